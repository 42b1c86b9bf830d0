"""Protocol selector, tuning tables and environment configuration."""

import json

import pytest

from numa_allreduce_b200.parallel.select import AlgoSelector, build_table, parse_table
from numa_allreduce_b200.utils.env import parse_groups, read_env


def test_builtin_defaults():
    s = AlgoSelector(8, has_nvls=True)
    assert s.choose(4096) == "oneshot"
    assert s.choose(64 << 20) == "twoshot_pipe"
    s = AlgoSelector(8, has_nvls=False)
    assert s.choose(64 << 20) == "twoshot_pipe"
    assert AlgoSelector(1).choose(123) == "copy"


def test_forced_and_capabilities():
    assert AlgoSelector(4, forced="nccl").choose(16) == "nccl"
    assert AlgoSelector(4, has_nvls=False, forced="nvls_twoshot").choose(16) == "twoshot"
    assert AlgoSelector(4, has_groups=False, forced="hier").choose(16) == "twoshot"
    assert AlgoSelector(4, has_groups=True, forced="hier").choose(16) == "hier"
    with pytest.raises(ValueError):
        AlgoSelector(4, forced="bogus").choose(16)


def test_table_round_trip(tmp_path):
    rows = []
    for size, winner in [(4096, "oneshot"), (65536, "oneshot"), (1 << 20, "twoshot"), (1 << 28, "nccl")]:
        for algo in ("oneshot", "twoshot", "nccl"):
            rows.append({"world_size": 4, "dtype": "bfloat16", "nvls": False, "bytes": size, "algo": algo,
                         "busbw_gbs": 100.0 if algo == winner else 10.0})
    table = build_table(rows)
    entries = parse_table(table)
    assert entries[0].steps[0] == (65536, "oneshot")
    path = tmp_path / "t.json"
    path.write_text(json.dumps(table))
    s = AlgoSelector.load(4, has_nvls=False, has_groups=False, path=str(path))
    assert s.choose(1000) == "oneshot"
    assert s.choose(1 << 20) == "twoshot"
    assert s.choose(1 << 28) == "nccl"
    assert s.choose(1 << 30) == "nccl"
    # other dtypes fall back to the built-in steps
    assert s.choose(1 << 30, dtype="float32") == "twoshot_pipe"


def test_table_custom_wins_at_top():
    rows = [{"world_size": 8, "dtype": "bfloat16", "nvls": True, "bytes": b, "algo": a,
             "busbw_gbs": {"nvls_twoshot": 900.0, "nccl": 700.0}[a]}
            for b in (1 << 20, 1 << 28) for a in ("nvls_twoshot", "nccl")]
    e = parse_table(build_table(rows))[0]
    assert e.fallback == "nvls_twoshot"
    s = AlgoSelector(8, has_nvls=True, entries=[e])
    assert s.choose(1 << 34) == "nvls_twoshot"


def test_env(monkeypatch):
    monkeypatch.setenv("NAB_ALGO", "hier")
    monkeypatch.setenv("NAB_HIER_GROUPS", "0,1,2,3|4,5,6,7")
    monkeypatch.setenv("NAB_MAX_SIZE", "0x1000")
    monkeypatch.setenv("NAB_NVLS", "0")
    e = read_env()
    assert e.algo == "hier" and e.hier_groups == [[0, 1, 2, 3], [4, 5, 6, 7]]
    assert e.max_size == 4096 and e.nvls is False
    monkeypatch.setenv("NAB_ALGO", "nope")
    with pytest.raises(ValueError):
        read_env()
    assert parse_groups(" 0,2 | 1,3 ") == [[0, 2], [1, 3]]
