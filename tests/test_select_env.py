"""Protocol selector, tuning tables and environment configuration."""

import json

import pytest

from numa_allreduce_b200.parallel.select import AlgoSelector, build_table, parse_table
from numa_allreduce_b200.utils.env import ALGO_IDS, ALGO_NAMES, parse_groups, read_env


def test_builtin_defaults():
    s = AlgoSelector(8, has_nvls=True)
    assert s.choose(4096) == "oneshot"
    assert s.choose(4 << 20) == "twoshot_pipe"
    assert s.choose(256 << 20) == "twoshot_pipe"
    assert AlgoSelector(2, has_nvls=True).choose(256 << 20) == "twoshot_pipe"
    s = AlgoSelector(8, has_nvls=False)
    assert s.choose(64 << 20) == "twoshot_pipe"
    assert s.choose(256 << 20) == "twoshot_pipe"
    assert AlgoSelector(1).choose(123) == "copy"


def _sizes():
    out = set()
    for k in range(4, 31):
        for d in (-16, 0, 16):
            if (1 << k) + d > 0:
                out.add((1 << k) + d)
    return sorted(out)


def _tables():
    """(label, world size, steps source) for the built-in steps and every
    entry of the shipped tuning table."""
    from numa_allreduce_b200.parallel.select import DEFAULT_TABLE_PATH

    cases = [("builtin", ws, None) for ws in range(2, 9)]
    if DEFAULT_TABLE_PATH.exists():
        for e in parse_table(json.loads(DEFAULT_TABLE_PATH.read_text())):
            cases.append((f"table ws{e.world_size} {e.dtype} nvls={e.nvls}", e.world_size, e))
    return cases


@pytest.mark.parametrize("label,ws,entry", _tables(), ids=lambda v: v if isinstance(v, str) else None)
def test_python_and_native_choice_agree(label, ws, entry):
    """The Python selector and the native planner's automatic choice (used by
    the C ABI) pick the same protocol for every size, with and without
    multicast and groups."""
    from numa_allreduce_b200.ops import _ext

    ops = _ext.load()
    for has_nvls in (True, False):
        if entry is not None and entry.nvls and not has_nvls:
            continue
        for has_groups in (True, False):
            s = AlgoSelector(ws, has_nvls=has_nvls, has_groups=has_groups,
                             entries=[entry] if entry is not None else [])
            dtype = entry.dtype if entry is not None else "bfloat16"
            limits, algos, fallback = s.native_table(dtype)
            for n in _sizes():
                py = s.choose(n, dtype)
                nat = ops.choose_auto(ws, n, has_nvls, has_groups, limits, algos, fallback)
                assert py == ("nccl" if nat == 100 else ALGO_NAMES[nat]), (label, has_nvls, has_groups, n)


def test_shipped_table_is_valid():
    from numa_allreduce_b200.parallel.select import DEFAULT_TABLE_PATH

    if not DEFAULT_TABLE_PATH.exists():
        pytest.skip("no tuning table shipped")
    obj = json.loads(DEFAULT_TABLE_PATH.read_text())
    entries = parse_table(obj)
    assert {e.world_size for e in entries} >= {8}
    for e in entries:
        assert all(a in ALGO_IDS or a == "nccl" for _, a in e.steps)
    for ws, split in obj.get("hybrid", {}).items():
        permille, cp, cn = split
        assert 0 < permille < 1000 and 1 <= cp and 1 <= cn and cp + cn <= 148


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


def test_table_ignores_noise_level_differences():
    # NCCL ahead by 1% at one size: keep this library's protocol (no extra step)
    speeds = {1 << 20: {"twoshot_pipe": 100.0, "nccl": 80.0}, 1 << 22: {"twoshot_pipe": 99.0, "nccl": 100.0},
              1 << 24: {"twoshot_pipe": 100.0, "nccl": 90.0}, 1 << 28: {"twoshot_pipe": 90.0, "nccl": 100.0}}
    rows = [{"world_size": 8, "dtype": "bfloat16", "nvls": True, "bytes": b, "algo": a, "busbw_gbs": v}
            for b, d in speeds.items() for a, v in d.items()]
    e = parse_table(build_table(rows))[0]
    assert e.steps == [(1 << 24, "twoshot_pipe"), (1 << 28, "nccl")] and e.fallback == "nccl"


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
    monkeypatch.setenv("NAB_HYBRID", "350,56,88")
    assert read_env().hybrid == (350, 56, 88)
    monkeypatch.setenv("NAB_HYBRID", "350,56")
    with pytest.raises(ValueError):
        read_env()
    monkeypatch.delenv("NAB_HYBRID")
    monkeypatch.setenv("NAB_ALGO", "nope")
    with pytest.raises(ValueError):
        read_env()
    assert parse_groups(" 0,2 | 1,3 ") == [[0, 2], [1, 3]]
