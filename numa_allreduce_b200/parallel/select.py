"""Protocol choice per (world size, dtype, message size).

The reference has a single gate: a fixed byte cap from vLLM's table
(src/numa_all_reduce.py:142-152) above which it returns ``None`` and the caller
uses NCCL. Here the cap is a measured crossover: the table lists, for each
world size and dtype, ascending ``[max_bytes, protocol]`` steps; a message
larger than the last step gets ``fallback`` (``"nccl"`` means: return ``None``
so the caller uses NCCL). Tables are JSON, produced by ``bench/sweep.py``
(``--write-table``) from device-timed bus bandwidth, and loaded from
``NAB_TUNING_FILE`` or the file shipped next to this module.

File format::

    {"version": 1,
     "entries": [{"world_size": 8, "dtype": "bfloat16", "nvls": true,
                  "steps": [[262144, "oneshot"], [17179869184, "nvls_twoshot"]],
                  "fallback": "nccl"}]}
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

from ..utils.env import ALGO_IDS, NCCL

DEFAULT_TABLE_PATH = Path(__file__).with_name("tuning_b200.json")
_BIG = 1 << 62


@dataclass
class Entry:
    world_size: int
    dtype: str
    nvls: bool
    steps: list[tuple[int, str]]
    fallback: str = NCCL


@dataclass
class AlgoSelector:
    world_size: int
    has_nvls: bool = False
    has_groups: bool = False
    entries: list[Entry] = field(default_factory=list)
    forced: str | None = None

    @staticmethod
    def builtin_steps(world_size: int, has_nvls: bool) -> list[tuple[int, str]]:
        """Defaults used when no measured table covers a configuration: the
        push one-shot up to 512 KiB, the pipelined store-based two-shot above
        (measured fastest on 2 and 8 B200s; NVLS two-shot trailed it)."""
        return [(512 << 10, "oneshot"), (_BIG, "twoshot_pipe")]

    @classmethod
    def load(cls, world_size: int, has_nvls: bool, has_groups: bool, path: str | None = None,
             forced: str | None = None) -> "AlgoSelector":
        entries: list[Entry] = []
        p = Path(path) if path else DEFAULT_TABLE_PATH
        if p.exists():
            entries = parse_table(json.loads(p.read_text()))
        return cls(world_size, has_nvls, has_groups, entries, forced)

    def _entry(self, dtype: str) -> Entry | None:
        best = None
        for e in self.entries:
            if e.world_size != self.world_size or e.dtype != dtype:
                continue
            if e.nvls and not self.has_nvls:
                continue
            # prefer the NVLS entry when NVLS is available
            if best is None or (e.nvls and not best.nvls):
                best = e
        return best

    def choose(self, nbytes: int, dtype: str = "bfloat16", registered: bool = False) -> str:
        """Protocol name, or ``"nccl"`` when NCCL should be used instead."""
        if self.world_size == 1:
            return "copy"
        if self.forced and self.forced != "auto":
            return self._validate(self.forced)
        e = self._entry(dtype)
        steps = e.steps if e else self.builtin_steps(self.world_size, self.has_nvls)
        fallback = e.fallback if e else NCCL
        for limit, algo in steps:
            if nbytes <= limit:
                return self._validate(algo)
        return fallback

    def _validate(self, algo: str) -> str:
        if algo == NCCL:
            return algo
        if algo not in ALGO_IDS:
            raise ValueError(f"unknown protocol {algo!r}")
        if algo.startswith("nvls") and not self.has_nvls:
            return "twoshot" if algo == "nvls_twoshot" else "oneshot"
        if algo == "hier" and not self.has_groups:
            return "twoshot"
        return algo


def parse_table(obj: dict) -> list[Entry]:
    if obj.get("version") != 1:
        raise ValueError("unsupported tuning table version")
    out = []
    for e in obj.get("entries", []):
        steps = [(int(a), str(b)) for a, b in e["steps"]]
        if steps != sorted(steps, key=lambda s: s[0]):
            raise ValueError("tuning steps must be ascending")
        out.append(Entry(int(e["world_size"]), str(e["dtype"]), bool(e.get("nvls", False)), steps,
                         str(e.get("fallback", NCCL))))
    return out


def build_table(results: list[dict], nccl_key: str = NCCL) -> dict:
    """Builds a table from sweep rows ``{"world_size", "dtype", "nvls", "bytes",
    "algo", "busbw_gbs"}``: for each size the fastest protocol wins; adjacent
    sizes with the same winner merge into one step."""
    groups: dict[tuple, dict[int, dict[str, float]]] = {}
    for r in results:
        k = (int(r["world_size"]), str(r["dtype"]), bool(r.get("nvls", False)))
        groups.setdefault(k, {}).setdefault(int(r["bytes"]), {})[str(r["algo"])] = float(r["busbw_gbs"])
    entries = []
    for (ws, dtype, nvls), by_size in sorted(groups.items()):
        steps: list[list] = []
        for size in sorted(by_size):
            algo = max(by_size[size].items(), key=lambda kv: kv[1])[0]
            if steps and steps[-1][1] == algo:
                steps[-1][0] = size
            else:
                steps.append([size, algo])
        fallback = NCCL
        if steps and steps[-1][1] != nccl_key:
            steps[-1][0] = _BIG  # the custom path wins at the largest size measured: keep it
            fallback = steps[-1][1]
        entries.append({"world_size": ws, "dtype": dtype, "nvls": nvls, "steps": steps, "fallback": fallback})
    return {"version": 1, "entries": entries}
