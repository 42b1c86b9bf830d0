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
                  "steps": [[262144, "oneshot"], [17179869184, "hybrid"]],
                  "fallback": "nccl"}],
     "hybrid": {"8": [350, 56, 88]}}

``hybrid`` (optional) gives, per world size, the hybrid protocol's split:
the P2P share of the message in per mille and the CTAs of its P2P and NVLS
parts.

The same steps drive the native communicator's automatic choice (the C ABI's
``numa_all_reduce_*`` calls): :class:`NumaAwareAllReduce` hands the entry of
each dtype to it, and without a table both sides use the built-in steps that
the native library defines (``builtin_auto_table``), so the Python path and
the C path pick the same protocol for every message.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

from ..ops import _ext
from ..utils.env import ALGO_IDS, ALGO_NAMES, NCCL, NCCL_ID

DEFAULT_TABLE_PATH = Path(__file__).with_name("tuning_b200.json")
_BIG = 1 << 62


def _algo_id(name: str) -> int:
    return NCCL_ID if name == NCCL else ALGO_IDS[name]


def _algo_name(algo_id: int) -> str:
    return NCCL if int(algo_id) == NCCL_ID else ALGO_NAMES[int(algo_id)]


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
    hybrid: tuple[int, int, int] | None = None  # measured split of the hybrid protocol

    @staticmethod
    def builtin_steps(world_size: int, has_nvls: bool) -> tuple[list[tuple[int, str]], str]:
        """Steps used when no measured table covers a configuration, as the
        native library defines them (one definition for both paths)."""
        limits, algos, fallback = _ext.load().builtin_auto_table(world_size, has_nvls)
        return [(int(b), ALGO_NAMES[int(a)]) for b, a in zip(limits, algos)], _algo_name(fallback)

    @classmethod
    def load(cls, world_size: int, has_nvls: bool, has_groups: bool, path: str | None = None,
             forced: str | None = None) -> "AlgoSelector":
        entries: list[Entry] = []
        hybrid = None
        p = Path(path) if path else DEFAULT_TABLE_PATH
        if p.exists():
            obj = json.loads(p.read_text())
            entries = parse_table(obj)
            h = obj.get("hybrid", {}).get(str(world_size))
            if h is not None:
                hybrid = tuple(int(v) for v in h)
        return cls(world_size, has_nvls, has_groups, entries, forced, hybrid)

    def steps_for(self, dtype: str) -> tuple[list[tuple[int, str]], str]:
        """The (steps, fallback) this selector uses for a dtype."""
        e = self._entry(dtype)
        if e is not None:
            return e.steps, e.fallback
        return self.builtin_steps(self.world_size, self.has_nvls)

    def native_table(self, dtype: str) -> tuple[list[int], list[int], int]:
        """The steps of a dtype as the native communicator takes them."""
        steps, fallback = self.steps_for(dtype)
        return [int(b) for b, _ in steps], [_algo_id(a) for _, a in steps], _algo_id(fallback)

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
        steps, fallback = self.steps_for(dtype)
        for limit, algo in steps:
            if nbytes <= limit:
                return self._validate(algo)
        return self._validate(fallback)

    def _validate(self, algo: str) -> str:
        """Substitutes what this group cannot run (same rules as the native
        ``choose_auto``)."""
        if algo == NCCL:
            return algo
        if algo not in ALGO_IDS:
            raise ValueError(f"unknown protocol {algo!r}")
        if not self.has_nvls:
            if algo == "nvls_twoshot":
                return "twoshot"
            if algo == "nvls_oneshot":
                return "oneshot"
            if algo == "hybrid":
                return "twoshot_pipe"
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


def build_table(results: list[dict], nccl_key: str = NCCL, hybrid: dict | None = None,
                margin: float = 0.03) -> dict:
    """Builds a table from sweep rows ``{"world_size", "dtype", "nvls", "bytes",
    "algo", "busbw_gbs"}``: for each size the fastest protocol wins, except
    that a protocol within ``margin`` of the winner is kept when it is the
    previous size's choice or when the winner is NCCL and it is this
    library's (differences that small are run-to-run noise and would only
    add steps); adjacent sizes with the same choice merge into one step.
    ``hybrid`` maps a world size to the measured split of the hybrid
    protocol."""
    groups: dict[tuple, dict[int, dict[str, float]]] = {}
    for r in results:
        k = (int(r["world_size"]), str(r["dtype"]), bool(r.get("nvls", False)))
        groups.setdefault(k, {}).setdefault(int(r["bytes"]), {})[str(r["algo"])] = float(r["busbw_gbs"])
    entries = []
    for (ws, dtype, nvls), by_size in sorted(groups.items()):
        steps: list[list] = []
        for size in sorted(by_size):
            cands = by_size[size]
            algo, best = max(cands.items(), key=lambda kv: kv[1])
            prev = steps[-1][1] if steps else None
            if prev is not None and prev != algo and cands.get(prev, 0.0) >= (1 - margin) * best:
                algo = prev
            elif algo == nccl_key:
                ours = {a: v for a, v in cands.items() if a != nccl_key}
                if ours:
                    a2, v2 = max(ours.items(), key=lambda kv: kv[1])
                    if v2 >= (1 - margin) * best:
                        algo = a2
            if steps and steps[-1][1] == algo:
                steps[-1][0] = size
            else:
                steps.append([size, algo])
        fallback = NCCL
        if steps and steps[-1][1] != nccl_key:
            steps[-1][0] = _BIG  # the custom path wins at the largest size measured: keep it
            fallback = steps[-1][1]
        entries.append({"world_size": ws, "dtype": dtype, "nvls": nvls, "steps": steps, "fallback": fallback})
    out = {"version": 1, "entries": entries}
    if hybrid:
        out["hybrid"] = {str(k): list(v) for k, v in hybrid.items()}
    return out
