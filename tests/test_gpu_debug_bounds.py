"""The device bounds checks of the debug build (-DNAB_DEBUG_BOUNDS=1).

``compute-sanitizer`` is closed on this pool; instead, a debug variant of the
library (``_C_debug.so``, loaded with ``NAB_DEBUG_BUILD=1``) checks on the
device the rank and world size of every launch, that each CTA's slots lie
inside the workspace (slot capacity), the RankData slot of the pull protocol,
and pack indices before the accesses they guard. A violation is recorded in
the error record (code 2, stage "bounds check") and the access is skipped: no
trap, no assert.

Run in a child process (the two variants register the same torch ops):
every emulable protocol must still be bit-exact with no check firing, and a
launch whose rank is out of range must be caught before that rank touches
memory, after which a reset makes the group usable again.
"""

import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = textwrap.dedent("""
    import torch
    from numa_allreduce_b200.ops import _ext
    from numa_allreduce_b200.ops.allreduce import EmulatedGroup
    from numa_allreduce_b200.parallel.schedule import HierSchedule, reference_allreduce

    ops = _ext.load()
    assert _ext.loaded_path().endswith("_C_debug.so"), _ext.loaded_path()
    assert ops.debug_bounds_build()
    torch.cuda.set_device(0)
    ws = 4
    groups = [[0, 1], [2, 3]]
    scheds = {"oneshot": HierSchedule.oneshot(ws), "twoshot": HierSchedule.twoshot(ws),
              "twoshot_pipe": HierSchedule.twoshot(ws), "hier": HierSchedule.from_groups(groups)}
    with EmulatedGroup(ws, chunk_max=16 << 10, groups=groups) as g:
        for algo, sched in scheds.items():
            for n in (8, 8 * 3 + 8, 4096 * 7 + 40, 1 << 20):
                if algo == "oneshot" and n * 2 > (1 << 20):
                    continue
                xs = [torch.randn(n, device="cuda", generator=torch.Generator(device="cuda").manual_seed(r + n))
                      .to(torch.bfloat16) for r in range(ws)]
                outs = g.all_reduce(xs, algo=algo)
                torch.cuda.synchronize()
                assert g.error_codes() == [0] * ws, (algo, n, g.error_states())
                ref = reference_allreduce([x.cpu() for x in xs], sched)
                assert all(torch.equal(o.cpu(), ref) for o in outs), (algo, n)
        # rank 0's view claims rank 4 of 4: its CTAs must stop before any access
        xs = [torch.ones(4096, device="cuda", dtype=torch.bfloat16) for _ in range(ws)]
        outs = [torch.zeros_like(x) for x in xs]
        ops.debug_emulate_bad_rank(g.fas, xs, outs, 8)  # twoshot_pipe
        torch.cuda.synchronize()
        code, rank, peer, stage, block, epoch, observed, count = g.error_states()[0]
        assert code == 2 and stage == 13 and observed == ws, g.error_states()[0]
        g.reset()
        outs = g.all_reduce(xs, algo="twoshot_pipe")
        torch.cuda.synchronize()
        assert g.error_codes() == [0] * ws
        assert all(torch.all(o == ws) for o in outs)
    print("debug bounds ok")
""")


def test_debug_build_checks_and_catches_bad_launch():
    env = dict(os.environ, NAB_DEBUG_BUILD="1", PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, "-c", SCRIPT], env=env, cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and "debug bounds ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
