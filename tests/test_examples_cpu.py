"""The example CLIs parse their arguments and refuse unsafe profiler use
without a GPU (their GPU paths run in the benchmarks)."""

import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    return subprocess.run([sys.executable, *args], cwd=ROOT, capture_output=True, text=True, timeout=120)


def test_demo_help():
    r = _run("examples/numa_allreduce_demo.py", "--help")
    assert r.returncode == 0 and "--sizes-mb" in r.stdout


def test_profile_help_and_modes():
    r = _run("examples/profile_allreduce.py", "--help")
    assert r.returncode == 0 and "benchmark" in r.stdout and "nvtx" in r.stdout


def test_profile_ncu_mode_needs_single_process():
    r = _run("examples/profile_allreduce.py", "--mode", "ncu")
    assert r.returncode != 0 and "--single" in r.stderr
