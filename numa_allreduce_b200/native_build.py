"""In-tree build of the native library for sm_100a (B200).

Produces two shared objects next to this file:

* ``_C.so``     the core plus the torch op bindings (``torch.ops.nab.*``),
                linked against torch and the CUDA runtime torch already loads;
* ``libnab.so`` the core plus the plain C ABI, with the CUDA runtime linked
                statically, for callers that do not use Python or torch.

Object files go to ``_build/`` and are rebuilt only when a source, any header
or the flags change (content hashes), so repeated calls are cheap. Every CUDA
file is compiled for ``sm_100a`` only; nvcc cross-compiles on hosts without a
GPU.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
TORCH_LIB = PKG_DIR / "_C.so"
PLAIN_LIB = PKG_DIR / "libnab.so"
# Debug variant: the same sources with the device bounds checks compiled in
# (-DNAB_DEBUG_BOUNDS=1); loaded instead of _C.so when NAB_DEBUG_BUILD=1.
DEBUG_TORCH_LIB = PKG_DIR / "_C_debug.so"
DEBUG_DEFINES = ["-DNAB_DEBUG_BOUNDS=1"]

CORE_SOURCES = [
    "nab_allreduce.cu",
    "nab_fused.cu",
    "nab_gemm_sm100.cu",
    "nab_llama.cu",
    "nab_attn_sm100.cu",
    "nab_comm.cpp",
    "nab_kerr.cpp",
    "nab_nvls.cpp",
    "nab_capi.cpp",
]
TORCH_SOURCES = ["nab_torch.cpp"]
# Linked into libnab.so only: the allocation-free entry point, whose static
# scratch array should not ride along in the torch extension.
PLAIN_ONLY_SOURCES = ["nab_noalloc.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cuda_home() -> Path:
    for cand in (os.environ.get("CUDA_HOME"), os.environ.get("CUDA_PATH"), "/usr/local/cuda"):
        if cand and (Path(cand) / "bin" / "nvcc").exists():
            return Path(cand)
    nvcc = shutil.which("nvcc")
    if nvcc:
        return Path(nvcc).resolve().parent.parent
    raise RuntimeError("nvcc not found: set CUDA_HOME")


def _torch_flags() -> tuple[list[str], list[str], str]:
    import torch
    from torch.utils import cpp_extension

    incs = [f"-I{p}" for p in cpp_extension.include_paths()]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    lib_dir = str(Path(torch.__file__).resolve().parent / "lib")
    return incs, [f"-D_GLIBCXX_USE_CXX11_ABI={abi}"], lib_dir


def _headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def _compile_cmd(src: Path, obj: Path, torch_src: bool, incs: list[str], defs: list[str]) -> list[str]:
    cuda = cuda_home()
    base_inc = [f"-I{CSRC}", f"-I{cuda / 'include'}"]
    if src.suffix == ".cu":
        cmd = [str(cuda / "bin" / "nvcc"), "-c", str(src), "-o", str(obj), "-O3", "-std=c++17",
               *ARCH_FLAGS, "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
               "-Xptxas", "-warn-spills", *base_inc, *defs]
    else:
        cmd = ["g++", "-c", str(src), "-o", str(obj), "-O3", "-std=c++17", "-fPIC", "-Wall",
               "-Wno-unused-function", *base_inc, *defs]
        if torch_src:
            cmd += incs
    return cmd


def _compile_one(src: Path, torch_src: bool, incs, defs, hdr_digest, verbose) -> Path:
    cmd_probe = _compile_cmd(src, Path("X"), torch_src, incs, defs)
    key = hashlib.sha256()
    key.update(src.read_bytes())
    key.update(hdr_digest.encode())
    # the key must not depend on where the tree lives (a copy elsewhere reuses the objects)
    key.update(" ".join(cmd_probe).replace(str(PKG_DIR), "<pkg>").encode())
    obj = BUILD_DIR / f"{src.stem}-{key.hexdigest()[:16]}.o"
    if obj.exists():
        return obj
    tmp = obj.with_suffix(".o.tmp")
    cmd = _compile_cmd(src, tmp, torch_src, incs, defs)
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compiling {src.name} failed:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout, res.stderr, file=sys.stderr)
    tmp.rename(obj)
    return obj


def _link(out: Path, objs: list[Path], extra: list[str], verbose: bool) -> None:
    key = hashlib.sha256(("\n".join(o.name for o in objs) + " ".join(extra)).encode()).hexdigest()[:16]
    stamp = BUILD_DIR / f"{out.name}.{key}.stamp"
    if out.exists() and stamp.exists():
        return
    tmp = out.with_suffix(".so.tmp")
    cmd = ["g++", "-shared", "-o", str(tmp), *[str(o) for o in objs], *extra]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"linking {out.name} failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out)
    for old in BUILD_DIR.glob(f"{out.name}.*.stamp"):
        old.unlink()
    stamp.write_text(key)


def ptxas_report(source: str = "nab_allreduce.cu") -> str:
    """Registers, spills and shared memory per kernel (``-Xptxas -v``)."""
    cuda = cuda_home()
    src = CSRC / source
    cmd = [str(cuda / "bin" / "nvcc"), "-c", str(src), "-o", os.devnull, "-O3", "-std=c++17",
           *ARCH_FLAGS, "-Xptxas", "-v", f"-I{CSRC}", "--expt-relaxed-constexpr"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    return res.stdout + res.stderr


def build(verbose: bool = False, jobs: int | None = None, debug: bool = False) -> dict[str, str]:
    """Compiles and links both libraries; returns their paths. ``debug``
    builds only the torch library, with the device bounds checks, as
    ``_C_debug.so``."""
    BUILD_DIR.mkdir(exist_ok=True)
    incs, defs, torch_lib = _torch_flags()
    if debug:
        defs = defs + DEBUG_DEFINES
    hdr = _headers_digest()
    cuda = cuda_home()
    jobs = jobs or min(8, os.cpu_count() or 2)
    plain_sources = [] if debug else PLAIN_ONLY_SOURCES
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        core_f = [ex.submit(_compile_one, CSRC / s, False, incs, defs, hdr, verbose) for s in CORE_SOURCES]
        torch_f = [ex.submit(_compile_one, CSRC / s, True, incs, defs, hdr, verbose) for s in TORCH_SOURCES]
        plain_f = [ex.submit(_compile_one, CSRC / s, False, incs, defs, hdr, verbose) for s in plain_sources]
        core = [f.result() for f in core_f]
        tobj = [f.result() for f in torch_f]
        pobj = [f.result() for f in plain_f]
    cuda_lib = str(cuda / "lib64")
    torch_out = DEBUG_TORCH_LIB if debug else TORCH_LIB
    _link(torch_out, core + tobj,
          [f"-L{torch_lib}", "-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda", "-ltorch_cuda",
           f"-L{cuda_lib}", "-lcudart", f"-Wl,-rpath,{torch_lib}"], verbose)
    if debug:
        return {"torch": str(torch_out)}
    _link(PLAIN_LIB, core + pobj,
          [f"-L{cuda_lib}", "-lcudart_static", "-ldl", "-lrt", "-lpthread"], verbose)
    # drop objects that no longer correspond to any current source (either variant)
    live = {o.name for o in core + tobj + pobj}
    dbg = {o.name for o in _objects(debug=True)} if DEBUG_TORCH_LIB.exists() else set()
    for o in BUILD_DIR.glob("*.o"):
        if o.name not in live and o.name not in dbg:
            o.unlink()
    return {"torch": str(TORCH_LIB), "plain": str(PLAIN_LIB)}


def _objects(debug: bool) -> list[Path]:
    """Object paths the given variant's current sources map to (no compiling)."""
    incs, defs, _ = _torch_flags()
    if debug:
        defs = defs + DEBUG_DEFINES
    hdr = _headers_digest()
    out = []
    for names, torch_src in ((CORE_SOURCES, False), (TORCH_SOURCES, True)):
        for n in names:
            src = CSRC / n
            key = hashlib.sha256()
            key.update(src.read_bytes())
            key.update(hdr.encode())
            key.update(" ".join(_compile_cmd(src, Path("X"), torch_src, incs, defs)).replace(str(PKG_DIR), "<pkg>")
                       .encode())
            out.append(BUILD_DIR / f"{src.stem}-{key.hexdigest()[:16]}.o")
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, debug="--debug" in sys.argv))
