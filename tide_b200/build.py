"""In-tree build of the native parts of tide_b200.

Produces, next to this file:
  libtide_b200.so  -- the C ABI (include/tide_b200.h) and every CUDA kernel,
                      compiled for sm_100a only, CUDA runtime linked statically;
  _C.so            -- the thin PyTorch operator layer (torch.ops.tide.*) that
                      links libtide_b200.so.

nvcc cross-compiles for sm_100a without a GPU, so this runs anywhere the CUDA
12.9 toolkit is installed.  Rebuilds only what is older than its sources.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libtide_b200.so"
EXT = PKG / "_C.so"
# The same kernels built with one test hook: tile TEST_TILE of every stable
# partition never publishes its look-back status, and look-back waits give up
# after a short bound, so tests can make a bounded device wait run out
# (TIDE_DEVERR_TIMEOUT) without any fault.  Only tests load it.
TEST_LIB = PKG / "libtide_b200_testhooks.so"
TEST_TILE = 3

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                     "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]

CU_SOURCES = ["capi.cu", "tc_checkpoint.cu", "tc_route_pair.cu", "tc_fused.cu", "move_bulk.cu",
              "noalloc.cu", "decode_attn.cu", "decode_layer.cu"]
HEADERS = ["common.cuh", "move_bulk.cuh", "simt_kernels.cuh", "tc_checkpoint.cuh", "tc_ptx.cuh"]


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr)


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in deps if d.exists())


def _headers() -> list[Path]:
    return [CSRC / h for h in HEADERS] + [INCLUDE / "tide_b200.h"]


def _lib_jobs(build_dir: Path, extra: list[str], force: bool) -> tuple[list[Path], list[list[str]]]:
    build_dir.mkdir(parents=True, exist_ok=True)
    objs, jobs = [], []
    for src in CU_SOURCES:
        s = CSRC / src
        o = build_dir / (src + ".o")
        objs.append(o)
        if force or not _newer(o, [s, *_headers(), Path(__file__)]):
            jobs.append([NVCC, *NVCC_FLAGS, *extra, "-c", str(s), "-o", str(o)])
    return objs, jobs


def build_lib(verbose: bool = False, force: bool = False) -> Path:
    """libtide_b200.so and its test-hook twin, compiled in parallel."""
    objs, jobs = _lib_jobs(BUILD, [], force)
    tobjs, tjobs = _lib_jobs(BUILD / "testhooks", [f"-DTIDE_TEST_UNPUBLISHED_TILE={TEST_TILE}"], force)
    all_jobs = jobs + tjobs
    with ThreadPoolExecutor(max_workers=max(1, min(len(all_jobs), os.cpu_count() or 1))) as ex:
        list(ex.map(lambda c: _run(c, verbose), all_jobs))
    if force or jobs or not _newer(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs)], verbose)
    if force or tjobs or not _newer(TEST_LIB, tobjs):
        _run([NVCC, *ARCH, "-shared", "-o", str(TEST_LIB), *map(str, tobjs)], verbose)
    return LIB


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths()
    if str(CUDA_HOME / "include") not in inc:
        inc.append(str(CUDA_HOME / "include"))
    libdir = cpp_extension.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = ["-O2", "-std=c++17", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
              f"-I{INCLUDE}", *[f"-I{p}" for p in inc],
              f"-I{sysconfig.get_paths()['include']}"]
    ldflags = [f"-L{libdir}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch",
               f"-Wl,-rpath,{libdir}", f"-L{PKG}", "-ltide_b200", "-Wl,-rpath,$ORIGIN"]
    return cflags, ldflags


def build_ext(verbose: bool = False, force: bool = False) -> Path:
    src = CSRC / "torch_ops.cpp"
    if not force and _newer(EXT, [src, INCLUDE / "tide_b200.h", LIB, Path(__file__)]):
        return EXT
    cflags, ldflags = _torch_flags()
    _run(["g++", *cflags, "-shared", str(src), "-o", str(EXT), *ldflags], verbose)
    return EXT


def build(verbose: bool = False, force: bool = False) -> None:
    build_lib(verbose, force)
    build_ext(verbose, force)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
