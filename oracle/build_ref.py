"""Test infrastructure: build the reference's own CUDA operators for sm_100a.

The reference ships its GPU path as a torch extension: csrc/extensions/
torch_bindings.cpp and the four kernels in csrc/kernels/ (fused_layernorm_route,
batch_compact, exit_scatter, exit_projection).  This recipe compiles those
files where they lie in the reference checkout (nothing is copied) into
oracle/_ref/tide_ref_C.so, with `-Dtide=tide_ref` so that the operators
register under `torch.ops.tide_ref` and load beside this repository's own
`torch.ops.tide` in one process.  The GPU tests use it as a checker: the
oracle and the product are compared against the reference's kernels run on
the same B200.  Nothing in the product imports, links or runs it.

Usage: python oracle/build_ref.py [reference checkout]   (default: the
TIDE_REFERENCE_ROOT environment variable).  Without a checkout it does
nothing; the .so built here travels with the repository to the GPU box.
The reference's batch_compact launches one block of n_tokens threads for its
prefix sums (csrc/kernels/batch_compact.cu:175), so it is only ever called
with n_tokens <= 1024 (above that the launch fails and the scatter that
follows would read unset prefix buffers).
"""
from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "tide_ref_C.so"
SOURCES = ["csrc/extensions/torch_bindings.cpp", "csrc/kernels/fused_layernorm_route.cu",
           "csrc/kernels/batch_compact.cu", "csrc/kernels/exit_scatter.cu",
           "csrc/kernels/exit_projection.cu"]


def _run(cmd: list[str], verbose: bool) -> None:
    import subprocess

    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(ref_root: str | None = None, verbose: bool = False) -> Path | None:
    """Compile the reference's kernels (nvcc, sm_100a) and its bindings (g++,
    against the installed torch) into oracle/_ref/tide_ref_C.so; returns its
    path, or None without a reference checkout."""
    ref_root = ref_root or os.environ.get("TIDE_REFERENCE_ROOT")
    if not ref_root or not Path(ref_root, SOURCES[0]).is_file():
        return None
    srcs = [Path(ref_root, s) for s in SOURCES]
    newest = max(p.stat().st_mtime for p in srcs + [Path(__file__)])
    if LIB.is_file() and LIB.stat().st_mtime >= newest:
        return LIB
    sys.path.insert(0, str(HERE.parent))
    from tide_b200.build import NVCC, _torch_flags

    tmp = OUT / "build"
    tmp.mkdir(parents=True, exist_ok=True)
    rename = "-Dtide=tide_ref"  # C++ namespace and operator namespace both become tide_ref
    objs = []
    for src in srcs:
        obj = tmp / (src.stem + ".o")
        if src.suffix == ".cu":
            _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                  "-Xcompiler", "-fPIC", rename, "-c", str(src), "-o", str(obj)], verbose)
        else:
            cflags, _ = _torch_flags()
            _run(["g++", *cflags, rename, "-c", str(src), "-o", str(obj)], verbose)
        objs.append(str(obj))
    _, ldflags = _torch_flags()
    ldflags = [f for f in ldflags if f not in ("-ltide_b200", "-Wl,-rpath,$ORIGIN")
               and not f.startswith("-L" + str(HERE.parent / "tide_b200"))]
    _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(LIB), *objs,
          *[f"-Xlinker={f[4:]}" if f.startswith("-Wl,") else f for f in ldflags]], verbose)
    shutil.rmtree(tmp, ignore_errors=True)
    return LIB


if __name__ == "__main__":
    path = build(sys.argv[1] if len(sys.argv) > 1 else None, verbose=True)
    print(path if path else "no reference checkout given: nothing built")
