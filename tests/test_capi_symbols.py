"""The C ABI library loads without a GPU, exports every function that
include/tide_b200.h declares, has a ctypes mirror with the header's struct
layout, and rejects bad arguments before touching the device."""
import ctypes
import re
import subprocess

import pytest

from tests.conftest import ROOT
from tide_b200 import _native, capi

HEADER = ROOT / "include" / "tide_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tide_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    names = declared_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), f"{n} declared in tide_b200.h but not exported"
    assert set(names) == set(capi.PROTOTYPES), "ctypes prototypes out of sync with the header"
    assert lib.tide_abi_version() == 1


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "probe.c"
    fields = [f for f, _ in capi.CheckpointArgs._fields_]
    body = "\n".join(f'  printf("{f} %zu\\n", offsetof(tide_checkpoint_args, {f}));' for f in fields)
    src.write_text(f"""#include <stdio.h>
#include <stddef.h>
#include "tide_b200.h"
int main(void) {{
  printf("size %zu\\n", sizeof(tide_checkpoint_args));
{body}
  return 0;
}}
""")
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    out = dict(line.split() for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                                        check=True).stdout.splitlines())
    assert int(out["size"]) == ctypes.sizeof(capi.CheckpointArgs)
    for f in fields:
        assert int(out[f]) == getattr(capi.CheckpointArgs, f).offset, f


def test_argument_errors_need_no_gpu():
    lib = _native.lib()
    # bad dtype
    rc = lib.tide_exit_scatter(7, None, None, None, 1, 8, 1, None, None)
    assert rc == 1 and b"dtype" in lib.tide_last_error()
    # bottleneck above 256
    rc = lib.tide_fused_layernorm_route(2, 1, 1, 1, 1, 1e-6, 1, 4, 64, 512, None)
    assert rc == 1
    # checkpoint without counts / workspace
    a = capi.CheckpointArgs(dtype=2, n_rows=4, hidden_dim=64, bottleneck_dim=16, n_total=4,
                            x=16, norm_weight=16, up=16)
    assert lib.tide_checkpoint(ctypes.byref(a), None) == 1
    a.counts_out = 16
    assert lib.tide_checkpoint(ctypes.byref(a), None) == 4  # workspace missing
    assert lib.tide_checkpoint_select_path(ctypes.byref(a)) < 0
    # zero-size requests are no-ops
    assert lib.tide_exit_scatter(2, None, None, None, 0, 8, 0, None, None) == 0
    assert lib.tide_norm_scatter(2, 0, None, None, None, None, None, 1e-5, 0, 8, 0, None, None) == 0


def test_workspace_sizes_grow_with_rows():
    lib = _native.lib()
    small = capi.CheckpointArgs(n_rows=128)
    big = capi.CheckpointArgs(n_rows=1 << 20)
    assert lib.tide_checkpoint_workspace_size(ctypes.byref(big)) > \
        lib.tide_checkpoint_workspace_size(ctypes.byref(small)) > 0
    assert lib.tide_batch_compact_workspace_size(0) > 0


def test_torch_extension_registers_operators():
    ops = _native.ops()
    for name in ("fused_layernorm_route", "batch_compact", "exit_scatter", "exit_projection",
                 "norm_scatter", "router_fold", "checkpoint", "checkpoint_workspace_size"):
        assert hasattr(ops, name), name
    assert ops.checkpoint_workspace_size(100000, 4096) > ops.checkpoint_workspace_size(1000, 4096) > 0


def test_operators_have_no_cpu_kernel():
    import torch
    ops = _native.ops()
    x = torch.zeros(4, 8)
    with pytest.raises(NotImplementedError):
        ops.exit_scatter(x, torch.zeros(4, dtype=torch.int32), x.clone())


def test_path_selection():
    """bf16/fp16 with folded weights: up to a row count set per hidden size
    from measured crossovers (5120 rows at H = 4096) the fused single-pass
    kernel when the router is 128 wide and a weight slice of H stays
    resident; above that, or when the fused kernel does not apply, the
    tensor-core split path (H % 64 == 0, B <= 256).  fp32 rows with folded
    fp32 weights and H % 32 == 0 take the split path too (error-compensated
    tf32 products); other shapes the SIMT path."""
    lib = _native.lib()

    def sel(**kw):
        base = dict(dtype=capi.DTYPE_BF16, n_rows=1000, hidden_dim=4096, bottleneck_dim=128,
                    n_total=1000, x=1 << 20, norm_weight=16, up=16, counts_out=16,
                    workspace=1 << 20, folded=1 << 21, colsum=16)
        base.update(kw)
        a = capi.CheckpointArgs(**base)
        return lib.tide_checkpoint_select_path(ctypes.byref(a))

    assert sel() == capi.PATH_TC                               # up to 5120 rows: fused single pass
    assert sel(n_rows=5120, n_total=5120) == capi.PATH_TC
    assert sel(n_rows=5121, n_total=5121) == capi.PATH_TC_SPLIT
    assert sel(n_rows=32768, n_total=32768) == capi.PATH_TC_SPLIT
    assert sel(dtype=capi.DTYPE_F16) == capi.PATH_TC
    assert sel(n_rows=32768, n_total=32768, dtype=capi.DTYPE_F16) == capi.PATH_TC_SPLIT
    assert sel(path=capi.PATH_TC) == capi.PATH_TC
    assert sel(dtype=capi.DTYPE_F32, folded=None) == capi.PATH_SIMT
    assert sel(dtype=capi.DTYPE_F32) == capi.PATH_TC_SPLIT     # fp32: 3 x tf32 split router
    assert sel(dtype=capi.DTYPE_F32, n_rows=8, n_total=8) == capi.PATH_TC_SPLIT
    assert sel(dtype=capi.DTYPE_F32, path=capi.PATH_TC) == capi.PATH_TC_SPLIT
    assert sel(dtype=capi.DTYPE_F32, hidden_dim=800) == capi.PATH_TC_SPLIT   # 800 = 25 x 32
    assert sel(dtype=capi.DTYPE_F32, hidden_dim=784) == capi.PATH_SIMT
    assert sel(dtype=capi.DTYPE_F32, path=capi.PATH_SIMT) == capi.PATH_SIMT
    assert sel(hidden_dim=4000) == capi.PATH_SIMT
    assert sel(bottleneck_dim=48) == capi.PATH_TC_SPLIT       # units padded to 128 (fused: 128 only)
    assert sel(bottleneck_dim=64) == capi.PATH_TC_SPLIT       # fused kernel: 128 units only
    assert sel(hidden_dim=8192, path=capi.PATH_TC) == capi.PATH_TC        # 16-CTA clusters, 8-chunk slices
    assert sel(hidden_dim=5120) == capi.PATH_TC                              # 16-CTA clusters, 5-chunk slices
    assert sel(hidden_dim=5120, n_rows=3584, n_total=3584) == capi.PATH_TC
    assert sel(hidden_dim=5120, n_rows=3585, n_total=3585) == capi.PATH_TC_SPLIT
    assert sel(hidden_dim=8192, n_rows=5632, n_total=5632) == capi.PATH_TC
    assert sel(hidden_dim=8192, n_rows=5633, n_total=5633) == capi.PATH_TC_SPLIT
    assert sel(hidden_dim=768, n_rows=8192, n_total=8192) == capi.PATH_TC     # GPT-2 width: SIMT mover on the split path
    assert sel(hidden_dim=768, n_rows=8193, n_total=8193) == capi.PATH_TC_SPLIT
    assert sel(hidden_dim=1024, n_rows=128, n_total=128) == capi.PATH_TC_SPLIT  # 2 KB rows: split wins
    assert sel(hidden_dim=1024, path=capi.PATH_TC) == capi.PATH_TC
    assert sel(hidden_dim=2048, n_rows=4096, n_total=4096) == capi.PATH_TC
    assert sel(hidden_dim=2048, n_rows=4097, n_total=4097) == capi.PATH_TC_SPLIT
    assert sel(hidden_dim=512, n_rows=128, n_total=128) == capi.PATH_TC_SPLIT
    assert sel(hidden_dim=512, path=capi.PATH_TC) == capi.PATH_TC
    assert sel(hidden_dim=16384, path=capi.PATH_TC) == capi.PATH_TC_SPLIT  # slice too large to stay resident
    assert sel(hidden_dim=768, path=capi.PATH_TC) == capi.PATH_TC   # cluster of 2
    assert sel(path=capi.PATH_TC_SPLIT) == capi.PATH_TC_SPLIT
    assert sel(folded=None) == capi.PATH_SIMT
    assert sel(path=capi.PATH_SIMT) == capi.PATH_SIMT
    assert sel(path=capi.PATH_TC, hidden_dim=4000) == -capi.ERR_UNSUPPORTED
    assert b"multiple of 64" in lib.tide_last_error()


def test_testhooks_library_mirrors_the_product_surface():
    """The test build (one look-back tile that never publishes, short wait
    bounds) loads without a GPU and exports the same C ABI."""
    from tide_b200 import build

    lib = ctypes.CDLL(str(build.TEST_LIB))
    capi.declare(lib)
    for n in declared_functions():
        assert hasattr(lib, n), n
    assert lib.tide_abi_version() == 1


def test_decode_entry_points_reject_bad_arguments_without_a_gpu():
    """The decode-side entry points (attention, cache append, norm scatter
    with a device count, the fused layer kernels) validate their arguments
    before any device call."""
    lib = _native.lib()
    ERR_INVALID, ERR_UNSUPPORTED = 1, 2
    # decode attention: head_dim 64, G = 3, a length past the cache
    assert lib.tide_decode_attention(2, 16, 16, 16, None, 16, 4, None, 8, 2, 64, 4, 32, 8, None,
                                     0.1, None, None) == ERR_UNSUPPORTED
    assert b"head_dim" in lib.tide_last_error()
    assert lib.tide_decode_attention(2, 16, 16, 16, None, 16, 4, None, 6, 2, 128, 4, 32, 8, None,
                                     0.1, None, None) == ERR_INVALID
    assert lib.tide_decode_attention(2, 16, 16, 16, None, 16, 4, None, 8, 2, 128, 4, 32, 33, None,
                                     0.1, None, None) == ERR_INVALID
    assert lib.tide_decode_attention(0, 16, 16, 16, None, 16, 4, None, 8, 2, 128, 4, 32, 8, None,
                                     0.1, None, None) == ERR_UNSUPPORTED  # fp32 caches
    # cache append: a host position past the cache
    assert lib.tide_kv_append(2, 16, 16, None, None, 4, 2, 128, 16, 16, 4, 32, 32, None, None,
                              None) == ERR_INVALID
    # norm scatter with a device count: bad norm type
    assert lib.tide_norm_scatter_rows(2, 9, 16, 16, None, 4, 64, 8, 16, 16, None, 1e-5, None,
                                      None) == ERR_INVALID
    # fused layer kernels: widths they do not take
    assert lib.tide_rms_norm(2, 16, None, None, 16, 16, 4, None, 100, 1e-6, None) == ERR_INVALID
    assert lib.tide_rms_norm(2, 16, None, None, 16, 16, 4, None, 16384, 1e-6, None) == ERR_INVALID
    assert lib.tide_silu_mul(2, 16, 16, 16, 4, None, 12, None) == ERR_INVALID
    assert lib.tide_qk_norm_rope(2, 16, 16, 16, 0, 0, None, None, 1e-6, 16, 1.0, 0, None, None,
                                 None, None, 4, 2, 1, 64, 16, 16, 16, 4, 8, None,
                                 None) == ERR_UNSUPPORTED
    # q/k/v row strides that do not cover the heads, or not multiples of 8
    assert lib.tide_qk_norm_rope(2, 16, 16, 16, 128, 0, None, None, 1e-6, 16, 1.0, 0, None, None,
                                 None, None, 4, 2, 1, 128, 16, 16, 16, 4, 8, None,
                                 None) == ERR_INVALID
    assert lib.tide_qk_norm_rope(2, 16, 16, 16, 0, 132, None, None, 1e-6, 16, 1.0, 0, None, None,
                                 None, None, 4, 2, 1, 128, 16, 16, 16, 4, 8, None,
                                 None) == ERR_INVALID
    # nothing to do: no rows
    assert lib.tide_rms_norm(2, None, None, None, None, None, 0, None, 64, 1e-6, None) == 0
