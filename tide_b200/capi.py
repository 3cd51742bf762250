"""ctypes declarations of the C ABI in include/tide_b200.h.

The structure and every prototype below mirror the header field for field;
tests/test_capi_symbols.py checks that each declared symbol is exported."""
from __future__ import annotations

import ctypes as C

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
NORM_RMS, NORM_LAYER = 0, 1
PATH_AUTO, PATH_SIMT, PATH_TC, PATH_TC_SPLIT = 0, 1, 2, 3
OK = 0
ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE, ERR_ALIGNMENT = 1, 2, 3, 4, 5
NOALLOC_MAX_ROWS = 1048576
DEVERR_POSITION, DEVERR_TIMEOUT, DEVERR_COUNT = 1, 2, 4

p = C.c_void_p
i32, i64, f32, sz = C.c_int32, C.c_int64, C.c_float, C.c_size_t


class CheckpointArgs(C.Structure):
    _fields_ = [
        ("dtype", i32), ("norm_type", i32), ("path", i32), ("reserved0", i32),
        ("n_rows", i64), ("hidden_dim", i64), ("bottleneck_dim", i64), ("n_total", i64),
        ("x", p), ("n_rows_dev", p),
        ("norm_weight", p), ("norm_bias", p), ("eps", f32), ("up_bias", f32),
        ("down_t", p), ("folded", p), ("colsum", p), ("bias_proj", p), ("up", p),
        ("threshold", f32), ("reserved1", i32),
        ("positions_in", p), ("slots_in", p),
        ("out_buffer", p), ("compact_out", p), ("positions_out", p), ("slots_out", p),
        ("exit_positions_out", p), ("scores_out", p), ("counts_out", p), ("error_word", p),
        ("workspace", p), ("workspace_bytes", sz),
    ]


# name -> (restype, argtypes); the exported surface of libtide_b200.so
PROTOTYPES = {
    "tide_abi_version": (C.c_int, []),
    "tide_last_error": (C.c_char_p, []),
    "tide_fused_layernorm_route": (C.c_int, [C.c_int, p, p, p, p, f32, p, i64, i64, i64, p]),
    "tide_batch_compact_workspace_size": (sz, [i64]),
    "tide_batch_compact": (C.c_int, [C.c_int, p, p, p, p, p, p, p, i64, i64, p, sz, p, p]),
    "tide_batch_compact_noalloc": (C.c_int, [C.c_int, p, p, p, p, p, p, p, i64, i64, p, p]),
    "tide_exit_scatter": (C.c_int, [C.c_int, p, p, p, i64, i64, i64, p, p]),
    "tide_exit_projection": (C.c_int, [C.c_int, p, p, p, p, f32, i64, i64, i64, p, p]),
    "tide_norm_scatter": (C.c_int, [C.c_int, C.c_int, p, p, p, p, p, f32, i64, i64, i64, p, p]),
    "tide_gather_rows": (C.c_int, [C.c_int, p, i64, p, p, i64, i64, p, p, p]),
    "tide_norm_at_positions": (C.c_int, [C.c_int, C.c_int, p, p, p, i64, i64, i64, p, p, p, f32,
                                         p, p]),
    "tide_decode_attention": (C.c_int, [C.c_int, p, p, p, p, p, i64, p, i64, i64, i64, i64, i64,
                                        i64, p, f32, p, p]),
    "tide_kv_append": (C.c_int, [C.c_int, p, p, p, p, i64, i64, i64, p, p, i64, i64, i64, p,
                                 p, p]),
    "tide_norm_scatter_rows": (C.c_int, [C.c_int, C.c_int, p, p, p, i64, i64, i64, p, p, p, f32,
                                         p, p]),
    "tide_rms_norm": (C.c_int, [C.c_int, p, p, p, p, p, i64, p, i64, f32, p]),
    "tide_qk_norm_rope": (C.c_int, [C.c_int, p, p, p, i64, i64, p, p, f32, p, f32, i64, p, p, p, p, i64,
                                    i64, i64, i64, p, p, p, i64, i64, p, p]),
    "tide_silu_mul": (C.c_int, [C.c_int, p, p, p, i64, p, i64, p]),
    "tide_router_fold": (C.c_int, [C.c_int, p, p, p, i64, i64, p, p, p, p, p]),
    "tide_checkpoint_workspace_size": (sz, [C.POINTER(CheckpointArgs)]),
    "tide_checkpoint": (C.c_int, [C.POINTER(CheckpointArgs), p]),
    "tide_checkpoint_select_path": (C.c_int, [C.POINTER(CheckpointArgs)]),
}


def declare(lib: C.CDLL) -> None:
    for name, (res, args) in PROTOTYPES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def check(lib: C.CDLL, rc: int, what: str) -> None:
    if rc != OK:
        raise RuntimeError(f"{what} failed ({rc}): {lib.tide_last_error().decode()}")
