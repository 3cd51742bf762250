"""Helpers for the GPU parity tests: call the C ABI (libtide_b200.so) through
ctypes with torch tensors as device memory, and build oracle inputs."""
from __future__ import annotations

import ctypes

import numpy as np
import torch

import tide_oracle as O
from tide_b200 import _native, capi

TORCH2C = {torch.float32: capi.DTYPE_F32, torch.float16: capi.DTYPE_F16,
           torch.bfloat16: capi.DTYPE_BF16}
TORCH2O = {torch.float32: O.F32, torch.float16: O.F16, torch.bfloat16: O.BF16}


def ptr(t):
    return None if t is None else t.data_ptr()


def stream():
    return torch.cuda.current_stream().cuda_stream


def lib():
    return _native.lib()


def storage_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def fold(down: torch.Tensor, norm_w: torch.Tensor, norm_b, dtype: torch.dtype):
    """tide_router_fold through the C ABI; returns (down_t, folded, colsum, bias_proj)."""
    B, H = down.shape
    dev = down.device
    down_t = torch.empty(H, B, device=dev)
    fdt = dtype if dtype != torch.float32 else torch.float32
    folded = torch.empty(B, H, device=dev, dtype=fdt)
    colsum = torch.empty(B, device=dev)
    bias_proj = torch.zeros(B, device=dev)
    rc = lib().tide_router_fold(TORCH2C[fdt], ptr(down.float().contiguous()), ptr(norm_w),
                                ptr(norm_b), H, B, ptr(down_t), ptr(folded), ptr(colsum),
                                ptr(bias_proj) if norm_b is not None else None, stream())
    capi.check(lib(), rc, "tide_router_fold")
    return down_t, folded, colsum, (bias_proj if norm_b is not None else None)


class Checkpoint:
    """One tide_checkpoint call through ctypes, owning all its buffers."""

    def __init__(self, x, norm_kind, norm_w, norm_b, eps, down, up, up_bias, threshold, *,
                 positions=None, slots=None, out_buffer=None, n_total=None, compact=True,
                 n_rows_dev=None, path=capi.PATH_AUTO, scores=True, exit_positions=True):
        dev = x.device
        n, H = x.shape
        self.x = x
        self.down_t, self.folded, self.colsum, self.bias_proj = fold(down, norm_w, norm_b, x.dtype)
        self.up = up.float().reshape(-1).contiguous()
        self.norm_w, self.norm_b = norm_w, norm_b
        self.positions, self.slots = positions, slots
        self.out_buffer = out_buffer
        self.compact_out = torch.empty_like(x) if compact else None
        self.positions_out = torch.full((n,), -7, dtype=torch.int64, device=dev)
        self.slots_out = torch.full((n,), -7, dtype=torch.int32, device=dev) if slots is not None else None
        self.exit_positions_out = torch.full((n,), -7, dtype=torch.int64, device=dev) if exit_positions else None
        self.scores_out = torch.full((n,), -1.0, device=dev) if scores else None
        self.counts = torch.full((2,), -1, dtype=torch.int32, device=dev)
        self.error_word = torch.zeros(1, dtype=torch.int32, device=dev)
        a = capi.CheckpointArgs()
        a.dtype = TORCH2C[x.dtype]
        a.norm_type = capi.NORM_RMS if norm_kind == "rms" else capi.NORM_LAYER
        a.path = path
        a.n_rows, a.hidden_dim, a.bottleneck_dim = n, H, down.shape[0]
        a.n_total = n_total if n_total is not None else (out_buffer.shape[0] if out_buffer is not None else 0)
        a.x = ptr(x)
        a.n_rows_dev = ptr(n_rows_dev)
        a.norm_weight, a.norm_bias, a.eps, a.up_bias = ptr(norm_w), ptr(norm_b), eps, up_bias
        a.down_t, a.folded, a.colsum, a.bias_proj, a.up = (ptr(self.down_t), ptr(self.folded),
                                                           ptr(self.colsum), ptr(self.bias_proj),
                                                           ptr(self.up))
        a.threshold = threshold
        a.positions_in, a.slots_in = ptr(positions), ptr(slots)
        a.out_buffer, a.compact_out = ptr(out_buffer), ptr(self.compact_out)
        a.positions_out, a.slots_out = ptr(self.positions_out), ptr(self.slots_out)
        a.exit_positions_out, a.scores_out = ptr(self.exit_positions_out), ptr(self.scores_out)
        a.counts_out, a.error_word = ptr(self.counts), ptr(self.error_word)
        need = lib().tide_checkpoint_workspace_size(ctypes.byref(a))
        self.workspace = torch.empty(need, dtype=torch.uint8, device=dev)
        a.workspace, a.workspace_bytes = ptr(self.workspace), need
        self.args = a

    def path(self) -> int:
        return lib().tide_checkpoint_select_path(ctypes.byref(self.args))

    def __call__(self):
        rc = lib().tide_checkpoint(ctypes.byref(self.args), stream())
        capi.check(lib(), rc, "tide_checkpoint")
        return self


def oracle_norm(kind, w, b, eps):
    return {"kind": kind, "weight": w.detach().cpu().numpy(),
            "bias": None if b is None else b.detach().cpu().numpy(), "eps": eps}
