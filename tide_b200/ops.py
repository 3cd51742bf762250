"""Python-side wrappers over torch.ops.tide for the early-exit path.

Everything here runs on CUDA tensors through the native operators; nothing
computes on the CPU.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from tide_b200 import _native
from tide_b200.capi import NORM_LAYER, NORM_RMS, PATH_AUTO


@dataclass
class NormSpec:
    """The final norm as the kernels see it: y = w * (x * rstd) (RMSNorm) or
    y = (x - mean) * rstd * w + b (LayerNorm), statistics in fp32."""
    kind: int
    weight: torch.Tensor          # fp32 [H]
    bias: Optional[torch.Tensor]  # fp32 [H] (LayerNorm) or None
    eps: float


def norm_spec(module: nn.Module, device: torch.device) -> NormSpec:
    """Read the final norm module found by the adapter (runtime.py:91).
    Understood: HF LlamaRMSNorm-family modules (weight * x_hat, with
    `variance_epsilon` or `eps`), torch.nn.RMSNorm and torch.nn.LayerNorm."""
    name = type(module).__name__
    w = getattr(module, "weight", None)
    if isinstance(module, nn.LayerNorm):
        if w is None:
            raise NotImplementedError("LayerNorm without elementwise affine is not supported")
        b = module.bias.detach().to(device, torch.float32).contiguous() if module.bias is not None else None
        return NormSpec(NORM_LAYER, w.detach().to(device, torch.float32).contiguous(), b,
                        float(module.eps))
    if "gemma" in name.lower():
        raise NotImplementedError(f"{name}: (1 + weight) RMSNorm is not supported by the kernels")
    is_rms = (hasattr(nn, "RMSNorm") and isinstance(module, nn.RMSNorm)) or "rmsnorm" in name.lower()
    if is_rms and w is not None:
        eps = getattr(module, "variance_epsilon", None)
        if eps is None:
            eps = getattr(module, "eps", None)
        if eps is None:
            eps = torch.finfo(torch.float32).eps
        return NormSpec(NORM_RMS, w.detach().to(device, torch.float32).contiguous(), None, float(eps))
    raise NotImplementedError(f"final norm module {name} is not one the kernels implement")


@dataclass
class PreparedRouter:
    """One router in the kernels' layout (tide_router_fold)."""
    down_t: torch.Tensor          # [H, B] fp32 (SIMT path)
    folded: Optional[torch.Tensor]  # [B, H] model dtype: down * norm_weight (tensor cores)
    colsum: torch.Tensor          # [B] fp32
    bias_proj: Optional[torch.Tensor]  # [B] fp32 (LayerNorm with bias)
    up: torch.Tensor              # [B] fp32
    up_bias: float
    bottleneck: int


def prepare_router(down: torch.Tensor, up: torch.Tensor, up_bias: float, norm: NormSpec,
                   dtype: torch.dtype) -> PreparedRouter:
    ops = _native.ops()
    _native.require_cuda(down, "router weights")
    fold_dtype = dtype if dtype in (torch.float16, torch.bfloat16) else torch.float32
    bias = norm.bias if norm.kind == NORM_LAYER else None
    down_t, folded, colsum, bias_proj = ops.router_fold(down.detach().float().contiguous(),
                                                        norm.weight, bias, fold_dtype)
    return PreparedRouter(down_t=down_t, folded=folded,
                          colsum=colsum, bias_proj=bias_proj if bias is not None else None,
                          up=up.detach().float().reshape(-1).contiguous(), up_bias=float(up_bias),
                          bottleneck=int(down.shape[0]))


class CheckpointRunner:
    """Owns the per-device workspace, counters and error word of
    torch.ops.tide.checkpoint and launches checkpoints on the current stream."""

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self.ops = _native.ops()
        self.workspace = torch.empty(0, dtype=torch.uint8, device=self.device)
        self.counts = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.error_word = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.last_path = None

    def _workspace(self, n_rows: int, hidden_dim: int) -> torch.Tensor:
        need = int(self.ops.checkpoint_workspace_size(n_rows, hidden_dim))
        if self.workspace.numel() < need:
            self.workspace = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self.workspace

    def run(self, x: torch.Tensor, router: PreparedRouter, norm: NormSpec, threshold: float, *,
            positions=None, slots=None, out_buffer=None, compact_out=None, positions_out=None,
            slots_out=None, exit_positions_out=None, scores_out=None, n_rows_dev=None,
            counts: Optional[torch.Tensor] = None, path: int = PATH_AUTO) -> torch.Tensor:
        """One checkpoint; returns the device counts tensor {survivors, exits}."""
        counts = self.counts if counts is None else counts
        ws = self._workspace(x.shape[0], x.shape[1])
        self.last_path = self.ops.checkpoint(
            x, n_rows_dev, norm.weight, norm.bias, norm.kind, norm.eps, router.down_t,
            router.folded, router.colsum, router.bias_proj, router.up, router.up_bias,
            float(threshold), positions, slots, out_buffer, compact_out, positions_out, slots_out,
            exit_positions_out, scores_out, counts, self.error_word, ws, path)
        return counts

    def norm_scatter(self, rows: torch.Tensor, positions: torch.Tensor, out_buffer: torch.Tensor,
                     norm: NormSpec) -> None:
        self.ops.norm_scatter(rows, positions, out_buffer, norm.weight, norm.bias, norm.kind,
                              norm.eps)

    def check_errors(self) -> None:
        """Read the device error word (one sync) and raise if a kernel flagged
        a fault; clears it."""
        e = int(self.error_word.item())
        if e:
            self.error_word.zero_()
            raise RuntimeError(f"tide_b200 kernel reported device error bits 0x{e:x} "
                               "(1: exit position out of range, 2: wait timeout, 4: bad row count)")
