"""Seeded synthetic inputs for the early-exit path.

The reference publishes no dataset for this path; these generators produce
the shapes and value distributions the benchmark configurations name:

* ``k1``: fp32 hidden states [4096, 768] drawn N(0,1) x per-row U(0.5, 2),
  RMSNorm weight N(1, 0.02), eps 1e-5, router down/up weights N(0, 0.02),
  all from one CPU ``torch.Generator`` seeded 0, in that draw order.
* ``rows``: bf16/fp16 rows N(0,1) of any [N, H] with a unit norm weight and
  N(0, 0.02) router weights (the bandwidth-sweep and 8B-arch checkpoint
  shapes).

Draws happen on the CPU generator unless ``device`` is given, so the same
seed yields bit-identical inputs on any machine with this torch version.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def k1(n: int = 4096, h: int = 768, b: int = 128, seed: int = 0) -> dict:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, h, generator=g) * (torch.rand(n, 1, generator=g) * 1.5 + 0.5)
    w_norm = 1.0 + 0.02 * torch.randn(h, generator=g)
    down = 0.02 * torch.randn(b, h, generator=g)
    up = 0.02 * torch.randn(1, b, generator=g)
    return {"x": x, "norm_weight": w_norm, "norm_bias": None, "eps": 1e-5,
            "norm_kind": "rms", "down": down, "up": up}


def rows(n: int, h: int, dtype: torch.dtype, b: int = 128, seed: int = 0,
         norm_kind: str = "rms", device: str | None = None,
         unit_norm_weight: bool = True) -> dict:
    """Rows N(0,1) of `dtype`; router weights N(0, 0.02) (fp32)."""
    g = torch.Generator(device=device or "cpu").manual_seed(seed)
    dev = device or "cpu"
    x = torch.randn(n, h, generator=g, device=dev).to(dtype)
    if unit_norm_weight:
        w_norm = torch.ones(h, device=dev)
    else:
        w_norm = (1.0 + 0.02 * torch.randn(h, generator=g, device=dev)).to(dtype).float()
    nb = None
    if norm_kind == "layer":
        nb = (0.02 * torch.randn(h, generator=g, device=dev)).to(dtype).float()
    down = 0.02 * torch.randn(b, h, generator=g, device=dev)
    up = 0.02 * torch.randn(1, b, generator=g, device=dev)
    return {"x": x, "norm_weight": w_norm, "norm_bias": nb, "eps": 1e-5,
            "norm_kind": norm_kind, "down": down, "up": up}


def logit(p: float) -> float:
    return math.log(p / (1.0 - p))


def bias_for_exit_fraction(logits: np.ndarray | torch.Tensor, fraction: float,
                           threshold: float) -> float:
    """Scalar up-projection bias b such that a `fraction` of the rows satisfy
    sigmoid(z + b) > threshold for the given pre-bias logits z.  The cut is
    placed midway between two consecutive sorted logits so that no row sits
    on the threshold.  fraction 0 -> every row stays; 1 -> every row exits."""
    z = np.sort(np.asarray(torch.as_tensor(logits).double().cpu().numpy(), dtype=np.float64))
    n = z.shape[0]
    if n == 0:
        return 0.0
    k = n - int(round(fraction * n))  # rows below the cut
    if k <= 0:
        cut = z[0] - 1.0
    elif k >= n:
        cut = z[-1] + 1.0
    else:
        cut = 0.5 * (z[k - 1] + z[k])
    return float(logit(threshold) - cut)


def prebias_logits_torch(x: torch.Tensor, norm_kind: str, norm_weight: torch.Tensor,
                         norm_bias: torch.Tensor | None, eps: float, down: torch.Tensor,
                         up: torch.Tensor, chunk: int = 16384) -> torch.Tensor:
    """fp32 router logits without bias, computed with torch on x's device
    (used only to place the bias of a synthetic workload)."""
    out = []
    for s in range(0, x.shape[0], chunk):
        xf = x[s:s + chunk].float()
        if norm_kind == "rms":
            var = xf.pow(2).mean(-1, keepdim=True)
            nrm = norm_weight.float() * (xf * torch.rsqrt(var + eps))
        else:
            nrm = torch.nn.functional.layer_norm(xf, (xf.shape[-1],), norm_weight.float(),
                                                 None if norm_bias is None else norm_bias.float(),
                                                 eps)
        h = torch.nn.functional.silu(nrm @ down.float().T)
        out.append((h @ up.float().reshape(1, -1).T)[:, 0])
    return torch.cat(out) if out else torch.zeros(0)
