"""CPU oracle for the TIDE early-exit hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, what the reference (RightNow-AI/TIDE v0.2.1)
computes on its PyTorch path for one early-exit checkpoint, so that the CUDA
kernels of tide_b200 can be checked against it on identical inputs.  Only
tests/, __graft_entry__.smoke() and the cpu_baseline leg of bench.py may
import it, and only as the checker or the timed CPU baseline: the product
path (tide_b200) never imports or calls it, and fails loudly when its CUDA
library is missing.

The oracle is pinned against golden vectors produced by running the
reference's own Python code (tests/golden/make_golden.py); see
tests/test_oracle_golden.py.

Conventions: all arithmetic is float32 (numpy BLAS for the router GEMM);
bfloat16 values travel as uint16 bit patterns (numpy has no bfloat16), float16
as numpy.float16.
"""
from __future__ import annotations

import numpy as np

F32, F16, BF16 = "f32", "f16", "bf16"

# --------------------------------------------------------------- dtypes


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, round-to-nearest-even (finite inputs),
    as torch's Tensor.to(torch.bfloat16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def to_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """Model-dtype storage -> float32, the `.float()` of runtime.py:129,177."""
    if dtype == BF16:
        return bf16_to_f32(x)
    return x.astype(np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    """float32 -> model-dtype storage, the `.to(dtype)` of runtime.py:177."""
    if dtype == BF16:
        return f32_to_bf16(x)
    if dtype == F16:
        return x.astype(np.float16)
    return x.astype(np.float32)


# --------------------------------------------------------------- final norm


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """HF LlamaRMSNorm / Qwen3RMSNorm applied to a float32 input, the
    `final_norm(hidden.float())` of python/TIDE/runtime.py:129,177,186:
    weight * (x * rsqrt(mean(x^2) + eps)), every step in float32.
    Also the `python_rmsnorm` of tests/test_kernels.py:42-47."""
    x = np.asarray(x, dtype=np.float32)
    var = np.mean(np.square(x), axis=-1, keepdims=True, dtype=np.float32)
    rstd = np.float32(1.0) / np.sqrt(var + np.float32(eps), dtype=np.float32)
    return np.asarray(weight, dtype=np.float32) * (x * rstd)


def layer_norm(x: np.ndarray, weight: np.ndarray, bias: np.ndarray | None,
               eps: float) -> np.ndarray:
    """torch.nn.LayerNorm on a float32 input with float32 parameters (GPT-2's
    ln_f, universal.py's 'transformer.ln_f'): (x - mean) * rstd * w + b with
    the biased variance.  The reference itself raises on an fp16 ln_f fed a
    float32 input; the oracle defines the intended fp32 computation."""
    x = np.asarray(x, dtype=np.float32)
    mean = np.mean(x, axis=-1, keepdims=True, dtype=np.float32)
    d = x - mean
    var = np.mean(np.square(d), axis=-1, keepdims=True, dtype=np.float32)
    rstd = np.float32(1.0) / np.sqrt(var + np.float32(eps), dtype=np.float32)
    y = (x * rstd + (-rstd * mean)) * np.asarray(weight, dtype=np.float32)
    if bias is not None:
        y = y + np.asarray(bias, dtype=np.float32)
    return y


def final_norm(x: np.ndarray, norm: dict) -> np.ndarray:
    """norm = {"kind": "rms"|"layer", "weight": [H], "bias": [H] or None,
    "eps": float}; input already float32."""
    if norm["kind"] == "rms":
        return rms_norm(x, norm["weight"], norm["eps"])
    return layer_norm(x, norm["weight"], norm.get("bias"), norm["eps"])


# --------------------------------------------------------------- router


def silu(z: np.ndarray) -> np.ndarray:
    return z / (np.float32(1.0) + np.exp(-z, dtype=np.float32))


def sigmoid(z: np.ndarray) -> np.ndarray:
    return np.float32(1.0) / (np.float32(1.0) + np.exp(-z, dtype=np.float32))


def router_logits(normed: np.ndarray, down: np.ndarray, up: np.ndarray,
                  up_bias: float = 0.0) -> np.ndarray:
    """Pre-sigmoid router output, python/TIDE/router.py:18-19:
    up(SiLU(down(h))) with down [B, H], up [1, B] (nn.Linear weights, no bias
    in the reference, router.py:14-15) plus an optional scalar up bias."""
    h = np.asarray(normed, dtype=np.float32) @ np.asarray(down, dtype=np.float32).T
    z = silu(h.astype(np.float32)) @ np.asarray(up, dtype=np.float32).reshape(1, -1).T
    return z[:, 0].astype(np.float32) + np.float32(up_bias)


def router_scores(normed, down, up, up_bias: float = 0.0) -> np.ndarray:
    """TokenRouter.forward, python/TIDE/router.py:18-19 (sigmoid of the
    logits, squeezed to [N])."""
    return sigmoid(router_logits(normed, down, up, up_bias))


def score_rows(x: np.ndarray, dtype: str, norm: dict, down, up, up_bias=0.0) -> np.ndarray:
    """_score_router's PyTorch path, python/TIDE/runtime.py:128-130:
    router(final_norm(flat.float()))."""
    return router_scores(final_norm(to_f32(x, dtype), norm), down, up, up_bias)


def exit_decision(scores: np.ndarray, threshold: float,
                  exited: np.ndarray | None = None) -> np.ndarray:
    """new_exits = (scores > threshold) & ~exited_mask,
    python/TIDE/runtime.py:174 (strict comparison)."""
    m = np.asarray(scores, dtype=np.float32) > np.float32(threshold)
    if exited is not None:
        m &= ~exited
    return m


# --------------------------------------------------------------- compaction


def stable_partition(mask: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Indices of rows kept (mask False) and exited (mask True), each in
    ascending source order: the boolean gathers h[~mask] / h[mask] of
    python/TIDE/scheduler.py:89-90,98-100 and the prefix-sum split of
    csrc/kernels/batch_compact.cu:66-146."""
    mask = np.asarray(mask, dtype=bool)
    idx = np.arange(mask.shape[0], dtype=np.int64)
    return idx[~mask], idx[mask]


def batch_compact(x: np.ndarray, exit_mask: np.ndarray):
    """torch.ops.tide.batch_compact semantics (torch_bindings.cpp:136-198):
    (compacted, exited, continue_indices, exit_indices, num_remaining)."""
    keep, ex = stable_partition(np.asarray(exit_mask) != 0)
    return (x[keep], x[ex], keep.astype(np.int32), ex.astype(np.int32),
            np.array([keep.shape[0]], dtype=np.int32))


def exit_scatter(exited: np.ndarray, positions: np.ndarray, out: np.ndarray) -> np.ndarray:
    """output_buffer[exit_positions[i]] = exited_states[i]
    (csrc/kernels/exit_scatter.cu:16-37)."""
    out = out.copy()
    out[np.asarray(positions, dtype=np.int64)] = exited
    return out


def exit_projection(exited: np.ndarray, dtype: str, norm_weight: np.ndarray,
                    positions: np.ndarray, out: np.ndarray, eps: float) -> np.ndarray:
    """output_buffer[pos[i]] = RMSNorm(exited[i]) * w in fp32, rounded to the
    storage dtype (csrc/kernels/exit_projection.cu:20-57)."""
    y = from_f32(rms_norm(to_f32(exited, dtype), norm_weight, eps), dtype)
    out = out.copy()
    out[np.asarray(positions, dtype=np.int64)] = y
    return out


def fused_layernorm_route(x: np.ndarray, dtype: str, norm_weight, down_t, up_t,
                          eps: float) -> np.ndarray:
    """torch.ops.tide.fused_layernorm_route with its python oracle,
    tests/test_kernels.py:42-61: RMSNorm (eps) then x @ down_t -> SiLU ->
    @ up_t -> sigmoid; down_t [H, B], up_t [B, 1]."""
    normed = rms_norm(to_f32(x, dtype), norm_weight, eps)
    return router_scores(normed, np.asarray(down_t).T, np.asarray(up_t).reshape(1, -1))


# --------------------------------------------------------------- checkpoint


def checkpoint(x: np.ndarray, dtype: str, norm: dict, down, up, up_bias: float,
               threshold: float, positions: np.ndarray | None = None,
               slots: np.ndarray | None = None, out_buffer: np.ndarray | None = None):
    """One early-exit checkpoint on the active rows x [N, H]:
      scores   = router(final_norm(x.float()))           runtime.py:128-130
      exits    = scores > threshold                       runtime.py:174
      out[pos] = final_norm(x.float()).to(dtype)[exits]   runtime.py:177-178
      survivors compacted with their positions and slots  scheduler.py:98-100
    Returns a dict with scores, exit mask, survivor rows/positions/slots,
    exit positions and the updated output buffer."""
    n = x.shape[0]
    if positions is None:
        positions = np.arange(n, dtype=np.int64)
    xf = to_f32(x, dtype)
    normed = final_norm(xf, norm)
    scores = router_scores(normed, down, up, up_bias)
    exits = exit_decision(scores, threshold)
    keep, ex = stable_partition(exits)
    res = {
        "scores": scores,
        "exits": exits,
        "compact": x[keep],
        "positions": np.asarray(positions, dtype=np.int64)[keep],
        "exit_positions": np.asarray(positions, dtype=np.int64)[ex],
        "n_survivors": int(keep.shape[0]),
        "n_exits": int(ex.shape[0]),
    }
    if slots is not None:
        res["slots"] = np.asarray(slots, dtype=np.int32)[keep]
    if out_buffer is not None:
        out = out_buffer.copy()
        out[res["exit_positions"]] = from_f32(normed[ex], dtype)
        res["out_buffer"] = out
    return res


def forward_posthoc(all_hidden: list[np.ndarray], dtype: str, norm: dict,
                    routers: dict[int, dict], threshold: float, min_layers: int,
                    detail: bool = False):
    """The post-hoc exit loop of TIDERuntime.forward, python/TIDE/runtime.py:
    163-188, on the flattened hidden states all_hidden[l] [N, H] (index 0 =
    embeddings, index l+1 = output of decoder layer l).  routers maps a layer
    index to {"down", "up", "up_bias"}.  Returns (output_buffer in storage
    dtype, exits_per_layer, remaining_tokens); with detail=True also a dict
    with each token's exit layer (-1: never) and every router's scores."""
    n, h = all_hidden[-1].shape
    out = np.zeros((n, h), dtype=all_hidden[-1].dtype)
    exited = np.zeros(n, dtype=bool)
    exit_layer = np.full(n, -1, dtype=np.int64)
    scores: dict[int, np.ndarray] = {}
    exits_per_layer: dict[int, int] = {}
    for layer in sorted(routers):
        if layer < min_layers:
            continue
        hid = all_hidden[layer + 1]
        r = routers[layer]
        s = score_rows(hid, dtype, norm, r["down"], r["up"], r.get("up_bias", 0.0))
        scores[layer] = s
        new = exit_decision(s, threshold, exited)
        if new.any():
            normed = from_f32(final_norm(to_f32(hid, dtype), norm), dtype)
            out[new] = normed[new]
            exited |= new
            exit_layer[new] = layer
            exits_per_layer[layer] = int(new.sum())
    remaining = ~exited
    if remaining.any():
        normed = from_f32(final_norm(to_f32(all_hidden[-1], dtype), norm), dtype)
        out[remaining] = normed[remaining]
    if detail:
        return out, exits_per_layer, int(remaining.sum()), {"exit_layer": exit_layer,
                                                            "scores": scores}
    return out, exits_per_layer, int(remaining.sum())


# --------------------------------------------------------------- comparison


def ulp_distance(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """Distance in units in the last place between two arrays of the storage
    dtype (monotone integer mapping of the bit patterns)."""
    if dtype == BF16:
        ia, ib = a.astype(np.int32), b.astype(np.int32)
        bits = 16
    elif dtype == F16:
        ia, ib = a.view(np.uint16).astype(np.int32), b.view(np.uint16).astype(np.int32)
        bits = 16
    else:
        ia = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.int64)
        ib = np.ascontiguousarray(b, dtype=np.float32).view(np.uint32).astype(np.int64)
        bits = 32
    sign = 1 << (bits - 1)

    def mono(v):
        return np.where(v & sign, -(v & (sign - 1)), v)

    return np.abs(mono(ia) - mono(ib))
