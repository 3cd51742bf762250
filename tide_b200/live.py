"""Live early exit: after each checkpoint the later layers run only on the
tokens that are still active.

The reference evaluates its routers post hoc: every layer runs on every
token and the exit buffer is assembled afterwards (python/TIDE/runtime.py:
151-188).  Its scheduler (python/TIDE/scheduler.py:39-120) and config
(`compaction_threshold`, `kv_cache_strategy`, python/TIDE/config.py:14-20)
describe the live variant without running it.  Here it runs: at each router
layer the checkpoint kernel scores the active rows, writes the exiting ones
final-normed to the output buffer and compacts the survivors (rows and
positions) into the dense buffer that the next layer takes as its input.

Exited tokens stay visible to the attention of later layers through the
reference's declared K/V policy, "zero_pad" (python/TIDE/runtime.py:194-221):
from the layer after its exit on, a token's key and value are zeros (not
masked).  Attention itself runs over the whole [batch, seq] layout (zeros
in the exited rows), so its cost does not shrink; the projections and the
MLP, which dominate a layer, run on the active rows only.

Supported layer families: Llama-style decoder layers (q/k/v/o projections,
optional per-head q/k RMSNorm as in Qwen3, rotary embeddings, gated MLP) and
GPT-2 blocks.  Inputs without padding only.  For 16-bit Llama-family models
the layers' elementwise work (RMSNorms with the residual adds, q/k norm +
rotary, SiLU gate) runs on fused kernels that round where the HF modules
round (tide_b200/csrc/decode_layer.cu); projections stay the modules' own.

LiveDecoder does the same for decoding: per-row exits whose later layers
skip the row, a KV cache addressed by slot, and steps free of host reads,
each one CUDA-graph replay.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, pos: Optional[torch.Tensor],
            B: int, S: int, scale: float) -> torch.Tensor:
    """Causal attention of the active rows q/k/v [n, heads, d] (token index
    b * S + s in `pos`; None = all B * S tokens in order) over the whole
    [B, S] layout, exited tokens' keys and values being zeros.  Returns
    [n, heads_q * d]."""
    n, nh, d = q.shape
    nkv = k.shape[1]
    if pos is not None:
        qf = q.new_zeros(B * S, nh, d)
        kf = k.new_zeros(B * S, nkv, d)
        vf = v.new_zeros(B * S, nkv, d)
        qf.index_copy_(0, pos, q)
        kf.index_copy_(0, pos, k)
        vf.index_copy_(0, pos, v)
        q, k, v = qf, kf, vf
    o = F.scaled_dot_product_attention(q.view(B, S, nh, d).transpose(1, 2),
                                       k.view(B, S, nkv, d).transpose(1, 2),
                                       v.view(B, S, nkv, d).transpose(1, 2),
                                       is_causal=True, scale=scale, enable_gqa=nh != nkv)
    o = o.transpose(1, 2).reshape(B * S, nh * d)
    return o if pos is None else o.index_select(0, pos)


class _LlamaFamily:
    """Llama / Qwen3 / Mistral-style decoder layers (HF modules' weights)."""

    def __init__(self, model: nn.Module):
        inner = model.model
        self.embed = inner.embed_tokens
        self.rotary = inner.rotary_emb
        self.layers = inner.layers
        self.norm = inner.norm
        cfg = model.config
        if getattr(cfg, "sliding_window", None) and getattr(cfg, "use_sliding_window", True) \
                and "mistral" in type(model).__name__.lower():
            raise NotImplementedError("sliding-window attention is not supported in live mode")

    def embed_tokens(self, ids: torch.Tensor) -> torch.Tensor:
        return self.embed(ids).reshape(ids.numel(), -1)

    def layer(self, i: int, h: torch.Tensor, pos: Optional[torch.Tensor], seq_pos: torch.Tensor,
              B: int, S: int) -> torch.Tensor:
        layer = self.layers[i]
        attn = layer.self_attn
        d = attn.head_dim
        n = h.shape[0]
        x = layer.input_layernorm(h)
        q = attn.q_proj(x).view(n, -1, d)
        k = attn.k_proj(x).view(n, -1, d)
        v = attn.v_proj(x).view(n, -1, d)
        if getattr(attn, "q_norm", None) is not None:
            q = attn.q_norm(q)
            k = attn.k_norm(k)
        cos, sin = self.rotary(v, seq_pos.view(1, -1))
        cos, sin = cos[0].unsqueeze(1), sin[0].unsqueeze(1)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        o = _attend(q, k, v, pos, B, S, float(attn.scaling))
        h = h + attn.o_proj(o)
        return h + layer.mlp(layer.post_attention_layernorm(h))


    # ---- decode with a KV cache addressed by slot (LiveDecoder)
    def kv_heads(self) -> int:
        a = self.layers[0].self_attn
        return a.k_proj.out_features // a.head_dim

    def head_dim(self) -> int:
        return self.layers[0].self_attn.head_dim

    def _qkv(self, layer, h: torch.Tensor, seq_pos: torch.Tensor):
        attn = layer.self_attn
        d = attn.head_dim
        n = h.shape[0]
        x = layer.input_layernorm(h)
        q = attn.q_proj(x).view(n, -1, d)
        k = attn.k_proj(x).view(n, -1, d)
        v = attn.v_proj(x).view(n, -1, d)
        if getattr(attn, "q_norm", None) is not None:
            q = attn.q_norm(q)
            k = attn.k_norm(k)
        cos, sin = self.rotary(v, seq_pos.view(1, -1))
        cos, sin = cos[0].unsqueeze(1), sin[0].unsqueeze(1)
        return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin, v

    def prefill_layer(self, i: int, h: torch.Tensor, B: int, S: int, kc: torch.Tensor,
                      vc: torch.Tensor) -> torch.Tensor:
        """Layer i on every token of B sequences of S positions ([B*S, H]),
        storing its keys and values in slots 0..B-1, positions 0..S-1."""
        layer = self.layers[i]
        attn = layer.self_attn
        seq = torch.arange(S, device=h.device).repeat(B)
        q, k, v = self._qkv(layer, h, seq)
        nkv, d = k.shape[1], k.shape[2]
        kc[:B, :, :S] = k.view(B, S, nkv, d).transpose(1, 2)
        vc[:B, :, :S] = v.view(B, S, nkv, d).transpose(1, 2)
        o = _attend(q, k, v, None, B, S, float(attn.scaling))
        h = h + attn.o_proj(o)
        return h + layer.mlp(layer.post_attention_layernorm(h))

    def decode_layer(self, i: int, h: torch.Tensor, slots: torch.Tensor, n_live: torch.Tensor,
                     pos: torch.Tensor, length: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor,
                     err: torch.Tensor) -> torch.Tensor:
        """Layer i for one new token of each row of h [B, H], of which the
        first n_live (device int32 [1]) are active; their sequences sit in
        cache `slots` (int32 [B]).  Their keys and values go to position
        `pos` (device int32 [1]) of those slots (tide_kv_append); attention
        reads positions [0, length) of those slots only (tide_decode_attention,
        length = pos + 1 on the device).  Rows past n_live go through the
        projections and the MLP (the GEMMs read the weights once whatever the
        row count of a decode batch) but neither write the cache nor attend;
        their outputs are not used."""
        from tide_b200 import _native

        ops = _native.ops()
        layer = self.layers[i]
        attn = layer.self_attn
        n = h.shape[0]
        q, k, v = self._qkv(layer, h, pos.long().expand(n).contiguous())
        ops.kv_append(k.to(kc.dtype).contiguous(), v.to(vc.dtype).contiguous(), slots, n_live,
                      kc, vc, 0, pos, err)
        o = torch.empty_like(q)
        ops.decode_attention(q.contiguous(), kc, vc, slots, o, kc.shape[2], float(attn.scaling),
                             err, n_live, length)
        h = h + attn.o_proj(o.view(n, -1))
        return h + layer.mlp(layer.post_attention_layernorm(h))


    # ---- the same decode layer on fused kernels (tide_b200/csrc/decode_layer.cu)
    def fused_decode_ok(self) -> bool:
        """True when every layer is one the fused kernels reproduce: RMSNorm
        input / post-attention / final norms, head_dim 128, optional q/k
        RMSNorm, a rotary embedding with a fixed inv_freq buffer, and a SiLU
        gated MLP."""
        rot = self.rotary
        if getattr(rot, "rope_type", "default") not in ("default", "llama3", "linear") or \
                not isinstance(getattr(rot, "inv_freq", None), torch.Tensor):
            return False
        H = self.embed.embedding_dim
        if H % 8 or H > 8192:  # tide_rms_norm's row layout
            return False
        norms = [self.norm]
        for layer in self.layers:
            a, m = layer.self_attn, layer.mlp
            if getattr(a, "head_dim", 0) != 128 or not all(
                    hasattr(m, n) for n in ("gate_proj", "up_proj", "down_proj")):
                return False
            if m.gate_proj.out_features % 8:  # tide_silu_mul's vectors
                return False
            # nn.SiLU, or transformers' SiLUActivation (F.silu)
            if type(getattr(m, "act_fn", None)).__name__ not in ("SiLU", "SiLUActivation"):
                return False
            norms += [layer.input_layernorm, layer.post_attention_layernorm]
            if getattr(a, "q_norm", None) is not None:
                norms += [a.q_norm, a.k_norm]
        return all(hasattr(n, "variance_epsilon") and isinstance(getattr(n, "weight", None),
                                                                  torch.Tensor) for n in norms)

    def _inv_freq(self) -> torch.Tensor:
        """The rotary module's inv_freq as its forward uses it (.float(): a
        model cast to 16 bits holds the buffer rounded to 16 bits)."""
        f = getattr(self, "_inv_freq_f32", None)
        if f is None or f.device != self.rotary.inv_freq.device:
            f = self._inv_freq_f32 = self.rotary.inv_freq.float().contiguous()
        return f

    def _qkv_weight(self, i: int, attn):
        """Layer i's q_proj, k_proj and v_proj weights stacked into one
        [q + k + v out, H] matrix (and their biases, if any), built once and
        rebuilt when a weight changes.  At a decode batch's row count one GEMM
        on the stacked weights runs faster than three: the k and v
        projections alone are too narrow to use the GPU well.  It costs a
        copy of those weights (1.7 GB for a 36-layer 8B model)."""
        projs = (attn.q_proj, attn.k_proj, attn.v_proj)
        tag = tuple((m.weight.data_ptr(), m.weight._version) for m in projs)
        cache = self.__dict__.setdefault("_qkv_cache", {})
        ent = cache.get(i)
        if ent is None or ent[0] != tag:
            w = torch.cat([m.weight.detach() for m in projs], 0)
            b = None
            if any(m.bias is not None for m in projs):
                b = torch.cat([m.bias.detach() if m.bias is not None else
                               torch.zeros(m.out_features, dtype=w.dtype, device=w.device)
                               for m in projs])
            ent = cache[i] = (tag, w, b)
        return ent[1], ent[2]

    def rms_norm(self, module, h: torch.Tensor, n_live: torch.Tensor,
                 delta: Optional[torch.Tensor] = None):
        """module's RMSNorm of h (of h + delta, also returned) for the live
        rows: (normed, sum or None)."""
        from tide_b200 import _native

        out = torch.empty_like(h)
        total = torch.empty_like(h) if delta is not None else None
        _native.ops().rms_norm(h, delta, total, module.weight, out, float(module.variance_epsilon),
                               n_live)
        return out, total

    def layer_fused(self, i: int, h: torch.Tensor, pos: Optional[torch.Tensor],
                    seq_pos: torch.Tensor, B: int, S: int) -> torch.Tensor:
        """layer() of the live prefill on the fused kernels: the input norm,
        the q/k norms with the rotary embedding at each row's own position,
        the residual add with the post-attention norm, and the SiLU gate are
        one kernel each; projections and attention as in layer()."""
        from tide_b200 import _native

        ops = _native.ops()
        layer = self.layers[i]
        attn = layer.self_attn
        n = h.shape[0]
        x, _ = self.rms_norm(layer.input_layernorm, h, None)
        q = attn.q_proj(x).view(n, -1, 128)
        k = attn.k_proj(x).view(n, -1, 128)
        v = attn.v_proj(x).view(n, -1, 128)
        hq, hkv = q.shape[1], k.shape[1]
        qn, kn = getattr(attn, "q_norm", None), getattr(attn, "k_norm", None)
        # q, k and v land at their tokens' places in [B * S] buffers (a one-
        # position "cache" per token, the tokens' indices as slots): the
        # exited tokens' keys and values stay zero, their queries are never
        # read back.  With every token active the rows are the tokens and v
        # is written onto itself.
        if pos is None:
            slots = torch.arange(n, dtype=torch.int32, device=h.device)
            q_full = torch.empty(n, hq, 128, dtype=q.dtype, device=q.device)
            k_full = torch.empty(n, hkv, 1, 128, dtype=k.dtype, device=k.device)
            v_full = v.view(n, hkv, 1, 128)
        else:
            slots = pos.to(torch.int32)
            q_full = torch.empty(B * S, hq, 128, dtype=q.dtype, device=q.device)
            k_full = torch.zeros(B * S, hkv, 1, 128, dtype=k.dtype, device=k.device)
            v_full = torch.zeros(B * S, hkv, 1, 128, dtype=v.dtype, device=v.device)
        ops.qk_norm_rope(q, k, v, qn.weight if qn is not None else None,
                         kn.weight if kn is not None else None,
                         float(qn.variance_epsilon) if qn is not None else 0.0,
                         self._inv_freq(), float(getattr(self.rotary, "attention_scaling", 1.0)),
                         0, None, seq_pos.long().contiguous(), slots, None, q_full,
                         k_full, v_full, None)
        o = _attend(q_full, k_full.view(-1, hkv, 128), v_full.view(-1, hkv, 128), None, B, S,
                    float(attn.scaling))
        if pos is not None:
            o = o.index_select(0, pos)
        x2, h1 = self.rms_norm(layer.post_attention_layernorm, h, None, delta=attn.o_proj(o))
        mlp = layer.mlp
        g = mlp.gate_proj(x2)
        act = torch.empty_like(g)
        ops.silu_mul(g, mlp.up_proj(x2), act, None)
        return h1 + mlp.down_proj(act)

    def decode_layer_fused(self, i: int, h: torch.Tensor, slots: torch.Tensor, n_live: torch.Tensor,
                           pos: torch.Tensor, length: torch.Tensor, kc: torch.Tensor,
                           vc: torch.Tensor, err: torch.Tensor) -> torch.Tensor:
        """decode_layer on fused kernels: the input norm, the q/k norms with the
        rotary embedding and the cache append, the residual add with the
        post-attention norm, and the SiLU gate are one kernel each; the
        projections are cuBLAS GEMMs on the model's weights, q, k and v in
        one (_qkv_weight)."""
        from tide_b200 import _native

        ops = _native.ops()
        layer = self.layers[i]
        attn = layer.self_attn
        n = h.shape[0]
        x, _ = self.rms_norm(layer.input_layernorm, h, n_live)
        # q, k and v from one GEMM on the stacked weights; the kernel below
        # takes them as column slices of its output
        w, b = self._qkv_weight(i, attn)
        qkv = torch.nn.functional.linear(x, w, b)
        dq, dk = attn.q_proj.out_features, attn.k_proj.out_features
        q = qkv[:, :dq].view(n, -1, 128)
        k = qkv[:, dq:dq + dk].view(n, -1, 128)
        v = qkv[:, dq + dk:].view(n, -1, 128)
        qn, kn = getattr(attn, "q_norm", None), getattr(attn, "k_norm", None)
        q_rot = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        ops.qk_norm_rope(q, k, v, qn.weight if qn is not None else None,
                         kn.weight if kn is not None else None,
                         float(qn.variance_epsilon) if qn is not None else 0.0,
                         self._inv_freq(), float(getattr(self.rotary, "attention_scaling", 1.0)),
                         0, pos, None, slots, n_live, q_rot, kc, vc, err)
        o = torch.empty_like(q_rot)
        ops.decode_attention(q_rot, kc, vc, slots, o, kc.shape[2], float(attn.scaling), err,
                             n_live, length)
        x2, h1 = self.rms_norm(layer.post_attention_layernorm, h, n_live,
                               delta=attn.o_proj(o.view(n, -1)))
        mlp = layer.mlp
        g = mlp.gate_proj(x2)
        act = torch.empty_like(g)
        ops.silu_mul(g, mlp.up_proj(x2), act, n_live)
        return h1 + mlp.down_proj(act)


class _GPT2Family:
    """GPT-2 blocks (fused c_attn, learned absolute positions)."""

    def __init__(self, model: nn.Module):
        tr = model.transformer
        self.wte, self.wpe = tr.wte, tr.wpe
        self.layers = tr.h
        self.norm = tr.ln_f

    def embed_tokens(self, ids: torch.Tensor) -> torch.Tensor:
        B, S = ids.shape
        p = torch.arange(S, device=ids.device)
        return (self.wte(ids) + self.wpe(p)[None]).reshape(B * S, -1)

    def layer(self, i: int, h: torch.Tensor, pos: Optional[torch.Tensor], seq_pos: torch.Tensor,
              B: int, S: int) -> torch.Tensor:
        blk = self.layers[i]
        attn = blk.attn
        n, H = h.shape
        nh = attn.num_heads
        d = H // nh
        q, k, v = attn.c_attn(blk.ln_1(h)).split(H, dim=1)
        scale = (d ** -0.5) if attn.scale_attn_weights else 1.0
        if getattr(attn, "scale_attn_by_inverse_layer_idx", False):
            scale /= float(i + 1)
        o = _attend(q.view(n, nh, d), k.view(n, nh, d), v.view(n, nh, d), pos, B, S, scale)
        h = h + attn.c_proj(o)
        return h + blk.mlp(blk.ln_2(h))


def family_of(model: nn.Module):
    """The live executor for a model's layer family, or NotImplementedError."""
    inner = getattr(model, "model", None)
    layers = getattr(inner, "layers", None)
    if layers is not None and len(layers) and hasattr(layers[0], "self_attn") \
            and hasattr(layers[0].self_attn, "q_proj") and hasattr(inner, "rotary_emb"):
        return _LlamaFamily(model)
    tr = getattr(model, "transformer", None)
    if tr is not None and hasattr(tr, "h") and len(tr.h) and hasattr(tr.h[0].attn, "c_attn"):
        return _GPT2Family(model)
    raise NotImplementedError(f"live early exit does not know the layers of {type(model).__name__}")


@torch.no_grad()
def live_forward(runtime, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor],
                 on_checkpoint: Optional[Callable[[int, int], None]] = None,
                 fused_layers: bool = True):
    """The live forward of TIDERuntime (see the module docstring): returns
    (out_buf [B*S, H] of final-normed rows at their token positions,
    ExitStats, exit_layer [B*S] int32).  One host read-back of the survivor
    count per checkpoint (the next layers' shapes depend on it).  Llama-
    family layers of a 16-bit model run on the fused elementwise kernels when
    they are ones those reproduce (fused_layers=False: the modules)."""
    from tide_b200.scheduler import ExitStats

    if attention_mask is not None and not bool(attention_mask.bool().all()):
        raise NotImplementedError("live early exit takes inputs without padding")
    fam = runtime._live_family()
    B, S = input_ids.shape
    N = B * S
    dev = input_ids.device
    h = fam.embed_tokens(input_ids)
    H = h.shape[1]
    dtype = h.dtype
    seq_all = torch.arange(S, device=dev).repeat(B)
    out_buf = torch.zeros(N, H, dtype=dtype, device=dev)
    exit_layer = torch.full((N,), -1, dtype=torch.int32, device=dev)
    stats = ExitStats(total_tokens=N)
    routers = {L for L in runtime.routers if L >= runtime.config.min_layers}
    thr = runtime.config.exit_threshold
    pos = None  # all tokens, in order
    pos_out = [torch.empty(N, dtype=torch.int64, device=dev) for _ in range(2)]
    exit_pos = torch.empty(N, dtype=torch.int64, device=dev)
    counts = torch.zeros(2, dtype=torch.int32, device=dev)
    fused = fused_layers and isinstance(fam, _LlamaFamily) and \
        dtype in (torch.bfloat16, torch.float16) and fam.fused_decode_ok()
    layer_fn = fam.layer_fused if fused else fam.layer
    n_ck = 0
    for i in range(len(fam.layers)):
        seq_pos = seq_all if pos is None else pos % S
        h = layer_fn(i, h, pos, seq_pos, B, S)
        if i not in routers:
            continue
        nxt = pos_out[n_ck % 2]
        comp = torch.empty_like(h)
        runtime._runner.run(h, runtime._router(i, dtype), runtime._norm, thr, positions=pos,
                            out_buffer=out_buf, compact_out=comp, positions_out=nxt,
                            exit_positions_out=exit_pos, counts=counts)
        n_surv, n_exit = (int(v) for v in counts.tolist())
        n_ck += 1
        if n_exit:
            stats.exits_per_layer[i] = n_exit
            exit_layer.index_fill_(0, exit_pos[:n_exit], i)
        if on_checkpoint is not None:
            on_checkpoint(i, n_surv)
        pos = nxt[:n_surv]
        h = comp[:n_surv]  # the survivors, compacted by the kernel: the next layer's input
        if n_surv == 0:
            break
    n_rem = h.shape[0]
    stats.remaining_tokens = n_rem
    if n_rem:
        # as the post-hoc path: the model's last hidden state (its final norm
        # applied, as HF reports it), final-normed once more
        last = fam.rms_norm(fam.norm, h, None)[0] if fused else fam.norm(h).contiguous()
        if pos is None:
            pos = torch.arange(N, device=dev)
        runtime._runner.norm_scatter(last, pos, out_buf, runtime._norm)
    runtime._runner.check_errors()
    return out_buf, stats, exit_layer


class _StepBuffers:
    """The fixed-size device buffers of one decode step of B rows."""

    def __init__(self, B: int, H: int, dtype: torch.dtype, dev: torch.device, checkpoints):
        self.B = B
        self.tokens = torch.zeros(B, dtype=torch.long, device=dev)
        self.rows0 = torch.arange(B, dtype=torch.long, device=dev)
        self.slots0 = torch.arange(B, dtype=torch.int32, device=dev)
        self.n0 = torch.full((1,), B, dtype=torch.int32, device=dev)
        self.out_buf = torch.zeros(B, H, dtype=dtype, device=dev)
        self.exit_layer = torch.full((B + 1,), -1, dtype=torch.int32, device=dev)  # [B]: sink
        self.ck = {i: (torch.empty(B, H, dtype=dtype, device=dev),           # compacted rows
                       torch.empty(B, dtype=torch.long, device=dev),         # their positions
                       torch.empty(B, dtype=torch.int32, device=dev),        # their KV slots
                       torch.empty(B, dtype=torch.long, device=dev),         # exit positions
                       torch.zeros(2, dtype=torch.int32, device=dev))        # {survivors, exits}
                   for i in checkpoints}
        self.graph = None
        self.logits = None
        self.threshold = None  # the exit threshold the graph was recorded with


class LiveDecoder:
    """Decode with per-row early exit that skips layers: after each checkpoint
    of a step, the later layers run only on the rows still active, their KV
    slot ids compacted by the checkpoint kernel, and attention reads only those
    slots (tide_decode_attention).  A row that exits leaves zeros in the cache
    at that position for every later layer (the reference's "zero_pad",
    python/TIDE/runtime.py:194-221).  Each row's logits come from its own exit
    layer (final norm, lm_head); the rows that never exit take the model's
    last layer, normalised as in the post-hoc path.

    A step reads nothing back: the live row count stays on the device from
    checkpoint to checkpoint (attention, the cache append and the final
    scatter read it there), buffers keep the batch's size, and the decode
    position is a device word.  The exit counts add up on the device until
    read_stats().  So a step can be captured: with graph=True the first step
    of a batch size is recorded as a CUDA graph and every later step replays
    it (one launch per step).  Llama-family layers with a head dimension of
    128, bf16 or fp16."""

    def __init__(self, runtime, n_slots: int, max_len: int, graph: bool = False,
                 fused_layers: bool = True):
        from tide_b200.ops import CheckpointRunner

        fam = runtime._live_family()
        if not isinstance(fam, _LlamaFamily) or fam.head_dim() != 128:
            raise NotImplementedError("the live decoder takes Llama-family layers with head_dim 128")
        self.rt, self.fam = runtime, fam
        p = next(runtime.model.parameters())
        if p.dtype not in (torch.bfloat16, torch.float16):
            raise NotImplementedError("the live decoder takes bf16 or fp16 models")
        self.dev, self.dtype = p.device, p.dtype
        shape = (n_slots, fam.kv_heads(), max_len, fam.head_dim())
        self.k = [torch.zeros(shape, dtype=p.dtype, device=p.device) for _ in fam.layers]
        self.v = [torch.zeros(shape, dtype=p.dtype, device=p.device) for _ in fam.layers]
        self.n_slots, self.max_len, self._length = n_slots, max_len, 0
        self.pos = torch.zeros(1, dtype=torch.int32, device=p.device)
        # its own checkpoint workspace and error word: a captured step keeps
        # their addresses, which a prefill elsewhere must not reallocate
        self.runner = CheckpointRunner(p.device)
        self.err = self.runner.error_word
        self.graph = graph
        # the layers' elementwise work on fused kernels where the model's
        # modules are ones they reproduce; otherwise the modules themselves
        self.fused = fused_layers and fam.fused_decode_ok()
        self._bufs = {}
        self.exits_dev = torch.zeros(len(fam.layers), dtype=torch.int64, device=p.device)
        self.remaining_dev = torch.zeros(1, dtype=torch.int64, device=p.device)
        self.last_exit_layer = None

    @property
    def length(self) -> int:
        """Positions held by every slot (the next token's position)."""
        return self._length

    @length.setter
    def length(self, value: int) -> None:
        self._length = int(value)
        self.pos.fill_(self._length)

    def fill_random(self, length: int, generator: torch.Generator) -> None:
        """Positions 0..length-1 of every slot hold N(0,1) keys and values."""
        for kc, vc in zip(self.k, self.v):
            for c in (kc, vc):
                c[:, :, :length] = torch.randn(c[:, :, :length].shape, generator=generator,
                                               device=c.device).to(c.dtype)
        self.length = length

    @torch.no_grad()
    def prefill(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Every layer on the prompt (no exits), filling slots 0..B-1; returns
        the last position's logits [B, V] (the model's own)."""
        B, S = input_ids.shape
        h = self.fam.embed_tokens(input_ids)
        for i in range(len(self.fam.layers)):
            h = self.fam.prefill_layer(i, h, B, S, self.k[i], self.v[i])
        self.length = S
        last = self.fam.norm(h.view(B, S, -1)[:, -1, :])
        return self.rt._lm_head(last)

    def _checkpoints(self):
        rt = self.rt
        return sorted(L for L in rt.routers if L >= rt.config.min_layers)

    def _body(self, b: _StepBuffers) -> torch.Tensor:
        """One step on b.tokens; every shape fixed by the batch size."""
        from tide_b200 import _native

        rt, fam, B = self.rt, self.fam, b.B
        norm = rt._norm
        h = fam.embed_tokens(b.tokens.view(B, 1))
        length = self.pos + 1
        rows, slots, n_live = b.rows0, b.slots0, b.n0
        b.exit_layer.fill_(-1)
        thr = rt.config.exit_threshold
        for i in range(len(fam.layers)):
            layer_fn = fam.decode_layer_fused if self.fused else fam.decode_layer
            h = layer_fn(i, h, slots, n_live, self.pos, length, self.k[i], self.v[i], self.err)
            if i not in b.ck:
                continue
            comp, rows_out, slots_out, exit_pos, counts = b.ck[i]
            self.runner.run(h, rt._router(i, self.dtype), norm, thr, positions=rows, slots=slots,
                            n_rows_dev=n_live, out_buffer=b.out_buf, compact_out=comp,
                            positions_out=rows_out, slots_out=slots_out,
                            exit_positions_out=exit_pos, counts=counts)
            # this checkpoint's exits: their layer, at their positions; the
            # entries past the exit count point at the sink entry B
            sink = torch.where(b.rows0 < counts[1], exit_pos, B)
            b.exit_layer.index_fill_(0, sink, i)
            self.exits_dev[i] += counts[1]
            h, rows, slots, n_live = comp, rows_out, slots_out, counts[0:1]
        # the rows that never exit: the model's last hidden state (its final
        # norm applied, as HF reports it), final-normed once more
        last = fam.rms_norm(fam.norm, h, n_live)[0] if self.fused else fam.norm(h).contiguous()
        _native.ops().norm_scatter_rows(last, rows, n_live, b.out_buf, norm.weight, norm.bias,
                                        norm.kind, norm.eps, self.err)
        self.remaining_dev += n_live
        self.pos += 1
        return rt._lm_head(b.out_buf)

    def _capture(self, b: _StepBuffers) -> None:
        """Record b's step as a CUDA graph.  One eager step first (library
        handles, workspaces, folded routers), on a side stream; its effects
        are undone (the position's cache entries, the counters) before the
        capture, which runs nothing."""
        p = self._length
        counters = (self.exits_dev.clone(), self.remaining_dev.clone())
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            self._body(b)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        for kc, vc in zip(self.k, self.v):
            kc[:, :, p].zero_()
            vc[:, :, p].zero_()
        self.length = p
        self.exits_dev.copy_(counters[0])
        self.remaining_dev.copy_(counters[1])
        b.graph = torch.cuda.CUDAGraph()
        b.threshold = self.rt.config.exit_threshold
        with torch.cuda.graph(b.graph):
            b.logits = self._body(b)

    @torch.no_grad()
    def step(self, tokens: torch.Tensor, stats=None) -> torch.Tensor:
        """One decode step for tokens [B] (slot i holds sequence i): the next
        logits [B, V] (with graph=True, a buffer the next step overwrites).
        `stats` (an ExitStats) counts the step's tokens; its exits stay on
        the device until read_stats()."""
        B = tokens.shape[0]
        if self._length >= self.max_len:
            raise RuntimeError("the live decoder's cache is full")
        if B > self.n_slots:
            raise ValueError("more rows than cache slots")
        b = self._bufs.get(B)
        if b is None:
            H = self.fam.embed.embedding_dim
            b = self._bufs[B] = _StepBuffers(B, H, self.dtype, self.dev, self._checkpoints())
        b.tokens.copy_(tokens.reshape(B))
        if self.graph:
            # the threshold is a constant of the recorded step: record again
            # when the engine's changes
            if b.graph is None or b.threshold != self.rt.config.exit_threshold:
                b.graph = None
                self._capture(b)
            b.graph.replay()
            logits = b.logits
        else:
            logits = self._body(b)
        self._length += 1
        self.last_exit_layer = b.exit_layer[:B]
        if stats is not None:
            stats.total_tokens += B
        return logits

    def read_stats(self, stats) -> None:
        """Add the exits and the never-exiting rows counted on the device
        since the last call to `stats` (one read-back) and reset them; also
        raises if a kernel flagged a device error."""
        per_layer = self.exits_dev.tolist()
        stats.remaining_tokens += int(self.remaining_dev.item())
        for i, c in enumerate(per_layer):
            if c:
                stats.exits_per_layer[i] = stats.exits_per_layer.get(i, 0) + int(c)
        self.exits_dev.zero_()
        self.remaining_dev.zero_()
        self.runner.check_errors()
