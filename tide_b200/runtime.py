"""TIDERuntime: the early-exit runtime, drop-in for the reference's
TIDE.TIDE (python/TIDE/runtime.py:56-389).

The model still runs every layer (the reference's post-hoc design,
runtime.py:151-156); what changes is each checkpoint.  The reference
normalises and scores the whole [B*S, H] tensor with PyTorch ops and
scatters exits with boolean indexing (runtime.py:168-188).  Here one native
call per checkpoint scores only the still-active rows, decides, writes the
exiting rows final-normed straight into the output buffer and compacts the
positions of the survivors (torch.ops.tide.checkpoint, sm_100a kernels).
The rows that never exit are final-normed and scattered by one more call
(torch.ops.tide.norm_scatter).

Semantics kept from the reference: router layer L scores hidden_states[L+1]
(runtime.py:172); layers below config.min_layers are skipped (:169); exits
are strict `score > exit_threshold` (:174) and sticky; the final norm is the
model's own module type and eps (:129,177); last_stats is an ExitStats
with exits recorded only for layers where some token exited (:176-180).
The only supported device is CUDA: there is no CPU path.
"""
from __future__ import annotations

import logging
from pathlib import Path
from typing import Dict, Optional

import torch
import torch.nn as nn

from tide_b200 import _native
from tide_b200.adapters.auto import get_adapter
from tide_b200.config import TIDEConfig
from tide_b200.ops import CheckpointRunner, PreparedRouter, norm_spec, prepare_router
from tide_b200.router import RouterCheckpoint, TokenRouter
from tide_b200.scheduler import ExitStats
from tide_b200.utils import setup_logging

logger = setup_logging()


class TIDERuntime(nn.Module):
    def __init__(self, model: nn.Module, router_path: str | Path,
                 config: Optional[TIDEConfig] = None, use_cuda_kernels: bool = True):
        super().__init__()
        self.model = model
        self.config = config or TIDEConfig()
        self.adapter = get_adapter(model)
        dev = self._device
        if dev.type != "cuda":
            raise RuntimeError("tide_b200.TIDE needs the model on a CUDA device: the early-exit "
                               "path exists only as sm_100a kernels")
        if not use_cuda_kernels:
            logger.warning("use_cuda_kernels=False has no effect: tide_b200 always runs its "
                           "CUDA kernels")
        self.use_cuda = True
        _native.ops()  # fail now, loudly, if the extension is missing
        ckpt = RouterCheckpoint.load(router_path, device=str(dev))
        self.routers: Dict[int, TokenRouter] = {}
        for layer, r in ckpt.routers.items():
            r.requires_grad_(False)
            self.routers[int(layer)] = r
        self._layers = self.adapter.get_layers(model)
        self._final_norm = self.adapter.get_final_norm(model)
        self._lm_head = self.adapter.get_lm_head(model)
        self._norm = norm_spec(self._final_norm, dev)
        self._prepared: Dict[tuple, PreparedRouter] = {}
        self._runner = CheckpointRunner(dev)
        self.last_stats: Optional[ExitStats] = None
        self.last_exit_layer: Optional[torch.Tensor] = None
        self._events = []
        self._family = None
        self._host_counts: list = []
        self._learned_exits()  # reject an unknown exit_strategy now
        # TIDEConfig.profile (declared by the reference, config.py:21, never
        # read there): NVTX ranges around every checkpoint and the device time
        # of each, in milliseconds, after a forward
        self.last_timings: Dict[str, float] = {}
        logger.info(f"TIDERuntime initialized: {len(self._layers)} layers, "
                    f"{len(self.routers)} routers, CUDA=on (sm_100a)")

    @property
    def _device(self) -> torch.device:
        return next(self.model.parameters()).device

    def _router(self, layer: int, dtype: torch.dtype) -> PreparedRouter:
        key = (layer, dtype)
        if key not in self._prepared:
            r = self.routers[layer]
            self._prepared[key] = prepare_router(r.down.weight, r.up.weight, r.up_bias_value,
                                                 self._norm, dtype)
        return self._prepared[key]

    def _score_router(self, hidden: torch.Tensor, layer_idx: int) -> torch.Tensor:
        """Router scores of hidden [..., H] in the leading shape
        (runtime.py:108-132), computed by the native checkpoint kernels."""
        flat = hidden.reshape(-1, hidden.shape[-1]).contiguous()
        _native.require_cuda(flat, "hidden states")
        scores = torch.empty(flat.shape[0], dtype=torch.float32, device=flat.device)
        self._runner.run(flat, self._router(layer_idx, flat.dtype), self._norm,
                         self.config.exit_threshold, scores_out=scores)
        return scores.view(hidden.shape[:-1])

    @torch.no_grad()
    def _hidden_states(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor]):
        """The model's per-layer hidden states.  Its own logits are not used
        (the exit buffer goes through lm_head below), so the model is asked
        for one position's logits where it takes `logits_to_keep`."""
        kw = dict(attention_mask=attention_mask, output_hidden_states=True, return_dict=True)
        try:
            return self.model(input_ids, logits_to_keep=1, **kw)
        except TypeError:
            return self.model(input_ids, **kw)

    def _checkpoint_chain(self, hidden_at, N: int, H: int, dtype: torch.dtype, final: torch.Tensor,
                          out_buf: torch.Tensor, slots: Optional[torch.Tensor] = None):
        """The post-hoc exit loop on N rows (runtime.py:163-188): for every
        router layer L >= min_layers, in order, route the still-active rows
        of hidden_at(L) ([N, H], row index = token position), write the
        exiting ones final-normed to out_buf at their positions and compact
        the positions (and KV slots) of the survivors; then final-norm the
        rows that never exit from `final`.  The live count chains on the
        device from checkpoint to checkpoint: nothing is read back here.
        Returns (layers, counts [n_layers, 2] device, exit position buffers,
        error word)."""
        ops = _native.ops()
        layers = [L for L in sorted(self.routers) if L >= self.config.min_layers]
        dev = out_buf.device
        counts = torch.zeros(len(layers), 2, dtype=torch.int32, device=dev)
        pos = [torch.empty(N, dtype=torch.int64, device=dev) for _ in range(2)]
        slot_buf = ([torch.empty(N, dtype=torch.int32, device=dev) for _ in range(2)]
                    if slots is not None else [None, None])
        exit_pos = [torch.empty(N, dtype=torch.int64, device=dev) for _ in layers]
        xbuf = torch.empty(N, H, dtype=dtype, device=dev) if len(layers) > 1 else None
        err = self._runner.error_word
        thr = self.config.exit_threshold
        prof = bool(self.config.profile)
        events = []
        pos_in, slot_in, cnt = None, slots, None
        for k, layer in enumerate(layers):
            if prof:
                torch.cuda.nvtx.range_push(f"tide.checkpoint.layer{layer}")
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            hidden = hidden_at(layer)
            if k == 0:
                x = hidden
            else:  # the still-active rows of this layer, by position, count on the device
                ops.gather_rows(hidden, pos_in, cnt, xbuf, err)
                x = xbuf
            self._runner.run(x, self._router(layer, dtype), self._norm, thr, positions=pos_in,
                             slots=slot_in, out_buffer=out_buf, positions_out=pos[k % 2],
                             slots_out=slot_buf[k % 2], exit_positions_out=exit_pos[k],
                             n_rows_dev=cnt, counts=counts[k])
            if prof:
                ev[1].record()
                torch.cuda.nvtx.range_pop()
                events.append((f"checkpoint.layer{layer}", ev))
            pos_in, slot_in, cnt = pos[k % 2], slot_buf[k % 2], counts[k, :1]
        if prof:
            torch.cuda.nvtx.range_push("tide.finalize")
            ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            ev[0].record()
        if pos_in is None:
            pos_in = torch.arange(N, dtype=torch.int64, device=dev)
        n = self._norm
        ops.norm_at_positions(final, pos_in, cnt, out_buf, n.weight, n.bias, n.kind, n.eps, err)
        if prof:
            ev[1].record()
            torch.cuda.nvtx.range_pop()
            events.append(("finalize", ev))
        self._events = events
        return layers, counts, exit_pos, (pos_in, slot_in)

    def _read_back(self, layers, counts, exit_pos, N: int, shape) -> ExitStats:
        """The forward's one host synchronisation: the exit counts and the
        device error word together; then ExitStats (layers with no exit are
        not recorded, runtime.py:176-180) and the per-token exit layer."""
        err = self._runner.error_word
        host = torch.cat([counts.reshape(-1), err]).cpu().tolist()
        if host[-1]:
            self._runner.error_word.zero_()
            raise RuntimeError(f"tide_b200 kernel reported device error bits 0x{host[-1]:x} "
                               "(1: position out of range, 2: wait timeout, 4: bad row count)")
        stats = ExitStats(total_tokens=N)
        exit_layer = torch.full((N,), -1, dtype=torch.int32, device=counts.device)
        remaining = N
        for k, layer in enumerate(layers):
            n_surv, n_exit = host[2 * k], host[2 * k + 1]
            if n_exit > 0:
                stats.exits_per_layer[layer] = n_exit
                exit_layer.index_fill_(0, exit_pos[k][:n_exit], layer)
            remaining = n_surv
        stats.remaining_tokens = remaining
        self.last_exit_layer = exit_layer.view(shape)
        if self.config.profile:
            torch.cuda.synchronize()
            self.last_timings = {name: a.elapsed_time(b) for name, (a, b) in self._events}
        self._host_counts = host
        return stats

    def _learned_exits(self) -> bool:
        """TIDEConfig.exit_strategy: "identity" (the reference's Mode A: an
        exiting row is final_norm(h)) or "learned" (its declared Mode B,
        csrc/kernels/exit_projection.cu:5-8: exit_proj(final_norm(h)) with
        the router file's per-layer exit_proj weights)."""
        strategy = self.config.exit_strategy
        if strategy not in ("identity", "learned"):
            raise ValueError(f"exit_strategy {strategy!r}: expected 'identity' or 'learned'")
        return strategy == "learned"

    def _project_exits(self, out_buf: torch.Tensor, layer: int, positions: torch.Tensor) -> None:
        """Mode B for the rows that exited at `layer` (their positions in
        out_buf, already final-normed there): gathered by the gather kernel,
        projected by one GEMM, written back in place."""
        r = self.routers[layer]
        if r.exit_proj is None or positions.numel() == 0:
            return
        key = ("proj", layer, out_buf.dtype)
        if key not in self._prepared:
            w = r.exit_proj.weight.detach().to(out_buf.device, out_buf.dtype).contiguous()
            b = (r.exit_proj.bias.detach().to(out_buf.device, out_buf.dtype)
                 if r.exit_proj.bias is not None else None)
            self._prepared[key] = (w, b)
        w, b = self._prepared[key]
        rows = torch.empty(positions.numel(), out_buf.shape[1], dtype=out_buf.dtype,
                           device=out_buf.device)
        _native.ops().gather_rows(out_buf, positions, None, rows, self._runner.error_word)
        out_buf.index_copy_(0, positions, torch.nn.functional.linear(rows, w, b))

    def _live_family(self):
        if self._family is None:
            from tide_b200.live import family_of

            self._family = family_of(self.model)
        return self._family

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None,
                logits_to_keep: int = 0, live: Optional[bool] = None, **kwargs) -> torch.Tensor:
        """Early-exit forward: logits [B, S, V].  By default the reference's
        post-hoc exit over the model's hidden states (runtime.py:134-192),
        with one host synchronisation per call (the exit counts, after the
        checkpoint chain is queued; the lm_head is queued after it and runs
        while the caller goes on).  With live=True (or config.live_compaction) the
        layers after each checkpoint run only on the tokens still active
        (tide_b200/live.py; logits then differ from the post-hoc ones by
        design, through the exited tokens' zero-padded K/V).  After a call,
        last_stats holds the ExitStats and last_exit_layer [B, S] the layer
        each token exited at (-1: ran every layer).  `logits_to_keep` > 0
        keeps only the last that many positions ([B, logits_to_keep, V]), so
        lm_head runs on the rows whose logits are used, e.g. 1 before
        sampling."""
        B, S = input_ids.shape
        if live if live is not None else self.config.live_compaction:
            from tide_b200.live import live_forward

            out_buf, stats, exit_layer = live_forward(self, input_ids, attention_mask)
            if self._learned_exits():
                for layer in stats.exits_per_layer:
                    self._project_exits(out_buf, layer, (exit_layer == layer).nonzero()[:, 0])
            rows = out_buf.view(B, S, -1)
            if logits_to_keep > 0:
                rows = rows[:, -logits_to_keep:, :]
            self.last_stats = stats
            self.last_exit_layer = exit_layer.view(B, S)
            return self._lm_head(rows)
        out = self._hidden_states(input_ids, attention_mask)
        hs = out.hidden_states
        H = hs[-1].shape[-1]
        dtype = hs[-1].dtype
        N = B * S
        out_buf = torch.zeros(N, H, device=hs[-1].device, dtype=dtype)
        layers, counts, exit_pos, _ = self._checkpoint_chain(
            lambda L: hs[L + 1].reshape(N, H), N, H, dtype, hs[-1].reshape(N, H), out_buf)
        rows = out_buf.view(B, S, H)
        if logits_to_keep > 0:
            rows = rows[:, -logits_to_keep:, :]
        if not self._learned_exits():
            # the read-back waits for the checkpoint chain only; the lm_head
            # queued after it then runs while the caller goes on
            self.last_stats = self._read_back(layers, counts, exit_pos, N, (B, S))
            return self._lm_head(rows)
        self.last_stats = self._read_back(layers, counts, exit_pos, N, (B, S))
        for k, layer in enumerate(layers):
            self._project_exits(out_buf, layer, exit_pos[k][: self._host_counts[2 * k + 1]])
        return self._lm_head(rows)

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int = 512,
                 temperature: float = 1.0, top_k: int = 50, top_p: float = 0.9,
                 per_row_exit: bool = False, past_key_values=None, live: bool = False,
                 **kwargs) -> torch.Tensor:
        """Autoregressive decode (runtime.py:223-313).  Every step runs all
        layers (the reference's post-hoc design).  With the reference's rule
        (default) the earliest checkpoint at which every row's score passes
        the threshold supplies all rows' next-token logits via
        lm_head(final_norm(h)).  With per_row_exit=True each row exits on its
        own: the step's rows go through the same checkpoint chain as a
        prefill (positions and KV slot ids of the survivors compacted on the
        device at every checkpoint), and each row's logits come from its own
        exit layer; the exit counts of every step add up on the device and
        are read back once, after the last step.  Generation stops when every
        sampled token equals `eos_token_id` (default 2, the reference's fixed
        id, runtime.py:257).  `past_key_values`: a model cache that already
        holds the context (e.g. an HF StaticCache); the model then runs only
        on input_ids[:, -1:] to start, instead of a prefill of input_ids.
        With live=True each row exits on its own and the layers after its
        exit are skipped for it (tide_b200.live.LiveDecoder: its own KV cache
        addressed by slot, exited rows' later keys and values zero-padded,
        each step one CUDA graph replay unless live_graph=False);
        Llama-family models with head_dim 128, bf16/fp16."""
        eos = kwargs.get("eos_token_id", 2)
        B = input_ids.shape[0]
        dev = input_ids.device
        n_layers = len(self._layers)
        generated = input_ids.clone()
        gen_stats = ExitStats(total_tokens=0)
        if live:
            from tide_b200.live import LiveDecoder

            dec = LiveDecoder(self, B, input_ids.shape[1] + max_new_tokens + 1,
                              graph=kwargs.get("live_graph", True))
            next_logits = dec.prefill(input_ids)
            for _ in range(max_new_tokens):
                nxt = sample_next_token(next_logits, temperature, top_k, top_p)
                generated = torch.cat([generated, nxt], dim=-1)
                if bool((nxt == eos).all()):
                    break
                next_logits = dec.step(nxt[:, 0], gen_stats)
            dec.read_stats(gen_stats)  # the one read-back of the exit counts
            self._runner.check_errors()
            self.last_stats = gen_stats
            return generated
        if past_key_values is None:
            pre = self.model(generated, use_cache=True, return_dict=True)
        else:
            pre = self.model(generated[:, -1:], past_key_values=past_key_values, use_cache=True,
                             return_dict=True)
        past = pre.past_key_values
        next_logits = pre.logits[:, -1, :]
        slots = torch.arange(B, device=dev, dtype=torch.int32)
        learned = self._learned_exits()
        step_counts = None  # per-row exits: {survivors, exits} per checkpoint, summed on the device
        row_layers: list = []
        for _ in range(max_new_tokens):
            nxt = sample_next_token(next_logits, temperature, top_k, top_p)
            generated = torch.cat([generated, nxt], dim=-1)
            if bool((nxt == eos).all()):
                break
            gen_stats.total_tokens += B
            out = self.model(nxt, past_key_values=past, use_cache=True, return_dict=True,
                             output_hidden_states=True)
            past = out.past_key_values
            hs = out.hidden_states
            if per_row_exit:
                H = hs[-1].shape[-1]
                out_buf = torch.zeros(B, H, device=dev, dtype=hs[-1].dtype)
                layers, counts, exit_pos, _ = self._checkpoint_chain(
                    lambda L: hs[L + 1][:, -1, :].contiguous(), B, H, hs[-1].dtype,
                    hs[-1][:, -1, :].contiguous(), out_buf, slots=slots)
                row_layers = layers
                if learned:  # the projection's GEMM shapes need the counts now
                    st = self._read_back(layers, counts, exit_pos, B, (B,))
                    for k, layer in enumerate(layers):
                        self._project_exits(out_buf, layer,
                                            exit_pos[k][: self._host_counts[2 * k + 1]])
                    for layer, c in st.exits_per_layer.items():
                        gen_stats.exits_per_layer[layer] = gen_stats.exits_per_layer.get(layer, 0) + c
                    gen_stats.remaining_tokens += st.remaining_tokens
                else:
                    step_counts = counts.to(torch.int64) if step_counts is None else step_counts + counts
                next_logits = self._lm_head(out_buf)
                continue
            exit_layer, exit_hidden = None, None
            for layer in sorted(self.routers):
                if layer < self.config.min_layers:
                    continue
                h = hs[layer + 1][:, -1, :]
                if bool((self._score_router(h, layer) > self.config.exit_threshold).all()):
                    exit_layer, exit_hidden = layer, h.contiguous()
                    break
            if exit_layer is not None:
                normed = torch.empty_like(exit_hidden)
                every = torch.arange(B, device=dev)
                self._runner.norm_scatter(exit_hidden, every, normed, self._norm)
                if self._learned_exits():
                    self._project_exits(normed, exit_layer, every)
                next_logits = self._lm_head(normed)
                gen_stats.exits_per_layer[exit_layer] = gen_stats.exits_per_layer.get(exit_layer, 0) + B
            else:
                next_logits = out.logits[:, -1, :]
                gen_stats.remaining_tokens += B
        if step_counts is not None:  # the one read-back of the per-row exit counts
            host = step_counts.cpu().tolist()
            for layer, (n_surv, n_exit) in zip(row_layers, host):
                if n_exit:
                    gen_stats.exits_per_layer[layer] = gen_stats.exits_per_layer.get(layer, 0) + n_exit
            gen_stats.remaining_tokens += host[-1][0] if host else gen_stats.total_tokens
        self._runner.check_errors()
        self.last_stats = gen_stats
        if gen_stats.total_tokens > 0:
            runs = sum((l + 1) * c for l, c in gen_stats.exits_per_layer.items())
            runs += gen_stats.remaining_tokens * n_layers
            speedup = gen_stats.total_tokens * n_layers / runs if runs > 0 else 1.0
            logger.info(f"Generation: {gen_stats.total_tokens} tokens, {gen_stats.total_exited} "
                        f"exits ({gen_stats.exit_rate:.1%}), estimated {speedup:.2f}x "
                        f"equivalent speedup")
        return generated

    @staticmethod
    def calibrate(*args, **kwargs):
        raise NotImplementedError(
            "router calibration (offline training) is not part of tide_b200; router.pt files "
            "written by the reference's calibrate() load here unchanged")


def sample_next_token(logits: torch.Tensor, temperature: float, top_k: int,
                      top_p: float) -> torch.Tensor:
    """Temperature, top-k and nucleus (top-p) sampling of one token per row
    (same rules as runtime.py:315-352); greedy when temperature <= 0."""
    if temperature <= 0:
        return logits.argmax(dim=-1, keepdim=True)
    z = logits / temperature
    if top_k > 0:
        k = min(top_k, z.shape[-1])
        kth = torch.topk(z, k, dim=-1).values[:, -1:]
        z = z.masked_fill(z < kth, float("-inf"))
    if top_p < 1.0:
        sz, idx = torch.sort(z, descending=True, dim=-1)
        cum = torch.softmax(sz, dim=-1).cumsum(dim=-1)
        drop = cum > top_p
        drop[:, 1:] = drop[:, :-1].clone()
        drop[:, 0] = False
        sz = sz.masked_fill(drop, float("-inf"))
        z = torch.empty_like(z).scatter_(1, idx, sz)
    return torch.multinomial(torch.softmax(z, dim=-1), num_samples=1)
