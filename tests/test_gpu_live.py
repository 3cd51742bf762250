"""Live early exit on the GPU (TIDEConfig.live_compaction / forward(live=
True)): the layers after each checkpoint run on the still-active tokens
only, compacted by the checkpoint kernel.  Checked against a dense emulation
built from the model's own HF layers on the whole batch, with the exited
tokens' K/V zeroed (the reference's "zero_pad" policy) and exits decided by
the oracle; and, with no exits, against the post-hoc forward."""
import numpy as np
import pytest
import torch

import tide_oracle as O
from tests.gpu_helpers import TORCH2O, storage_np
from tests.test_gpu_runtime import gpt2, llama, norm_of, tuned_routers, write_routers
from tests.test_live_layers import hf_layer
from tide_b200 import TIDEConfig
from tide_b200.live import family_of
from tide_b200.runtime import TIDERuntime

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("family", ["llama", "gpt2"])
def test_live_without_exits_is_the_posthoc_forward(tmp_path, family):
    model = llama() if family == "llama" else gpt2()
    write_routers(tmp_path / "router.pt", 256, [1, 2], bias=-20.0)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.5,
                                                                       min_layers=0))
    ids = torch.randint(0, 512, (3, 33), generator=torch.Generator().manual_seed(6)).to(DEV)
    with torch.no_grad():
        post = rt(ids)
        live = rt(ids, live=True)
    assert rt.last_stats.total_exited == 0 and rt.last_stats.remaining_tokens == 99
    torch.testing.assert_close(live.float(), post.float(), atol=3e-2, rtol=3e-2)


def dense_emulation(model, rt, ids, routers, threshold, min_layers):
    """Every token through every layer of the model's own HF modules; from the
    layer after a token's exit on, its K/V are zeros; exits decided by the
    oracle's scores of the rows still active; exit rows and the last rows
    final-normed by the oracle.  Returns (logits, exit layer per token,
    scores per router layer)."""
    fam = family_of(model)
    B, S = ids.shape
    N = B * S
    dt = TORCH2O[next(model.parameters()).dtype]
    norm = norm_of(rt._final_norm, "rms")
    keep = torch.ones(B, S, dtype=torch.bool, device=DEV)
    exit_layer = np.full(N, -1)
    scores = {}
    with torch.no_grad():
        h = fam.embed_tokens(ids)
        out = np.zeros((N, h.shape[1]), dtype=storage_np(h[:1]).dtype)
        for i in range(len(fam.layers)):
            h = hf_layer(model, fam, i, h, keep, B, S)
            if i not in routers or i < min_layers:
                continue
            r = routers[i]
            x = storage_np(h)
            s = O.score_rows(x, dt, norm, r.down.weight.numpy(), r.up.weight.numpy(),
                             float(r.up.bias))
            scores[i] = s
            act = keep.reshape(-1).cpu().numpy()
            new = act & (s > threshold)
            out[new] = O.from_f32(O.final_norm(O.to_f32(x, dt), norm), dt)[new]
            exit_layer[new] = i
            keep = keep & ~torch.from_numpy(new).to(DEV).view(B, S)
        rem = keep.reshape(-1).cpu().numpy()
        last = storage_np(fam.norm(h))
        out[rem] = O.from_f32(O.final_norm(O.to_f32(last, dt), norm), dt)[rem]
        t = torch.from_numpy(out.view(np.int16)).view(torch.bfloat16) if dt == O.BF16 \
            else torch.from_numpy(out)
        logits = rt._lm_head(t.to(DEV).view(B, S, -1))
    return logits, exit_layer, scores


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_live_matches_dense_emulation(tmp_path, dtype):
    model = llama(dtype=dtype, layers=6)
    ids = torch.randint(0, 512, (4, 48), generator=torch.Generator().manual_seed(7)).to(DEV)
    routers = tuned_routers(tmp_path / "router.pt", model, ids, [1, 3], [0.3, 0.4], 0.7)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.7,
                                                                       min_layers=0,
                                                                       live_compaction=True))
    with torch.no_grad():
        logits = rt(ids)
    ref, theirs, scores = dense_emulation(model, rt, ids, routers, 0.7, 0)
    ours = rt.last_exit_layer.reshape(-1).cpu().numpy()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    differ = np.nonzero(ours != theirs)[0]
    # a token decided differently sits on the threshold at the first layer
    # where the two disagree; with bf16 the rows after a disagreement drift
    # (other tokens see different K/V), so only the first is checked strictly
    if len(differ):
        i = differ[0]
        first = min(x for x in (ours[i], theirs[i]) if x >= 0)
        assert abs(scores[first][i] - 0.7) <= tol
    assert len(differ) <= 3
    st = rt.last_stats
    assert st.total_exited == int((ours >= 0).sum()) and st.total_exited > 0
    if len(differ) == 0:
        atol = 1e-3 if dtype == torch.float32 else 5e-2
        torch.testing.assert_close(logits.float(), ref.float(), atol=atol, rtol=atol)


@pytest.mark.parametrize("G,L", [(4, 1), (4, 17), (4, 1025), (8, 300), (1, 64), (2, 5000),
                                 (8, 2100), (4, 4166)])
def test_decode_attention_matches_torch(G, L):
    """tide_decode_attention over slot-addressed caches against an fp32 torch
    softmax attention of the gathered rows (bf16 in and out)."""
    from tide_b200 import _native

    ops = _native.ops()
    n, hkv, d, n_slots = 37, 2, 128, 50
    hq, max_len = G * hkv, L + 3
    g = torch.Generator(device=DEV).manual_seed(G * 10007 + L)
    kc = torch.randn(n_slots, hkv, max_len, d, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(n_slots, hkv, max_len, d, generator=g, device=DEV).to(torch.bfloat16)
    q = torch.randn(n, hq, d, generator=g, device=DEV).to(torch.bfloat16)
    slots = torch.randperm(n_slots, generator=torch.Generator().manual_seed(L))[:n].to(torch.int32).to(DEV)
    out = torch.empty_like(q)
    scale = d ** -0.5
    ops.decode_attention(q, kc, vc, slots, out, L, scale, None)
    K = kc[slots.long(), :, :L].float().repeat_interleave(G, dim=1)
    V = vc[slots.long(), :, :L].float().repeat_interleave(G, dim=1)
    p = torch.softmax(torch.einsum("nhd,nhld->nhl", q.float(), K) * scale, dim=-1)
    ref = torch.einsum("nhl,nhld->nhd", p, V)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)


def test_decode_attention_reads_row_count_and_length_from_the_device():
    """n_rows_dev: rows at and past it are left alone; length_dev: the length
    read on the device (clamped to [1, length]) against the torch reference
    at that length."""
    from tide_b200 import _native

    ops = _native.ops()
    n, hkv, G, d, n_slots, max_len = 37, 2, 4, 128, 40, 1100
    g = torch.Generator(device=DEV).manual_seed(77)
    kc = torch.randn(n_slots, hkv, max_len, d, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(n_slots, hkv, max_len, d, generator=g, device=DEV).to(torch.bfloat16)
    q = torch.randn(n, G * hkv, d, generator=g, device=DEV).to(torch.bfloat16)
    slots = torch.randperm(n_slots, generator=torch.Generator().manual_seed(3))[:n]
    slots = slots.to(torch.int32).to(DEV)
    scale = d ** -0.5
    for live, L in [(20, 300), (0, 5), (37, 1025), (1, 1)]:
        out = torch.full_like(q, 5.0)
        n_dev = torch.tensor([live], dtype=torch.int32, device=DEV)
        len_dev = torch.tensor([L], dtype=torch.int32, device=DEV)
        ops.decode_attention(q, kc, vc, slots, out, 1025, scale, None, n_dev, len_dev)
        K = kc[slots.long(), :, :L].float().repeat_interleave(G, dim=1)
        V = vc[slots.long(), :, :L].float().repeat_interleave(G, dim=1)
        p = torch.softmax(torch.einsum("nhd,nhld->nhl", q.float(), K) * scale, dim=-1)
        ref = torch.einsum("nhl,nhld->nhd", p, V)
        torch.testing.assert_close(out[:live].float(), ref[:live], atol=2e-2, rtol=2e-2)
        assert torch.all(out[live:] == 5.0)


def test_decode_attention_flags_a_slot_outside_the_cache():
    from tide_b200 import _native

    ops = _native.ops()
    kc = torch.zeros(4, 1, 8, 128, dtype=torch.bfloat16, device=DEV)
    q = torch.ones(3, 2, 128, dtype=torch.bfloat16, device=DEV)
    out = torch.full_like(q, 5.0)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    slots = torch.tensor([0, 4, 2], dtype=torch.int32, device=DEV)
    ops.decode_attention(q, kc, kc, slots, out, 8, 0.1, err)
    torch.cuda.synchronize()
    assert int(err.item()) & 1
    assert torch.all(out[1] == 5.0) and torch.all(out[0] == 0.0) and torch.all(out[2] == 0.0)


def _qwen3_hd128(dtype=torch.bfloat16):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                      num_attention_heads=2, num_key_value_heads=1, head_dim=128,
                      rms_norm_eps=1e-6, max_position_embeddings=256)
    torch.manual_seed(0)
    return Qwen3ForCausalLM(cfg).to(DEV, dtype).eval()


@pytest.mark.parametrize("graph", [False, True])
def test_live_decoder_first_step_matches_posthoc(tmp_path, graph):
    """One decode step of the live decoder (layers skipped per row after its
    exit) against the post-hoc chain on the model's own hidden states: on the
    first step a row's computation up to its exit reads only its own cache,
    so both give the same logits and exit layers (bf16, within tolerance).
    With graph=True the step is the replay of its captured CUDA graph."""
    from tide_b200.live import LiveDecoder
    from tide_b200.scheduler import ExitStats

    model = _qwen3_hd128()
    B, S = 6, 12
    ids = torch.randint(0, 512, (B, S), generator=torch.Generator().manual_seed(17)).to(DEV)
    tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.3, 0.3], 0.6)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.6,
                                                                       min_layers=0))
    dec = LiveDecoder(rt, B, S + 4, graph=graph)
    with torch.no_grad():
        first = dec.prefill(ids)
        pre = model(ids, use_cache=True)
    torch.testing.assert_close(first.float(), pre.logits[:, -1].float(), atol=5e-2, rtol=5e-2)
    nxt = first.argmax(-1)
    st = ExitStats()
    live_logits = dec.step(nxt, st).clone()
    live_exit = dec.last_exit_layer.clone()
    dec.read_stats(st)
    with torch.no_grad():
        out = model(nxt[:, None], past_key_values=pre.past_key_values, use_cache=True,
                    output_hidden_states=True)
        hs = out.hidden_states
        H = hs[-1].shape[-1]
        out_buf = torch.zeros(B, H, dtype=hs[-1].dtype, device=DEV)
        layers, counts, exit_pos, _ = rt._checkpoint_chain(
            lambda L: hs[L + 1][:, -1, :].contiguous(), B, H, hs[-1].dtype,
            hs[-1][:, -1, :].contiguous(), out_buf)
        rt._read_back(layers, counts, exit_pos, B, (B,))
        ref_logits = rt._lm_head(out_buf)
    same = live_exit == rt.last_exit_layer
    assert int(same.sum()) >= B - 1
    assert st.total_tokens == B and st.total_exited + st.remaining_tokens == B
    torch.testing.assert_close(live_logits[same].float(), ref_logits[same].float(), atol=6e-2,
                               rtol=6e-2)


def test_generate_live_skips_layers_per_row(tmp_path):
    """generate(live=True): greedy tokens with per-row exits that skip the
    later layers; exit counts add up and rows exit."""
    model = _qwen3_hd128()
    ids = torch.randint(0, 512, (4, 10), generator=torch.Generator().manual_seed(23)).to(DEV)
    tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.4, 0.4], 0.6)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.6,
                                                                       min_layers=0))
    out = rt.generate(ids, max_new_tokens=6, temperature=0, live=True, eos_token_id=-1)
    assert out.shape == (4, 16)
    st = rt.last_stats
    assert st.total_tokens == 4 * 6 and st.total_exited + st.remaining_tokens == st.total_tokens
    assert st.total_exited > 0


def _decoder_case(tmp_path, B=5, S=9):
    model = _qwen3_hd128()
    ids = torch.randint(0, 512, (B, S), generator=torch.Generator().manual_seed(29)).to(DEV)
    tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.35, 0.35], 0.6)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.6,
                                                                       min_layers=0))
    return model, rt, ids


def test_live_decoder_graph_replays_the_eager_step(tmp_path):
    """Four decode steps, captured once and replayed, against the same steps
    launched kernel by kernel: the same logits, exit layers and caches, and
    the exit counts read back once agree."""
    from tide_b200.live import LiveDecoder
    from tide_b200.scheduler import ExitStats

    model, rt, ids = _decoder_case(tmp_path)
    B, S = ids.shape
    runs = []
    for graph in (False, True):
        dec = LiveDecoder(rt, B, S + 6, graph=graph)
        st = ExitStats()
        with torch.no_grad():
            tok = dec.prefill(ids).argmax(-1)
            logits, layers = [], []
            for _ in range(4):
                lg = dec.step(tok, st)
                logits.append(lg.float().clone())
                layers.append(dec.last_exit_layer.clone())
                tok = lg.argmax(-1)
        dec.read_stats(st)
        runs.append((logits, layers, st, dec))
    (l0, e0, s0, d0), (l1, e1, s1, d1) = runs
    for a, b in zip(l0, l1):
        torch.testing.assert_close(a, b, atol=1e-3, rtol=1e-3)
    for a, b in zip(e0, e1):
        assert torch.equal(a, b)
    assert s0.total_tokens == s1.total_tokens == 4 * B
    assert s0.exits_per_layer == s1.exits_per_layer and s0.remaining_tokens == s1.remaining_tokens
    assert s1.total_exited + s1.remaining_tokens == 4 * B and s1.total_exited > 0
    for i in range(len(d0.k)):
        torch.testing.assert_close(d0.k[i].float(), d1.k[i].float(), atol=1e-3, rtol=1e-3)


def test_live_decoder_zero_pads_the_layers_after_an_exit(tmp_path):
    """After a step, a row that exited at layer e holds this position's key
    and value in the caches of layers 0..e and zeros above (the reference's
    "zero_pad"); a row that never exited holds them in every layer."""
    from tide_b200.live import LiveDecoder
    from tide_b200.scheduler import ExitStats

    model, rt, ids = _decoder_case(tmp_path, B=8)
    B, S = ids.shape
    dec = LiveDecoder(rt, B, S + 4, graph=True)
    st = ExitStats()
    with torch.no_grad():
        tok = dec.prefill(ids).argmax(-1)
        dec.step(tok, st)
    dec.read_stats(st)
    exit_layer = dec.last_exit_layer.cpu().tolist()
    assert any(e >= 0 for e in exit_layer)
    n_layers = len(dec.k)
    for r, e in enumerate(exit_layer):
        top = n_layers - 1 if e < 0 else e
        for i in range(n_layers):
            written = bool(dec.k[i][r, :, S].abs().sum() > 0) and bool(dec.v[i][r, :, S].abs().sum() > 0)
            assert written == (i <= top), (r, e, i)


def test_kv_append_writes_the_live_rows_at_the_device_position():
    from tide_b200 import _native

    ops = _native.ops()
    n, hkv, d, n_slots, max_len = 11, 3, 128, 16, 20
    g = torch.Generator(device=DEV).manual_seed(5)
    kn = torch.randn(n, hkv, d, generator=g, device=DEV).to(torch.float16)
    vn = torch.randn(n, hkv, d, generator=g, device=DEV).to(torch.float16)
    slots = torch.randperm(n_slots, generator=torch.Generator().manual_seed(1))[:n].to(torch.int32).to(DEV)
    kc = torch.zeros(n_slots, hkv, max_len, d, dtype=torch.float16, device=DEV)
    vc = torch.zeros_like(kc)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    live, pos = 7, 13
    ops.kv_append(kn, vn, slots, torch.tensor([live], dtype=torch.int32, device=DEV), kc, vc, 0,
                  torch.tensor([pos], dtype=torch.int32, device=DEV), err)
    ek, ev = torch.zeros_like(kc), torch.zeros_like(vc)
    ek[slots[:live].long(), :, pos] = kn[:live]
    ev[slots[:live].long(), :, pos] = vn[:live]
    assert torch.equal(kc, ek) and torch.equal(vc, ev) and int(err.item()) == 0
    ops.kv_append(kn, vn, slots, None, kc, vc, 0, torch.tensor([max_len], dtype=torch.int32,
                                                              device=DEV), err)
    torch.cuda.synchronize()
    assert int(err.item()) & 1 and torch.equal(kc, ek)  # a position past the cache: nothing written


@pytest.mark.parametrize("dtype,kind", [(torch.bfloat16, "rms"), (torch.float16, "layer"),
                                        (torch.float32, "rms")])
def test_norm_scatter_rows_with_a_device_count(dtype, kind):
    """output[positions[i]] = final_norm(rows[i]) for i below the device count,
    against the oracle's norm scatter of those rows (<= 1 ulp of the output
    type); rows past the count leave the buffer alone."""
    from tide_b200 import _native
    from tide_b200.capi import NORM_LAYER, NORM_RMS

    ops = _native.ops()
    n, H, total, live = 40, 768, 64, 23
    g = torch.Generator().manual_seed(8)
    rows = torch.randn(n, H, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(H, generator=g)).float()
    b = (0.1 * torch.randn(H, generator=g)).float() if kind == "layer" else None
    pos = torch.randperm(total, generator=g)[:n]
    out = torch.full((total, H), 7.0, dtype=dtype)
    ref = out.clone()
    dt = TORCH2O[dtype]
    norm = {"kind": kind, "weight": w.numpy(), "bias": None if b is None else b.numpy(), "eps": 1e-5}
    normed = O.from_f32(O.final_norm(O.to_f32(storage_np(rows[:live]), dt), norm), dt)
    if dt == O.BF16:
        ref[pos[:live]] = torch.from_numpy(normed.view(np.int16)).view(torch.bfloat16)
    else:
        ref[pos[:live]] = torch.from_numpy(normed)
    dev_out = out.to(DEV)
    ops.norm_scatter_rows(rows.to(DEV), pos.to(DEV), torch.tensor([live], dtype=torch.int32, device=DEV),
                          dev_out, w.to(DEV), None if b is None else b.to(DEV),
                          NORM_LAYER if kind == "layer" else NORM_RMS, 1e-5, None)
    got = dev_out.cpu()
    untouched = sorted(set(range(total)) - set(pos[:live].tolist()))
    assert torch.equal(got[untouched], out[untouched])
    ulp = torch.finfo(dtype).eps  # 1 ulp (16-bit), 8 ulp (fp32: another summation order)
    k = 8 if dtype == torch.float32 else 1
    torch.testing.assert_close(got.float(), ref.float(), atol=4 * k * ulp, rtol=k * ulp)


def _close16(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Within 2 ulp everywhere and bit-equal in at least 99 % of the elements:
    an fp32 sum in another order than torch's moves a statistic by an fp32
    ulp, which can flip one rounding of a chain of two (x * rstd to 16 bits,
    then times the weight)."""
    return _ulp16(a, b) <= 2 and (a == b).float().mean().item() >= 0.99


def _ulp16(a: torch.Tensor, b: torch.Tensor) -> int:
    """Largest distance in units in the last place between two 16-bit tensors."""
    ia = a.contiguous().view(torch.int16).to(torch.int32)
    ib = b.contiguous().view(torch.int16).to(torch.int32)
    ia = torch.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = torch.where(ib < 0, -(ib & 0x7FFF), ib)
    return int((ia - ib).abs().max().item()) if ia.numel() else 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_rms_norm_is_the_hf_module(dtype):
    """tide_rms_norm against the model's RMSNorm module (Qwen3RMSNorm), with
    and without the fused residual add (_close16), rows past the live count
    untouched; the residual sum bit-equal."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm

    from tide_b200 import _native

    ops = _native.ops()
    n, H, live = 37, 4096, 30
    mod = Qwen3RMSNorm(H, eps=1e-6).to(DEV, dtype)
    g = torch.Generator(device=DEV).manual_seed(9)
    with torch.no_grad():
        mod.weight.copy_((1 + 0.2 * torch.randn(H, generator=g, device=DEV)).to(dtype))
        x = (3 * torch.randn(n, H, generator=g, device=DEV)).to(dtype)
        d = torch.randn(n, H, generator=g, device=DEV).to(dtype)
        n_dev = torch.tensor([live], dtype=torch.int32, device=DEV)
        for delta in (None, d):
            out = torch.full_like(x, 7.0)
            tot = torch.full_like(x, 7.0) if delta is not None else None
            ops.rms_norm(x, delta, tot, mod.weight, out, 1e-6, n_dev)
            s = x if delta is None else x + delta
            assert _close16(out[:live], mod(s)[:live])
            assert torch.all(out[live:] == 7.0)
            if delta is not None:
                assert torch.equal(tot[:live], s[:live]) and torch.all(tot[live:] == 7.0)


@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("qk_norm", [True, False])
def test_fused_qk_norm_rope_is_the_hf_modules(qk_norm, packed):
    """tide_qk_norm_rope against the model's q_norm / k_norm and rotary
    modules (apply_rotary_pos_emb), with k and v landing in the cache at the
    rows' slots and the device position; packed: q, k and v as column slices
    of one [n, (hq + 2 hkv) * 128] projection output (strided rows)."""
    from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb

    from tide_b200 import _native

    ops = _native.ops()
    model = _qwen3_hd128()
    attn = model.model.layers[1].self_attn
    rot = model.model.rotary_emb
    n, hq, hkv, d, n_slots, max_len, pos = 9, 2, 1, 128, 12, 40, 33
    g = torch.Generator(device=DEV).manual_seed(10)
    with torch.no_grad():
        q = torch.randn(n, hq, d, generator=g, device=DEV).to(torch.bfloat16)
        k = torch.randn(n, hkv, d, generator=g, device=DEV).to(torch.bfloat16)
        v = torch.randn(n, hkv, d, generator=g, device=DEV).to(torch.bfloat16)
        if packed:
            qkv = torch.cat([q.view(n, -1), k.view(n, -1), v.view(n, -1)], 1)
            q = qkv[:, :hq * d].view(n, hq, d)
            k = qkv[:, hq * d:(hq + hkv) * d].view(n, hkv, d)
            v = qkv[:, (hq + hkv) * d:].view(n, hkv, d)
            assert not q.is_contiguous() and k.stride(0) == (hq + 2 * hkv) * d
        for mod in (attn.q_norm, attn.k_norm):
            mod.weight.copy_((1 + 0.3 * torch.randn(d, generator=g, device=DEV)).to(torch.bfloat16))
        slots = torch.randperm(n_slots, generator=torch.Generator().manual_seed(2))[:n]
        slots = slots.to(torch.int32).to(DEV)
        kc = torch.zeros(n_slots, hkv, max_len, d, dtype=torch.bfloat16, device=DEV)
        vc = torch.zeros_like(kc)
        q_out = torch.empty(q.shape, dtype=q.dtype, device=DEV)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        ops.qk_norm_rope(q, k, v, attn.q_norm.weight if qk_norm else None,
                         attn.k_norm.weight if qk_norm else None, float(attn.q_norm.variance_epsilon),
                         rot.inv_freq.float(), float(rot.attention_scaling), 0,
                         torch.tensor([pos], dtype=torch.int32, device=DEV), None, slots, None, q_out,
                         kc, vc, err)
        qn = attn.q_norm(q) if qk_norm else q
        kn = attn.k_norm(k) if qk_norm else k
        cos, sin = rot(v, torch.full((1, n), pos, dtype=torch.long, device=DEV))
        q_ref, k_ref = apply_rotary_pos_emb(qn, kn, cos[0], sin[0], unsqueeze_dim=1)
        assert _close16(q_out, q_ref)
        assert _close16(kc[slots.long(), :, pos], k_ref)
        assert torch.equal(vc[slots.long(), :, pos], v)
        assert int(err.item()) == 0
        others = torch.ones(n_slots, dtype=torch.bool)
        others[slots.cpu().long()] = False
        assert torch.all(kc[others.to(DEV)] == 0) and torch.all(kc[:, :, :pos] == 0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_qk_norm_rope_prefill_at_token_places(dtype):
    """A prefill-sized call (2048 rows x 48 heads: eight heads per warp, the
    cos/sin computed once per row and head group): each row's own rotary
    position, and q, k, v written at the row's token index (the slots) of
    [tokens, heads, 1, 128] buffers; tokens no row maps to stay untouched.
    Against the model's q_norm / k_norm and rotary modules."""
    from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb

    from tide_b200 import _native

    ops = _native.ops()
    model = _qwen3_hd128(dtype)
    attn = model.model.layers[1].self_attn
    rot = model.model.rotary_emb
    n, hq, hkv, d, tokens = 2048, 32, 8, 128, 3000
    g = torch.Generator(device=DEV).manual_seed(12)
    with torch.no_grad():
        q = torch.randn(n, hq, d, generator=g, device=DEV).to(dtype)
        k = torch.randn(n, hkv, d, generator=g, device=DEV).to(dtype)
        v = torch.randn(n, hkv, d, generator=g, device=DEV).to(dtype)
        for mod in (attn.q_norm, attn.k_norm):
            mod.weight.copy_((1 + 0.3 * torch.randn(d, generator=g, device=DEV)).to(dtype))
        place = torch.randperm(tokens, generator=torch.Generator().manual_seed(5))[:n].to(DEV)
        seq_pos = torch.randint(0, 240, (n,), generator=torch.Generator().manual_seed(6)).to(DEV)
        q_full = torch.full((tokens, hq, d), 3.0, dtype=dtype, device=DEV)
        k_full = torch.zeros(tokens, hkv, 1, d, dtype=dtype, device=DEV)
        v_full = torch.zeros_like(k_full)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        ops.qk_norm_rope(q, k, v, attn.q_norm.weight, attn.k_norm.weight,
                         float(attn.q_norm.variance_epsilon), rot.inv_freq.float(),
                         float(rot.attention_scaling), 0, None, seq_pos, place.to(torch.int32),
                         None, q_full, k_full, v_full, err)
        cos, sin = rot(v, seq_pos[None])
        q_ref, k_ref = apply_rotary_pos_emb(attn.q_norm(q), attn.k_norm(k), cos[0], sin[0],
                                            unsqueeze_dim=1)
        assert int(err.item()) == 0
        assert _close16(q_full[place], q_ref)
        assert _close16(k_full[place, :, 0], k_ref)
        assert torch.equal(v_full[place, :, 0], v)
        others = torch.ones(tokens, dtype=torch.bool, device=DEV)
        others[place] = False
        assert torch.all(q_full[others] == 3.0) and torch.all(k_full[others] == 0)


def test_fused_silu_mul_is_the_hf_mlp_gate():
    from tide_b200 import _native

    ops = _native.ops()
    g = torch.Generator(device=DEV).manual_seed(11)
    gate = (2 * torch.randn(33, 1536, generator=g, device=DEV)).to(torch.bfloat16)
    up = torch.randn(33, 1536, generator=g, device=DEV).to(torch.bfloat16)
    out = torch.full_like(gate, 7.0)
    ops.silu_mul(gate, up, out, torch.tensor([20], dtype=torch.int32, device=DEV))
    ref = torch.nn.functional.silu(gate) * up
    assert _close16(out[:20], ref[:20]) and torch.all(out[20:] == 7.0)


def test_live_decoder_fused_layers_match_the_module_layers(tmp_path):
    """Four decode steps with the fused layer kernels against the same steps
    on the model's own modules: the same exits, logits within bf16 noise."""
    from tide_b200.live import LiveDecoder
    from tide_b200.scheduler import ExitStats

    model, rt, ids = _decoder_case(tmp_path, B=6)
    B, S = ids.shape
    runs = []
    for fused in (False, True):
        dec = LiveDecoder(rt, B, S + 6, graph=fused, fused_layers=fused)
        assert dec.fused == fused
        st = ExitStats()
        with torch.no_grad():
            tok = dec.prefill(ids).argmax(-1)
            out = []
            for _ in range(4):
                lg = dec.step(tok, st)
                out.append((lg.float().clone(), dec.last_exit_layer.clone()))
                tok = lg.argmax(-1)
        dec.read_stats(st)
        runs.append((out, st))
    (a, sa), (b, sb) = runs
    same_exit = [torch.equal(ea, eb) for (_, ea), (_, eb) in zip(a, b)]
    assert all(same_exit[:2])
    for (la, ea), (lb, eb) in zip(a[:2], b[:2]):
        torch.testing.assert_close(la, lb, atol=6e-2, rtol=6e-2)
    assert sa.total_tokens == sb.total_tokens


def test_live_decoder_restacks_changed_projection_weights(tmp_path):
    """The fused decode layer's stacked q/k/v weights follow the model's: after
    an in-place change of one layer's k_proj weight, an eager fused step gives
    what the model's own modules give with the changed weight."""
    from tide_b200.live import LiveDecoder
    from tide_b200.scheduler import ExitStats

    model, rt, ids = _decoder_case(tmp_path, B=4)
    B, S = ids.shape
    with torch.no_grad():
        dec0 = LiveDecoder(rt, B, S + 4, graph=False, fused_layers=True)
        dec0.prefill(ids)
        dec0.step(ids[:, -1], ExitStats())  # builds the stacked weights
        model.model.layers[0].self_attn.k_proj.weight.mul_(-0.5)
        outs = []
        for fused in (True, False):
            dec = LiveDecoder(rt, B, S + 4, graph=False, fused_layers=fused)
            tok = dec.prefill(ids).argmax(-1)
            outs.append(dec.step(tok, ExitStats()).float().clone())
    torch.testing.assert_close(outs[0], outs[1], atol=6e-2, rtol=6e-2)


@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_live_forward_fused_layers_match_the_module_layers(tmp_path, family):
    """The live prefill on the fused layer kernels against the same forward on
    the model's own modules (bf16): the same exits, logits within bf16 noise."""
    from tide_b200.live import live_forward

    # head_dim 128: Llama at hidden 512 with 4 heads
    model = llama(dtype=torch.bfloat16, layers=4, hidden=512) if family == "llama" else _qwen3_hd128()
    H = model.config.hidden_size
    ids = torch.randint(0, 512, (3, 40), generator=torch.Generator().manual_seed(31)).to(DEV)
    tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.3, 0.3], 0.6)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.6,
                                                                       min_layers=0))
    assert family_of(model).fused_decode_ok()
    outs = [live_forward(rt, ids, None, fused_layers=f) for f in (False, True)]
    (oa, sa, ea), (ob, sb, eb) = outs
    assert torch.equal(ea, eb) and sa.exits_per_layer == sb.exits_per_layer
    torch.testing.assert_close(ob.float(), oa.float(), atol=5e-2, rtol=5e-2)
    assert H % 8 == 0


def test_live_decoder_when_every_row_exits_at_the_first_checkpoint(tmp_path):
    """A threshold every score passes: all rows exit at the first checkpoint,
    the live count drops to 0 and the later layers touch no row (their
    attention and cache appends are skipped); every row's logits come from
    that exit, the same as the post-hoc chain's, graph or not."""
    from tide_b200.live import LiveDecoder
    from tide_b200.scheduler import ExitStats

    model = _qwen3_hd128()
    B, S = 5, 10
    ids = torch.randint(0, 512, (B, S), generator=torch.Generator().manual_seed(41)).to(DEV)
    tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.3, 0.3], 0.6)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=-1.0,
                                                                       min_layers=0))
    for graph in (False, True):
        dec = LiveDecoder(rt, B, S + 3, graph=graph)
        st = ExitStats()
        with torch.no_grad():
            first = dec.prefill(ids)
            lg = dec.step(first.argmax(-1), st).float().clone()
        dec.read_stats(st)
        assert st.exits_per_layer == {1: B} and st.remaining_tokens == 0
        assert torch.all(dec.last_exit_layer == 1)
        for i in range(2, len(dec.k)):  # nothing written above the exit layer
            assert torch.all(dec.k[i][:, :, S] == 0) and torch.all(dec.v[i][:, :, S] == 0)
        with torch.no_grad():
            pre = model(ids, use_cache=True)
            out = model(first.argmax(-1)[:, None], past_key_values=pre.past_key_values,
                        use_cache=True, output_hidden_states=True)
            h1 = out.hidden_states[2][:, -1, :].contiguous()
            ref = torch.empty_like(h1)
            rt._runner.norm_scatter(h1, torch.arange(B, device=DEV), ref, rt._norm)
            ref_logits = rt._lm_head(ref).float()
        torch.testing.assert_close(lg, ref_logits, atol=6e-2, rtol=6e-2)


def test_live_decoder_fp16(tmp_path):
    """The live decoder on an fp16 model (fused layers, graph) against the same
    decoder on the model's own modules."""
    from tide_b200.live import LiveDecoder
    from tide_b200.scheduler import ExitStats

    model = _qwen3_hd128(torch.float16)
    B, S = 4, 9
    ids = torch.randint(0, 512, (B, S), generator=torch.Generator().manual_seed(43)).to(DEV)
    tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.3, 0.3], 0.6)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.6,
                                                                       min_layers=0))
    outs = []
    for fused in (False, True):
        dec = LiveDecoder(rt, B, S + 3, graph=fused, fused_layers=fused)
        assert dec.fused == fused
        with torch.no_grad():
            tok = dec.prefill(ids).argmax(-1)
            outs.append((dec.step(tok, ExitStats()).float().clone(), dec.last_exit_layer.clone()))
    (la, ea), (lb, eb) = outs
    assert torch.equal(ea, eb)
    torch.testing.assert_close(lb, la, atol=2e-2, rtol=2e-2)


def test_live_decoder_records_again_when_the_threshold_changes(tmp_path):
    """A graph decoder whose engine's threshold changes between steps records
    the step again: the steps after the change follow the new threshold, and
    the exit counts of the steps before it are kept."""
    from tide_b200.live import LiveDecoder
    from tide_b200.scheduler import ExitStats

    model, rt, ids = _decoder_case(tmp_path, B=6)
    B, S = ids.shape
    dec = LiveDecoder(rt, B, S + 6, graph=True)
    st = ExitStats()
    with torch.no_grad():
        tok = dec.prefill(ids).argmax(-1)
        tok = dec.step(tok, st).argmax(-1)
        before = dec.exits_dev.clone()
        rt.config.exit_threshold = 2.0  # no score passes: no row exits
        dec.step(tok, st)
        assert torch.all(dec.last_exit_layer == -1)
        assert torch.equal(dec.exits_dev, before)
    dec.read_stats(st)
    rt.config.exit_threshold = 0.6
    assert st.total_tokens == 2 * B and st.total_exited == int(before.sum())
    assert st.remaining_tokens == 2 * B - st.total_exited
