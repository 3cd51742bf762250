"""TIDE runtime on the GPU (drop-in API of the reference's TIDE.TIDE):
logits and exit statistics against the oracle's post-hoc exit loop
(runtime.py:163-192) applied to the same model's hidden states, plus the
behavioural pins of the reference's runtime tests (test_runtime.py:58-116)."""
import numpy as np
import pytest
import torch

import tide_oracle as O
from tests.gpu_helpers import TORCH2O, storage_np
from tide_b200 import TIDEConfig
from tide_b200.router import RouterCheckpoint, TokenRouter
from tide_b200.runtime import TIDERuntime

pytestmark = pytest.mark.gpu
DEV = "cuda"


def llama(dtype=torch.bfloat16, layers=4, hidden=256):
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=512, hidden_size=hidden, intermediate_size=2 * hidden,
                      num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=2,
                      rms_norm_eps=1e-5, max_position_embeddings=256)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(DEV, dtype).eval()


def qwen3(dtype=torch.bfloat16, layers=4, hidden=256):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = Qwen3Config(vocab_size=512, hidden_size=hidden, intermediate_size=2 * hidden,
                      num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=hidden // 4, rms_norm_eps=1e-6, max_position_embeddings=256)
    torch.manual_seed(0)
    return Qwen3ForCausalLM(cfg).to(DEV, dtype).eval()


def gpt2(dtype=torch.float16, layers=4, hidden=256):
    from transformers import GPT2Config, GPT2LMHeadModel

    cfg = GPT2Config(vocab_size=512, n_embd=hidden, n_layer=layers, n_head=4, n_positions=256)
    torch.manual_seed(0)
    m = GPT2LMHeadModel(cfg).to(DEV, dtype).eval()
    with torch.no_grad():  # non-trivial final LayerNorm parameters
        m.transformer.ln_f.weight.normal_(1.0, 0.1)
        m.transformer.ln_f.bias.normal_(0.0, 0.1)
    return m


def write_routers(path, hidden, layers, bias, seed=0):
    g = torch.Generator().manual_seed(seed)
    routers = {}
    for L in layers:
        r = TokenRouter(hidden, 64, up_bias=True)
        with torch.no_grad():
            r.down.weight.normal_(0, 0.05, generator=g)
            r.up.weight.normal_(0, 0.2, generator=g)
            r.up.bias.fill_(bias)
        routers[L] = r
    RouterCheckpoint(routers, hidden, 64).save(path)
    return routers


def oracle_logits(model, runtime, input_ids, routers, threshold, min_layers, norm):
    out = model(input_ids, output_hidden_states=True, return_dict=True)
    hs = [storage_np(h.reshape(-1, h.shape[-1])) for h in out.hidden_states]
    dtype = out.hidden_states[-1].dtype
    dt = TORCH2O[dtype]
    r_np = {L: {"down": r.down.weight.detach().numpy(), "up": r.up.weight.detach().numpy(),
                "up_bias": float(r.up.bias.detach())} for L, r in routers.items()}
    buf, exits, remaining = O.forward_posthoc(hs, dt, norm, r_np, threshold, min_layers)
    if dt == O.BF16:
        t = torch.from_numpy(buf.view(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(buf)
    B, S = input_ids.shape
    logits = runtime._lm_head(t.to(DEV).view(B, S, -1))
    return logits, exits, remaining, buf


def norm_of(module, kind):
    return {"kind": kind, "weight": module.weight.detach().float().cpu().numpy(),
            "bias": None if kind == "rms" else module.bias.detach().float().cpu().numpy(),
            "eps": float(getattr(module, "variance_epsilon", getattr(module, "eps", 1e-5)))}


def tuned_routers(path, model, ids, layers, fractions, threshold, bottleneck=64, seed=0,
                  down_std=0.05, up_std=0.2):
    """Routers at `layers` whose output biases exit the given share of the
    rows still active at each layer (on this model's own hidden states, the
    reference's post-hoc order), saved as a router.pt with `up.bias`."""
    from tide_b200 import workloads

    with torch.no_grad():
        out = model(ids, output_hidden_states=True, return_dict=True)
    hs = out.hidden_states
    fn = model.model.norm if hasattr(model, "model") else model.transformer.ln_f
    kind = "layer" if isinstance(fn, torch.nn.LayerNorm) else "rms"
    eps = float(getattr(fn, "variance_epsilon", getattr(fn, "eps", 1e-5)))
    H = hs[-1].shape[-1]
    N = ids.numel()
    g = torch.Generator().manual_seed(seed)
    exited = torch.zeros(N, dtype=torch.bool)
    routers = {}
    for L, f in zip(layers, fractions):
        r = TokenRouter(H, bottleneck, up_bias=True)
        with torch.no_grad():
            r.down.weight.normal_(0, down_std, generator=g)
            r.up.weight.normal_(0, up_std, generator=g)
        h = hs[L + 1].reshape(N, H)
        with torch.no_grad():
            z = workloads.prebias_logits_torch(h, kind, fn.weight.float(),
                                               None if kind == "rms" else fn.bias.float(), eps,
                                               r.down.weight.to(h.device),
                                               r.up.weight.to(h.device)).cpu()
        active = (~exited).nonzero()[:, 0]
        bias = workloads.bias_for_exit_fraction(z[active], f, threshold)
        with torch.no_grad():
            r.up.bias.fill_(bias)
        exited[active[(z[active] + bias) > workloads.logit(threshold)]] = True
        routers[L] = r
    RouterCheckpoint(routers, H, bottleneck).save(path)
    return routers


def check_against_oracle(rt, model, ids, routers, threshold, min_layers, kind, tol):
    """Runtime logits and per-token exit layers against the oracle's
    post-hoc loop on the same hidden states.  Tokens whose exit layer
    differs must have an oracle score within `tol` of the threshold at the
    first layer where the two disagree; every other token's logits must
    match.  Returns (number of disagreeing tokens, max logit difference)."""
    with torch.no_grad():
        logits = rt(ids)
        out = model(ids, output_hidden_states=True, return_dict=True)
    hs = [storage_np(h.reshape(-1, h.shape[-1])) for h in out.hidden_states]
    dt = TORCH2O[out.hidden_states[-1].dtype]
    norm = norm_of(rt._final_norm, kind)
    r_np = {L: {"down": r.down.weight.detach().numpy(), "up": r.up.weight.detach().numpy(),
                "up_bias": float(r.up.bias.detach())} for L, r in routers.items()}
    buf, exits, remaining, det = O.forward_posthoc(hs, dt, norm, r_np, threshold, min_layers,
                                                   detail=True)
    if dt == O.BF16:
        t = torch.from_numpy(buf.view(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(buf)
    B, S = ids.shape
    with torch.no_grad():
        ref_logits = rt._lm_head(t.to(DEV).view(B, S, -1))
    ours = rt.last_exit_layer.reshape(-1).cpu().numpy()
    theirs = det["exit_layer"]
    st = rt.last_stats
    assert st.total_tokens == B * S
    assert st.total_exited + st.remaining_tokens == st.total_tokens
    assert st.total_exited == int((ours >= 0).sum())
    differ = np.nonzero(ours != theirs)[0]
    for i in differ:
        # the first router layer at which one of the two exits
        first = min(x for x in (ours[i], theirs[i]) if x >= 0)
        assert abs(det["scores"][first][i] - threshold) <= tol, (i, ours[i], theirs[i])
    same = torch.from_numpy(ours == theirs).to(DEV).view(B, S)
    diff = (logits.float() - ref_logits.float()).abs()[same]
    max_diff = float(diff.max()) if diff.numel() else 0.0
    print(f"{len(differ)} of {B * S} tokens differ in exit layer; max logit difference "
          f"elsewhere {max_diff:.3e}; exits {st.exits_per_layer} (oracle {exits})")
    assert len(differ) <= max(2, (B * S) // 200)
    return len(differ), max_diff


@pytest.mark.parametrize("family", ["llama", "gpt2"])
def test_forward_matches_oracle(tmp_path, family):
    model = llama() if family == "llama" else gpt2()
    ids = torch.randint(0, 512, (3, 40), generator=torch.Generator().manual_seed(5)).to(DEV)
    routers = tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.3, 0.3], 0.7)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.7,
                                                                       min_layers=0))
    _, max_diff = check_against_oracle(rt, model, ids, routers, 0.7, 0,
                                       "rms" if family == "llama" else "layer", 1e-2)
    assert max_diff <= 2e-2


def test_forward_gpt2_small_config(tmp_path):
    """GPT-2-small architecture (12 layers, H 768, 12 heads, MLP 3072, vocab
    50257), random-init fp16, routers at layers 4 and 8 exiting ~20 % of the
    active rows each, prefill 8 x 512 uniform random ids (seed 1)."""
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.manual_seed(0)
    model = GPT2LMHeadModel(GPT2Config()).to(DEV, torch.float16).eval()
    ids = torch.randint(0, 50257, (8, 512), generator=torch.Generator().manual_seed(1)).to(DEV)
    routers = tuned_routers(tmp_path / "router.pt", model, ids, [4, 8], [0.2, 0.2], 0.85,
                            bottleneck=128, down_std=0.02, up_std=0.2)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.85,
                                                                       min_layers=0))
    _, max_diff = check_against_oracle(rt, model, ids, routers, 0.85, 0, "layer", 1e-2)
    st = rt.last_stats
    assert 0.15 < st.exits_per_layer[4] / 4096 < 0.25
    assert max_diff <= 5e-2


def test_forward_llama_h4096_reduced_depth(tmp_path):
    """Llama-3.1-8B layer shapes (H 4096, 32/8 heads, head_dim 128, SwiGLU
    14336, RMSNorm eps 1e-5, RoPE theta 5e5) at reduced depth (4 layers) and
    vocabulary (32000), bf16, routers at layers 1 and 2 with 5 % and 20 %
    exits, 2 x 512 tokens."""
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=32000, hidden_size=4096, intermediate_size=14336,
                      num_hidden_layers=4, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, rms_norm_eps=1e-5, rope_theta=500000.0,
                      max_position_embeddings=4096)
    torch.manual_seed(0)
    model = LlamaForCausalLM(cfg).to(DEV, torch.bfloat16).eval()
    ids = torch.randint(0, 32000, (2, 512), generator=torch.Generator().manual_seed(2)).to(DEV)
    routers = tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.05, 0.2], 0.85,
                            bottleneck=128, down_std=0.02, up_std=0.2)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.85,
                                                                       min_layers=0))
    _, max_diff = check_against_oracle(rt, model, ids, routers, 0.85, 0, "rms", 1e-2)
    assert max_diff <= 5e-2


def test_score_router_matches_oracle(tmp_path):
    """_score_router (runtime.py:108-132) keeps the leading shape and gives
    the oracle's scores of final_norm(h) within the 16-bit bar."""
    model = llama()
    routers = write_routers(tmp_path / "router.pt", 256, [1, 2], bias=0.3)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(min_layers=0))
    h = torch.randn(3, 17, 256, generator=torch.Generator().manual_seed(9)).to(DEV, torch.bfloat16)
    s = rt._score_router(h, 2)
    assert s.shape == (3, 17) and s.dtype == torch.float32
    r = routers[2]
    ref = O.score_rows(storage_np(h.reshape(-1, 256)), O.BF16, norm_of(rt._final_norm, "rms"),
                       r.down.weight.detach().numpy(), r.up.weight.detach().numpy(),
                       float(r.up.bias.detach()))
    assert np.abs(s.reshape(-1).cpu().numpy() - ref).max() <= 1e-2


def test_logits_to_keep(tmp_path):
    """logits_to_keep = k: lm_head on the last k positions only.  Against the
    oracle's post-hoc output rows at those positions through the model's
    lm_head (bf16 rows: identical where the exit layers agree), and against
    the full logits' last k positions (bit-identical: the same exit buffer)."""
    model = llama()
    ids = torch.randint(0, 512, (2, 24), generator=torch.Generator().manual_seed(4)).to(DEV)
    routers = tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.3, 0.3], 0.7)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.7,
                                                                       min_layers=0))
    with torch.no_grad():
        full = rt(ids)
        stats = rt.last_stats
        ours_exit = rt.last_exit_layer.reshape(2, 24).clone()
        last = rt(ids, logits_to_keep=1)
        last3 = rt(ids, logits_to_keep=3)
        ref, _, _, _ = oracle_logits(model, rt, ids, routers, 0.7, 0, norm_of(rt._final_norm, "rms"))
    assert last.shape == (2, 1, 512) and last3.shape == (2, 3, 512)
    torch.testing.assert_close(last, full[:, -1:, :], atol=0, rtol=0)
    torch.testing.assert_close(last3, full[:, -3:, :], atol=0, rtol=0)
    assert rt.last_stats == stats and stats.total_exited > 0
    torch.testing.assert_close(last3.float(), ref[:, -3:, :].float(), atol=2e-2, rtol=2e-2)


def test_threshold_pins(tmp_path):
    model = llama()
    write_routers(tmp_path / "router.pt", 256, [1, 3], bias=0.0)
    ids = torch.randint(0, 512, (2, 16), generator=torch.Generator().manual_seed(1)).to(DEV)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=1.0,
                                                                       min_layers=0))
    assert rt(ids).shape == (2, 16, 512)
    assert rt.last_stats.total_exited == 0
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.0,
                                                                       min_layers=0))
    rt(ids)
    assert rt.last_stats.exits_per_layer == {1: 32}
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.0,
                                                                       min_layers=2))
    rt(ids)
    assert rt.last_stats.exits_per_layer == {3: 32}


def test_profile_timings(tmp_path):
    """TIDEConfig.profile: NVTX ranges and the device time of every checkpoint
    (and of the final scatter of the rows that never exit) after a forward;
    the outputs are those of an unprofiled forward."""
    model = llama()
    write_routers(tmp_path / "router.pt", 256, [1, 2], bias=0.8)
    ids = torch.randint(0, 512, (2, 24), generator=torch.Generator().manual_seed(3)).to(DEV)
    plain = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.7,
                                                                          min_layers=0))
    prof = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.7,
                                                                         min_layers=0, profile=True))
    with torch.no_grad():
        a = plain(ids)
        b = prof(ids)
    assert torch.equal(a, b)
    assert plain.last_timings == {}
    t = prof.last_timings
    assert set(t) >= {"checkpoint.layer1", "checkpoint.layer2"}
    if prof.last_stats.remaining_tokens > 0:
        assert "finalize" in t
    assert all(v > 0 for v in t.values())


def test_reference_router_file_loads(tmp_path):
    """A router.pt written by the reference (no bias key) drives the runtime."""
    from tests.conftest import GOLDEN

    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=8,
                      num_attention_heads=4, num_key_value_heads=4)
    model = LlamaForCausalLM(cfg).to(DEV, torch.float32).eval()
    rt = TIDERuntime(model, GOLDEN / "router_ref.pt", config=TIDEConfig(exit_threshold=0.5,
                                                                         min_layers=0))
    ids = torch.randint(0, 256, (2, 16)).to(DEV)
    assert rt(ids).shape == (2, 16, 256)
    st = rt.last_stats
    assert st.total_exited + st.remaining_tokens == 32


def test_generate(tmp_path):
    model = llama()
    write_routers(tmp_path / "router.pt", 256, [1, 2], bias=3.0)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.5,
                                                                       min_layers=0))
    ids = torch.randint(0, 512, (2, 4)).to(DEV)
    out = rt.generate(ids, max_new_tokens=6, temperature=0)
    assert out.shape[0] == 2 and out.shape[1] >= 5
    st = rt.last_stats
    assert st.total_exited + st.remaining_tokens == st.total_tokens
    out = rt.generate(ids, max_new_tokens=4, temperature=0.8, top_k=20, top_p=0.9)
    assert out.shape[1] >= 5


def _oracle_generate(model, rt, ids, routers, threshold, steps, per_row):
    """Greedy decode by the oracle: the model's own cached steps; each step's
    next-token logits from lm_head of the oracle's exit rows (whole-batch
    rule of runtime.py:273-297, or each row on its own)."""
    norm = norm_of(rt._final_norm, "rms")
    r_np = {L: {"down": r.down.weight.detach().numpy(), "up": r.up.weight.detach().numpy(),
                "up_bias": float(r.up.bias.detach())} for L, r in routers.items()}
    gen = ids.clone()
    with torch.no_grad():
        pre = model(gen, use_cache=True, return_dict=True)
        past, logits = pre.past_key_values, pre.logits[:, -1, :]
        exits = {}
        for _ in range(steps):
            nxt = logits.argmax(-1, keepdim=True)
            gen = torch.cat([gen, nxt], -1)
            out = model(nxt, past_key_values=past, use_cache=True, return_dict=True,
                        output_hidden_states=True)
            past = out.past_key_values
            hs = [h[:, -1, :].float().cpu().numpy() for h in out.hidden_states]
            if per_row:
                buf, ex, _ = O.forward_posthoc(hs, O.F32, norm, r_np, threshold, 0)
                for k, v in ex.items():
                    exits[k] = exits.get(k, 0) + v
                logits = rt._lm_head(torch.from_numpy(buf).to(DEV))
                continue
            layer = None
            for L in sorted(r_np):
                s = O.score_rows(hs[L + 1], O.F32, norm, r_np[L]["down"], r_np[L]["up"],
                                 r_np[L]["up_bias"])
                if (s > threshold).all():
                    layer = L
                    break
            if layer is None:
                logits = out.logits[:, -1, :]
            else:
                exits[layer] = exits.get(layer, 0) + ids.shape[0]
                logits = rt._lm_head(torch.from_numpy(O.final_norm(hs[layer + 1], norm)).to(DEV))
    return gen, exits


@pytest.mark.parametrize("family,per_row", [("llama", False), ("llama", True), ("qwen3", True)])
def test_generate_greedy_matches_oracle(tmp_path, family, per_row):
    """Greedy decode (temperature 0) of an fp32 model against the oracle's
    decode: the same tokens and the same exit counts.  Whole-batch rule:
    routers that every row passes at layer 1 on most steps.  Per-row rule
    (Llama, and the Qwen3 architecture with its QK-norm): routers that split
    the rows between layers 1, 2 and no exit, positions and KV slot ids
    compacted on the device at every checkpoint of every step."""
    model = (llama if family == "llama" else qwen3)(dtype=torch.float32)
    ids = torch.randint(0, 512, (4, 6), generator=torch.Generator().manual_seed(8)).to(DEV)
    if per_row:
        routers = tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.4, 0.4], 0.6)
    else:
        routers = write_routers(tmp_path / "router.pt", 256, [1, 2], bias=4.0)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.6,
                                                                       min_layers=0))
    steps = 8
    out = rt.generate(ids, max_new_tokens=steps, temperature=0, per_row_exit=per_row,
                      eos_token_id=-1)
    ref, exits = _oracle_generate(model, rt, ids, routers, 0.6, steps, per_row)
    assert torch.equal(out, ref[:, : out.shape[1]]) and out.shape == ref.shape
    st = rt.last_stats
    assert st.exits_per_layer == exits
    assert st.total_exited > 0
    if not per_row:
        assert set(st.exits_per_layer) == {1}
    else:
        assert st.total_exited + st.remaining_tokens == st.total_tokens


@pytest.mark.parametrize("n,H", [(1, 2048), (300, 800), (4096, 768), (5000, 4096), (64, 784)])
def test_torch_op_router_fp32_tensor_cores(n, H):
    """torch.ops.tide.fused_layernorm_route on fp32 rows takes the tensor-core
    router (three tf32 products) when H % 32 == 0, and the SIMT router
    otherwise (H = 784): scores within the fp32 bar of 1e-5 of the oracle and
    of the C ABI's SIMT router, on router weights at the reference's scale of
    0.02."""
    from tests.gpu_helpers import lib, ptr, stream
    from tide_b200 import _native, capi

    ops = _native.ops()
    g = torch.Generator().manual_seed(n + H)
    x = (torch.randn(n, H, generator=g) * (torch.rand(n, 1, generator=g) * 1.5 + 0.5)).to(DEV)
    nw = (1.0 + 0.02 * torch.randn(H, generator=g)).to(DEV)
    dw = (0.02 * torch.randn(H, 128, generator=g)).to(DEV)
    uw = (0.02 * torch.randn(128, 1, generator=g)).to(DEV)
    s = ops.fused_layernorm_route(x, nw, dw, uw, 1e-5)
    simt = torch.empty(n, device=DEV)
    capi.check(lib(), lib().tide_fused_layernorm_route(capi.DTYPE_F32, ptr(x), ptr(nw), ptr(dw), ptr(uw),
                                                       1e-5, ptr(simt), n, H, 128, stream()),
               "fused_layernorm_route")
    ref = O.fused_layernorm_route(storage_np(x), O.F32, nw.cpu().numpy(), dw.cpu().numpy(),
                                  uw.cpu().numpy(), 1e-5)
    torch.cuda.synchronize()
    np.testing.assert_allclose(s.cpu().numpy(), ref, atol=1e-5, rtol=0)
    np.testing.assert_allclose(s.cpu().numpy(), simt.cpu().numpy(), atol=1e-5, rtol=0)


def test_torch_ops_reference_semantics():
    """torch.ops.tide.* with the reference's calling conventions
    (tests/test_kernels.py:64-186 of the reference), seeded."""
    from tide_b200 import _native

    ops = _native.ops()
    g = torch.Generator().manual_seed(3)
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        x = torch.randn(32, 2048, generator=g).to(dtype).to(DEV)
        nw = torch.randn(2048, generator=g).to(DEV)
        dw = torch.randn(2048, 128, generator=g).to(DEV)
        uw = torch.randn(128, 1, generator=g).to(DEV)
        s = ops.fused_layernorm_route(x, nw, dw, uw, 1e-6)
        ref = O.fused_layernorm_route(storage_np(x), TORCH2O[dtype], nw.cpu().numpy(),
                                      dw.cpu().numpy(), uw.cpu().numpy(), 1e-6)
        np.testing.assert_allclose(s.cpu().numpy(), ref, atol=2e-3)
        m = torch.randint(0, 2, (32,), generator=g, dtype=torch.int32).to(DEV)
        comp, exd, ci, ei, nr = ops.batch_compact(x[:, :256].contiguous(), m)
        keep = np.nonzero(m.cpu().numpy() == 0)[0]
        assert nr.item() == len(keep) and comp.shape == (len(keep), 256) and comp.dtype == dtype
        assert np.array_equal(ci.cpu().numpy(), keep)
        out = torch.zeros(32, 256, dtype=dtype, device=DEV)
        pos = torch.tensor([2, 5, 8, 11, 15, 20, 25, 30], device=DEV, dtype=torch.int32)
        ops.exit_scatter(x[:8, :256].contiguous(), pos, out)
        assert torch.equal(out[pos.long()], x[:8, :256])
        out.zero_()
        ops.exit_projection(x[:4, :256].contiguous(), torch.ones(256, device=DEV), pos[:4], out, 1e-6)
        ref = O.rms_norm(O.to_f32(storage_np(x[:4, :256]), TORCH2O[dtype]), np.ones(256, np.float32), 1e-6)
        np.testing.assert_allclose(out[pos[:4].long()].float().cpu().numpy(), ref, atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H", [2048, 4096])
@pytest.mark.parametrize("n", [1, 8, 32, 128, 5000])
def test_torch_op_router_16bit_tensor_cores(n, H, dtype):
    """torch.ops.tide.fused_layernorm_route on the reference runtime's own
    inputs (runtime.py:120-126: rows and the final norm's weight in the model
    dtype, pre-transposed fp32 router weights, eps 1e-6) at the reference
    op test's shapes (tests/test_kernels.py:64-87) runs a tensor-core router
    (fused single pass or split) and stays within the 1e-2 score bar of the
    oracle; the observed margin is printed."""
    from tide_b200 import _native, capi

    ops = _native.ops()
    g = torch.Generator().manual_seed(n * 7 + H)
    x = torch.randn(n, H, generator=g).to(dtype).to(DEV)
    nw = (1.0 + 0.02 * torch.randn(H, generator=g)).to(dtype).to(DEV)
    dw = (0.02 * torch.randn(H, 128, generator=g)).to(DEV)
    uw = (0.15 * torch.randn(128, 1, generator=g)).to(DEV)
    s = ops.fused_layernorm_route(x, nw, dw, uw, 1e-6)
    path = ops.last_route_path()
    ref = O.fused_layernorm_route(storage_np(x), TORCH2O[dtype], nw.float().cpu().numpy(),
                                  dw.cpu().numpy(), uw.cpu().numpy(), 1e-6)
    err = float(np.abs(s.cpu().numpy() - ref).max())
    print(f"n={n} H={H} {dtype}: path {path}, max score error {err:.2e}")
    assert path in (capi.PATH_TC, capi.PATH_TC_SPLIT)
    assert err <= 1e-2


def test_torch_op_router_refolds_after_update_and_falls_back():
    """The op's folded-weight cache: an in-place update of the router weights
    (version bump) refolds; weights whose 16-bit rounding could move a score
    by more than the bar (N(0,1) weights, as in the reference's op test) take
    the fp32 SIMT router and stay exact to 1e-4."""
    from tide_b200 import _native, capi

    ops = _native.ops()
    g = torch.Generator().manual_seed(11)
    n, H = 256, 4096
    x = torch.randn(n, H, generator=g).to(torch.bfloat16).to(DEV)
    nw = torch.ones(H, device=DEV)
    dw = (0.02 * torch.randn(H, 128, generator=g)).to(DEV)
    uw = (0.15 * torch.randn(128, 1, generator=g)).to(DEV)

    def ref():
        return O.fused_layernorm_route(storage_np(x), O.BF16, nw.cpu().numpy(), dw.cpu().numpy(),
                                       uw.cpu().numpy(), 1e-6)

    s0 = ops.fused_layernorm_route(x, nw, dw, uw, 1e-6).cpu().numpy()
    assert ops.last_route_path() in (capi.PATH_TC, capi.PATH_TC_SPLIT)
    np.testing.assert_allclose(s0, ref(), atol=1e-2, rtol=0)
    dw.mul_(-1.5)  # same tensor, new values
    s1 = ops.fused_layernorm_route(x, nw, dw, uw, 1e-6).cpu().numpy()
    np.testing.assert_allclose(s1, ref(), atol=1e-2, rtol=0)
    assert np.abs(s1 - s0).max() > 1e-2
    big = torch.randn(H, 128, generator=g).to(DEV)
    ub = torch.randn(128, 1, generator=g).to(DEV)
    s2 = ops.fused_layernorm_route(x, torch.randn(H, generator=g).to(DEV), big, ub, 1e-6)
    assert ops.last_route_path() == capi.PATH_SIMT
    assert torch.isfinite(s2).all()


def test_learned_exit_projection(tmp_path):
    """exit_strategy 'learned' (the reference's declared Mode B): an exiting
    row is exit_proj(final_norm(h)), the projection taken from the router
    file; rows that never exit keep final_norm(h).  Against the oracle's
    post-hoc loop with the projection applied to its exit rows (normed rows
    rounded to the model dtype, weights in the model dtype, fp32 sums)."""
    model = llama()
    ids = torch.randint(0, 512, (2, 40), generator=torch.Generator().manual_seed(12)).to(DEV)
    routers = tuned_routers(tmp_path / "r0.pt", model, ids, [1, 2], [0.3, 0.3], 0.7)
    g = torch.Generator().manual_seed(13)
    for r in routers.values():
        r.exit_proj = torch.nn.Linear(256, 256, bias=True)
        with torch.no_grad():
            r.exit_proj.weight.normal_(0, 0.06, generator=g)
            r.exit_proj.bias.normal_(0, 0.1, generator=g)
    RouterCheckpoint(routers, 256, 64).save(tmp_path / "router.pt")
    rt = TIDERuntime(model, tmp_path / "router.pt",
                     config=TIDEConfig(exit_threshold=0.7, min_layers=0, exit_strategy="learned"))
    with torch.no_grad():
        logits = rt(ids)
        out = model(ids, output_hidden_states=True, return_dict=True)
    hs = [storage_np(h.reshape(-1, h.shape[-1])) for h in out.hidden_states]
    norm = norm_of(rt._final_norm, "rms")
    r_np = {L: {"down": r.down.weight.detach().numpy(), "up": r.up.weight.detach().numpy(),
                "up_bias": float(r.up.bias.detach())} for L, r in routers.items()}
    buf, _, _, det = O.forward_posthoc(hs, O.BF16, norm, r_np, 0.7, 0, detail=True)
    for L, r in routers.items():
        sel = det["exit_layer"] == L
        w = O.to_f32(O.from_f32(r.exit_proj.weight.detach().numpy(), O.BF16), O.BF16)
        b = O.to_f32(O.from_f32(r.exit_proj.bias.detach().numpy(), O.BF16), O.BF16)
        buf[sel] = O.from_f32(O.to_f32(buf[sel], O.BF16) @ w.T + b, O.BF16)
    ref = rt._lm_head(torch.from_numpy(buf.view(np.int16)).view(torch.bfloat16).to(DEV).view(2, 40, -1))
    ours = rt.last_exit_layer.reshape(-1).cpu().numpy()
    assert (ours >= 0).sum() > 0
    same = torch.from_numpy(ours == det["exit_layer"]).to(DEV).view(2, 40)
    assert int(same.sum()) >= 78
    torch.testing.assert_close(logits[same].float(), ref[same].float(), atol=5e-2, rtol=5e-2)
    # identity (Mode A) differs exactly on the exit rows
    rt_a = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.7,
                                                                         min_layers=0))
    with torch.no_grad():
        plain = rt_a(ids)
    exited = torch.from_numpy(ours >= 0).to(DEV).view(2, 40)
    assert torch.equal(plain[~exited], logits[~exited])
    assert not torch.allclose(plain[exited].float(), logits[exited].float(), atol=1e-2)


@pytest.mark.parametrize("per_row", [False, True])
def test_generate_from_a_prefilled_cache(tmp_path, per_row):
    """generate(past_key_values=cache) with the context already in the cache
    (all but the last prompt token) gives the tokens and exit counts of a
    generate that prefills the whole prompt itself."""
    from transformers import DynamicCache

    model = qwen3(dtype=torch.float32)
    ids = torch.randint(0, 512, (4, 9), generator=torch.Generator().manual_seed(21)).to(DEV)
    routers = tuned_routers(tmp_path / "router.pt", model, ids, [1, 2], [0.4, 0.4], 0.6)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.6,
                                                                       min_layers=0))
    a = rt.generate(ids, max_new_tokens=6, temperature=0, per_row_exit=per_row, eos_token_id=-1)
    sa = rt.last_stats
    cache = DynamicCache(config=model.config)
    with torch.no_grad():
        model(ids[:, :-1], past_key_values=cache, use_cache=True)
    b = rt.generate(ids, max_new_tokens=6, temperature=0, per_row_exit=per_row, eos_token_id=-1,
                    past_key_values=cache)
    assert torch.equal(a, b)
    assert rt.last_stats == sa
    assert sa.total_exited + sa.remaining_tokens == sa.total_tokens
