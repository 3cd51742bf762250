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


@pytest.mark.parametrize("family", ["llama", "gpt2"])
def test_forward_matches_oracle(tmp_path, family):
    model = llama() if family == "llama" else gpt2()
    hidden = 256
    routers = write_routers(tmp_path / "router.pt", hidden, [1, 2], bias=0.8)
    cfg = TIDEConfig(exit_threshold=0.7, min_layers=0)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=cfg)
    ids = torch.randint(0, 512, (3, 40), generator=torch.Generator().manual_seed(5)).to(DEV)
    with torch.no_grad():
        logits = rt(ids)
        norm = norm_of(rt._final_norm, "rms" if family == "llama" else "layer")
        ref_logits, exits, remaining, _ = oracle_logits(model, rt, ids, routers, 0.7, 0, norm)
    st = rt.last_stats
    assert st.total_tokens == 120
    assert st.total_exited + st.remaining_tokens == st.total_tokens
    # exit counts agree up to rows sitting on the threshold (fp32 scores)
    assert abs(st.remaining_tokens - remaining) <= 1
    if st.exits_per_layer == exits:
        torch.testing.assert_close(logits.float(), ref_logits.float(), atol=2e-2, rtol=2e-2)


def test_logits_to_keep(tmp_path):
    """logits_to_keep = k gives the last k positions of the full logits (the
    same exit decisions and buffer; lm_head only on the kept rows)."""
    model = llama()
    write_routers(tmp_path / "router.pt", 256, [1, 2], bias=0.8)
    rt = TIDERuntime(model, tmp_path / "router.pt", config=TIDEConfig(exit_threshold=0.7,
                                                                       min_layers=0))
    ids = torch.randint(0, 512, (2, 24), generator=torch.Generator().manual_seed(4)).to(DEV)
    with torch.no_grad():
        full = rt(ids)
        stats = rt.last_stats
        last = rt(ids, logits_to_keep=1)
        last3 = rt(ids, logits_to_keep=3)
    assert last.shape == (2, 1, 512) and last3.shape == (2, 3, 512)
    torch.testing.assert_close(last, full[:, -1:, :], atol=0, rtol=0)
    torch.testing.assert_close(last3, full[:, -3:, :], atol=0, rtol=0)
    assert rt.last_stats == stats


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
