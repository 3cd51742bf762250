"""Host-side pieces of bench.py that need no GPU: the workload table, the
algorithmic bytes of a checkpoint, the e2e step count and the engine
workloads' router tuning."""
import importlib.util
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_module", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_workload_table(bench):
    for name, wk in bench.WORKLOADS.items():
        assert len(wk["layers"]) == len(wk["exit_fractions"]), name
        assert wk["of"] in ("batch", "active"), name
        assert wk.get("dtype", "bf16") in bench.DTYPE_NAMES, name
        assert wk.get("hidden", 4096) % 32 == 0, name
    # the reference's kernel-level case: 4096 fp32 rows of H = 768, one router, 30 % exits
    k = bench.WORKLOADS["kernel_fp32_4096x768"]
    assert (k["rows"], k["hidden"], k["dtype"], k["exit_fractions"]) == (4096, 768, "f32", [0.30])


def test_algorithmic_bytes(bench):
    # every row read and written once, 21 B per row, 12 B per survivor
    n, exits, h = 32768, 1638, 4096
    assert bench.algorithmic_bytes(n, exits, h, 2) == n * 2 * h * 2 + 21 * n + 12 * (n - exits)
    assert bench.algorithmic_bytes(4096, 4096, 768, 4) == 4096 * 2 * 768 * 4 + 21 * 4096


def test_e2e_step_count(bench):
    # the headline sweep copies ~1.6 GB per step: ~8 GB over 6 steps (the minimum)
    assert bench.e2e_step_count(None, 32768 * 4096 * 2 * 6) == 6
    # a 12.6 MB workload: the cap of 200 steps
    assert bench.e2e_step_count(None, 4096 * 768 * 4) == 200
    assert bench.e2e_step_count(None, 1) == 200
    assert bench.e2e_step_count(5, 1) == 5
    assert bench.e2e_step_count(1, 10 ** 12) == 1


def test_nominal_schedule(bench):
    bench.configure("llama8b_prefill_checkpoints")
    active, exits = bench.nominal_schedule(32768)
    assert active[0] == 32768 and sum(exits) == 32768  # everything exits by the last router
    assert [round(e / 32768, 2) for e in exits[:-1]] == [0.05, 0.10, 0.15, 0.20, 0.20]
    bench.configure("qwen3_8b_decode_checkpoints")
    active, exits = bench.nominal_schedule(256)
    assert all(e == round(0.1 * a) for a, e in zip(active, exits))
    bench.configure("llama8b_prefill_checkpoints")


def test_checkpoint_setup_is_shared_and_places_the_bias(bench):
    """Both arms draw a checkpoint's leading rows, router and bias from the CPU
    generator: the same call gives bit-identical results, and the bias exits
    the scheduled share of the calibration rows."""
    from tide_b200 import workloads

    bench.configure("llama8b_prefill_checkpoints")
    a = bench.checkpoint_setup(1, 0, 31130, 3277)
    b = bench.checkpoint_setup(1, 0, 31130, 3277)
    assert torch.equal(a["x_head"].view(torch.int16), b["x_head"].view(torch.int16))
    assert torch.equal(a["down"], b["down"]) and a["bias"] == b["bias"]
    z = workloads.prebias_logits_torch(a["x_head"], "rms", torch.ones(4096), None, 1e-5,
                                       a["down"], a["up"])
    frac = float(((z + a["bias"]) > workloads.logit(0.85)).float().mean())
    assert abs(frac - 3277 / 31130) < 1e-3
    c = bench.checkpoint_setup(1, 1, 31130, 3277)  # another rank: other rows
    assert not torch.equal(a["x_head"].view(torch.int16), c["x_head"].view(torch.int16))


def test_cpu_reference_step_chains_survivors(bench):
    bench.configure("llama8b_prefill_checkpoints")
    inp = bench.cpu_sweep_inputs(64)
    t, routed = bench.cpu_sweep_step(inp)
    assert t > 0 and 64 <= routed <= 6 * 64
    t2, routed2 = bench.cpu_sweep_step(inp)
    assert routed2 == routed  # deterministic


@pytest.mark.parametrize("last_takes_rest", [False, True])
def test_engine_router_tuning_places_the_exit_schedule(bench, last_takes_rest):
    """The engine workloads' routers (bench._tuned_routers) exit the scheduled
    share of the tokens at each checkpoint on the model's own hidden states
    (here a small GPT-2-architecture model on the CPU, LayerNorm final norm),
    and with last_takes_rest every token still active at the last one."""
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.manual_seed(0)
    m = GPT2LMHeadModel(GPT2Config(vocab_size=101, n_embd=64, n_layer=6, n_head=4,
                                   n_positions=128)).eval()
    ids = torch.randint(0, 101, (4, 64), generator=torch.Generator().manual_seed(1))
    ln = m.transformer.ln_f
    layers, fracs = [1, 3], [0.25, 0.15]
    with torch.inference_mode():
        routers = bench._tuned_routers(m, ids, layers, fracs, 64,
                                       ("ln", ln.weight.float(), ln.bias.float(), ln.eps), 7,
                                       last_takes_rest=last_takes_rest)
        hs = m(ids, output_hidden_states=True).hidden_states
        N = ids.numel()
        exited = torch.zeros(N, dtype=torch.bool)
        for L, f in zip(layers, fracs):
            h = torch.nn.functional.layer_norm(hs[L + 1].reshape(N, -1).float(), (64,),
                                               ln.weight, ln.bias, ln.eps)
            new = (routers[L](h) > bench.THRESHOLD) & ~exited
            want = int((~exited).sum()) if (last_takes_rest and L == layers[-1]) else round(f * N)
            assert abs(int(new.sum()) - want) <= 2, (L, int(new.sum()), want)
            exited |= new
