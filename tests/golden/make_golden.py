"""Generate the golden vectors that pin the oracle to the reference.

Runs the reference's own Python code (RightNow-AI/TIDE v0.2.1, imported from
the `python/` folder of a checkout of it, named by the environment variable
TIDE_REFERENCE_PYTHON; the reference is read, never modified) on seeded
inputs from tide_b200.workloads and stores its outputs here as .npz files.
Nothing that runs on a GPU runs this script: the fixtures are committed.

  TIDE_REFERENCE_PYTHON=<reference checkout>/python python tests/golden/make_golden.py

Reference code exercised:
  TIDE.router.TokenRouter / RouterCheckpoint      (router.py:11-52)
  TIDE.scheduler.SkipScheduler.process_exits      (scheduler.py:63-102)
  TIDE.runtime.TIDERuntime.forward                (runtime.py:134-192)
  HF LlamaRMSNorm (transformers, as the runtime's final_norm)
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if "TIDE_REFERENCE_PYTHON" not in os.environ:
    sys.exit("set TIDE_REFERENCE_PYTHON to the reference checkout's python/ folder")
REF = Path(os.environ["TIDE_REFERENCE_PYTHON"])
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(REF))

from TIDE.config import TIDEConfig  # noqa: E402  (reference)
from TIDE.router import RouterCheckpoint, TokenRouter  # noqa: E402  (reference)
from TIDE.scheduler import SkipScheduler  # noqa: E402  (reference)
from transformers.models.llama.modeling_llama import LlamaRMSNorm  # noqa: E402

from tide_b200 import workloads  # noqa: E402

THRESHOLD = 0.85


def ref_router(down: torch.Tensor, up: torch.Tensor, bias: float) -> TokenRouter:
    """The reference TokenRouter with its weights set; the scalar bias that
    places the exit fraction rides on an up projection with a bias term."""
    b, h = down.shape
    r = TokenRouter(h, b)
    with torch.no_grad():
        r.down.weight.copy_(down)
        up_lin = torch.nn.Linear(b, 1, bias=True)
        up_lin.weight.copy_(up)
        up_lin.bias.fill_(bias)
        r.up = up_lin
    return r.eval()


def rms_module(weight: torch.Tensor, eps: float, dtype: torch.dtype) -> LlamaRMSNorm:
    m = LlamaRMSNorm(weight.shape[0], eps=eps)
    with torch.no_grad():
        m.weight.copy_(weight.to(dtype).float())
    return m.to(dtype)


def layer_module(weight, bias, eps, dtype) -> torch.nn.LayerNorm:
    """GPT-2 ln_f semantics on a float32 input: fp32 parameters holding the
    model-dtype values (the reference's own call raises on mixed dtypes)."""
    m = torch.nn.LayerNorm(weight.shape[0], eps=eps)
    with torch.no_grad():
        m.weight.copy_(weight.to(dtype).float())
        m.bias.copy_(bias.to(dtype).float())
    return m


def storage(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@torch.no_grad()
def checkpoint_case(name, x, norm_mod, down, up, fraction, dtype, n_keep_rows=64):
    """Score -> strict threshold -> SkipScheduler.process_exits on the
    reference; the normed exit rows follow runtime.py:177 (norm of x.float(),
    then .to(dtype))."""
    n, h = x.shape
    normed0 = norm_mod(x.float())
    r0 = ref_router(down, up, 0.0)
    logits = torch.logit(r0(normed0).double())
    bias = workloads.bias_for_exit_fraction(logits, fraction, THRESHOLD)
    router = ref_router(down, up, bias)
    scores = router(norm_mod(x.float()))  # runtime.py:128-130
    mask = scores > THRESHOLD  # runtime.py:174
    cfg = TIDEConfig()
    sched = SkipScheduler(1, n, h, cfg, torch.device("cpu"), dtype)

    def final_norm_runtime(hs):
        return norm_mod(hs.float()).to(dtype)  # runtime.py:177

    compact = sched.process_exits(x, mask, 0, final_norm_runtime)
    out = {
        "bias": np.float32(bias),
        "scores": scores.numpy().astype(np.float32),
        "mask": mask.numpy(),
        "positions": sched.active_positions.numpy().astype(np.int64),
        "n_survivors": np.int64(compact.shape[0]),
    }
    ex = np.nonzero(out["mask"])[0]
    out["exit_positions"] = ex.astype(np.int64)
    rows = ex[:n_keep_rows]
    out["normed_exit_rows_idx"] = rows.astype(np.int64)
    out["normed_exit_rows"] = storage(sched.output_buffer[torch.as_tensor(rows)])
    buf = sched.output_buffer.float()
    out["out_sum"] = np.float64(buf.double().sum().item())
    out["out_sumsq"] = np.float64(buf.double().pow(2).sum().item())
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"{name}: n={n} h={h} exits={int(mask.sum())} bias={bias:.6f}")


@torch.no_grad()
def compaction_kats():
    """Stable compaction known answers on the reference scheduler: masks of
    sizes around warp/tile/1024 boundaries, all-exit, none-exit, alternating,
    and a three-stage chain (positions carried across checkpoints)."""
    out = {}
    sizes = [0, 1, 2, 31, 32, 33, 127, 128, 129, 1023, 1024, 1025, 4097]
    g = torch.Generator().manual_seed(7)
    cfg = TIDEConfig()
    h = 8
    for n in sizes:
        for pat in ("rand", "all", "none", "alt"):
            if pat == "rand":
                mask = torch.rand(n, generator=g) < 0.3
            elif pat == "all":
                mask = torch.ones(n, dtype=torch.bool)
            elif pat == "none":
                mask = torch.zeros(n, dtype=torch.bool)
            else:
                mask = (torch.arange(n) % 2) == 1
            x = torch.arange(n * h, dtype=torch.float32).reshape(n, h)
            sched = SkipScheduler(1, n, h, cfg, torch.device("cpu"), torch.float32)
            kept = sched.process_exits(x, mask, 0, torch.nn.Identity())
            key = f"n{n}_{pat}"
            out[key + "_mask"] = mask.numpy()
            out[key + "_positions"] = sched.active_positions.numpy().astype(np.int64)
            out[key + "_kept_first_col"] = kept[:, 0].numpy().astype(np.float32)
            out[key + "_out_first_col"] = sched.output_buffer[:, 0].numpy().astype(np.float32)
    # chain of three checkpoints over 300 rows
    n = 300
    x = torch.arange(n * h, dtype=torch.float32).reshape(n, h)
    sched = SkipScheduler(1, n, h, cfg, torch.device("cpu"), torch.float32)
    hs = x
    for stage in range(3):
        m = torch.rand(hs.shape[0], generator=g) < 0.25
        out[f"chain{stage}_mask"] = m.numpy()
        hs = sched.process_exits(hs, m, stage, torch.nn.Identity())
        out[f"chain{stage}_positions"] = sched.active_positions.numpy().astype(np.int64)
    out["chain_out_first_col"] = sched.output_buffer[:, 0].numpy().astype(np.float32)
    np.savez_compressed(HERE / "compaction_kats.npz", **out)
    print(f"compaction_kats: {len(out)} arrays")


@torch.no_grad()
def router_file():
    """A router.pt written by the reference's RouterCheckpoint.save (integer
    layer keys 3 and 7, hidden 64, bottleneck 32)."""
    torch.manual_seed(11)
    routers = {3: TokenRouter(64, 32), 7: TokenRouter(64, 32)}
    RouterCheckpoint(routers=routers, hidden_dim=64, bottleneck_dim=32).save(HERE / "router_ref.pt")
    x = torch.randn(5, 64, generator=torch.Generator().manual_seed(12))
    np.savez_compressed(HERE / "router_ref_scores.npz",
                        x=x.numpy(), s3=routers[3](x).numpy(), s7=routers[7](x).numpy())
    print("router_ref.pt written")


def main():
    torch.set_num_threads(8)
    # the fp32 kernel-level case (4096 x 768): RMSNorm eps 1e-5, 30% exit at threshold 0.85
    k = workloads.k1()
    checkpoint_case("k1_fp32_rms", k["x"], rms_module(k["norm_weight"], 1e-5, torch.float32),
                    k["down"], k["up"], 0.30, torch.float32)
    # bf16 H=4096 RMSNorm (Llama-3.1-8B final norm), 25% exit
    r = workloads.rows(256, 4096, torch.bfloat16, seed=3, unit_norm_weight=False)
    checkpoint_case("bf16_rms_h4096", r["x"], rms_module(r["norm_weight"], 1e-5, torch.bfloat16),
                    r["down"], r["up"], 0.25, torch.bfloat16, n_keep_rows=48)
    # fp16 H=768 LayerNorm (GPT-2 ln_f), 20% exit
    r = workloads.rows(256, 768, torch.float16, seed=4, norm_kind="layer",
                       unit_norm_weight=False)
    checkpoint_case("fp16_ln_h768", r["x"], layer_module(r["norm_weight"], r["norm_bias"], 1e-5,
                                                         torch.float16),
                    r["down"], r["up"], 0.20, torch.float16, n_keep_rows=48)
    compaction_kats()
    router_file()


if __name__ == "__main__":
    main()
