"""The oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py): router scores, strict-threshold decisions,
stable compaction and the runtime's normed exit rows."""
import numpy as np
import pytest
import torch

import tide_oracle as O
from tests.conftest import GOLDEN
from tide_b200 import workloads

THR = 0.85


def _norm(kind, w, b, eps):
    return {"kind": kind, "weight": w, "bias": b, "eps": eps}


def _storage(t: torch.Tensor, dtype: str) -> np.ndarray:
    if dtype == O.BF16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


CASES = {
    "k1_fp32_rms": (lambda: workloads.k1(), O.F32, torch.float32, 1e-5),
    "bf16_rms_h4096": (lambda: workloads.rows(256, 4096, torch.bfloat16, seed=3,
                                              unit_norm_weight=False), O.BF16, torch.bfloat16, 1e-5),
    "fp16_ln_h768": (lambda: workloads.rows(256, 768, torch.float16, seed=4, norm_kind="layer",
                                            unit_norm_weight=False), O.F16, torch.float16, 1e-5),
}


@pytest.mark.parametrize("name", list(CASES))
def test_checkpoint_matches_reference(name):
    make, dt, tdt, score_tol = CASES[name]
    g = np.load(GOLDEN / f"{name}.npz")
    w = make()
    x = _storage(w["x"].to(tdt), dt)
    if w["norm_kind"] == "rms":
        nw = w["norm_weight"].to(tdt).float().numpy()
        norm = _norm("rms", nw, None, w["eps"])
    else:
        norm = _norm("layer", w["norm_weight"].to(tdt).float().numpy(),
                     w["norm_bias"].to(tdt).float().numpy(), w["eps"])
    res = O.checkpoint(x, dt, norm, w["down"].numpy(), w["up"].numpy(), float(g["bias"]), THR,
                       out_buffer=np.zeros_like(x))
    # scores: fp32 restatement vs the reference's torch fp32 path
    np.testing.assert_allclose(res["scores"], g["scores"], atol=score_tol, rtol=0)
    # decisions identical except for scores within tolerance of the threshold
    near = np.abs(g["scores"] - THR) <= score_tol
    assert np.array_equal(res["exits"][~near], g["mask"][~near])
    if np.array_equal(res["exits"], g["mask"]):
        # compaction: bit-exact positions, stable order
        assert np.array_equal(res["positions"], g["positions"])
        assert np.array_equal(res["exit_positions"], g["exit_positions"])
        assert res["n_survivors"] == int(g["n_survivors"])
        rows = g["normed_exit_rows_idx"]
        ours = res["out_buffer"][rows]
        ulp = O.ulp_distance(ours, g["normed_exit_rows"], dt)
        assert ulp.max() <= (8 if dt == O.F32 else 1), ulp.max()


def test_compaction_kats():
    g = np.load(GOLDEN / "compaction_kats.npz")
    keys = sorted({k.rsplit("_mask", 1)[0] for k in g.files if k.endswith("_mask")
                   and not k.startswith("chain")})
    assert len(keys) == 13 * 4
    for k in keys:
        mask = g[k + "_mask"]
        n = mask.shape[0]
        x = np.arange(n * 8, dtype=np.float32).reshape(n, 8)
        comp, ex, ci, ei, nr = O.batch_compact(x, mask)
        assert np.array_equal(ci.astype(np.int64), g[k + "_positions"]), k
        assert np.array_equal(comp[:, 0], g[k + "_kept_first_col"]), k
        out = O.exit_scatter(ex, ei, np.zeros_like(x))
        assert np.array_equal(out[:, 0], g[k + "_out_first_col"]), k
        assert int(nr[0]) == n - int(mask.sum())
    # three chained checkpoints carry positions
    pos = np.arange(300, dtype=np.int64)
    for stage in range(3):
        keep, _ = O.stable_partition(g[f"chain{stage}_mask"])
        pos = pos[keep]
        assert np.array_equal(pos, g[f"chain{stage}_positions"])


def test_router_file_scores():
    from tide_b200.router import RouterCheckpoint

    ck = RouterCheckpoint.load(GOLDEN / "router_ref.pt")
    ref = np.load(GOLDEN / "router_ref_scores.npz")
    for layer, key in ((3, "s3"), (7, "s7")):
        r = ck.routers[layer]
        s = O.router_scores(ref["x"], r.down.weight.detach().numpy(), r.up.weight.detach().numpy())
        np.testing.assert_allclose(s, ref[key], atol=1e-6, rtol=0)


def test_bf16_rounding_matches_torch():
    x = torch.randn(4096) * 3
    ours = O.f32_to_bf16(x.numpy())
    ref = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)


def test_ulp_distance():
    a = np.array([1.0, -1.0, 0.0], dtype=np.float32)
    b = np.nextafter(a, np.float32(2.0))
    assert O.ulp_distance(a, b, O.F32).tolist() == [1, 1, 1]
