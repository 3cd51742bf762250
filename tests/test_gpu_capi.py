"""GPU parity of the C ABI against the oracle and the reference's golden
vectors.  Bars: compaction indices, survivor rows and copies bit-exact;
router scores within 1e-5 (fp32 inputs, and every input on the fp32 SIMT
path) or 1e-2 (bf16/fp16 inputs on the tensor-core path) absolute; exit
decisions identical except for rows whose oracle score lies within that
tolerance of the threshold; final-normed exit rows within 1 ulp of the
storage dtype (bf16/fp16) or 8 ulp (fp32, ~1e-6 relative: the row
statistics are sums whose order differs from the reference's)."""
import types

import numpy as np
import pytest
import torch

import tide_oracle as O
from tests.conftest import GOLDEN
from tests.gpu_helpers import (TORCH2O, Checkpoint, lib, oracle_norm, ptr, storage_np, stream)
from tide_b200 import capi, workloads

pytestmark = pytest.mark.gpu
THR = 0.85
DEV = "cuda"

GOLDEN_CASES = {
    "k1_fp32_rms": lambda: workloads.k1(),
    "bf16_rms_h4096": lambda: workloads.rows(256, 4096, torch.bfloat16, seed=3, unit_norm_weight=False),
    "fp16_ln_h768": lambda: workloads.rows(256, 768, torch.float16, seed=4, norm_kind="layer",
                                           unit_norm_weight=False),
}
GOLDEN_DTYPE = {"k1_fp32_rms": torch.float32, "bf16_rms_h4096": torch.bfloat16,
                "fp16_ln_h768": torch.float16}


def score_tol(dtype, path):
    tc = path in (capi.PATH_TC, capi.PATH_TC_SPLIT)
    return 1e-2 if (dtype != torch.float32 and tc) else 1e-5


def skip_unless_path(ck, path):
    used = ck.path()
    if path not in (capi.PATH_AUTO,) and used < 0:
        pytest.skip("path does not take these arguments")
    return used


def norm_tensors(w, dtype):
    nw = w["norm_weight"].to(dtype).float().to(DEV).contiguous()
    nb = None if w["norm_bias"] is None else w["norm_bias"].to(dtype).float().to(DEV).contiguous()
    return nw, nb


def check_against_oracle(ck: Checkpoint, res: dict, dtype, kind, tol, out_ref=None):
    torch.cuda.synchronize()
    assert int(ck.error_word.item()) == 0
    n = ck.x.shape[0]
    scores = ck.scores_out.cpu().numpy()
    np.testing.assert_allclose(scores, res["scores"], atol=tol, rtol=0)
    near = np.abs(res["scores"] - THR) <= tol
    ours_exit = scores > THR
    assert np.array_equal(ours_exit[~near], res["exits"][~near])
    counts = ck.counts.cpu().numpy()
    assert counts[0] + counts[1] == n
    assert counts[1] == int(ours_exit.sum())
    # compaction is exact given our own decisions
    keep = np.nonzero(~ours_exit)[0]
    ex = np.nonzero(ours_exit)[0]
    pos_in = np.arange(n) if ck.positions is None else ck.positions.cpu().numpy()
    assert np.array_equal(ck.positions_out.cpu().numpy()[: len(keep)], pos_in[keep])
    if ck.exit_positions_out is not None:
        assert np.array_equal(ck.exit_positions_out.cpu().numpy()[: len(ex)], pos_in[ex])
    if ck.slots is not None:
        assert np.array_equal(ck.slots_out.cpu().numpy()[: len(keep)], ck.slots.cpu().numpy()[keep])
    x_np = storage_np(ck.x)
    assert np.array_equal(storage_np(ck.compact_out)[: len(keep)], x_np[keep])
    if ck.out_buffer is not None:
        out = storage_np(ck.out_buffer)
        dt = TORCH2O[dtype]
        normed = O.from_f32(O.final_norm(O.to_f32(x_np, dt), oracle_norm(kind, ck.norm_w, ck.norm_b, 0)
                                         | {"eps": res["eps"]}), dt)
        ulp = O.ulp_distance(out[pos_in[ex]], normed[ex], dt)
        bad = ulp > (8 if dtype == torch.float32 else 1)
        if kind == "layer" and bad.any():
            # LayerNorm's bias can cancel the normalised term: an output near
            # zero then has ulps far below the fp32 rounding of its two terms.
            # There the bar is the absolute fp32 error of those terms.
            diff = np.abs(O.to_f32(out[pos_in[ex]], dt) - O.to_f32(normed[ex], dt))
            scale = np.abs(O.to_f32(x_np[ex], dt)).max(axis=1, keepdims=True) * 4 + 1
            bad &= diff > scale * 2.0 ** -20
        assert not bad.any(), int(ulp.max())
        if out_ref is not None:  # rows nobody exited to stay untouched
            untouched = np.setdiff1d(np.arange(out.shape[0]), pos_in[ex])
            assert np.array_equal(out[untouched], out_ref[untouched])


@pytest.mark.parametrize("path", [capi.PATH_SIMT, capi.PATH_TC, capi.PATH_TC_SPLIT])
@pytest.mark.parametrize("name", list(GOLDEN_CASES))
def test_checkpoint_golden(name, path):
    dtype = GOLDEN_DTYPE[name]
    g = np.load(GOLDEN / f"{name}.npz")
    w = GOLDEN_CASES[name]()
    x = w["x"].to(dtype).to(DEV).contiguous()
    nw, nb = norm_tensors(w, dtype)
    n, H = x.shape
    out = torch.zeros_like(x)
    ck = Checkpoint(x, w["norm_kind"], nw, nb, w["eps"], w["down"].to(DEV), w["up"].to(DEV),
                    float(g["bias"]), THR, out_buffer=out, path=path)
    used = skip_unless_path(ck, path)
    ck()
    tol = score_tol(dtype, used)
    # against the reference's own outputs
    torch.cuda.synchronize()
    s = ck.scores_out.cpu().numpy()
    np.testing.assert_allclose(s, g["scores"], atol=tol, rtol=0)
    near = np.abs(g["scores"] - THR) <= tol
    assert np.array_equal((s > THR)[~near], g["mask"][~near])
    if np.array_equal(s > THR, g["mask"]):
        assert np.array_equal(ck.positions_out.cpu().numpy()[: int(g["n_survivors"])], g["positions"])
        rows = g["normed_exit_rows_idx"]
        ulp = O.ulp_distance(storage_np(out)[rows], g["normed_exit_rows"], TORCH2O[dtype])
        assert ulp.max() <= (8 if dtype == torch.float32 else 1)
    # against the oracle on the same inputs
    dt = TORCH2O[dtype]
    norm = oracle_norm(w["norm_kind"], nw, nb, w["eps"])
    res = O.checkpoint(storage_np(x), dt, norm, w["down"].numpy(), w["up"].numpy(),
                       float(g["bias"]), THR)
    res["eps"] = w["eps"]
    check_against_oracle(ck, res, dtype, w["norm_kind"], tol, out_ref=np.zeros_like(storage_np(out)))


@pytest.mark.parametrize("n", [0, 1, 31, 32, 33, 63, 64, 65, 127, 128, 129, 1023, 1024, 1025, 5000])
@pytest.mark.parametrize("dtype,H", [(torch.bfloat16, 256), (torch.float16, 256),
                                     (torch.float32, 256), (torch.bfloat16, 1024)])
@pytest.mark.parametrize("path", [capi.PATH_AUTO, capi.PATH_TC_SPLIT])
def test_checkpoint_sizes_positions_slots(n, dtype, H, path):
    """Sizes around the warp, tile and 1024 boundaries on the automatic path
    (fused single pass / SIMT at these sizes) and on the split path (its
    mover: 16-byte SIMT rows at H = 256, bulk copies at H = 1024)."""
    w = workloads.rows(max(n, 1), H, dtype, b=128, seed=100 + n, unit_norm_weight=False)
    x = w["x"][:n].to(DEV).contiguous()
    nw, nb = norm_tensors(w, dtype)
    g = torch.Generator().manual_seed(n)
    n_total = 3 * n + 5
    positions = torch.randperm(n_total, generator=g)[:n].to(DEV)
    slots = torch.randint(0, 1 << 30, (n,), generator=g, dtype=torch.int32).to(DEV)
    out = torch.randn(n_total, H, generator=g).to(dtype).to(DEV)
    out0 = storage_np(out).copy()
    dt = TORCH2O[dtype]
    norm = oracle_norm("rms", nw, nb, 1e-5)
    z = O.router_logits(O.final_norm(O.to_f32(storage_np(x), dt), norm), w["down"].numpy(),
                        w["up"].numpy()) if n else np.zeros(0)
    bias = workloads.bias_for_exit_fraction(z, 0.4, THR)
    ck = Checkpoint(x, "rms", nw, None, 1e-5, w["down"].to(DEV), w["up"].to(DEV), bias, THR,
                    positions=positions, slots=slots, out_buffer=out, path=path)
    used = skip_unless_path(ck, path)
    ck()
    res = O.checkpoint(storage_np(x), dt, norm, w["down"].numpy(), w["up"].numpy(), bias, THR,
                       positions=positions.cpu().numpy(), slots=slots.cpu().numpy())
    res["eps"] = 1e-5
    check_against_oracle(ck, res, dtype, "rms", score_tol(dtype, used), out_ref=out0)


@pytest.mark.parametrize("fraction", [0.0, 1.0])
def test_checkpoint_all_or_nothing(fraction):
    n, H = 700, 512
    w = workloads.rows(n, H, torch.bfloat16, seed=9)
    x = w["x"].to(DEV)
    up_bias = -50.0 if fraction == 0.0 else 50.0
    out = torch.zeros_like(x)
    ck = Checkpoint(x, "rms", w["norm_weight"].to(DEV), None, 1e-5, w["down"].to(DEV),
                    w["up"].to(DEV), up_bias, THR, out_buffer=out)()
    c = ck.counts.cpu().tolist()
    assert c == ([n, 0] if fraction == 0.0 else [0, n])
    if fraction == 1.0:
        assert np.array_equal(ck.exit_positions_out.cpu().numpy(), np.arange(n))
    else:
        assert np.array_equal(ck.positions_out.cpu().numpy(), np.arange(n))
        assert torch.equal(ck.compact_out, x)
        assert int(out.abs().sum().item()) == 0


def test_checkpoint_device_row_count():
    """n_rows_dev < capacity: rows past the device count are ignored."""
    n_cap, n_live, H = 3000, 1777, 384
    w = workloads.rows(n_cap, H, torch.bfloat16, seed=21)
    x = w["x"].to(DEV)
    cnt = torch.tensor([n_live], dtype=torch.int32, device=DEV)
    out = torch.zeros_like(x)
    nw = w["norm_weight"].to(DEV)
    ck = Checkpoint(x, "rms", nw, None, 1e-5, w["down"].to(DEV), w["up"].to(DEV), 0.0, 0.5,
                    out_buffer=out, n_rows_dev=cnt)()
    torch.cuda.synchronize()
    s = ck.scores_out.cpu().numpy()
    c = ck.counts.cpu().tolist()
    assert c[0] + c[1] == n_live
    assert c[1] == int((s[:n_live] > 0.5).sum())
    assert np.all(s[n_live:] == -1.0)  # untouched
    keep = np.nonzero(s[:n_live] <= 0.5)[0]
    assert np.array_equal(ck.positions_out.cpu().numpy()[: len(keep)], keep)


@pytest.mark.parametrize("dtype,path", [(torch.bfloat16, capi.PATH_SIMT), (torch.bfloat16, capi.PATH_TC),
                                        (torch.bfloat16, capi.PATH_TC_SPLIT),
                                        (torch.float32, capi.PATH_TC_SPLIT)])
@pytest.mark.parametrize("live", [0, 1, 63, 64, 65])
def test_device_row_count_edges(dtype, path, live):
    """A live count on the device of 0 (an earlier checkpoint exited every
    row), 1, and around a 64-row tile, below a launch capacity of 1000 rows:
    nothing past the live rows is read or written; with no live rows the
    counts are {0, 0} and every output stays untouched.  fp32 rows on the
    split path (the tf32 router) too."""
    n_cap, H = 1000, 512
    w = workloads.rows(n_cap, H, dtype, seed=70 + live, unit_norm_weight=False)
    x = w["x"].to(DEV)
    nw = w["norm_weight"].to(DEV)
    norm = oracle_norm("rms", nw, None, 1e-5)
    x_live = storage_np(x)[:live]
    z = O.router_logits(O.final_norm(O.to_f32(storage_np(x), TORCH2O[dtype]), norm),
                        w["down"].numpy(), w["up"].numpy())
    bias = workloads.bias_for_exit_fraction(z, 0.4, THR)
    out = torch.zeros_like(x)
    out0 = storage_np(out).copy()
    cnt = torch.tensor([live], dtype=torch.int32, device=DEV)
    ck = Checkpoint(x, "rms", nw, None, 1e-5, w["down"].to(DEV), w["up"].to(DEV), bias, THR,
                    out_buffer=out, n_rows_dev=cnt, path=path)
    assert ck.path() == path
    ck()
    torch.cuda.synchronize()
    assert int(ck.error_word.item()) == 0
    assert np.all(ck.scores_out.cpu().numpy()[live:] == -1.0)
    if live == 0:
        assert ck.counts.cpu().tolist() == [0, 0]
        assert np.all(ck.positions_out.cpu().numpy() == -7)
        assert np.all(ck.exit_positions_out.cpu().numpy() == -7)
        assert np.array_equal(storage_np(out), out0)
        return
    res = O.checkpoint(x_live, TORCH2O[dtype], norm, w["down"].numpy(), w["up"].numpy(), bias, THR)
    res["eps"] = 1e-5
    view = types.SimpleNamespace(
        x=ck.x[:live], scores_out=ck.scores_out[:live], counts=ck.counts, error_word=ck.error_word,
        positions=None, slots=None, positions_out=ck.positions_out,
        exit_positions_out=ck.exit_positions_out, compact_out=ck.compact_out, out_buffer=out,
        norm_w=ck.norm_w, norm_b=ck.norm_b)
    check_against_oracle(view, res, dtype, "rms", score_tol(dtype, path), out_ref=out0)


@pytest.mark.parametrize("path", [capi.PATH_SIMT, capi.PATH_TC, capi.PATH_TC_SPLIT])
def test_checkpoint_chain_on_device_counts(path):
    """Three checkpoints chained on device-side counts with no host sync in
    between; afterwards each stage is checked against the oracle on the rows
    it actually received (compaction exact given the stage's decisions)."""
    n, H = 6000, 512
    dtype = torch.bfloat16
    dt = TORCH2O[dtype]
    ws = [workloads.rows(n, H, dtype, seed=40 + i, unit_norm_weight=False) for i in range(3)]
    fractions = [0.2, 0.3, 0.5]
    nw = ws[0]["norm_weight"].to(DEV)
    norm = oracle_norm("rms", nw, None, 1e-5)
    # biases placed on the oracle's own chain
    pos = np.arange(n, dtype=np.int64)
    biases = []
    for k in range(3):
        xk = storage_np(ws[k]["x"])[pos]
        z = O.router_logits(O.final_norm(O.to_f32(xk, dt), norm), ws[k]["down"].numpy(),
                            ws[k]["up"].numpy())
        b = workloads.bias_for_exit_fraction(z, fractions[k], THR)
        biases.append(b)
        pos = O.checkpoint(xk, dt, norm, ws[k]["down"].numpy(), ws[k]["up"].numpy(), b, THR,
                           positions=pos)["positions"]
    # device chain
    out = torch.zeros(n, H, dtype=dtype, device=DEV)
    positions = torch.arange(n, device=DEV)
    count = torch.tensor([n], dtype=torch.int32, device=DEV)
    stages = []
    for k in range(3):
        xk = ws[k]["x"].to(DEV)[positions]
        ck = Checkpoint(xk, "rms", nw, None, 1e-5, ws[k]["down"].to(DEV), ws[k]["up"].to(DEV),
                        biases[k], THR, positions=positions, out_buffer=out, n_rows_dev=count,
                        path=path)()
        stages.append(ck)
        positions = ck.positions_out.clone()
        positions[positions < 0] = 0
        count = ck.counts[:1].clone()
    torch.cuda.synchronize()
    # stage-by-stage verification
    pos = np.arange(n, dtype=np.int64)
    out_o = np.zeros((n, H), dtype=np.uint16)
    for k, ck in enumerate(stages):
        assert int(ck.error_word.item()) == 0
        live = len(pos)
        tol = score_tol(dtype, ck.path())
        xk = storage_np(ws[k]["x"])[pos]
        r = O.checkpoint(xk, dt, norm, ws[k]["down"].numpy(), ws[k]["up"].numpy(), biases[k], THR,
                         positions=pos)
        s = ck.scores_out.cpu().numpy()[:live]
        np.testing.assert_allclose(s, r["scores"], atol=tol, rtol=0)
        near = np.abs(r["scores"] - THR) <= tol
        ours = s > THR
        assert np.array_equal(ours[~near], r["exits"][~near])
        c = ck.counts.cpu().tolist()
        assert c == [int((~ours).sum()), int(ours.sum())]
        assert np.array_equal(ck.positions_out.cpu().numpy()[: c[0]], pos[~ours])
        normed = O.from_f32(O.final_norm(O.to_f32(xk, dt), norm), dt)
        out_o[pos[ours]] = normed[ours]
        pos = pos[~ours]
    assert O.ulp_distance(storage_np(out), out_o, dt).max() <= 1


def test_bad_exit_position_is_flagged_not_written():
    n, H = 64, 128
    w = workloads.rows(n, H, torch.bfloat16, seed=5)
    x = w["x"].to(DEV)
    out = torch.zeros(n, H, dtype=torch.bfloat16, device=DEV)
    positions = torch.arange(n, device=DEV)
    positions[3] = -1
    positions[10] = n  # one past the end
    ck = Checkpoint(x, "rms", w["norm_weight"].to(DEV), None, 1e-5, w["down"].to(DEV),
                    w["up"].to(DEV), 50.0, THR, positions=positions, out_buffer=out)()
    torch.cuda.synchronize()
    assert int(ck.error_word.item()) & capi.DEVERR_POSITION
    written = out.float().abs().sum(dim=1).cpu().numpy() > 0
    expect = np.ones(n, dtype=bool)
    expect[[3, 10]] = False
    assert np.array_equal(written, expect)
    assert ck.counts.cpu().tolist() == [0, n]


@pytest.mark.parametrize("H", [256, 512, 768, 1024, 2048, 4096, 5120, 8192])
def test_fused_cluster_sizes(H):
    """The fused kernel at every cluster size it uses (H 256/512 -> 1 CTA,
    768/1024 -> 2, 2048 -> 4, 4096 -> 8, 5120/8192 -> 16, a non-portable
    cluster size), RMSNorm and LayerNorm."""
    dtype = torch.bfloat16
    n = 3000
    for kind in ("rms", "layer"):
        w = workloads.rows(n, H, dtype, seed=H + (kind == "layer"), norm_kind=kind,
                           unit_norm_weight=False)
        x = w["x"].to(DEV)
        nw, nb = norm_tensors(w, dtype)
        dt = TORCH2O[dtype]
        norm = oracle_norm(kind, nw, nb, 1e-5)
        z = O.router_logits(O.final_norm(O.to_f32(storage_np(x), dt), norm), w["down"].numpy(),
                            w["up"].numpy())
        bias = workloads.bias_for_exit_fraction(z, 0.35, THR)
        g = torch.Generator().manual_seed(H)
        positions = torch.randperm(2 * n, generator=g)[:n].to(DEV)
        slots = torch.randint(0, 1 << 20, (n,), generator=g, dtype=torch.int32).to(DEV)
        out = torch.zeros(2 * n, H, dtype=dtype, device=DEV)
        out0 = storage_np(out).copy()
        ck = Checkpoint(x, kind, nw, nb, 1e-5, w["down"].to(DEV), w["up"].to(DEV), bias, THR,
                        positions=positions, slots=slots, out_buffer=out, path=capi.PATH_TC)
        assert ck.path() == capi.PATH_TC
        ck()
        res = O.checkpoint(storage_np(x), dt, norm, w["down"].numpy(), w["up"].numpy(), bias, THR,
                           positions=positions.cpu().numpy(), slots=slots.cpu().numpy())
        res["eps"] = 1e-5
        check_against_oracle(ck, res, dtype, kind, 1e-2, out_ref=out0)


@pytest.mark.parametrize("B", [1, 48, 100, 128, 160, 256])
def test_split_router_widths(B):
    """The tensor-core split router at router widths that are not one full
    128-unit block (padded units) and at two blocks (B > 128), RMSNorm and
    LayerNorm, bf16 and fp16, ragged row counts."""
    H, n = 1024, 2000 + B
    for kind, dtype in (("rms", torch.bfloat16), ("layer", torch.float16)):
        w = workloads.rows(n, H, dtype, b=B, seed=500 + B, norm_kind=kind, unit_norm_weight=False)
        x = w["x"].to(DEV)
        nw, nb = norm_tensors(w, dtype)
        dt = TORCH2O[dtype]
        norm = oracle_norm(kind, nw, nb, 1e-5)
        z = O.router_logits(O.final_norm(O.to_f32(storage_np(x), dt), norm), w["down"].numpy(),
                            w["up"].numpy())
        bias = workloads.bias_for_exit_fraction(z, 0.25, THR)
        out = torch.zeros_like(x)
        ck = Checkpoint(x, kind, nw, nb, 1e-5, w["down"].to(DEV), w["up"].to(DEV), bias, THR,
                        out_buffer=out, path=capi.PATH_TC_SPLIT)
        assert ck.path() == capi.PATH_TC_SPLIT
        ck()
        res = O.checkpoint(storage_np(x), dt, norm, w["down"].numpy(), w["up"].numpy(), bias, THR)
        res["eps"] = 1e-5
        check_against_oracle(ck, res, dtype, kind, 1e-2, out_ref=np.zeros_like(storage_np(out)))


@pytest.mark.parametrize("units", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("device_count", [False, True])
def test_split_router_tile_geometry(units, device_count):
    """The split router sizes its pipeline from the live row count: the
    largest CTA tile (1-8 units of 32 rows, also the MMA's N), the K chunks
    per stage and the 128/64/32-row boxes follow from it.  Row counts that
    give every tile size on this GPU, ragged last units, and a live count on
    the device below the launch capacity; parity with the oracle."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    H = 1024
    n_cap = sms * 32 * units
    n = n_cap - 17 if device_count else n_cap - 5
    w = workloads.rows(n_cap, H, torch.bfloat16, seed=900 + units, unit_norm_weight=False)
    x = w["x"].to(DEV)
    nw, nb = norm_tensors(w, torch.bfloat16)
    norm = oracle_norm("rms", nw, nb, 1e-5)
    x_live = storage_np(x)[:n]
    z = O.router_logits(O.final_norm(O.to_f32(x_live, O.BF16), norm), w["down"].numpy(), w["up"].numpy())
    bias = workloads.bias_for_exit_fraction(z, 0.2, THR)
    out = torch.zeros_like(x)
    if device_count:
        cnt = torch.tensor([n], dtype=torch.int32, device=DEV)
        ck = Checkpoint(x, "rms", nw, nb, 1e-5, w["down"].to(DEV), w["up"].to(DEV), bias, THR,
                        out_buffer=out, n_rows_dev=cnt, path=capi.PATH_TC_SPLIT)
    else:
        ck = Checkpoint(x[:n], "rms", nw, nb, 1e-5, w["down"].to(DEV), w["up"].to(DEV), bias, THR,
                        out_buffer=out, n_total=n_cap, path=capi.PATH_TC_SPLIT)
    assert ck.path() == capi.PATH_TC_SPLIT
    ck()
    res = O.checkpoint(x_live, O.BF16, norm, w["down"].numpy(), w["up"].numpy(), bias, THR)
    res["eps"] = 1e-5
    live = types.SimpleNamespace(
        x=ck.x[:n], scores_out=ck.scores_out[:n], counts=ck.counts, error_word=ck.error_word,
        positions=None, slots=None, positions_out=ck.positions_out,
        exit_positions_out=ck.exit_positions_out, compact_out=ck.compact_out, out_buffer=out,
        norm_w=ck.norm_w, norm_b=ck.norm_b)
    check_against_oracle(live, res, torch.bfloat16, "rms", 1e-2)


@pytest.mark.parametrize("kind", ["rms", "layer"])
@pytest.mark.parametrize("n,H,B", [(1, 768, 128), (100, 768, 128), (4096, 768, 128),
                                   (5000, 1024, 200), (12000, 4096, 128), (777, 800, 48),
                                   (25000, 512, 128), (40000, 256, 128)])
def test_fp32_tensor_core_router(n, H, B, kind):
    """fp32 rows on the split path: kind::tf32 MMAs on hi/lo operand splits,
    three products per K step.  Scores within 1e-5 of the oracle (the fp32
    bar), exits final-normed within 8 ulp, stable compaction.  Tiles of 1-8
    units (6 at 25000 rows; two tiles per CTA, 8 units and 1, at 40000), a
    router wider than 128 (two 128-unit blocks) and narrower (padded units),
    H = 800 (25 chunks of 32 columns).  LayerNorm rows carry a mean
    of 3: the statistics are taken about each row's first value, so the
    variance does not cancel away."""
    w = workloads.rows(n, H, torch.float32, b=B, seed=1300 + n, norm_kind=kind,
                       unit_norm_weight=False)
    x = (w["x"] + 3.0 if kind == "layer" else w["x"]).to(DEV).contiguous()
    nw, nb = norm_tensors(w, torch.float32)
    norm = oracle_norm(kind, nw, nb, 1e-5)
    z = O.router_logits(O.final_norm(O.to_f32(storage_np(x), O.F32), norm), w["down"].numpy(),
                        w["up"].numpy())
    bias = workloads.bias_for_exit_fraction(z, 0.3, THR)
    out = torch.zeros(n + 3, H, device=DEV)
    ck = Checkpoint(x, kind, nw, nb, 1e-5, w["down"].to(DEV), w["up"].to(DEV), bias, THR,
                    out_buffer=out, n_total=n + 3, path=capi.PATH_TC_SPLIT)
    assert ck.path() == capi.PATH_TC_SPLIT
    ck()
    res = O.checkpoint(storage_np(x), O.F32, norm, w["down"].numpy(), w["up"].numpy(), bias, THR)
    res["eps"] = 1e-5
    check_against_oracle(ck, res, torch.float32, kind, 1e-5, out_ref=np.zeros((n + 3, H), np.float32))


@pytest.mark.parametrize("path", [capi.PATH_TC, capi.PATH_TC_SPLIT, capi.PATH_SIMT])
def test_full_size_properties(path):
    """32768 x 4096 bf16 (one 8B-architecture prefill batch): properties that
    hold at any size -- counts add up, positions are a stable partition,
    survivors are bit-exact copies, exits are the final norm of their row
    (<= 1 ulp against a torch fp32 evaluation), decisions follow the scores,
    scores match a torch fp32 router within 1e-2."""
    n, H = 32768, 4096
    w = workloads.rows(n, H, torch.bfloat16, seed=77, device=DEV)
    x = w["x"]
    nw = w["norm_weight"]
    z = workloads.prebias_logits_torch(x, "rms", nw, None, 1e-5, w["down"], w["up"])
    bias = workloads.bias_for_exit_fraction(z, 0.3, THR)
    out = torch.zeros_like(x)
    ck = Checkpoint(x, "rms", nw, None, 1e-5, w["down"], w["up"], bias, THR, out_buffer=out,
                    path=path)
    assert ck.path() == path
    ck()
    torch.cuda.synchronize()
    assert int(ck.error_word.item()) == 0
    s = ck.scores_out
    ref = torch.sigmoid(z + bias)
    assert float((s - ref).abs().max()) <= (1e-2 if path != capi.PATH_SIMT else 1e-5)
    ex = s > THR
    c = ck.counts.cpu().tolist()
    assert c == [int((~ex).sum()), int(ex.sum())]
    assert abs(c[1] - 0.3 * n) < 0.01 * n
    keep_idx = torch.nonzero(~ex).flatten()
    ex_idx = torch.nonzero(ex).flatten()
    assert torch.equal(ck.positions_out[: c[0]], keep_idx)
    assert torch.equal(ck.exit_positions_out[: c[1]], ex_idx)
    assert torch.equal(ck.compact_out[: c[0]], x[keep_idx])
    xf = x[ex_idx].float()
    normed = (nw * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5))).to(torch.bfloat16)
    got = out[ex_idx]
    diff = (got.view(torch.int16).int() - normed.view(torch.int16).int()).abs()
    assert int(diff.max()) <= 1
    untouched = torch.ones(n, dtype=torch.bool, device=DEV)
    untouched[ex_idx] = False
    assert int(out[untouched].abs().sum()) == 0


def test_full_size_properties_fp32():
    """32768 x 4096 fp32 rows on the split path (the tf32 router, three
    products): counts add up, positions are a stable partition, survivors are
    bit-exact copies, exits are the final norm of their row (<= 8 ulp against
    a torch fp32 evaluation), decisions follow the scores, scores match a
    torch fp32 router (no tf32) within 1e-5."""
    assert not torch.backends.cuda.matmul.allow_tf32
    n, H = 32768, 4096
    w = workloads.rows(n, H, torch.float32, seed=78, device=DEV, unit_norm_weight=False)
    x = w["x"]
    nw = w["norm_weight"]
    z = workloads.prebias_logits_torch(x, "rms", nw, None, 1e-5, w["down"], w["up"])
    bias = workloads.bias_for_exit_fraction(z, 0.3, THR)
    out = torch.zeros_like(x)
    ck = Checkpoint(x, "rms", nw, None, 1e-5, w["down"], w["up"], bias, THR, out_buffer=out,
                    path=capi.PATH_TC_SPLIT)
    assert ck.path() == capi.PATH_TC_SPLIT
    ck()
    torch.cuda.synchronize()
    assert int(ck.error_word.item()) == 0
    s = ck.scores_out
    assert float((s - torch.sigmoid(z + bias)).abs().max()) <= 1e-5
    ex = s > THR
    c = ck.counts.cpu().tolist()
    assert c == [int((~ex).sum()), int(ex.sum())]
    assert abs(c[1] - 0.3 * n) < 0.01 * n
    keep_idx = torch.nonzero(~ex).flatten()
    ex_idx = torch.nonzero(ex).flatten()
    assert torch.equal(ck.positions_out[: c[0]], keep_idx)
    assert torch.equal(ck.exit_positions_out[: c[1]], ex_idx)
    assert torch.equal(ck.compact_out[: c[0]], x[keep_idx])
    xe = x[ex_idx]
    normed = nw * (xe * torch.rsqrt(xe.pow(2).mean(-1, keepdim=True) + 1e-5))
    diff = (out[ex_idx].view(torch.int32).long() - normed.view(torch.int32).long()).abs()
    assert int(diff.max()) <= 8
    untouched = torch.ones(n, dtype=torch.bool, device=DEV)
    untouched[ex_idx] = False
    assert int(out[untouched].abs().sum()) == 0


# the bandwidth sweep's shapes: N up to 1M rows, H 2048..8192, exit fractions
# 0..0.9 (the largest case holds 3 x 16 GiB of rows on the device)
SWEEP = [(65536, 2048, 0.0), (65536, 5120, 0.1), (16384, 8192, 0.5), (262144, 4096, 0.9),
         (1048576, 2048, 0.1), (1048576, 8192, 0.5)]


@pytest.mark.parametrize("n,H,f", SWEEP)
def test_bandwidth_sweep_properties(n, H, f):
    """Size-independent properties at the sweep's shapes, default path:
    decisions follow the scores, scores within 1e-2 of a torch fp32 router,
    counts add up, positions are the stable partition, survivors are
    bit-exact copies, exits are their row's final norm (<= 1 ulp), rows
    nobody exited to stay zero."""
    w = workloads.rows(n, H, torch.bfloat16, seed=n % 1000 + H, device=DEV)
    x, nw = w["x"], w["norm_weight"]
    z = workloads.prebias_logits_torch(x, "rms", nw, None, 1e-5, w["down"], w["up"])
    bias = workloads.bias_for_exit_fraction(z, f, THR)
    out = torch.zeros_like(x)
    ck = Checkpoint(x, "rms", nw, None, 1e-5, w["down"], w["up"], bias, THR, out_buffer=out)
    ck()
    torch.cuda.synchronize()
    assert int(ck.error_word.item()) == 0
    s = ck.scores_out
    assert float((s - torch.sigmoid(z + bias)).abs().max()) <= 1e-2
    ex = s > THR
    c = ck.counts.cpu().tolist()
    assert c == [int((~ex).sum()), int(ex.sum())]
    assert abs(c[1] - f * n) <= max(2, 0.001 * n)
    keep_idx = torch.nonzero(~ex).flatten()
    ex_idx = torch.nonzero(ex).flatten()
    assert torch.equal(ck.positions_out[: c[0]], keep_idx)
    assert torch.equal(ck.exit_positions_out[: c[1]], ex_idx)
    step = 65536
    for a in range(0, c[0], step):
        assert torch.equal(ck.compact_out[a:a + step][: c[0] - a], x[keep_idx[a:a + step]])
    for a in range(0, c[1], step):
        idx = ex_idx[a:a + step]
        xf = x[idx].float()
        normed = (nw * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5))).to(torch.bfloat16)
        diff = (out[idx].view(torch.int16).int() - normed.view(torch.int16).int()).abs()
        assert int(diff.max()) <= 1
    untouched = torch.ones(n, dtype=torch.bool, device=DEV)
    untouched[ex_idx] = False
    for a in range(0, n, step):
        sel = untouched[a:a + step]
        assert int(out[a:a + step][sel].abs().sum()) == 0


def test_layernorm_fp16_large_split():
    """LayerNorm on fp16 rows at 65536 x 2048 on the split path (bulk mover,
    LayerNorm exits): decisions follow the scores, scores within 1e-2 of a
    torch fp32 router, stable compaction, exits equal to the oracle's final
    norm of their row (the same bar as the small cases)."""
    n, H, dtype = 65536, 2048, torch.float16
    w = workloads.rows(n, H, dtype, seed=2049, norm_kind="layer", unit_norm_weight=False,
                       device=DEV)
    x = w["x"]
    nw, nb = norm_tensors(w, dtype)
    z = workloads.prebias_logits_torch(x, "layer", nw, nb, 1e-5, w["down"], w["up"])
    bias = workloads.bias_for_exit_fraction(z, 0.3, THR)
    out = torch.zeros_like(x)
    ck = Checkpoint(x, "layer", nw, nb, 1e-5, w["down"], w["up"], bias, THR, out_buffer=out,
                    path=capi.PATH_TC_SPLIT)
    assert ck.path() == capi.PATH_TC_SPLIT
    ck()
    torch.cuda.synchronize()
    assert int(ck.error_word.item()) == 0
    s = ck.scores_out
    assert float((s - torch.sigmoid(z + bias)).abs().max()) <= 1e-2
    ex = s > THR
    c = ck.counts.cpu().tolist()
    assert c == [int((~ex).sum()), int(ex.sum())]
    keep_idx = torch.nonzero(~ex).flatten()
    ex_idx = torch.nonzero(ex).flatten()
    assert torch.equal(ck.positions_out[: c[0]], keep_idx)
    assert torch.equal(ck.compact_out[: c[0]], x[keep_idx])
    dt = TORCH2O[dtype]
    norm = oracle_norm("layer", nw, nb, 1e-5)
    x_ex = storage_np(x[ex_idx])
    normed = O.from_f32(O.final_norm(O.to_f32(x_ex, dt), norm), dt)
    got = storage_np(out[ex_idx])
    ulp = O.ulp_distance(got, normed, dt)
    bad = ulp > 1
    if bad.any():  # cancellation in x - mean: fp32-level absolute error is the bar
        diff = np.abs(O.to_f32(got, dt) - O.to_f32(normed, dt))
        scale = np.abs(O.to_f32(x_ex, dt)).max(axis=1, keepdims=True) * 4 + 1
        bad &= diff > scale * 2.0 ** -20
    assert not bad.any(), int(ulp.max())


# ---------------------------------------------------------- reference ops


def test_batch_compact_kats():
    g = np.load(GOLDEN / "compaction_kats.npz")
    keys = sorted({k.rsplit("_mask", 1)[0] for k in g.files if k.endswith("_mask")
                   and not k.startswith("chain")})
    for k in keys:
        mask = torch.from_numpy(g[k + "_mask"].astype(np.int32)).to(DEV)
        n = mask.shape[0]
        x = torch.arange(n * 8, dtype=torch.float32, device=DEV).reshape(n, 8)
        comp = torch.empty_like(x)
        exd = torch.empty_like(x)
        ci = torch.full((max(n, 1),), -1, dtype=torch.int32, device=DEV)
        ei = torch.full((max(n, 1),), -1, dtype=torch.int32, device=DEV)
        nr = torch.full((1,), -1, dtype=torch.int32, device=DEV)
        wsz = lib().tide_batch_compact_workspace_size(n)
        ws = torch.empty(wsz, dtype=torch.uint8, device=DEV)
        rc = lib().tide_batch_compact(capi.DTYPE_F32, ptr(x), ptr(mask), ptr(comp), ptr(exd),
                                      ptr(ci), ptr(ei), ptr(nr), n, 8, ptr(ws), wsz, None, stream())
        capi.check(lib(), rc, "batch_compact")
        torch.cuda.synchronize()
        r = int(nr.item())
        assert r == n - int(g[k + "_mask"].sum()), k
        assert np.array_equal(ci[:r].cpu().numpy().astype(np.int64), g[k + "_positions"]), k
        assert np.array_equal(comp[:r, 0].cpu().numpy(), g[k + "_kept_first_col"]), k
        ex_ref = np.nonzero(g[k + "_mask"])[0]
        assert np.array_equal(ei[: n - r].cpu().numpy(), ex_ref), k
        assert torch.equal(exd[: n - r], x[torch.as_tensor(ex_ref, device=DEV)]), k


@pytest.mark.parametrize("n,H,dtype", [(100003, 96, torch.float32), (40000, 13, torch.bfloat16),
                                       (65536, 4096, torch.bfloat16), (2, 6, torch.float16)])
def test_batch_compact_large_and_ragged(n, H, dtype):
    g = torch.Generator().manual_seed(n)
    x = torch.randn(n, H, generator=g).to(dtype).to(DEV)
    mask_np = (torch.rand(n, generator=g) < 0.37).numpy()
    mask = torch.from_numpy(mask_np.astype(np.int32)).to(DEV)
    comp, exd = torch.empty_like(x), torch.empty_like(x)
    ci = torch.empty(n, dtype=torch.int32, device=DEV)
    ei = torch.empty(n, dtype=torch.int32, device=DEV)
    nr = torch.empty(1, dtype=torch.int32, device=DEV)
    wsz = lib().tide_batch_compact_workspace_size(n)
    ws = torch.empty(wsz, dtype=torch.uint8, device=DEV)
    ew = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib().tide_batch_compact({torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype],
                                  ptr(x), ptr(mask), ptr(comp), ptr(exd), ptr(ci), ptr(ei), ptr(nr),
                                  n, H, ptr(ws), wsz, ptr(ew), stream())
    capi.check(lib(), rc, "batch_compact")
    keep, ex = O.stable_partition(mask_np)
    torch.cuda.synchronize()
    r = int(nr.item())
    assert r == len(keep) and int(ew.item()) == 0
    assert np.array_equal(ci[:r].cpu().numpy(), keep)
    assert np.array_equal(ei[: n - r].cpu().numpy(), ex)
    assert torch.equal(comp[:r], x[torch.as_tensor(keep, device=DEV)])
    assert torch.equal(exd[: n - r], x[torch.as_tensor(ex, device=DEV)])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H", [256, 4096, 250])
def test_exit_scatter_and_projection(dtype, H):
    n_total, n_exit = 97, 41
    g = torch.Generator().manual_seed(H)
    ex = torch.randn(n_exit, H, generator=g).to(dtype).to(DEV)
    pos = torch.randperm(n_total, generator=g)[:n_exit].to(torch.int32).to(DEV)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(DEV)
    dt = TORCH2O[dtype]
    for norm in (False, True):
        out = torch.zeros(n_total, H, dtype=dtype, device=DEV)
        if norm:
            rc = lib().tide_exit_projection(capi.DTYPE_F32 if dtype == torch.float32 else
                                            (1 if dtype == torch.float16 else 2), ptr(ex), ptr(w),
                                            ptr(pos), ptr(out), 1e-6, n_exit, H, n_total, None,
                                            stream())
            ref = O.exit_projection(storage_np(ex), dt, w.cpu().numpy(), pos.cpu().numpy(),
                                    storage_np(torch.zeros(n_total, H, dtype=dtype)), 1e-6)
            torch.cuda.synchronize()
            assert O.ulp_distance(storage_np(out), ref, dt).max() <= (8 if dt == O.F32 else 1)
        else:
            rc = lib().tide_exit_scatter(0 if dtype == torch.float32 else
                                         (1 if dtype == torch.float16 else 2), ptr(ex), ptr(pos),
                                         ptr(out), n_exit, H, n_total, None, stream())
            ref = O.exit_scatter(storage_np(ex), pos.cpu().numpy(),
                                 storage_np(torch.zeros(n_total, H, dtype=dtype)))
            torch.cuda.synchronize()
            assert np.array_equal(storage_np(out), ref)
        capi.check(lib(), rc, "scatter")


@pytest.mark.parametrize("kind", ["rms", "layer"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_norm_scatter(kind, dtype):
    n, n_total, H = 300, 512, 768
    w = workloads.rows(n, H, dtype, seed=77, norm_kind=kind, unit_norm_weight=False)
    x = w["x"].to(DEV)
    nw, nb = norm_tensors(w, dtype)
    pos = torch.randperm(n_total, generator=torch.Generator().manual_seed(1))[:n].to(DEV)
    out = torch.zeros(n_total, H, dtype=dtype, device=DEV)
    rc = lib().tide_norm_scatter(1 if dtype == torch.float16 else 2,
                                 capi.NORM_RMS if kind == "rms" else capi.NORM_LAYER, ptr(x),
                                 ptr(pos), ptr(out), ptr(nw), ptr(nb), 1e-5, n, H, n_total, None,
                                 stream())
    capi.check(lib(), rc, "norm_scatter")
    dt = TORCH2O[dtype]
    ref = O.from_f32(O.final_norm(O.to_f32(storage_np(x), dt), oracle_norm(kind, nw, nb, 1e-5)), dt)
    torch.cuda.synchronize()
    got = storage_np(out)[pos.cpu().numpy()]
    assert O.ulp_distance(got, ref, dt).max() <= 1


def test_fused_layernorm_route_reference_op():
    """tide_fused_layernorm_route against test_kernels.py's python oracle
    (RMSNorm eps 1e-6 with fp32 weights, pre-transposed down [H, B])."""
    for n, H, dtype in [(1, 2048, torch.float32), (8, 4096, torch.float16),
                        (128, 4096, torch.bfloat16), (32, 1000, torch.bfloat16)]:
        g = torch.Generator().manual_seed(n * H)
        x = torch.randn(n, H, generator=g).to(dtype).to(DEV)
        nw = torch.randn(H, generator=g).to(DEV)
        dt_ = torch.randn(H, 128, generator=g).to(DEV)
        ut = torch.randn(128, 1, generator=g).to(DEV)
        s = torch.empty(n, device=DEV)
        rc = lib().tide_fused_layernorm_route({torch.float32: 0, torch.float16: 1,
                                               torch.bfloat16: 2}[dtype], ptr(x), ptr(nw), ptr(dt_),
                                              ptr(ut), 1e-6, ptr(s), n, H, 128, stream())
        capi.check(lib(), rc, "fused_layernorm_route")
        ref = O.fused_layernorm_route(storage_np(x), TORCH2O[dtype], nw.cpu().numpy(),
                                      dt_.cpu().numpy(), ut.cpu().numpy(), 1e-6)
        torch.cuda.synchronize()
        np.testing.assert_allclose(s.cpu().numpy(), ref, atol=2e-3, rtol=0)


def test_paired_router_parity_in_its_own_process():
    """The paired-CTA router (tcgen05.mma cta_group::2, TIDE_ROUTER=pair) on
    the split path's parity cases (golden vectors, tile geometry of 1 to 8
    units per CTA, the 32768 x 4096 properties), in a fresh process with the
    switch set."""
    import os
    import subprocess
    import sys

    from tests.conftest import ROOT

    env = dict(os.environ, TIDE_ROUTER="pair")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", str(ROOT / "tests" / "test_gpu_capi.py"),
                        "-k", "golden and TC_SPLIT or split_router or full_size_properties"],
                       cwd=str(ROOT), env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
