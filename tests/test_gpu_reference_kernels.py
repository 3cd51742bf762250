"""The reference's own CUDA operators, built for sm_100a from its sources
(oracle/build_ref.py: torch.ops.tide_ref), as a checker on the GPU: the
oracle is pinned against them, and this repository's torch.ops.tide
operators are compared with them on the same inputs.

Shapes follow the reference's kernel tests (tests/test_kernels.py:64-156:
N in {1, 8, 32, 128}, H in {2048, 4096}, every input dtype) plus the
configs' widths.  The reference's batch_compact is only called with
N <= 1024 (its prefix sums run in one block of N threads,
csrc/kernels/batch_compact.cu:175)."""
from pathlib import Path

import numpy as np
import pytest
import torch

import tide_oracle as O
from tests.gpu_helpers import TORCH2O, storage_np

pytestmark = pytest.mark.gpu
DEV = "cuda"
REF_LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "tide_ref_C.so"


@pytest.fixture(scope="module")
def ops():
    if not REF_LIB.is_file():
        pytest.skip("the reference's operators were not built (oracle/build_ref.py)")
    from tide_b200 import _native

    torch.ops.load_library(str(REF_LIB))
    return torch.ops.tide_ref, _native.ops()


def _router(H, B=128, seed=0):
    g = torch.Generator().manual_seed(seed)
    nw = (1 + 0.1 * torch.randn(H, generator=g)).float()
    down = (0.02 * torch.randn(B, H, generator=g)).float()
    up = (0.2 * torch.randn(1, B, generator=g)).float()
    return nw, down, up


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("N,H", [(1, 2048), (8, 4096), (32, 2048), (128, 4096), (4096, 768),
                                 (3000, 4096), (2048, 8192)])
def test_router_against_the_reference_kernel(ops, dtype, N, H):
    """Scores of the reference's fused_layernorm_route kernel and of this
    repository's operator, each against the oracle (which pins the oracle on
    the reference's own GPU code): 1e-5 for fp32 rows, 1e-2 for 16-bit rows;
    so the two kernels agree within twice that."""
    ref, ours = ops
    nw, down, up = _router(H, seed=N + H)
    g = torch.Generator().manual_seed(7 * N + H)
    x = (torch.randn(N, H, generator=g) * (0.5 + 1.5 * torch.rand(N, 1, generator=g))).to(dtype)
    args = (x.to(DEV), nw.to(DEV), down.t().contiguous().to(DEV), up.t().contiguous().to(DEV), 1e-5)
    s_ref = ref.fused_layernorm_route(*args).cpu().numpy()
    s_ours = ours.fused_layernorm_route(*args).cpu().numpy()
    norm = {"kind": "rms", "weight": nw.numpy(), "bias": None, "eps": 1e-5}
    s_or = O.score_rows(storage_np(x), TORCH2O[dtype], norm, down.numpy(), up.numpy())
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert np.abs(s_ref - s_or).max() <= tol, np.abs(s_ref - s_or).max()
    assert np.abs(s_ours - s_or).max() <= tol, np.abs(s_ours - s_or).max()
    assert np.abs(s_ours - s_ref).max() <= 2 * tol, np.abs(s_ours - s_ref).max()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("N", [1, 17, 32, 33, 500, 1024])
def test_batch_compact_against_the_reference_kernel(ops, dtype, N):
    """All five outputs bit-identical to the reference kernel's (N <= 1024)."""
    ref, ours = ops
    H = 256
    g = torch.Generator().manual_seed(N)
    x = torch.randn(N, H, generator=g).to(dtype).to(DEV)
    mask = (torch.rand(N, generator=g) < 0.4).to(torch.int32).to(DEV)
    a = ref.batch_compact(x, mask)
    b = ours.batch_compact(x, mask)
    assert len(a) == len(b) == 5
    for ta, tb in zip(a, b):
        assert ta.shape == tb.shape and ta.dtype == tb.dtype
        assert torch.equal(ta, tb)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_exit_scatter_against_the_reference_kernel(ops, dtype):
    ref, ours = ops
    n_total, n_exit, H = 300, 77, 4096
    g = torch.Generator().manual_seed(3)
    ex = torch.randn(n_exit, H, generator=g).to(dtype).to(DEV)
    pos = torch.randperm(n_total, generator=g)[:n_exit].to(torch.int32).to(DEV)
    base = torch.randn(n_total, H, generator=g).to(dtype).to(DEV)
    a, b = base.clone(), base.clone()
    ref.exit_scatter(ex, pos, a)
    ours.exit_scatter(ex, pos, b)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_exit_projection_against_the_reference_kernel(ops, dtype):
    """Normed exit rows of the reference kernel against the oracle, and of
    this repository's operator against the reference kernel: within 1 ulp
    (16-bit) or 8 ulp (fp32) of the oracle each (the reference takes the
    hardware rsqrt, this repository a correctly rounded one, and the sums run
    in different orders), rows elsewhere untouched in both."""
    ref, ours = ops
    n_total, n_exit, H = 256, 64, 2048
    g = torch.Generator().manual_seed(4)
    ex = (torch.randn(n_exit, H, generator=g) * 3).to(dtype).to(DEV)
    nw = (1 + 0.1 * torch.randn(H, generator=g)).float().to(DEV)
    pos = torch.randperm(n_total, generator=g)[:n_exit].to(torch.int32).to(DEV)
    base = torch.randn(n_total, H, generator=g).to(dtype).to(DEV)
    a, b = base.clone(), base.clone()
    ref.exit_projection(ex, nw, pos, a, 1e-5)
    ours.exit_projection(ex, nw, pos, b, 1e-5)
    torch.cuda.synchronize()
    dt = TORCH2O[dtype]
    bar = 8 if dtype == torch.float32 else 1
    want = O.exit_projection(storage_np(ex.cpu()), dt, nw.cpu().numpy(), pos.cpu().numpy(),
                             storage_np(base.cpu()), 1e-5)
    d_ref = O.ulp_distance(storage_np(a.cpu()), want, dt)
    d_ours = O.ulp_distance(storage_np(b.cpu()), want, dt)
    assert d_ref.max() <= bar, d_ref.max()
    assert d_ours.max() <= bar, d_ours.max()
    rest = np.setdiff1d(np.arange(n_total), pos.cpu().numpy())
    assert torch.equal(a[rest], base[rest]) and torch.equal(b[rest], base[rest])
