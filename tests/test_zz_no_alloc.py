"""tide_batch_compact_noalloc: the row split for callers that cannot allocate
device memory (an FFI host whose GPU memory belongs to another runtime, code
running where allocation is forbidden).  It must give exactly what
tide_batch_compact gives with a caller workspace, call after call, even
though every call reuses one built-in scratch array.

This file is named so that pytest collects it last."""
import numpy as np
import pytest
import torch

from tide_b200 import _native, capi

DTYPES = {torch.float32: capi.DTYPE_F32, torch.float16: capi.DTYPE_F16,
          torch.bfloat16: capi.DTYPE_BF16}


def _outputs(n, H, dtype):
    dev = "cuda"
    return (torch.full((n, H), 7, dtype=dtype, device=dev), torch.full((n, H), 7, dtype=dtype, device=dev),
            torch.full((max(n, 1),), -1, dtype=torch.int32, device=dev),
            torch.full((max(n, 1),), -1, dtype=torch.int32, device=dev),
            torch.full((1,), -1, dtype=torch.int32, device=dev))


def _split(x, mask, noalloc: bool):
    lib = _native.lib()
    n, H = x.shape
    comp, exd, ci, ei, nr = _outputs(n, H, x.dtype)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    if noalloc:
        rc = lib.tide_batch_compact_noalloc(DTYPES[x.dtype], x.data_ptr(), mask.data_ptr(),
                                            comp.data_ptr(), exd.data_ptr(), ci.data_ptr(),
                                            ei.data_ptr(), nr.data_ptr(), n, H, err.data_ptr(), s)
    else:
        wsz = lib.tide_batch_compact_workspace_size(n)
        ws = torch.empty(wsz, dtype=torch.uint8, device="cuda")
        rc = lib.tide_batch_compact(DTYPES[x.dtype], x.data_ptr(), mask.data_ptr(), comp.data_ptr(),
                                    exd.data_ptr(), ci.data_ptr(), ei.data_ptr(), nr.data_ptr(), n,
                                    H, ws.data_ptr(), wsz, err.data_ptr(), s)
    capi.check(lib, rc, "noalloc" if noalloc else "batch_compact")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    r = int(nr.item())
    return r, comp[:r].clone(), exd[: n - r].clone(), ci[:r].clone(), ei[: n - r].clone()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,H", [(torch.bfloat16, 4096), (torch.float32, 13)])
def test_noalloc_matches_workspace_version_two_calls(dtype, H):
    g = torch.Generator().manual_seed(H)
    # a large call first, then a smaller one: the second must not see the
    # first call's tile states left in the shared scratch
    for n, p in ((70_001 if H < 100 else 40_000, 0.35), (5_000, 0.6)):
        x = torch.randn(n, H, generator=g).to(dtype).cuda()
        mask = (torch.rand(n, generator=g) < p).to(torch.int32).cuda()
        ref = _split(x, mask, noalloc=False)
        got = _split(x, mask, noalloc=True)
        assert got[0] == ref[0] == int((mask == 0).sum().item())
        for a, b in zip(got[1:], ref[1:]):
            assert torch.equal(a, b)
        keep = np.nonzero(mask.cpu().numpy() == 0)[0]
        assert np.array_equal(got[3].cpu().numpy(), keep)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [capi.NOALLOC_MAX_ROWS, 0])
def test_noalloc_at_its_limit_and_empty(n):
    """The largest call the built-in scratch takes (its last status word in
    use) and an empty call, each twice in a row, against the workspace
    version and np.nonzero.  Rows of 4 fp32 values keep the limit case at
    16 MB per tensor."""
    g = torch.Generator().manual_seed(n + 1)
    x = torch.randn(n, 4, generator=g).cuda()
    mask = (torch.rand(n, generator=g) < 0.5).to(torch.int32).cuda()
    ref = _split(x, mask, noalloc=False)
    for _ in range(2):
        got = _split(x, mask, noalloc=True)
        assert got[0] == ref[0] == int((mask == 0).sum().item())
        for a, b in zip(got[1:], ref[1:]):
            assert torch.equal(a, b)
        keep = np.nonzero(mask.cpu().numpy() == 0)[0]
        assert np.array_equal(got[3].cpu().numpy(), keep)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _native.lib()
    n = capi.NOALLOC_MAX_ROWS + 1
    rc = lib.tide_batch_compact_noalloc(capi.DTYPE_BF16, 16, 16, 16, 16, 16, 16, 16, n, 64, None,
                                        None)
    assert rc == capi.ERR_INVALID
    assert b"exceed the limit" in lib.tide_last_error()
