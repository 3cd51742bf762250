"""A bounded device wait that runs out, on purpose and without any fault.

The look-back of the stable partition waits for the status word of the tile
before it.  In the test build of the library (libtide_b200_testhooks.so, the
same kernels compiled with TIDE_TEST_UNPUBLISHED_TILE) one tile computes its
own prefix but never publishes its status: the tiles after it wait on a word
that nothing sets.  Their waits must give up after the bound, set
TIDE_DEVERR_TIMEOUT in the error word and let the kernel return; nothing may
be written outside the outputs, and the context must stay usable (a call
through the product library right after gives exact results).  This replaces
the unbounded single-block scan of the reference's batch_compact kernel
(csrc/kernels/batch_compact.cu:171-175), whose failure mode is a hang.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

import tide_oracle as O
from tests.gpu_helpers import TORCH2C, Checkpoint, oracle_norm, ptr, storage_np, stream
from tide_b200 import _native, build, capi

pytestmark = pytest.mark.gpu
DEV = "cuda"
CANARY_ROWS = 64


@pytest.fixture(scope="module")
def hooks():
    if not build.TEST_LIB.exists():
        pytest.fail(f"{build.TEST_LIB} is missing: build it with python tide_b200/build.py")
    lib = ctypes.CDLL(str(build.TEST_LIB))
    capi.declare(lib)
    return lib


def _with_canary(n, H, dtype, fill):
    t = torch.full((n + CANARY_ROWS, H), fill, dtype=dtype, device=DEV)
    return t


def test_split_timeout_is_reported_not_hung(hooks):
    """tide_batch_compact (SIMT partition, 128-row tiles) with tile 3 silent."""
    n, H = 128 * 12 + 5, 64
    assert n > 128 * (build.TEST_TILE + 1)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(n, H, generator=g).to(DEV)
    mask = (torch.rand(n, generator=g) < 0.4).to(torch.int32).to(DEV)
    comp = _with_canary(n, H, torch.float32, 7.0)
    exd = _with_canary(n, H, torch.float32, 7.0)
    ci = torch.full((n + CANARY_ROWS,), -9, dtype=torch.int32, device=DEV)
    ei = torch.full((n + CANARY_ROWS,), -9, dtype=torch.int32, device=DEV)
    nr = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    wsz = hooks.tide_batch_compact_workspace_size(n)
    ws = torch.empty(wsz, dtype=torch.uint8, device=DEV)
    t0 = time.perf_counter()
    rc = hooks.tide_batch_compact(capi.DTYPE_F32, ptr(x), ptr(mask), ptr(comp), ptr(exd), ptr(ci),
                                  ptr(ei), ptr(nr), n, H, ptr(ws), wsz, ptr(err), stream())
    capi.check(hooks, rc, "tide_batch_compact (test build)")
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30.0
    assert int(err.item()) & capi.DEVERR_TIMEOUT
    assert torch.all(comp[n:] == 7.0) and torch.all(exd[n:] == 7.0)
    assert torch.all(ci[n:] == -9) and torch.all(ei[n:] == -9)
    # the context is intact: the product library gives the exact split
    lib = _native.lib()
    err.zero_()
    rc = lib.tide_batch_compact(capi.DTYPE_F32, ptr(x), ptr(mask), ptr(comp), ptr(exd), ptr(ci),
                                ptr(ei), ptr(nr), n, H, ptr(ws), wsz, ptr(err), stream())
    capi.check(lib, rc, "tide_batch_compact")
    torch.cuda.synchronize()
    keep = np.nonzero(mask.cpu().numpy() == 0)[0]
    assert int(err.item()) == 0 and int(nr.item()) == len(keep)
    assert np.array_equal(ci[: len(keep)].cpu().numpy(), keep)
    assert torch.equal(comp[: len(keep)], x[torch.from_numpy(keep).to(DEV)])


@pytest.mark.parametrize("H,path", [(4096, capi.PATH_TC_SPLIT), (4096, capi.PATH_TC),
                                    (768, capi.PATH_TC), (2048, capi.PATH_TC)])
def test_checkpoint_timeout_is_reported_not_hung(hooks, H, path):
    """tide_checkpoint with tile 3 silent: the bulk mover (32-row tiles, one
    look-back thread, abort and drain), and the fused cluster kernel (64-row
    tiles; one look-back thread with 8 CTAs per cluster at H = 4096, the
    warp-wide look-back with 2 and 4 at H = 768 and 2048)."""
    n = 1024
    g = torch.Generator().manual_seed(H + path)
    x = torch.randn(n, H, generator=g).to(torch.bfloat16).to(DEV)
    nw = torch.ones(H, device=DEV)
    down = 0.02 * torch.randn(128, H, generator=g)
    up = 0.02 * torch.randn(1, 128, generator=g)
    norm = oracle_norm("rms", nw, None, 1e-5)
    z = O.router_logits(O.final_norm(O.to_f32(storage_np(x), O.BF16), norm), down.numpy(), up.numpy())
    from tide_b200 import workloads

    bias = workloads.bias_for_exit_fraction(z, 0.3, 0.85)
    out = _with_canary(n, H, torch.bfloat16, 3.0)
    ck = Checkpoint(x, "rms", nw, None, 1e-5, down.to(DEV), up.to(DEV), bias, 0.85,
                    out_buffer=out[:n], path=path)
    ck.compact_out = _with_canary(n, H, torch.bfloat16, 5.0)
    ck.args.compact_out = ptr(ck.compact_out)
    assert ck.path() == path
    t0 = time.perf_counter()
    rc = hooks.tide_checkpoint(ctypes.byref(ck.args), stream())
    capi.check(hooks, rc, "tide_checkpoint (test build)")
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30.0
    assert int(ck.error_word.item()) & capi.DEVERR_TIMEOUT
    assert torch.all(out[n:] == 3.0) and torch.all(ck.compact_out[n:] == 5.0)
    # the product library, same arguments, same context: exact again
    ck.error_word.zero_()
    ck()
    torch.cuda.synchronize()
    assert int(ck.error_word.item()) == 0
    res = O.checkpoint(storage_np(x), O.BF16, norm, down.numpy(), up.numpy(), bias, 0.85)
    s = ck.scores_out.cpu().numpy()
    ours = s > 0.85
    assert np.array_equal(ours, res["exits"]) or np.all(np.abs(res["scores"][ours != res["exits"]] - 0.85) <= 1e-2)
    keep = np.nonzero(~ours)[0]
    assert np.array_equal(ck.positions_out.cpu().numpy()[: len(keep)], keep)
    assert np.array_equal(storage_np(ck.compact_out)[: len(keep)], storage_np(x)[keep])
    assert torch.all(out[n:] == 3.0) and torch.all(ck.compact_out[n:] == 5.0)
