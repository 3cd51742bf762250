"""The multi-rank host logic on CPU: two gloo ranks on 127.0.0.1.

Covers what a multi-GPU run does outside the kernels (the path itself shards
by rows with no exchange): the max over ranks of a timed region, the sum of
per-rank exit counts for global ExitStats, balanced row shards, and a rank
that never joins a collective being detected by the process-group timeout
instead of hanging the others."""
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

from tide_b200.dist import shard_range


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _env(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))


def _collectives(rank: int, world: int, port: int, q) -> None:
    _env(rank, world, port)
    import torch.distributed as dist

    from tide_b200 import dist as td
    from tide_b200.scheduler import ExitStats

    w, r, _ = td.init("gloo", timeout_s=60)
    out = {"world": w, "rank": r}
    out["max"] = td.max_over_ranks(w, 1.5 + r)
    out["sum"] = td.sum_counts(w, torch.tensor([[10 + r, 1], [5, r]], dtype=torch.int32)).tolist()
    st = ExitStats(total_tokens=100 * (r + 1), exits_per_layer={4: r + 1, 8: 2},
                   remaining_tokens=100 * (r + 1) - (r + 3))
    g = td.global_stats(w, st)
    out["stats"] = (g.total_tokens, dict(g.exits_per_layer), g.remaining_tokens, g.summary())
    # ranks that recorded different layers (a layer with no exit on a rank is
    # not recorded there): summed over the full router layer list
    st2 = ExitStats(total_tokens=10, exits_per_layer={8: 3} if r == 0 else {8: 1, 12: 2},
                    remaining_tokens=7 if r == 0 else 7)
    g2 = td.global_stats(w, st2, layers=[8, 12, 16])
    out["stats_uneven"] = (g2.total_tokens, dict(g2.exits_per_layer), g2.remaining_tokens)
    rows = torch.full((3, 4), float(r), dtype=torch.bfloat16)
    out["rows"] = td.all_gather_rows(w, rows).float().tolist()
    out["gcounts"] = td.all_gather_counts(w, torch.tensor([[r, 2 * r]], dtype=torch.int32)).tolist()
    td.barrier(w)
    dist.destroy_process_group()
    q.put(out)


def _put_and_exit(q, item) -> None:
    """Deliver `item` before the process ends without any cleanup (the queue's
    feeder thread is flushed first)."""
    q.put(item)
    q.close()
    q.join_thread()
    os._exit(0)


def _dead_peer(rank: int, world: int, port: int, q, ready) -> None:
    _env(rank, world, port)
    import torch.distributed as dist

    from tide_b200 import dist as td

    # both ranks have imported torch before the short-timeout rendezvous (a
    # cold first import can take far longer than the 3 s timeout)
    ready.wait(timeout=300)
    w, r, _ = td.init("gloo", timeout_s=3)
    if r == 1:
        # leaves between steps, never joins the next collective
        _put_and_exit(q, {"rank": 1, "left": True})
    t0 = time.time()
    try:
        td.max_over_ranks(w, 1.0)
        item = {"rank": 0, "raised": False}
    except Exception as e:  # the timeout or the closed peer connection
        item = {"rank": 0, "raised": True, "after_s": time.time() - t0, "err": type(e).__name__}
    _put_and_exit(q, item)


def _run(target, world=2, timeout=120, sync=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    extra = (ctx.Barrier(world),) if sync else ()
    ps = [ctx.Process(target=target, args=(r, world, port, q) + extra) for r in range(world)]
    for p in ps:
        p.start()
    res = []
    deadline = time.time() + timeout
    while len(res) < world and time.time() < deadline:
        try:
            res.append(q.get(timeout=1))
        except Exception:
            if all(not p.is_alive() for p in ps) and q.empty():
                break
    for p in ps:
        p.join(timeout=max(1, deadline - time.time()))
        if p.is_alive():
            p.kill()
    return sorted(res, key=lambda d: d["rank"]), [p.exitcode for p in ps]


def test_two_rank_collectives():
    res, codes = _run(_collectives)
    assert codes == [0, 0], codes
    assert [d["rank"] for d in res] == [0, 1]
    for d in res:
        assert d["world"] == 2
        assert d["max"] == 2.5
        assert d["sum"] == [[21, 2], [10, 1]]
        total, exits, remaining, text = d["stats"]
        assert total == 300 and exits == {4: 3, 8: 4} and remaining == 300 - 7
        assert text.startswith("Total tokens: 300, Exited: 7")
        assert d["stats_uneven"] == (20, {8: 4, 12: 2}, 14)
        assert d["rows"] == [[0.0] * 4] * 3 + [[1.0] * 4] * 3
        assert d["gcounts"] == [[[0, 0]], [[1, 2]]]


def test_rank_that_never_joins_is_detected():
    res, _ = _run(_dead_peer, timeout=400, sync=True)
    r0 = [d for d in res if d["rank"] == 0]
    assert r0 and r0[0]["raised"], res
    assert r0[0]["after_s"] < 60


@pytest.mark.parametrize("n", [0, 1, 7, 148, 32768, 1 << 20])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_range_tiles_rows(n, world):
    spans = [shard_range(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    for (a, b), (c, _) in zip(spans, spans[1:]):
        assert b == c
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(n, world, world)
