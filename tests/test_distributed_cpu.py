"""Row sharding + all-gather host logic on CPU: world_size 2 over gloo, with a
dense fp64 stand-in for each rank's tile pass, checked against the full
single-process operator."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashdiffusion_b200.distributed import RowGather, ShardedDMAP, all_shards, shard_rows
from oracle import fd_oracle as O


def test_shard_rows_cover_exactly_once():
    for n in (1, 255, 256, 257, 1000, 200_000):
        for w in (1, 2, 3, 4, 8):
            sh = all_shards(n, w)
            assert sh[0][0] == 0 and sh[-1][1] == n
            for (a, b), (c, _) in zip(sh, sh[1:]):
                assert b == c and a <= b
            sizes = [b - a for a, b in sh]
            assert max(sizes) - min(sizes) <= 256


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, X, beta, alpha, v, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Xt = torch.from_numpy(X)
        Kfull = torch.from_numpy(O.dense_kernel(X, beta))
        a, b = shard_rows(X.shape[0], world, rank)

        def local_apply(V, cs, rs, dt):
            U = torch.ones((Xt.shape[0], 1), dtype=torch.float64) if V is None else V.double().reshape(Xt.shape[0], -1)
            if cs is not None:
                U = U * cs.double()[:, None]
            out = Kfull[a:b] @ U
            if rs is not None:
                out = out * rs.double()[:, None]
            return out.to(dt)

        op = ShardedDMAP(Xt, beta, alpha, local_apply=local_apply).fit()
        mv = op.matvec_device(torch.from_numpy(v))
        blk = op.matvec_device(torch.from_numpy(np.stack([v, 2 * v], 1)))
        out_q.put((rank, op.rscale.double().numpy(), mv.numpy(), blk.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [300, 513])
def test_sharded_dmap_two_ranks_matches_dense(n):
    from tests.golden.make_golden import test_roll
    X = test_roll(n)
    beta, alpha = 1.0, 0.5
    v = np.random.default_rng(0).standard_normal(n)
    M, rs = O.dense_dmap_operator(X, beta, alpha)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, X, beta, alpha, v, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, rscale, mv, blk in res:
        np.testing.assert_allclose(rscale, rs, rtol=1e-5)
        np.testing.assert_allclose(mv, M @ v, rtol=1e-5, atol=1e-7)
        np.testing.assert_allclose(blk[:, 1], 2 * (M @ v), rtol=1e-5, atol=1e-7)
    # replicas hold bit-identical vectors after the gather
    assert np.array_equal(res[0][2], res[1][2])


def test_row_gather_single_rank_is_identity():
    g = RowGather(10, 1)
    x = torch.arange(10.0)
    assert g(x) is x


def _dropout_worker(rank, world, port, out_q):
    import datetime
    import time as _t
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    g = RowGather(600, world)
    a, b = shard_rows(600, world, rank)
    first = g(torch.full((b - a,), float(rank), dtype=torch.float64))   # one good product
    if rank == 1:
        out_q.put((rank, "left", float(first.sum())))
        out_q.close()
        out_q.join_thread()       # the message is out before the process goes
        os._exit(0)               # leaves between products, with nothing in flight
    t0 = _t.perf_counter()
    try:
        g(torch.zeros(b - a, dtype=torch.float64))
        out_q.put((rank, "no error", _t.perf_counter() - t0))
    except Exception as e:    # the collective ends with an error instead of hanging
        out_q.put((rank, type(e).__name__, _t.perf_counter() - t0))


def test_rank_that_leaves_is_detected_by_the_next_gather():
    """Failure detection on the host: a rank exits between products; the other rank's next
    all-gather ends with an error within the process-group timeout instead of hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (what, val)) for r, what, val in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
    assert res[1][0] == "left"
    assert res[0][0] != "no error", res[0]
    assert res[0][1] < 60.0


def _gather_worker(rank, world, port, n, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = RowGather(n, world)
        a, b = g.shards[rank]
        res = []
        for step in range(2):                     # the buffer is reused between gathers
            for dt in (torch.float32, torch.float64):
                slot = g.slot(3, dt, torch.device("cpu"))
                slot.copy_(torch.arange(a, b, dtype=dt)[:, None] * (step + 1) + torch.arange(3, dtype=dt))
                full = g.gather_slot(3, dt, torch.device("cpu")).clone()
                res.append(full.numpy())
        first = g(torch.arange(a, b, dtype=torch.float32))
        second = g(torch.arange(a, b, dtype=torch.float32) * 2)
        out_q.put((rank, res, first.numpy(), second.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [512, 700])          # equal shards (views) and uneven shards (gather-copy)
def test_row_gather_slots_in_place(n):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gather_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    rows = np.arange(n, dtype=np.float64)
    for _, res, first, second in outs:
        k = 0
        for step in range(2):
            for _dt in range(2):
                want = rows[:, None] * (step + 1) + np.arange(3)
                assert np.array_equal(res[k], want)
                k += 1
        assert np.array_equal(first, rows) and np.array_equal(second, 2 * rows)   # no aliasing
