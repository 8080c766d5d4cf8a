"""Data-parallel exchange on 2 CPU ranks (gloo): the backward's collectives reproduce
the single-process accumulators and maxima exactly.

Runs ``ecoint8.parallel.reduce_backward`` with int32/int64 CPU tensors; the
max-abs reduction is supplied by the oracle (the library's reduction is CUDA
only), so this checks the host logic and the collective arithmetic, not kernels.
"""

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import fixedpoint as ofp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from ecoint8 import parallel

        parallel.init()
        gen = torch.Generator().manual_seed(42)
        B, out, inn = 64, 10, 24
        g = torch.randint(-127, 128, (B, out), dtype=torch.int8, generator=gen)
        x = torch.randint(-127, 128, (B, inn), dtype=torch.int8, generator=gen)
        w = torch.randint(-127, 128, (out, inn), dtype=torch.int8, generator=gen)
        lo, hi = rank * B // world, (rank + 1) * B // world
        gl, xl = g[lo:hi].numpy(), x[lo:hi].numpy()
        dw = torch.from_numpy(ofp.int_mm(gl.T, xl))
        dx = ofp.int_mm(gl, w.numpy())
        gb = torch.from_numpy(gl.astype(np.int64).sum(0))
        amax = torch.tensor([0, ofp.int_amax(dx)], dtype=torch.int32)
        a_dw, a_dx, dw, gb = parallel.reduce_backward(
            dw, gb, amax, amax_fn=lambda t: torch.tensor([ofp.int_amax(t.numpy())]))
        full_dw = ofp.int_mm(g.numpy().T, x.numpy())
        ok = (np.array_equal(dw.numpy(), full_dw) and a_dw == ofp.int_amax(full_dw)
              and a_dx == ofp.int_amax(ofp.int_mm(g.numpy(), w.numpy()))
              and np.array_equal(gb.numpy(), g.numpy().astype(np.int64).sum(0))
              and parallel.allreduce_max_int(rank * 7 + 1, device=torch.device("cpu")) == (world - 1) * 7 + 1)
        q.put((rank, ok))
        parallel.shutdown()
    finally:
        dist.destroy_process_group()


def test_two_rank_backward_exchange_is_exact():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(res) == [(0, True), (1, True)]


def _gather_worker(rank, world, port, q):
    """The "gather" exchange: all-gathered inputs and all-to-all dY columns give each
    rank exactly its rows of the full-batch dW and of the bias sums."""
    import types

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        from ecoint8 import parallel

        parallel.init(dw_exchange="gather")
        gen = torch.Generator().manual_seed(5)
        b, out, inn = 16, 8 * world, 20
        g = torch.randint(-127, 128, (b * world, out), dtype=torch.int8, generator=gen)
        x = torch.randint(-127, 128, (b * world, inn), dtype=torch.int8, generator=gen)
        layer = types.SimpleNamespace(out_features=out)
        ok = parallel.gathers_input(layer) and parallel.exchange() == "gather"
        parallel.gather_input(layer, x[rank * b:(rank + 1) * b])
        # the column blocks of this rank's dY (a CUDA copy in the library; built here on the CPU)
        mine = g[rank * b:(rank + 1) * b]
        dy_cols, a2a = parallel.exchange_blocks(mine.reshape(b, world, out // world).transpose(0, 1).contiguous())
        full, work = layer._input_gather
        a2a.wait()
        work.wait()
        lo, hi = parallel.shard_rows(out)
        rows = ofp.int_mm(dy_cols.numpy().T, full.numpy())
        ok &= np.array_equal(rows, ofp.int_mm(g.numpy().T, x.numpy())[lo:hi])
        ok &= np.array_equal(dy_cols.numpy().astype(np.int64).sum(0), g.numpy()[:, lo:hi].astype(np.int64).sum(0))
        q.put((rank, bool(ok)))
        parallel.shutdown()
    finally:
        dist.destroy_process_group()


def test_three_rank_gather_exchange_gives_row_shards_of_full_dw():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert sorted(res) == [(0, True), (1, True), (2, True)]
