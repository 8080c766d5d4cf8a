"""Data parallelism on 2 GPUs reproduces the single-GPU run bit for bit (NCCL),
with every dW exchange (int32 reduce-scatter; gathered inputs + dY all-to-all
through NCCL; the same through the library's NVLink peer stores).

Two ranks split a batch of 96 rows; rank 0 also trains an identical net on the
whole batch on its own.  Both use the same Philox key sequence, so after
several training steps every weight, momentum, bias and momentum scale must
agree exactly.  The fp32 loss boundary is either made deterministic (round-to-nearest
quantization of the gradient on its global scale) or is the fused boundary
(``cross_entropy_grad_i8``: global maximum over the ranks, Philox uniforms on
global rows), so both sides feed the same int8 gradient.  Skipped with fewer
than 2 GPUs.
"""

import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

B, D, H, C = 96, 40, 48, 5


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _net(dev):
    from ecoint8 import I8Linear, I8ReLU, I8Sequential

    torch.manual_seed(0)
    return I8Sequential(I8Linear(D, H), I8ReLU(), I8Linear(H, H), I8ReLU(), I8Linear(H, C)).to(dev)


def _boundary(logits, s_out, y, world):
    """CE grad over the global batch, int8 by round-to-nearest on the global amax."""
    import torch.distributed as dist

    from ecoint8.quant import calc_scale, quantize_symmetric

    lf = (logits.to(torch.float32) * s_out).requires_grad_()
    loss = torch.nn.functional.cross_entropy(lf, y, reduction="sum") / B
    (g,) = torch.autograd.grad(loss, lf)
    amax = g.abs().max().reshape(1)
    if world > 1:
        dist.all_reduce(amax, op=dist.ReduceOp.MAX)
    s = calc_scale(float(amax.item()))
    return quantize_symmetric(g, s, stochastic=False), s


def _train(net, x8, sx, y, world, row_base, gen_seed, steps, fused=False):
    from ecoint8 import I8ECO
    from ecoint8._sr import batch_rows, set_generator
    from ecoint8.quant import cross_entropy_grad_i8

    set_generator(torch.Generator().manual_seed(gen_seed))
    with batch_rows(row_base):
        net.calibrate(x8, sx)  # the accumulator maxima are all-reduced across ranks
        opt = I8ECO(net.int8_layers(), lr=0.3, momentum=0.9)
        for _ in range(steps):
            logits, s_out = net.forward_i8(x8)
            if fused:
                _, g8, sg = cross_entropy_grad_i8(logits, s_out, y, count=B)
            else:
                g8, sg = _boundary(logits, s_out, y, world)
            net.backward_i8(g8, sg)
            opt.step()
            opt.zero_grad()
    set_generator(None)
    return opt


def _worker(rank, port, q):
    import sys

    sys.path[:0] = [os.environ["ECO_PKG"], os.environ["ECO_REPO"]]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import torch.distributed as dist

    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from ecoint8 import parallel
        from ecoint8.quant import quantize_tensor_dynamic

        gen = torch.Generator().manual_seed(7)
        X = torch.randn(B, D, generator=gen) * 2.0
        Y = torch.randint(0, C, (B,), generator=gen)
        X8, sx = quantize_tensor_dynamic(X)  # entry scale of the global batch, identical on both ranks
        lo, hi = rank * B // 2, (rank + 1) * B // 2
        runs = {}
        for exchange, fused in (("reduce", False), ("gather", False), ("peer", False), ("peer", True)):
            parallel.init(dw_exchange=exchange)
            net = _net(dev)
            opt = _train(net, X8[lo:hi].to(dev), sx, Y[lo:hi].to(dev), 2, lo, 123, 4, fused)
            parallel.synchronize(net.int8_layers())  # the last step's row all-gathers
            parallel.gather_momentum(opt)  # momentum rows live on their owner rank
            runs[exchange + ("+fused" if fused else "")] = (net, opt, opt.stats["mean_abs_e"])
            parallel.shutdown()
        if rank == 0:
            res = {}
            for exchange, (net, opt, stats) in runs.items():
                single = _net(dev)
                sopt = _train(single, X8.to(dev), sx, Y.to(dev), 1, 0, 123, 4, exchange.endswith("+fused"))
                ok = all(torch.equal(a.w_i8, b.w_i8) for a, b in zip(net.int8_layers(), single.int8_layers()))
                ok &= all(torch.equal(a.b_acc, b.b_acc) for a, b in zip(net.int8_layers(), single.int8_layers()))
                ok &= all(torch.equal(a, b) for a, b in zip(opt.m_i8, sopt.m_i8))
                ok &= opt.s_m == sopt.s_m
                ok &= stats == sopt.stats["mean_abs_e"]
                res[exchange] = bool(ok)
            q.put(res)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_data_parallel_equals_single_gpu():
    import pathlib

    import torch.multiprocessing as mp

    repo = pathlib.Path(__file__).resolve().parent.parent
    os.environ["ECO_PKG"] = str(repo / "eco-int8-opt_b200")
    os.environ["ECO_REPO"] = str(repo)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    ok = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert ok == {"reduce": True, "gather": True, "peer": True, "peer+fused": True}


# ---------------------------------------------------------------------------- CUDA graphs
GH, GC = 48, 16  # every layer splits into row shards of at least 8 over 2 ranks


def _graph_net(dev):
    from ecoint8 import I8Linear, I8ReLU, I8Sequential

    torch.manual_seed(0)
    return I8Sequential(I8Linear(D, GH), I8ReLU(), I8Linear(GH, GH), I8ReLU(), I8Linear(GH, GC)).to(dev)


def _graph_train(net, x8, sx, y, row_base, steps, graph):
    """``steps`` steps of the fused-boundary loop, eagerly or as one eager step plus
    replays of a captured graph, with a changing learning rate."""
    from ecoint8 import I8ECO
    from ecoint8._sr import batch_rows, set_generator
    from ecoint8.graphs import StepGraph
    from ecoint8.quant import cross_entropy_grad_i8

    set_generator(torch.Generator().manual_seed(321))
    with batch_rows(row_base):
        net.calibrate(x8, sx)
        opt = I8ECO(net.int8_layers(), lr=0.3, momentum=0.9)

        def step():
            logits, s_out = net.forward_i8(x8)
            loss, g8, sg = cross_entropy_grad_i8(logits, s_out, y, count=B)
            net.backward_i8(g8, sg)
            opt.step()
            opt.zero_grad()
            return loss

        g = StepGraph(step, warmup=1) if graph else None
        for t in range(steps):
            opt.set_lr(0.3 - 0.02 * t)
            if g is None:
                step()
            elif t == 0:
                g.capture()
            else:
                g.replay()
    set_generator(None)
    return opt


def _graph_worker(rank, port, q):
    import sys

    sys.path[:0] = [os.environ["ECO_PKG"], os.environ["ECO_REPO"]]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import torch.distributed as dist

    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from ecoint8 import parallel
        from ecoint8.quant import quantize_tensor_dynamic

        gen = torch.Generator().manual_seed(8)
        X = torch.randn(B, D, generator=gen) * 2.0
        Y = torch.randint(0, GC, (B,), generator=gen)
        X8, sx = quantize_tensor_dynamic(X)
        lo, hi = rank * B // 2, (rank + 1) * B // 2
        parallel.init(dw_exchange="peer")
        net = _graph_net(dev)
        opt = _graph_train(net, X8[lo:hi].to(dev), sx, Y[lo:hi].to(dev), lo, 5, graph=True)
        parallel.synchronize(net.int8_layers())
        parallel.gather_momentum(opt)
        stats = opt.stats["mean_abs_e"]
        steps = opt.step_count
        parallel.shutdown()
        if rank == 0:
            single = _graph_net(dev)
            sopt = _graph_train(single, X8.to(dev), sx, Y.to(dev), 0, 5, graph=False)
            ok = all(torch.equal(a.w_i8, b.w_i8) for a, b in zip(net.int8_layers(), single.int8_layers()))
            ok &= all(torch.equal(a.b_acc, b.b_acc) for a, b in zip(net.int8_layers(), single.int8_layers()))
            ok &= all(torch.equal(a, b) for a, b in zip(opt.m_i8, sopt.m_i8))
            ok &= opt.s_m == sopt.s_m
            ok &= stats == sopt.stats["mean_abs_e"]
            ok &= steps == sopt.step_count == 5
            q.put(bool(ok))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_graph_replay_equals_single_gpu():
    """The data-parallel step (peer exchange) captured as a CUDA graph on each rank and
    replayed reproduces the single-GPU eager run bit for bit."""
    import pathlib

    import torch.multiprocessing as mp

    repo = pathlib.Path(__file__).resolve().parent.parent
    os.environ["ECO_PKG"] = str(repo / "eco-int8-opt_b200")
    os.environ["ECO_REPO"] = str(repo)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_graph_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    ok = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert ok
