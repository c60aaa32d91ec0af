"""Multi-rank host logic on CPU (gloo, world_size 2).

The per-shard compute is the NumPy oracle (the CUDA kernels need a GPU); what
is tested is the partition and the reductions: batch-sharded parameter
gradients summed by one all-reduce, and channel-sharded scans whose replicated
B / C gradients are summed across ranks, both equal to the unsharded gradients.
A rank that fails is reported on the host without hanging the others.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import selectssm_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _inputs():
    inp = O.make_scan_inputs(4, 24, 16, 16, seed=7)
    inp["bias"] = np.linspace(-0.3, 0.3, 16)
    return inp


def _grads(inp, sl_b=slice(None), sl_c=slice(None)):
    kw = dict(D=inp["D"][sl_c], z=inp["z"][sl_b][:, :, sl_c], delta_bias=inp["bias"][sl_c], delta_softplus=True)
    return O.selective_scan_bwd(inp["u"][sl_b][:, :, sl_c], inp["delta"][sl_b][:, :, sl_c], inp["A"][sl_c],
                                inp["B"][sl_b], inp["C"][sl_b], inp["dout"][sl_b][:, :, sl_c], **kw)


def _batch_worker(rank, world, port, q):
    try:
        from selectssm_b200.parallel import allreduce_grads, shard_range
        _init(rank, world, port)
        inp = _inputs()
        s, e = shard_range(4, rank, world)
        g = _grads(inp, sl_b=slice(s, e))
        params = [torch.nn.Parameter(torch.zeros(16, 16, dtype=torch.float64)),
                  torch.nn.Parameter(torch.zeros(16, dtype=torch.float64)),
                  torch.nn.Parameter(torch.zeros(16, dtype=torch.float64))]
        for p, k in zip(params, ("dA", "dD", "ddelta_bias")):
            p.grad = torch.from_numpy(g[k].copy())
        allreduce_grads(params)
        sync = [p.grad.numpy().copy() for p in params]
        # the asynchronous form writes the same sums into the gradients captured at the call
        grads = [torch.from_numpy(g[k].copy()) for k in ("dA", "dD", "ddelta_bias")]
        for p, gr in zip(params, grads):
            p.grad = gr
        handle = allreduce_grads(params, async_op=True)
        for p in params:
            p.grad = None  # the caller may move on before waiting
        handle.wait()
        assert all(np.array_equal(a, b.numpy()) for a, b in zip(sync, grads))
        q.put((rank, sync))
        dist.destroy_process_group()
    except Exception as ex:  # pragma: no cover - reported to the parent
        q.put((rank, repr(ex)))


def _channel_worker(rank, world, port, q):
    try:
        from selectssm_b200.parallel import replicated_bc, shard_channels
        _init(rank, world, port)
        inp = _inputs()
        c = shard_channels(torch.arange(16), rank, world)
        sl_c = slice(int(c[0]), int(c[-1]) + 1)
        g = _grads(inp, sl_c=sl_c)
        # the autograd node sums the B / C gradients of the channel shards
        Bt = torch.from_numpy(inp["B"]).requires_grad_()
        Ct = torch.from_numpy(inp["C"]).requires_grad_()
        Br, Cr = replicated_bc(Bt, Ct)
        (Br * torch.from_numpy(g["dB"])).sum().backward(retain_graph=True)
        (Cr * torch.from_numpy(g["dC"])).sum().backward()
        q.put((rank, (Bt.grad.numpy(), Ct.grad.numpy(), sl_c.start, sl_c.stop, g["dA"])))
        dist.destroy_process_group()
    except Exception as ex:  # pragma: no cover
        q.put((rank, repr(ex)))


def _failing_worker(rank, world, port, q):
    _init(rank, world, port)
    if rank == 1:
        q.put((rank, "failed"))
        raise SystemExit(3)  # leaves before the collective
    try:
        t = torch.ones(4)
        work = dist.all_reduce(t, async_op=True)
        done = work.wait(timeout=__import__("datetime").timedelta(seconds=3))
        q.put((rank, "completed" if done else "timeout"))
    except Exception as ex:
        q.put((rank, "error: " + type(ex).__name__))


def _run(worker, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, v = q.get(timeout=timeout)
        out[r] = v
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out


def test_batch_sharded_param_grads_allreduce():
    out = _run(_batch_worker)
    full = _grads(_inputs())
    for r in (0, 1):
        assert not isinstance(out[r], str), out[r]
        for got, k in zip(out[r], ("dA", "dD", "ddelta_bias")):
            np.testing.assert_allclose(got, full[k], rtol=1e-10, atol=1e-12)


def test_channel_sharded_bc_grads_summed():
    out = _run(_channel_worker)
    full = _grads(_inputs())
    for r in (0, 1):
        assert not isinstance(out[r], str), out[r]
        dB, dC, s, e, dA = out[r]
        np.testing.assert_allclose(dB, full["dB"], rtol=1e-10, atol=1e-12)
        np.testing.assert_allclose(dC, full["dC"], rtol=1e-10, atol=1e-12)
        np.testing.assert_allclose(dA, full["dA"][s:e], rtol=1e-10, atol=1e-12)   # per channel, local


def test_shard_ranges_cover_everything():
    from selectssm_b200.parallel import shard_range
    for n in (0, 1, 7, 8, 1536):
        for w in (1, 2, 3, 8):
            spans = [shard_range(n, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


@pytest.mark.timeout(120)
def test_dead_rank_is_seen_on_the_host():
    """A rank that exits before a collective: the survivor's bounded wait ends
    with an error or timeout instead of hanging."""
    out = _run(_failing_worker, timeout=90)
    assert out[1] == "failed"
    assert out[0] in ("timeout",) or out[0].startswith("error")
