"""Data-parallel plumbing on CPU ranks (gloo, world size 2): the flat-bucket gradient all-reduce equals the
reference's per-tensor all-reduce, weights broadcast from rank 0, the checksum check catches divergence, and a rank
that fails is seen by the others as an error instead of a hang."""

from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))  # fmt: skip
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))


def _model(seed):
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.Tanh(), torch.nn.Linear(16, 3))


def _worker_allreduce(rank, world, port, q):
    from ebr_b200 import runtime

    _init(rank, world, port)
    try:
        m = _model(100 + rank)  # different weights per rank
        runtime.broadcast_model(m)
        runtime.check_param_sync(m)  # identical after the broadcast
        x = torch.randn(4, 8, generator=torch.Generator().manual_seed(rank))
        m(x).square().sum().backward()
        ref = [p.grad.clone() for p in m.parameters()]
        for g in ref:  # the reference's per-tensor all-reduce
            dist.all_reduce(g)
        n = runtime.allreduce_gradients(list(m.parameters()))
        ok = all(torch.allclose(p.grad, r, atol=1e-6) for p, r in zip(m.parameters(), ref))
        q.put((rank, ok, n))
    finally:
        dist.destroy_process_group()


def _worker_diverge(rank, world, port, q):
    from ebr_b200 import runtime

    _init(rank, world, port)
    try:
        m = _model(5)
        if rank == 1:
            with torch.no_grad():
                next(m.parameters()).add_(1.0)
        try:
            runtime.check_param_sync(m)
            q.put((rank, "no error"))
        except RuntimeError as e:
            q.put((rank, "diverged" if "diverged" in str(e) else str(e)))
    finally:
        dist.destroy_process_group()


def _worker_fail(rank, world, port, q):
    _init(rank, world, port)
    if rank == 1:
        os._exit(3)  # a rank that dies between steps, with nothing in flight
    try:
        dist.all_reduce(torch.ones(1))
        q.put((rank, "completed"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, type(e).__name__))


def _run(target, world=2, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    out = []
    while not q.empty():
        out.append(q.get())
    return sorted(out)


def test_flat_bucket_allreduce_matches_per_tensor():
    res = _run(_worker_allreduce)
    assert len(res) == 2 and all(ok for _, ok, _ in res), res
    assert res[0][2] == 8 * 16 + 16 + 16 * 3 + 3


def test_param_sync_detects_divergence():
    res = _run(_worker_diverge)
    assert res == [(0, "diverged"), (1, "diverged")], res


def test_dead_rank_is_an_error_not_a_hang():
    res = _run(_worker_fail)
    assert len(res) == 1 and res[0][0] == 0 and res[0][1] != "completed", res
