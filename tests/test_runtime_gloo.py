"""Data-parallel plumbing on CPU ranks (gloo, world size 2): the flat-bucket and the overlapped bucketed gradient
all-reduces equal the reference's per-tensor all-reduce, a parameter no rank produced a gradient for stays without
one (as the reference skips it), weights broadcast from rank 0, the checksum check catches divergence, and a rank
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


class _TwoHeads(torch.nn.Module):
    """A trunk and two heads; ``head_b`` is used only by rank 1, ``unused`` by no rank."""

    def __init__(self):
        super().__init__()
        torch.manual_seed(7)
        self.unused = torch.nn.Linear(16, 3)  # registered first: it lands in the last bucket
        self.trunk = torch.nn.Linear(8, 16)
        self.head_a = torch.nn.Linear(16, 3)
        self.head_b = torch.nn.Linear(16, 3)

    def forward(self, x, use_b):
        h = torch.tanh(self.trunk(x))
        y = self.head_a(h).square().sum()
        return y + self.head_b(h).square().sum() if use_b else y


def _worker_buckets(rank, world, port, q):
    from ebr_b200 import runtime

    _init(rank, world, port)
    try:
        results = {}
        x = torch.randn(4, 8, generator=torch.Generator().manual_seed(rank))
        # The reference's result: per-tensor SUM, a missing gradient counting as zero (from a plain backward).
        m = _TwoHeads()
        m(x, use_b=rank == 1).backward()
        exp = []
        for p in m.parameters():
            t = torch.zeros_like(p) if p.grad is None else p.grad.clone()
            dist.all_reduce(t)
            exp.append(t)
        for mode in ("flat", "buckets"):
            m = _TwoHeads()
            buckets = runtime.GradientBuckets(list(m.parameters()), bucket_mb=0.0003) if mode == "buckets" else None
            if buckets:
                buckets.start()  # no other collective may run between start() and finish()
            m(x, use_b=rank == 1).backward()
            if buckets:
                buckets.finish()
                results["early"] = buckets.launched_early
                results["nbuckets"] = len(buckets.buckets)
            else:
                runtime.allreduce_gradients(list(m.parameters()))
            for (n, p), e in zip(m.named_parameters(), exp):
                if n.startswith("unused"):
                    results[f"{mode}:{n}"] = p.grad is None
                else:
                    results[f"{mode}:{n}"] = p.grad is not None and torch.allclose(p.grad, e, atol=1e-6)
        q.put((rank, results))
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


def test_bucketed_overlapped_allreduce_and_missing_gradients():
    """Both all-reduce forms give the per-tensor sums; a gradient only rank 1 has is summed onto both ranks; a
    parameter no rank used keeps grad None; with tiny buckets several are launched from the hooks mid-backward."""
    res = _run(_worker_buckets)
    assert len(res) == 2, res
    for rank, r in res:
        bad = {k: v for k, v in r.items() if k not in ("early", "nbuckets") and not v}
        assert not bad, (rank, bad)
        assert r["nbuckets"] > 2, r
        if rank == 1:  # every gradient but the unused one: buckets go out during the backward
            assert r["early"] >= 1, r
