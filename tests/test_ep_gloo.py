"""Expert-parallel host logic on CPU: two gloo ranks, each holding half of the routed experts, against the
single-process layer. The expert computation is a fake (a fixed function per expert id) so the test checks the
sharding, dispatch, return and shared-expert handling, not the kernels (the GPU tests cover those)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from glmx import ep

H, E, K = 64, 8, 3


def f_expert(e, x):
    return torch.sin(x * (0.1 * (e + 1))) + 0.01 * e


class FakeShard:
    """A shard's layer over LOCAL ids: 0..n-1 are global experts first..first+n-1, id n is the shared expert."""

    def __init__(self, first, n):
        self.first, self.n = first, n
        self.device = torch.device("cpu")

    def forward(self, x, sel, w, mode=2, out=None, accumulate=False):
        y = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32)
        for t in range(x.shape[0]):
            for j in range(sel.shape[1]):
                e = int(sel[t, j])
                if 0 <= e <= self.n:
                    y[t] += float(w[t, j]) * f_expert(99 if e == self.n else e + self.first, x[t].float())
        if accumulate:
            out += y
        else:
            out.copy_(y)
        return out


def inputs(rank, B):
    g = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(B, H, generator=g)
    sel = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(B)]).int()
    sel[0, 1] = -1
    w = torch.rand(B, K, generator=g)
    return x, sel, w


def reference(x, sel, w):
    out = torch.zeros(x.shape[0], H)
    for t in range(x.shape[0]):
        for j in range(K):
            if sel[t, j] >= 0:
                out[t] += float(w[t, j]) * f_expert(int(sel[t, j]), x[t])
        out[t] += f_expert(99, x[t])
    return out


def _worker(rank, world, port, B, q, exchange):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        first, n = ep.shard_range(E, world, rank)
        layer = ep.ExpertParallelLayer(FakeShard(first, n), first, n, has_shared=True, E=E, exchange=exchange)
        x, sel, w = inputs(rank, B)
        out = layer.forward(x, sel, w)
        err = float((out - reference(x, sel, w)).abs().max())
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,exchange", [(2, "a2a"), (2, "allgather"), (4, "a2a")])
def test_ep_ranks_match_single_process(world, exchange):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 5, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert set(res) == set(range(world))
    assert all(e < 1e-5 for e in res.values()), res


def test_shard_range():
    assert ep.shard_range(288, 8, 3) == (108, 36)
    assert ep.shard_range(288, 1, 0) == (0, 288)
    with pytest.raises(ValueError):
        ep.shard_range(288, 5, 0)
