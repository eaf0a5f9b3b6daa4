"""The collective skeleton of the vocab-parallel screen (g4.screen_dist) over torch.distributed on
CPU: two gloo ranks, each with a host stand-in for the three device phases over its rows.  Checks
that H is broadcast, that the bound and the candidate max are all-reduced before the phases that
use them, and that the winner is the lowest global index among the rows holding the global max."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from g4pkg import g4  # noqa: E402

M, NR, WORLD = 3, 50, 2


def tables():
    rng = np.random.default_rng(7)
    v = rng.integers(0, 20, size=(M, NR * WORLD)).astype(np.float32)  # candidate values, many ties
    Lr = rng.standard_normal((WORLD, M)).astype(np.float32)
    H = rng.standard_normal((M, 8)).astype(np.float32)
    return v, Lr, H


class HostPhases:
    def __init__(self, rank):
        self.rank = rank
        self.v, self.Lr, self.H = tables()
        self.rows = slice(rank * NR, (rank + 1) * NR)

    def bound(self, H):
        assert np.array_equal(H.numpy(), self.H)  # broadcast before the first phase
        return torch.from_numpy(self.Lr[self.rank].copy())

    def select(self, H, L):
        assert np.array_equal(L.numpy(), self.Lr.max(0))  # all-reduced bound
        return torch.from_numpy(self.v[:, self.rows].max(1).copy())

    def pick(self, gmax):
        assert np.array_equal(gmax.numpy(), self.v.max(1))  # all-reduced candidate max
        out = np.full(M, g4.INT_MAX, np.int32)
        for m in range(M):
            hit = np.nonzero(self.v[m, self.rows] == gmax[m].item())[0]
            if hit.size:
                out[m] = self.rank * NR + hit[0]
        return torch.from_numpy(out)


def _worker(rank, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        v, _, H = tables()
        Ht = torch.from_numpy(H.copy()) if rank == 0 else torch.zeros(M, 8)
        idx = g4.screen_dist(HostPhases(rank), Ht, dist)
        q.put((rank, idx.numpy().tolist()))
    finally:
        dist.destroy_process_group()


def test_screen_dist_two_gloo_ranks():
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = dict(q.get(timeout=10) for _ in range(WORLD))
    v, _, _ = tables()
    want = [int(np.nonzero(v[m] == v[m].max())[0][0]) for m in range(M)]
    assert got[0] == want and got[1] == want
