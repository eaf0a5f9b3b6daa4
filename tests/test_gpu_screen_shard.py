"""Vocab-parallel head screen (configs[2]'s sharded mode) on one GPU: G shards of the head's rows
run the three device phases with the reductions done in this process; the winners must equal the
single-device screen's (itself pinned to the oracle by test_gpu_head.py), on the fallback path, on
the survivor path and across shard boundaries.  The collective skeleton over torch.distributed is
covered on CPU by test_screen_dist.py."""
import numpy as np
import pytest

from oracle_lib import bf16_bits, bf16_to_f32

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

N, K = 32768, 2048


@pytest.fixture(scope="module")
def head_and_shards():
    g4.device_init()
    rng = np.random.default_rng(32768)
    E = bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    Ed = torch.from_numpy(E.view(np.int16)).cuda()
    head = g4.PackedHead(Ed)
    screen = g4.screen_build(Ed)
    shards = {}
    for G, lim in ((2, 30000), (4, 30000), (4, 2048)):
        bounds = np.linspace(0, N, G + 1).astype(int)
        shards[(G, lim)] = [g4.ScreenShard(Ed[bounds[i]:bounds[i + 1]], bounds[i], lim=lim) for i in range(G)]
    torch.cuda.synchronize()
    return E, head, screen, shards, rng


def planted(E, rows, rng, a=24.0, b=8.0):
    H = []
    for j in rows:
        w = bf16_to_f32(E[j])
        u = w / np.float32(np.linalg.norm(w))
        noise = rng.standard_normal(K, dtype=np.float32) / np.float32(np.sqrt(K))
        H.append((np.float32(a) * u + np.float32(b) * noise).astype(np.float32))
    return np.stack(H)


@pytest.mark.parametrize("key", [(2, 30000), (4, 30000), (4, 2048)])
def test_sharded_random_rows_match_single_device(head_and_shards, key):
    """configs[2]'s h ~ N(0,1)/sqrt(K): the single device falls back (every row survives); shards of
    16,384 or 8,192 rows keep all of them below lim=30000 (rescoring path) or overflow lim=2048
    (per-shard fallback).  Same winners either way."""
    E, head, screen, shards, rng = head_and_shards
    H = torch.from_numpy((rng.standard_normal((4, K), dtype=np.float32) / np.float32(np.sqrt(K))).astype(np.float32)).cuda()
    idx_ref, ns_ref = g4.head_screen(screen, head, H)
    idx, ns = g4.screen_sharded(shards[key], H)
    assert list(idx.cpu().numpy()) == list(idx_ref.cpu().numpy())
    ns = ns.cpu().numpy()
    if key[1] == 2048:
        assert (ns == -1).all()  # every shard fell back
    else:
        assert (ns == N // key[0]).all()  # every row of every shard survived and was rescored


@pytest.mark.parametrize("key", [(2, 30000), (4, 30000)])
def test_sharded_planted_winners(head_and_shards, key):
    """Planted hidden states: winners in different shards (global indices across the boundaries),
    few survivors; same winners as the single device."""
    E, head, screen, shards, rng = head_and_shards
    rows = [5, 16383, 16384, 32767]
    H = torch.from_numpy(planted(E, rows, rng)).cuda()
    idx_ref, _ = g4.head_screen(screen, head, H)
    idx, ns = g4.screen_sharded(shards[key], H)
    assert list(idx.cpu().numpy()) == list(idx_ref.cpu().numpy()) == rows
    assert (ns.cpu().numpy() >= 0).all()


def test_native_dist_screen_one_rank_matches_single_device():
    """g4_head_screen_dist (broadcast, three phases, three all-reduces on the stream) over a
    one-rank NCCL communicator gives the single-device screen's winners, eagerly and replayed from a
    CUDA graph that records the whole call."""
    rng = np.random.default_rng(77)
    N, K = 32768, 2048
    E = bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    Ed = torch.from_numpy(E.view(np.int16)).cuda()
    shard = g4.ScreenShard(Ed, 0, lim=30000, M=4)
    H = torch.from_numpy((rng.standard_normal((4, K), dtype=np.float32) / np.float32(45.0)).astype(np.float32)).cuda()
    ref, _ = g4.head_screen(shard.screen, shard.head, H.clone())
    comm = g4.NcclComm()
    try:
        idx = g4.screen_dist_native(shard, H, comm)
        assert list(idx.cpu().numpy()) == list(ref.cpu().numpy())
        out = torch.empty(4, dtype=torch.int32, device="cuda")
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            g4.screen_dist_native(shard, H, comm, out=out)
        g.replay()
        torch.cuda.synchronize()
        assert list(out.cpu().numpy()) == list(ref.cpu().numpy())
        del g
    finally:
        comm.close()
    assert g4.device_status() == 0
