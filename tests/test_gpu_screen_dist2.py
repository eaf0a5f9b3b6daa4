"""g4_head_screen_dist across two GPUs: two processes, one NCCL communicator of the library, each
rank holding half of a 32,768 x 2,048 head.  Only rank 0 is given the hidden rows (the call
broadcasts them).  The winners must equal the single-device screen's over the whole head (itself
pinned to the oracle by test_gpu_head.py) on the survivor path, the per-shard fallback path and
planted rows on either side of the shard boundary, eagerly and replayed from a CUDA graph that
records the call.  NVLS is off (NCCL_NVLS_ENABLE=0).  Runs only where two GPUs are visible."""
import json
import pathlib
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

N, K, M = 32768, 2048, 4
TESTS = pathlib.Path(__file__).resolve().parent


def _cases(E, rng):
    from oracle_lib import bf16_to_f32
    out = []
    rnd = (rng.standard_normal((M, K), dtype=np.float32) / np.float32(np.sqrt(K))).astype(np.float32)
    out.append(("random", rnd))
    rows = [5, N // 2 - 1, N // 2, N - 3]  # both sides of the boundary between the two shards
    H = []
    for j in rows:
        w = bf16_to_f32(E[j])
        u = w / np.float32(np.linalg.norm(w))
        noise = rng.standard_normal(K, dtype=np.float32) / np.float32(np.sqrt(K))
        H.append((np.float32(24.0) * u + np.float32(8.0) * noise).astype(np.float32))
    out.append(("planted", np.stack(H)))
    return out


def _worker(rank, world, port, outfile):
    import datetime
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, str(TESTS))
    import torch
    import torch.distributed as dist
    from g4pkg import g4
    from oracle_lib import bf16_bits
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=90),
                            device_id=torch.device("cuda", rank))
    g4.device_init()
    rng = np.random.default_rng(2048 * 16)
    E = bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    n_loc = N // world
    Ed = torch.from_numpy(E.view(np.int16)).cuda()
    shards = {lim: g4.ScreenShard(Ed[rank * n_loc:(rank + 1) * n_loc].contiguous(), rank * n_loc, lim=lim, M=M)
              for lim in (30000, 2048)}
    full = None
    if rank == 0:
        full = (g4.screen_build(Ed), g4.PackedHead(Ed))
    del Ed
    comm = g4.NcclComm(dist)
    results = {}
    try:
        for name, Hn in _cases(E, rng):
            for lim, shard in shards.items():
                Hd = torch.from_numpy(Hn).cuda() if rank == 0 else torch.zeros(M, K, dtype=torch.float32, device="cuda")
                idx = g4.screen_dist_native(shard, Hd, comm).cpu().numpy().tolist()
                out = torch.full((M,), -7, dtype=torch.int32, device="cuda")
                Hg = torch.from_numpy(Hn).cuda() if rank == 0 else torch.zeros(M, K, dtype=torch.float32, device="cuda")
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    g4.screen_dist_native(shard, Hg, comm, out=out)
                g.replay()
                torch.cuda.synchronize()
                idx_g = out.cpu().numpy().tolist()
                del g
                if rank == 0:
                    ref, _ = g4.head_screen(full[0], full[1], torch.from_numpy(Hn).cuda())
                    results[f"{name}/{lim}"] = {"dist": idx, "graph": idx_g, "single": ref.cpu().numpy().tolist()}
        status = g4.device_status()
    finally:
        torch.cuda.synchronize()
        comm.close()
        dist.destroy_process_group()
    if rank == 0:
        pathlib.Path(outfile).write_text(json.dumps({"results": results, "status": status}))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def test_native_dist_screen_two_gpus(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    outfile = tmp_path / "dist2.json"
    mp.start_processes(_worker, args=(2, _free_port(), str(outfile)), nprocs=2, join=True, start_method="spawn")
    res = json.loads(outfile.read_text())
    assert res["status"] == 0
    assert len(res["results"]) == 4
    for key, r in res["results"].items():
        assert r["dist"] == r["single"], key
        assert r["graph"] == r["single"], key
    assert res["results"]["planted/30000"]["single"] == [5, N // 2 - 1, N // 2, N - 3]
