"""Benchmark driver (one JSON line on stdout from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl g4|reference] [--workload decode|gemv|head]

Workloads:
  decode (default) configs[4]: greedy speculative decode of the synthetic E2B model (30 layers,
         hidden 2048, 262,144-token tied head, int4 W4G32 weights with int8 activations, 4-layer
         MTP drafter, k = 3, prompt lookup n-gram 2) after a 6,841-token prompt (Zipf(1.1) with
         copied spans).  A step is one decode round: drafts (prompt lookup or MTP) -> one verify
         pass over the k+1 rows -> greedy acceptance.  Value = committed tokens / device time of
         the timed rounds; every verify pass streams ~1.37 GB (all weights + KV + the int4 head
         screen), far above the 126 MB L2.
  gemv   configs[0]: one W4G32 GEMV, 8192 x 2048 int4 weights, x ~ N(0,1), M = 1.  A step is one
         GEMV over the next of 64 rotating weight copies (604 MB, > 4x the 126 MB L2), so every
         step streams its weights from HBM.

The g4 arm times the sm_100a kernels with CUDA events on the launching stream (inputs resident
in HBM); its `e2e` key is the same workload through the C ABI from host buffers, host<->device
copies inside every step.  `--impl reference` times the reference's CPU path on the host's cores
for the same workload (decode: the oracle's restatement of the engine, whose reference sources do
not build without their model files; gemv: the reference's own AVX2 kernels from oracle/_ref).
Under torchrun every rank runs its own replica (no data-path collective); the value is the sum
over ranks and the time the max over ranks.
"""
import argparse
import ctypes
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

# independent request streams run one CUDA stream each: give the device enough hardware queues that
# up to 32 of them do not alias onto the default 8 (read when CUDA initialises)
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gemma4-e2b-laptop-cpu_b200"))
sys.path.insert(0, str(ROOT / "tests"))

METRIC = "greedy spec-decode tok/s @6.8k ctx; W4G32 GEMV HBM GB/s vs B200 peak"
FALLBACK_HBM_GBS = 6650.0


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>.md, or None."""
    p = ROOT / "profiles" / f"{name}.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi samples (every 200 ms) during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        self.out = tempfile.TemporaryFile(mode="w+")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        t0 = time.perf_counter()  # the sampler's start-up can take a while: wait for its first sample
        while time.perf_counter() - t0 < 5.0 and self.proc.poll() is None:
            self.out.flush()
            if os.fstat(self.out.fileno()).st_size > 0:
                break
            time.sleep(0.05)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if self.proc is None:
            return None
        self.out.seek(0)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- distributed
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def init_pg(world, local):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    if world > 1 and not dist.is_initialized():
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    return dist if world > 1 else None


def max_over_ranks(x, dist_):
    if dist_ is None:
        return x
    import torch
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist_.all_reduce(t, op=dist_.ReduceOp.MAX)
    return float(t.item())


def barrier(dist_):
    if dist_ is not None:
        dist_.barrier()


# --------------------------------------------------------------------------- gemv workload
N_CFG0, K_CFG0, NCOPY = 8192, 2048, 64
GEMV_BYTES = N_CFG0 * K_CFG0 // 2 + N_CFG0 * (K_CFG0 // 32) * 2 + K_CFG0 * 4 + N_CFG0 * 4  # 9,478,144


def gemv_inputs(seed=0):
    from oracle_lib import w4g32_weights
    rng = np.random.default_rng(seed)
    W, S = w4g32_weights(rng, N_CFG0, K_CFG0)
    X = rng.standard_normal((1, K_CFG0), dtype=np.float32)
    return W, S, X


def run_gemv_g4(args, world, rank, local, dist_=None, steps=None, warmup=None):
    import torch
    import g4
    torch.cuda.set_device(local)
    if dist_ is None:
        dist_ = init_pg(world, local)
    steps = steps if steps is None else steps
    warmup = warmup if warmup is None else warmup
    W, S, X = gemv_inputs(rank)
    Wd = torch.from_numpy(W).cuda()
    Wp0 = g4.w4_pack(Wd)
    Sd0 = torch.from_numpy(S).cuda()
    Wps = [Wp0] + [Wp0.clone() for _ in range(NCOPY - 1)]
    Sds = [Sd0] + [Sd0.clone() for _ in range(NCOPY - 1)]
    Xd = torch.from_numpy(X).cuda()
    Y = torch.empty((1, N_CFG0), device="cuda")
    lib = g4.lib()
    stream = torch.cuda.Stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    xp, yp = ctypes.c_void_p(Xd.data_ptr()), ctypes.c_void_p(Y.data_ptr())
    wps = [ctypes.c_void_p(t.data_ptr()) for t in Wps]
    sps = [ctypes.c_void_p(t.data_ptr()) for t in Sds]

    def step(i):
        rc = lib.g4_w4g32_gemm(wps[i % NCOPY], sps[i % NCOPY], xp, None, 1, N_CFG0, K_CFG0, yp, N_CFG0, sp)
        if rc:
            raise RuntimeError(lib.g4_last_error().decode())

    # the K timed steps are launched as one CUDA graph (no host launch gaps between kernels)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(warmup):
            step(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            step(i)
    with torch.cuda.stream(stream):
        graph.replay()  # warm replay
    torch.cuda.synchronize()
    barrier(dist_)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # nvidia-smi samples every 200 ms, so the timed replay sits in the middle of a ~1.2 s window of
    # back-to-back replays of the same graph, and the clock record covers that window.
    t_one = time.perf_counter()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    t_one = max(time.perf_counter() - t_one, 1e-5)
    roll = max(1, int(0.6 / t_one))
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            for _ in range(roll):
                graph.replay()
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            for _ in range(roll):
                graph.replay()
        torch.cuda.synchronize()
    barrier(dist_)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms, dist_)
    del graph

    # e2e: the same GEMV through the C ABI from pinned host buffers, H2D x + D2H y every step
    xh = torch.from_numpy(X).pin_memory()
    yh = torch.empty((1, N_CFG0), dtype=torch.float32).pin_memory()
    with torch.cuda.stream(stream):
        for i in range(warmup):
            Xd.copy_(xh, non_blocking=True)
            step(i)
            yh.copy_(Y, non_blocking=True)
            stream.synchronize()
        barrier(dist_)
        t0 = time.perf_counter()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for i in range(steps):
            Xd.copy_(xh, non_blocking=True)
            step(i)
            yh.copy_(Y, non_blocking=True)
            stream.synchronize()
        f1.record(stream)
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), dist_)
    wall_ms = (time.perf_counter() - t0) * 1e3
    ok = np.array_equal(yh.numpy(), Y.cpu().numpy())
    out = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        per_gpu_gbs = GEMV_BYTES * steps / (ms / 1e3) / 1e9
        out = {
            "metric": METRIC, "value": GEMV_BYTES * steps * world / (ms_max / 1e3) / 1e9, "unit": "GB/s",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms_max / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded int4 weights uniform in [-8,7], bf16 scales |N(0,1)|*0.01, x ~ N(0,1))",
            "config": {"workload": "configs[0] W4G32 GEMV 8192x2048, M=1", "N": N_CFG0, "K": K_CFG0,
                       "timing": "K launches replayed as one CUDA graph, CUDA events on its stream",
                       "bytes_per_step": GEMV_BYTES, "l2": f"{NCOPY} rotating weight copies "
                       f"({NCOPY * GEMV_BYTES / 1e6:.0f} MB > L2)", "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "achieved": per_gpu_gbs, "peak": peak, "unit": "GB/s",
                         "frac": per_gpu_gbs / peak, "peak_kind": peak_kind,
                         "traffic": profile_traffic("w4g32_gemv_cfg0"), "kernel": "k_w4g32<1>"},
            "e2e": {"value": GEMV_BYTES * steps * world / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": K_CFG0 * 4, "d2h_bytes_per_step": N_CFG0 * 4,
                    "wall_ms": wall_ms, "result_matches_device": bool(ok)},
            "gpu_launches": steps,
            "clocks": dict(clk.summary() or {}, window="1.2 s of back-to-back replays around the timed one"),
        }
    return out, dist_


# --------------------------------------------------------------------------- head workload
N_CFG2, K_CFG2, M_CFG2 = 262144, 2048, 4


def run_head_g4(args, world, rank, local):
    """configs[2]'s exact head: the bf16p logits of M=4 hidden states against the 262,144 x 2048 head
    (the screen's fallback), through the split-nibble copy the engine reads (g4_bf16p_nib_gemm, 48 B
    per group).  Bytes counted: the bf16p rows (44 per group), the exceptions, x and the logits."""
    import torch
    import g4
    torch.cuda.set_device(local)
    dist_ = init_pg(world, local)
    g4.device_init()
    gen = torch.Generator(device="cuda").manual_seed(262144 + rank)
    E = (torch.randn(N_CFG2, K_CFG2, device="cuda", generator=gen) * 0.02).to(torch.bfloat16).view(torch.int16)
    head = g4.PackedHead(E)
    del E
    torch.cuda.empty_cache()
    nib = head.nibbled()
    Xd = torch.randn(M_CFG2, K_CFG2, device="cuda", generator=gen) / float(np.sqrt(K_CFG2))
    Y = torch.empty((M_CFG2, N_CFG2), device="cuda")
    nbytes = (N_CFG2 * (K_CFG2 // 32) * 44 + head.n_exc * 6 + (N_CFG2 + 1) * 8 + M_CFG2 * K_CFG2 * 4
              + M_CFG2 * N_CFG2 * 4)
    lib = g4.lib()
    stream = torch.cuda.Stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    cargs = (ctypes.c_void_p(nib.data_ptr()), head.cb, ctypes.c_void_p(head.exc_ptr.data_ptr()),
             ctypes.c_void_p(head.exc_col.data_ptr()), ctypes.c_void_p(head.exc_delta.data_ptr()), N_CFG2, K_CFG2,
             ctypes.c_void_p(Xd.data_ptr()), M_CFG2, ctypes.c_void_p(Y.data_ptr()), N_CFG2, sp)

    def step():
        if lib.g4_bf16p_nib_gemm(*cargs):
            raise RuntimeError(lib.g4_last_error().decode())

    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(args.steps):
            step()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    barrier(dist_)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_one = time.perf_counter()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    roll = max(1, int(0.6 / max(time.perf_counter() - t_one, 1e-5)))  # the clock record spans ~1.2 s
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            for _ in range(roll):
                graph.replay()
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            for _ in range(roll):
                graph.replay()
        torch.cuda.synchronize()
    barrier(dist_)
    ms = e0.elapsed_time(e1)
    ms_max = max_over_ranks(ms, dist_)
    del graph
    # e2e: x from pinned host memory, the logits back to it, every step
    xh = Xd.cpu().pin_memory()
    yh = torch.empty((M_CFG2, N_CFG2), dtype=torch.float32).pin_memory()
    with torch.cuda.stream(stream):
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            Xd.copy_(xh, non_blocking=True)
            step()
            yh.copy_(Y, non_blocking=True)
        f1.record(stream)
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), dist_)
    out = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        per_gpu = nbytes * args.steps / (ms / 1e3) / 1e9
        out = {
            "metric": METRIC, "value": nbytes * args.steps * world / (ms_max / 1e3) / 1e9, "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded head ~ N(0, 0.02) bf16, x ~ N(0,1)/sqrt(2048))",
            "config": {"workload": "configs[2] exact head (bf16p) 262144x2048, M=4", "N": N_CFG2, "K": K_CFG2,
                       "M": M_CFG2, "exceptions": int(head.n_exc), "bytes_per_step": nbytes,
                       "timing": "K launches replayed as one CUDA graph, CUDA events on its stream",
                       "l2": "every step reads the 805 MB split-nibble head (> L2)", "parallelism": f"replicas x{world}"},
            "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                         "peak_kind": peak_kind, "traffic": profile_traffic("head_nib_gemv_cfg2"),
                         "kernel": "k_bf16n_rows_tma<4>"},
            "e2e": {"value": nbytes * args.steps * world / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": M_CFG2 * K_CFG2 * 4, "d2h_bytes_per_step": M_CFG2 * N_CFG2 * 4},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
        }
    return out, (dist_, head, Xd)


def cpu_head_port(head_and_x, rows=8192, seconds=10.0):
    """The oracle's bf16p logits (the restatement of bf16p::rows_tile, OpenMP over rows) for the first
    `rows` rows of the same head and x, on the host's cores."""
    from oracle_lib import or_head_logits
    head, Xd = head_and_x
    K = head.K
    data = head.data[: rows * (K // 32) * 44].cpu().numpy()
    ep = head.exc_ptr[: rows + 1].cpu().numpy()
    ne = int(ep[-1])
    col = head.exc_col[:max(ne, 1)].cpu().numpy().view(np.uint16)
    dl = head.exc_delta[:max(ne, 1)].cpu().numpy()
    X = Xd.cpu().numpy()
    cb = np.frombuffer(head.cb_host, np.uint8)
    nbytes = rows * (K // 32) * 44 + ne * 6 + (rows + 1) * 8 + X.size * 4 + X.shape[0] * rows * 4
    or_head_logits((data, ep, col, dl), cb, rows, K, X)
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < seconds and n < 1000:
        or_head_logits((data, ep, col, dl), cb, rows, K, X)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": nbytes * n / dt / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} calls of the oracle's bf16p logits over the first {rows} rows, M=4 (OpenMP)"}


# --------------------------------------------------------------------------- screen workload
SCREEN_BYTES = N_CFG2 * (K_CFG2 // 2) + N_CFG2 * (K_CFG2 // 32) * 2 + N_CFG2 * 4  # int4 + scales + coef


def run_screen_g4(args, world, rank, local, dist_=None, steps=None, warmup=None, planted=None, min_seconds=1.0):
    """configs[2]'s certified head screen, vocab-parallel: rank r holds rows [r N/W, (r+1) N/W) of
    the 262,144 x 2,048 head (screen copy, packed rows, unpacked copy) and one call is the library's
    g4_head_screen_dist over its own NCCL communicator: the hidden broadcast, the shard's screen, the
    all-reduced bound, survivors or the shard's full exact head, the all-reduced candidate max and the
    all-reduced winner, all on the stream.  The timed calls are replays of a CUDA graph that records
    16 calls (collectives included), repeated until the timed region lasts >= min_seconds.  Total
    work is fixed as W grows ("strong").  Bytes counted per call: the int4 screen and the hidden rows,
    plus the bf16p rows and exceptions of every shard when a shard fell back."""
    import torch
    import g4
    steps = steps or args.steps
    warmup = warmup or args.warmup
    planted = args.planted if planted is None else planted
    torch.cuda.set_device(local)
    if dist_ is None:
        dist_ = init_pg(world, local)
    g4.device_init()
    n_loc = N_CFG2 // world
    gen = torch.Generator(device="cuda").manual_seed(262144 * 16 + rank)
    E = (torch.randn(n_loc, K_CFG2, device="cuda", generator=gen) * 0.02).to(torch.bfloat16).view(torch.int16)
    shard = g4.ScreenShard(E, rank * n_loc, lim=30000, M=M_CFG2)
    hgen = torch.Generator(device="cuda").manual_seed(2048)
    H = torch.randn(M_CFG2, K_CFG2, device="cuda", generator=hgen) / float(np.sqrt(K_CFG2))
    if planted:  # h = a w_j / |w_j| + sqrt(1 - a^2) noise for rows j of rank 0's shard (broadcast by the call)
        rows = [5 + 9973 * m for m in range(M_CFG2)]
        Wj = E[rows].view(torch.bfloat16).float()
        a = float(args.plant_weight)
        H = a * Wj / Wj.norm(dim=1, keepdim=True) + float(np.sqrt(max(0.0, 1.0 - a * a))) * H
    del E
    torch.cuda.empty_cache()
    comm = g4.NcclComm(dist_) if dist_ is not None else g4.NcclComm()
    idx = torch.empty(M_CFG2, dtype=torch.int32, device="cuda")

    def step():
        return g4.screen_dist_native(shard, H, comm, root=0, out=idx)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    _, ns = shard.select(H, shard.bound(H))  # survivors of this shard (fallback = -1), local bound
    fell_back = bool((ns < 0).any().item())
    nsurv = [int(v) for v in ns.cpu().numpy()]
    nb = torch.tensor([shard.head.n_exc, float(fell_back)], dtype=torch.float64, device="cuda")
    if dist_ is not None:
        dist_.all_reduce(nb)
    n_exc, any_fallback = int(nb[0].item()), bool(nb[1].item() > 0)
    nbytes = SCREEN_BYTES + M_CFG2 * K_CFG2 * 4 + (N_CFG2 * (K_CFG2 // 32) * 44 + n_exc * 6 if any_fallback else 0)
    inner = 16
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(inner):
            step()
    graph.replay()  # calibration replay (also the graph's warm-up)
    torch.cuda.synchronize()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    graph.replay()
    c1.record()
    torch.cuda.synchronize()
    per_replay = max_over_ranks(c0.elapsed_time(c1), dist_)
    reps = int(max(-(-steps // inner), np.ceil(min_seconds * 1e3 / max(per_replay, 1e-3))))
    barrier(dist_)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
    barrier(dist_)
    calls = reps * inner
    ms_max = max_over_ranks(e0.elapsed_time(e1), dist_)
    del graph  # graphs holding NCCL calls go before the communicator
    # e2e: the hidden rows from pinned host memory on rank 0 (the call broadcasts them), the winners
    # back to host every call; eager calls
    hh = H.cpu().pin_memory()
    ih = torch.empty(M_CFG2, dtype=torch.int32).pin_memory()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(steps):
        if rank == 0:
            H.copy_(hh, non_blocking=True)
        step()
        ih.copy_(idx, non_blocking=True)
        torch.cuda.current_stream().synchronize()
    f1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1), dist_)
    winners = [int(i) for i in idx.cpu().numpy()]
    barrier(dist_)
    comm.close()
    out = None
    if rank == 0:
        peak, peak_kind = measured_peaks()
        per_gpu = nbytes / world * calls / (ms_max / 1e3) / 1e9
        out = {
            "metric": METRIC, "value": nbytes * calls / (ms_max / 1e3) / 1e9, "unit": "GB/s",
            "n_gpus": world, "steps": calls, "warmup": warmup, "ms_per_step": ms_max / calls,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded head ~ N(0, 0.02) bf16 per shard, h ~ N(0,1)/sqrt(2048))",
            "config": {"workload": f"configs[2] certified head screen 262144x2048, M=4, vocab-parallel x{world}"
                                   + (f", planted hidden states (weight {args.plant_weight})" if planted else ""),
                       "rows_per_gpu": n_loc, "lim": 30000, "fallback": any_fallback, "bytes_per_step": nbytes,
                       "rank0_survivors_local_bound": nsurv,
                       "collectives": ("NCCL (the library's own communicator) broadcast h, all-reduce max (bound, "
                                       "candidate max), all-reduce min (winner) between the device phases"),
                       "timing": f"CUDA events around {reps} replays of a graph of {inner} calls (collectives "
                                 "captured), max over ranks",
                       "parallelism": f"vocab-parallel x{world}"},
            "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                         "peak_kind": peak_kind, "traffic": None,
                         "kernel": "whole screen call per GPU (screen GEMV + exact-head fallback + collectives)"},
            "e2e": {"value": nbytes * steps / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": M_CFG2 * K_CFG2 * 4, "d2h_bytes_per_step": M_CFG2 * 4,
                    "api": "g4_head_screen_dist per call, eager"},
            "gpu_launches": 14 * calls,  # per call: bound 4, select 8, pick 1, sentinel 1 (per GPU; NCCL's not counted)
            "clocks": clk.summary(),
            "winners": winners,
        }
    return out, dist_


def cpu_screen_port(rows=16384, seconds=10.0):
    """The oracle's screen row (screen_task's bound and survivor list, restated) over the first
    `rows` rows of a configs[2]-distributed head, for M=4 hidden rows, on the host's cores."""
    from oracle_lib import bf16_bits, or_screen_build, or_screen_row
    rng = np.random.default_rng(2)
    E = bf16_bits(rng.standard_normal((rows, K_CFG2), dtype=np.float32) * np.float32(0.02))
    W4, S4, coef = or_screen_build(E)
    H = (rng.standard_normal((M_CFG2, K_CFG2), dtype=np.float32) / np.float32(np.sqrt(K_CFG2))).astype(np.float32)
    nbytes = rows * (K_CFG2 // 2) + rows * (K_CFG2 // 32) * 2 + rows * 4
    t0 = time.perf_counter()
    n = 0
    while time.perf_counter() - t0 < seconds and n < 200:
        for m in range(M_CFG2):
            or_screen_row(W4, S4, coef, H[m], lim=rows)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": nbytes * n / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{n} screens of {rows} rows x M=4 (oracle restatement of screen_task, scalar; no exact head)"}


# --------------------------------------------------------------------------- decode workload
PROMPT_SEED, N_PROMPT = 4, 6841
TOKENS_METRIC_UNIT = "tok/s"


def pass_bytes(P, M, H=2048, NL=30, I=8192, NQ=8, HD=256, V=262144, WINDOW=512, head=True):
    """Algorithmic HBM bytes of one verify pass of M rows after position P: every int4 weight and
    bf16 group scale of the 30 layers, the K and V rows the attention reads (global layers: all
    P+M positions; sliding: the last 511+M), the K/V rows written, and (head=True) the int4 head
    screen (weights, scales, row coefficients).  Exact rescoring of the few survivors is not
    counted."""
    QD = NQ * HD

    def lin(N, K):
        return N * K // 2 + N * (K // 32) * 2

    per_layer = lin(QD + 2 * HD, H) + lin(H, QD) + lin(2 * I, H) + lin(H, I) + 4 * H * 4 + 2 * HD * 4
    n_glob = sum(1 for l in range(NL) if l % 5 == 4)
    keys = n_glob * (P + M) + (NL - n_glob) * min(P + M, WINDOW - 1 + M)
    kv = keys * HD * 2 * 2 + NL * M * HD * 2 * 2
    screen = V * H // 2 + V * (H // 32) * 2 + V * 4
    return NL * per_layer + kv + (screen if head else 0)


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def timed_decode(eng, args, dist_, local, pad=True):
    """W warm-up rounds, then K timed rounds in one g4_engine_decode call (one graph launch of the
    device-side round loop), with untimed padding rounds around it so that the clock record covers
    the timed call.  Returns (tokens, stats delta, wall ms, clock summary)."""
    import torch
    _, st_w = eng.decode(args.warmup, 1 << 30)
    barrier(dist_)
    torch.cuda.synchronize()
    pad_s = 0.4 if pad else 0.0
    with Clocks(local) as clk:
        t_pad, n_pad = time.perf_counter(), 0
        while time.perf_counter() - t_pad < pad_s and n_pad < 60:  # <= 60 rounds: the context must hold them
            eng.decode(4, 1 << 30)
            n_pad += 4
        _, st_w = eng.decode(0, 1 << 30)
        barrier(dist_)
        t1 = time.perf_counter()
        n_tok, st = eng.decode(args.steps, 1 << 30)
        wall_s = time.perf_counter() - t1
        t_pad, n_pad = time.perf_counter(), 0
        while time.perf_counter() - t_pad < pad_s and n_pad < 60:
            eng.decode(4, 1 << 30)
            n_pad += 4
    keys = ("rounds", "ngram_rounds", "drafted", "accepted", "decode_tokens", "verify_passes", "verify_rows",
            "draft_steps", "verify_gpu_ms", "draft_gpu_ms", "decode_gpu_ms", "h2d_bytes", "d2h_bytes",
            "kernel_launches", "head_fallbacks", "screen_skipped")
    d = {k: st[k] - st_w[k] for k in keys}
    d["P_end"] = st["decode_tokens"]
    return n_tok, d, wall_s * 1e3, clk.summary()


def decode_roofline(eng, d, M_pass, P_mid, peak, peak_kind):
    """Roofline of the verify pass: its algorithmic bytes over its device time, the pass replayed
    with CUDA events around it on the engine stream (g4_engine_time_verify) right after the timed
    call.  algorithmic_bytes, per pass: every weight, the K/V rows read and written, plus the head
    as the timed rounds ran it: the int4 screen on the passes that screened, the bf16p exact head
    on the passes that read the full head (the screen fell back, or its back-off skipped it), as
    fractions of the timed passes.  screen_every_pass gives the figure of a pass that screens and
    whose screen certifies (no exact head): the definition used before the back-off existed."""
    ms_pass = eng.time_verify(M_pass, reps=20)
    n = max(1, d["verify_passes"])
    f_screen = 1.0 - d["screen_skipped"] / n
    f_full = d["head_fallbacks"] / n
    base = pass_bytes(P_mid, M_pass, head=False)
    screen = pass_bytes(P_mid, M_pass) - base
    alg = int(base + f_screen * screen + f_full * HEAD_BF16P_BYTES)
    achieved = alg / (ms_pass / 1e3) / 1e9
    alg_s = base + screen
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "peak_kind": peak_kind, "M": M_pass, "ms_per_pass": ms_pass, "algorithmic_bytes": alg,
            "frac_uses": "algorithmic_bytes",
            "head_path": {"screened_frac": f_screen, "full_head_frac": f_full, "layers_kv_bytes": base,
                          "screen_bytes": screen, "exact_head_bf16p_bytes": HEAD_BF16P_BYTES},
            "screen_every_pass": {"bytes": alg_s, "achieved": alg_s / (ms_pass / 1e3) / 1e9,
                                  "frac": alg_s / (ms_pass / 1e3) / 1e9 / peak},
            "traffic": profile_traffic(f"verify_pass_cfg4_m{M_pass}") or profile_traffic("verify_pass_cfg4"),
            "traffic_kind": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one pass (cold, serialised)",
            "kernel": f"target verify pass of M={M_pass} rows (30 layers + int4 head screen + exact-head fallback), "
                      "CUDA events around 20 replays of its graph"}


def run_prefill_g4(args, world, rank, local):
    """configs[4]'s prompt prefill: the 6,841-token prompt through the tensor-core path (full blocks
    in chunks of 2,048 rows, the last block through the GEMV path), W untimed prefills first (the
    first builds the int8 weight copies), then K timed prefills on the engine stream.  A step is
    one prefill of the whole prompt; value = prompt tokens / second, summed over replicas."""
    import torch
    import g4
    from oracle_lib import make_prompt
    torch.cuda.set_device(local)
    dist_ = init_pg(world, local)
    n_prompt = args.prompt_tokens or N_PROMPT
    eng = g4.Engine(g4.engine_config(prefill_tc=args.prefill_tc, ctx_max=max(8192, n_prompt + 64)))
    prompt = make_prompt(PROMPT_SEED + rank, n_prompt)
    for _ in range(args.warmup):
        eng.prefill(prompt)
    torch.cuda.synchronize()
    barrier(dist_)
    times = []
    with Clocks(local) as clk:
        for _ in range(args.steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            eng.prefill(prompt)  # host token ids in; the first token back (one H2D and one D2H copy)
            times.append(time.perf_counter() - t0)
    s_max = max_over_ranks(sum(times), dist_)
    eng.close()
    out = None
    if rank == 0:
        out = {
            "metric": "prompt prefill tok/s (configs[4] prompt)", "value": n_prompt * args.steps * world / s_max,
            "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": s_max / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32+int8", "data": "synthetic (seeded random-init E2B weights; Zipf(1.1) prompt with copied spans)",
            "config": {"workload": f"configs[4] prefill of a {n_prompt}-token prompt", "prefill_tc": args.prefill_tc,
                       "timing": "host wall clock around each g4_engine_prefill call (it synchronises), max over "
                                 "ranks", "parallelism": f"replicas x{world}"},
            "e2e": {"value": n_prompt * args.steps * world / s_max, "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * n_prompt, "d2h_bytes_per_step": 4},
            "clocks": clk.summary(),
        }
    return out, dist_

HEAD_BF16P_BYTES = 262144 * (2048 // 32) * 44  # the exact head rows the fallback reads


def run_decode_g4(args, world, rank, local):
    import torch
    import g4
    from oracle_lib import make_prompt
    torch.cuda.set_device(local)
    dist_ = init_pg(world, local)
    eng = g4.Engine(g4.engine_config(graphs=args.graphs))
    prompt = make_prompt(PROMPT_SEED + rank, N_PROMPT)
    if args.fake_ctx:  # the reference's ENGINE_FAKE_CTX mode: LCG K/V for 6,837 positions, then 4 prompt tokens
        eng.fake_ctx(N_PROMPT - 4)
        prompt = prompt[-4:]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.prefill(prompt)
    prefill_s = time.perf_counter() - t0
    state = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not args.fake_ctx:
        state = eng.export_state(N_PROMPT)  # the CPU baseline continues from this prefilled context
    n_tok, d, wall_ms, clocks = timed_decode(eng, args, dist_, local, pad=not args.no_clock_window)
    gpu_ms = d["decode_gpu_ms"]
    ms_max = max_over_ranks(gpu_ms, dist_)
    wall_max = max_over_ranks(wall_ms, dist_)
    tok_all = float(n_tok)  # tokens committed by all replicas in the timed rounds
    if dist_ is not None:
        t = torch.tensor([float(n_tok)], dtype=torch.float64, device="cuda")
        dist_.all_reduce(t)
        tok_all = float(t.item())
    rounds = max(1, d["rounds"])
    M_avg = d["verify_rows"] / max(1, d["verify_passes"])
    M_pass = max(1, min(4, round(M_avg)))
    P_mid = N_PROMPT + 60  # mid-run context (the warm-up, padding and timed rounds commit ~100-250 tokens)
    peak, peak_kind = measured_peaks()
    roof = decode_roofline(eng, d, M_pass, P_mid, peak, peak_kind)
    streams = None
    if not args.no_subrecords:
        streams = run_streams_subrecord(eng, args, world, rank, local, dist_)
    eng.close()
    del eng
    torch.cuda.empty_cache()
    # the M = 4 path: prompt lookup off, every round drafts k = 3 tokens with the MTP drafter
    mtp = None
    if not args.no_subrecords:
        mtp = run_mtp_subrecord(args, world, rank, local, dist_, peak, peak_kind)
    gemv = None
    if not args.no_subrecords:
        gemv, _ = run_gemv_g4(args, world, rank, local, dist_=dist_, steps=200, warmup=10)
        if gemv is not None:
            gemv = {k: gemv[k] for k in ("value", "unit", "ms_per_step", "config", "roofline", "e2e", "clocks")}
    screen = None
    if not args.no_subrecords:  # configs[2]'s head screen split over the N GPUs (one library call per screen)
        screen, _ = run_screen_g4(args, world, rank, local, dist_=dist_, steps=64, warmup=5, planted=False)
        if screen is not None:
            screen = {k: screen[k] for k in ("value", "unit", "n_gpus", "scaling", "ms_per_step", "config", "roofline",
                                             "e2e", "clocks", "winners")}
        torch.cuda.empty_cache()
    out = None
    if rank == 0:
        out = {
            "metric": METRIC, "value": tok_all / (ms_max / 1e3), "unit": TOKENS_METRIC_UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / rounds,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+int8",
            "data": "synthetic (seeded random-init E2B weights, generator g4-e2b-synth v1; Zipf(1.1) prompt with "
                    "copied spans)",
            "config": {"workload": "configs[4] greedy speculative decode @6.8k ctx, synthetic E2B, 1 stream per GPU",
                       "prompt_tokens": N_PROMPT, "context": ("ENGINE_FAKE_CTX 6,837 + 4 prompt tokens" if args.fake_ctx
                                                               else "6,841-token prompt prefilled"), "k_draft": 3, "ngram": 2, "int8_activations": True,
                       "step": "one decode round (drafts -> verify pass of k+1 rows -> greedy accept), the K timed "
                               "rounds one launch of the device-side round-loop graph",
                       "tokens": n_tok, "rounds": d["rounds"], "ngram_rounds": d["ngram_rounds"],
                       "accepted_drafts": d["accepted"], "tokens_per_round": n_tok / rounds,
                       "verify_ms_per_pass_in_decode": d["verify_gpu_ms"] / max(1, d["verify_passes"]),
                       "draft_ms_per_round": d["draft_gpu_ms"] / rounds, "head_fallbacks": d["head_fallbacks"],
                       "screen_skipped": d["screen_skipped"],
                       "head_screen": "2: certified screen with back-off after fallbacks (same tokens as screening every pass)",
                       "prefill_s": prefill_s, "l2": "every verify pass streams ~1.37 GB of weights, KV and head "
                       "screen (> 10x the 126 MB L2)", "parallelism": f"replicas x{world}",
                       "timing": "CUDA events on the engine stream around the timed decode call (max over ranks)"},
            "roofline": roof,
            "e2e": {"value": tok_all / (wall_max / 1e3), "unit": TOKENS_METRIC_UNIT,
                    "h2d_bytes_per_step": d["h2d_bytes"] / rounds, "d2h_bytes_per_step": d["d2h_bytes"] / rounds,
                    "api": "g4_engine_decode (host token buffer; the K rounds are one graph launch, then one copy of "
                           "the round state and the committed tokens)", "wall_ms": wall_max},
            "gpu_launches": d["kernel_launches"],
            "clocks": clocks,
            "mtp": mtp,
            "streams": streams,
            "gemv_cfg0": gemv,
            "screen_sharded": screen,
        }
    return out, (dist_, state)


def run_streams_subrecord(eng, args, world, rank, local, dist_, totals=(8, 64)):
    """configs[4] as independent request streams: S streams in total split over the N GPUs (S/N per
    GPU), each an engine of its own (KV cache, round state, CUDA stream, round-loop graph) over the
    weights of the GPU's first engine (g4_engine_create_shared), all decoding at once
    (g4_engine_decode_async).  Up to 8 distinct prompts are prefilled per GPU; further streams continue
    copies of those contexts (g4_engine_copy_state).  A step is one round of every stream; value =
    tokens committed by all streams / the device time from a common start event to the last
    stream's end (max over ranks)."""
    import torch
    import g4
    from oracle_lib import make_prompt
    n_ctx = max(1, min(8, max(totals) // world))
    ctxs = [eng]
    for i in range(1, n_ctx):
        e2 = g4.Engine(g4.engine_config(), share=eng)
        e2.prefill(make_prompt(PROMPT_SEED + 100 * rank + i, N_PROMPT))
        ctxs.append(e2)
    pool = list(ctxs)
    out = {}
    try:
        for S in totals:
            s_loc = max(1, S // world)
            while len(pool) < s_loc:
                e2 = g4.Engine(g4.engine_config(), share=eng)
                e2.copy_state_from(ctxs[len(pool) % n_ctx])
                pool.append(e2)
            active = pool[:s_loc]
            for e in active:  # warm-up (and graph capture of new engines)
                e.decode_async(args.warmup, 1 << 30)
            for e in active:
                e.decode_wait()
            barrier(dist_)
            torch.cuda.synchronize()
            start = torch.cuda.Event(enable_timing=True)
            with Clocks(local) as clk:
                start.record()
                t0 = time.perf_counter()
                for e in active:
                    e.decode_async(args.steps, 1 << 30, start)
                res = [e.decode_wait(start) for e in active]
                wall = time.perf_counter() - t0
            ms = max(r[2] for r in res)
            ntok = sum(len(r[0]) for r in res)
            ms_max = max_over_ranks(ms, dist_)
            tok_all = float(ntok)
            if dist_ is not None:
                t = torch.tensor([tok_all], dtype=torch.float64, device="cuda")
                dist_.all_reduce(t)
                tok_all = float(t.item())
            out[f"s{S}"] = {"value": tok_all / (ms_max / 1e3), "unit": TOKENS_METRIC_UNIT, "streams_total": S,
                            "streams_per_gpu": s_loc, "distinct_prompts_per_gpu": min(n_ctx, s_loc),
                            "rounds_per_stream": args.steps, "tokens": tok_all, "ms": ms_max,
                            "wall_ms": wall * 1e3, "clocks": clk.summary()}
    finally:
        for e in pool[1:]:
            e.close()
    out["timing"] = ("CUDA events: a start event that every stream waits on, to each stream's end; max over streams "
                     "and ranks")
    return out


def run_mtp_subrecord(args, world, rank, local, dist_, peak, peak_kind):
    """configs[4] with prompt lookup off: every round runs the MTP drafter (k = 3) and a verify pass
    of M = 4 rows."""
    import torch
    import g4
    from oracle_lib import make_prompt
    eng = g4.Engine(g4.engine_config(ngram=0))
    eng.prefill(make_prompt(PROMPT_SEED + rank, N_PROMPT))
    n_tok, d, wall_ms, clocks = timed_decode(eng, args, dist_, local, pad=not args.no_clock_window)
    ms_max = max_over_ranks(d["decode_gpu_ms"], dist_)
    roof = decode_roofline(eng, d, 4, N_PROMPT + 60, peak, peak_kind)
    eng.close()
    del eng
    torch.cuda.empty_cache()
    rounds = max(1, d["rounds"])
    return {"value": n_tok * world / (ms_max / 1e3), "unit": TOKENS_METRIC_UNIT, "ngram": 0, "tokens": n_tok,
            "rounds": d["rounds"], "accepted_drafts": d["accepted"], "ms_per_round": ms_max / rounds,
            "verify_ms_per_pass_in_decode": d["verify_gpu_ms"] / max(1, d["verify_passes"]),
            "draft_ms_per_round": d["draft_gpu_ms"] / rounds, "roofline": roof, "clocks": clocks,
            "gpu_launches": d["kernel_launches"]}


def cpu_decode_reference(state=None, seconds=25.0, rounds_min=16, rounds_max=64, warm_rounds=2):
    """configs[4] decode on the host's cores through the reference's own compiled kernels: the
    linears (lin_task / i8_task), split-KV attention (attn_task + attn_merge) and the exact head
    (head_task) from oracle/_ref/libg4ref.so on the reference's thread pool, the rest of the round
    (norms, RoPE, drafter glue, prompt lookup, acceptance) from the oracle's C restatement
    (OpenMP).  state: the GPU arm's prefilled context (K/V, history, hidden, P), so both arms decode
    the same rounds; without it the CPU prefills the prompt itself (untimed).  The reference cannot
    run its certified screen at K = 2048 (hard-coded 1536), so the CPU reads the full exact head every
    round, which the screen falls back to on this model anyway."""
    from oracle_lib import OracleModel, e2e_config, make_prompt, oracle, reference
    threads = host_threads()
    reference(min(threads, 16))  # the reference's pool: all host threads, at most the 16 it has slots for (:78, :145)
    oracle().or_set_threads(threads)
    om = OracleModel(e2e_config())
    kind = "reference" if om.use_reference_kernels() else "port"
    t0 = time.perf_counter()
    if state is not None:
        K, V, seq, h, P = state
        om.set_state(K, V, seq, h, P)
        how = "the GPU arm's prefilled 6,841-token context (K/V, history, hidden state) handed over"
    else:
        om.prefill(make_prompt(PROMPT_SEED, N_PROMPT))
        how = f"the 6,841-token prompt prefilled on the CPU first ({time.perf_counter() - t0:.0f} s, untimed)"
    om.decode(warm_rounds, 1 << 30)
    toks_all = []
    t0 = time.perf_counter()
    r = 0
    while r < rounds_max and (r < rounds_min or time.perf_counter() - t0 < seconds):
        toks, _ = om.decode(1, 1 << 30)
        toks_all += list(toks)
        r += 1
    dt = time.perf_counter() - t0
    om.close()
    ref = reference()
    pool = getattr(ref, "pool_threads", threads) if ref is not None else threads
    return {"value": len(toks_all) / dt, "unit": TOKENS_METRIC_UNIT, "cores": int(pool), "kind": kind,
            "rounds": r, "tokens": len(toks_all), "seconds": dt,
            "sample": f"{len(toks_all)} tokens in {r} decode rounds after {warm_rounds} warm-up rounds, from {how}; "
                      f"linears, split-KV attention and exact head = the reference's AVX2 kernels on its pool of "
                      f"{pool} threads, the rest the oracle's C restatement (OpenMP x{threads})"}


def cpu_gemv_reference(seconds=10.0, max_calls=2000):
    """The reference's own W4G32 path (lin_task over its thread pool) on the host's cores, over
    rotating weight copies larger than the last-level cache."""
    from oracle_lib import ptr, reference
    ref = reference(min(host_threads(), 16))  # the reference's pool holds at most 16 threads (:78)
    if ref is None:
        return None
    W, S, X = gemv_inputs(0)
    ncopy = 32
    Ws = [W.copy() for _ in range(ncopy)]
    Ss = [S.copy() for _ in range(ncopy)]
    Y = np.empty((1, N_CFG0), np.float32)
    for i in range(5):
        ref.ref_w4g32_gemm(ptr(Ws[i % ncopy]), ptr(Ss[i % ncopy]), ptr(X), 1, N_CFG0, K_CFG0, ptr(Y))
    t0 = time.perf_counter()
    n = 0
    while n < max_calls and time.perf_counter() - t0 < seconds:
        ref.ref_w4g32_gemm(ptr(Ws[n % ncopy]), ptr(Ss[n % ncopy]), ptr(X), 1, N_CFG0, K_CFG0, ptr(Y))
        n += 1
    dt = time.perf_counter() - t0
    return {"value": GEMV_BYTES * n / dt / 1e9, "unit": "GB/s", "cores": int(getattr(ref, "pool_threads", 0)),
            "kind": "reference", "calls": n, "ms_per_call": dt / n * 1e3,
            "sample": f"{n} GEMV calls over {ncopy} rotating weight copies ({ncopy * GEMV_BYTES / 1e6:.0f} MB), "
                      f"reference lin_task via its pool (oracle/_ref, AVX2)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="g4", choices=["g4", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "gemv", "head", "screen", "prefill"])
    ap.add_argument("--prefill-tc", type=int, default=1, choices=[0, 1, 2, 3],
                    help="prefill: the engine's prefill_tc (1 tensor-core GEMMs + eight-lanes-per-key attention)")
    ap.add_argument("--prompt-tokens", type=int, default=0, help="prefill: prompt length (default 6,841)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--planted", action="store_true",
                    help="screen: planted hidden states a * w_j/|w_j| + sqrt(1 - a^2) * noise (a = --plant-weight)")
    ap.add_argument("--plant-weight", type=float, default=0.3)
    ap.add_argument("--no-clock-window", action="store_true",
                    help="decode: no untimed padding rounds around the timed call (for profiling; clocks unsampled)")
    ap.add_argument("--no-subrecords", action="store_true",
                    help="decode: skip the M=4 MTP and configs[0] GEMV sub-records")
    ap.add_argument("--graphs", type=int, default=1, choices=[0, 1, 2],
                    help="decode: 1 = a decode call is one launch of the round-loop graph (default), 2 = one graph "
                         "launch per verify pass and draft chain, 0 = eager launches")
    ap.add_argument("--fake-ctx", action="store_true",
                    help="decode: build the 6.8k context with the reference's ENGINE_FAKE_CTX values instead of a "
                         "prefill (short, for profiling)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"decode": 64, "gemv": 200, "head": 20, "screen": 20, "prefill": 5}[args.workload]
    if args.warmup is None:
        args.warmup = 3 if args.workload in ("decode", "prefill") else 10
    args.warmup = max(args.warmup, 3)
    if args.workload == "decode":
        args.steps = min(args.steps, 120)  # 6,841 + 4 x (W + K + ~2 x 0.4 s of padding rounds) tokens fit 8,192
    world, rank, local = dist_setup()

    if args.impl == "reference":
        if rank != 0:
            return
        if args.workload == "decode":
            reference_decode(args)
        elif args.workload in ("head", "screen", "prefill"):
            print(json.dumps({"impl": "reference", "unavailable": f"the {args.workload} workload has no reference "
                              "arm; its cpu_baseline is the oracle's restatement"}))
        else:
            reference_gemv(args)
        return

    if args.workload == "decode":
        out, (dist_, state) = run_decode_g4(args, world, rank, local)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_decode_reference(state)
    elif args.workload == "screen":
        out, dist_ = run_screen_g4(args, world, rank, local)
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_screen_port()
    elif args.workload == "prefill":
        out, dist_ = run_prefill_g4(args, world, rank, local)
    elif args.workload == "head":
        out, (dist_, head, Xd) = run_head_g4(args, world, rank, local)
        if rank == 0 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_head_port((head, Xd))
    else:
        out, dist_ = run_gemv_g4(args, world, rank, local)
        if rank == 0 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_gemv_reference()
    if rank == 0:
        print(json.dumps(out))
    if dist_ is not None:
        dist_.destroy_process_group()


def reference_decode(args):
    """The reference arm for configs[4]: the reference's own CPU kernels (cpu_decode_reference) on all
    host threads, the prompt prefilled on the CPU (untimed), then W warm-up rounds and K timed rounds
    (at most ~60 s of rounds); value = committed tokens / time of the timed rounds."""
    r = cpu_decode_reference(None, seconds=60.0, rounds_min=min(args.steps, 16), rounds_max=args.steps,
                             warm_rounds=args.warmup)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": r["value"], "unit": TOKENS_METRIC_UNIT, "n_gpus": args.gpus,
        "steps": r["rounds"], "warmup": args.warmup, "ms_per_step": r["seconds"] * 1e3 / max(1, r["rounds"]),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+int8", "data": "synthetic",
        "config": {"workload": "configs[4] greedy speculative decode @6.8k ctx, synthetic E2B, 1 stream",
                   "context": "6,841-token prompt prefilled (same prompt as the g4 arm)", "k_draft": 3, "ngram": 2,
                   "int8_activations": True},
        "cpu_baseline": {"value": r["value"], "unit": TOKENS_METRIC_UNIT, "cores": r["cores"], "kind": r["kind"],
                         "sample": r["sample"]},
        "e2e": {"value": r["value"], "unit": TOKENS_METRIC_UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


def reference_gemv(args):
    per_step = []
    res = None
    for i in range(args.warmup + args.steps):
        r = cpu_gemv_reference(seconds=1.0, max_calls=50)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libg4ref.so was not built "
                              "(needs the reference sources at build time)"}))
            return
        if i >= args.warmup:
            per_step.append(r)
        res = r
    value = statistics.median(r["value"] for r in per_step)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.median(r["ms_per_call"] for r in per_step),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "configs[0] W4G32 GEMV 8192x2048, M=1", "N": N_CFG0,
                                        "K": K_CFG0, "bytes_per_step": GEMV_BYTES},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": res["cores"], "kind": "reference",
                         "sample": res["sample"]},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))


if __name__ == "__main__":
    main()
