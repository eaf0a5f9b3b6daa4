"""Generate the golden fixtures in tests/golden/ from the reference's own compiled kernels.

Run in a container that has the reference checkout and `make -C oracle` done:

    python tests/golden/make_golden.py

Each fixture stores its seeded inputs and the outputs of oracle/_ref/libg4ref.so (the
reference's kernels compiled from its sources, see oracle/Makefile).  tests/test_oracle_golden.py
checks the plain-C oracle against them bit-for-bit; GPU tests then check the CUDA path against
the oracle.  The reference ships no golden vectors of its own, so these are the pins.
"""
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from oracle_lib import (bf16_bits, or_codebook, or_pack, ptr, reference,  # noqa: E402
                        w4g32_weights)


def gemm_cases(rng):
    out = {}
    shapes = [(1, 128, 2048), (4, 128, 2048), (3, 64, 8192), (8, 64, 2048), (2, 256, 256)]
    for i, (M, N, K) in enumerate(shapes):
        W, S = w4g32_weights(rng, N, K)
        X = rng.standard_normal((M, K), dtype=np.float32)
        if i == 1:
            X[0, :32] = 0.0          # an all-zero group
            X[1, 32:64] *= 1e-30     # a tiny group
            X[2, 64:96] *= 1e4       # a large group
        out[f"c{i}"] = (W, S, X)
    return out


def main():
    ref = reference()
    if ref is None:
        sys.exit("oracle/_ref/libg4ref.so not built: run `make -C oracle`")
    rng = np.random.default_rng(20261201)
    fx = {}

    # W4G32 float GEMM and W4A8 (quant + integer-exact GEMM) on the same inputs.
    for name, (W, S, X) in gemm_cases(rng).items():
        M, K = X.shape
        N = W.shape[0]
        Yf = np.empty((M, N), np.float32)
        ref.ref_w4g32_gemm(ptr(W), ptr(S), ptr(X), M, N, K, ptr(Yf))
        Yi = np.empty((M, N), np.float32)
        ref.ref_w4a8_gemm(ptr(W), ptr(S), ptr(X), M, N, K, ptr(Yi))
        q = np.empty((M, K), np.int8)
        sx = np.empty((M, K // 32), np.float32)
        sm = np.empty((M, K // 32), np.int32)
        ref.ref_w4a8_quant(ptr(X), M, K, ptr(q), ptr(sx), ptr(sm))
        np.savez_compressed(HERE / f"gemm_{name}.npz", W=W, S=S, X=X, Y_w4g32=Yf, Y_w4a8=Yi, q=q, sx=sx, sum=sm)
        fx[name] = (M, N, K)

    # Quantisation edge cases: exact .5 midpoints (RNE), zeros, negative zero, huge and tiny groups.
    X = rng.standard_normal((4, 256), dtype=np.float32)
    sx0 = np.float32(1.0) / np.float32(127.0)
    X[0, :32] = (np.arange(32, dtype=np.float32) - 16 + 0.5) * sx0
    X[0, 31] = 127 * sx0
    X[1, :32] = 0.0
    X[1, 32:64] = -0.0
    X[2, :32] *= 3e38 / 4
    X[3, :32] *= 1e-38
    q = np.empty((4, 256), np.int8)
    sx = np.empty((4, 8), np.float32)
    sm = np.empty((4, 8), np.int32)
    ref.ref_w4a8_quant(ptr(X), 4, 256, ptr(q), ptr(sx), ptr(sm))
    np.savez_compressed(HERE / "quant_edges.npz", X=X, q=q, sx=sx, sum=sm)

    # bf16-exp3 packed head: codebook, pack bytes, CSR exceptions, logits, argmax rule.
    N, K = 192, 2048
    E = bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    E[3, :40] = 0                                   # zero weights (exponent 0 -> exceptions)
    E[4, :8] = bf16_bits(np.full(8, 3.0, np.float32))  # outlier exponents
    E[5, 100] = 0x8000                              # negative zero
    cb = or_codebook(E)
    data, ep, col, dl = or_pack(E, cb)               # only for sizing; the stored pack is the reference's
    d_r = np.zeros_like(data)
    ep_r = np.zeros_like(ep)
    col_r = np.zeros(len(col) + 1, np.uint16)
    dl_r = np.zeros(len(col) + 1, np.float32)
    ne = ref.ref_bf16p_pack(ptr(E), N, K, ptr(cb), ptr(d_r), ptr(ep_r), ptr(col_r), ptr(dl_r), len(col_r))
    Xh = (rng.standard_normal((4, K), dtype=np.float32) / np.float32(np.sqrt(K))).astype(np.float32)
    Y = np.empty((4, N), np.float32)
    ref.ref_bf16p_gemm(ptr(E), N, K, ptr(cb), ptr(Xh), 4, ptr(Y))
    np.savez_compressed(HERE / "bf16p.npz", E=E, cb=cb, data=d_r, exc_ptr=ep_r, exc_col=col_r[:ne],
                        exc_delta=dl_r[:ne], X=Xh, Y=Y)

    # Split-KV attention through attn_task + attn_merge with the pool's T threads.
    hd, nh = 256, 8
    cases = [(300, 1, False), (700, 4, True), (1000, 3, False), (520, 4, True)]
    for i, (ctx, M, sliding) in enumerate(cases):
        Kc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
        Vc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
        q = (rng.standard_normal((M, nh, hd), dtype=np.float32) * np.float32(0.0625)).astype(np.float32)
        pos = np.arange(ctx - M, ctx, dtype=np.int32)
        lo = (np.maximum(0, pos - 511) if sliding else np.zeros(M)).astype(np.int32)
        out = np.empty((M, nh, hd), np.float32)
        ref.ref_attn_splitkv(ptr(Kc), ptr(Vc), hd, nh, M, ptr(q), ptr(pos), ptr(lo), int(lo.min()), int(pos.max()),
                             ptr(out))
        np.savez_compressed(HERE / f"attn_c{i}.npz", K=Kc, V=Vc, q=q, pos=pos, lo=lo, out=out,
                            T=np.int32(ref.ref_pool_start(0)))

    # exp8 / gelu8 on edge inputs.
    x = np.concatenate([np.linspace(-100, 100, 4000, dtype=np.float32),
                        rng.standard_normal(96, dtype=np.float32) * 4]).astype(np.float32)
    e8 = np.empty_like(x)
    g8 = np.empty_like(x)
    ref.ref_exp8(ptr(np.minimum(x, 0).astype(np.float32)), x.size, ptr(e8))
    ref.ref_gelu8(ptr(x), x.size, ptr(g8))
    np.savez_compressed(HERE / "exp8_gelu.npz", x=x, exp8=e8, gelu=g8)

    # The reference screen_task runs only at its hard-coded N=262144, K=1536: store its outputs
    # for one seeded head and a planted-winner hidden state (few survivors) plus a random one
    # (every row survives, so the reference falls back).  The inputs are regenerated from the seed.
    if "--no-screen" not in sys.argv:
        screen_fixture(ref)
    print("golden fixtures written to", HERE)


def screen_inputs(seed=7):
    """262144 x 1536 head ~ N(0, 0.02) and three hidden states: a strongly planted winner (one
    survivor), a moderately planted one (h = 8 (0.3 w_j/|w_j| + sqrt(0.91) n): a few hundred
    survivors) and a random one (every row survives: fallback)."""
    rng = np.random.default_rng(seed)
    N, K = 262144, 1536
    E = bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    j = 123457
    wj = (E[j].astype(np.uint32) << 16).view(np.float32)
    u = wj / np.float32(np.linalg.norm(wj))
    noise = rng.standard_normal(K, dtype=np.float32) / np.float32(np.sqrt(K))
    h_strong = np.float32(24.0) * u + np.float32(8.0) * noise
    h_mod = np.float32(8.0) * (np.float32(0.3) * u + np.float32(np.sqrt(0.91)) * noise)
    h_rand = rng.standard_normal(K, dtype=np.float32) / np.float32(np.sqrt(K))
    return E, np.stack([h_strong, h_mod, h_rand]).astype(np.float32)


def screen_fixture(ref):
    from oracle_lib import or_screen_build
    E, H = screen_inputs()
    W4, S4, coef = or_screen_build(E)
    M, lim = H.shape[0], 30000
    L = np.empty(M, np.float32)
    cnt = np.empty(M, np.int32)
    surv = np.zeros((M, lim), np.int32)
    from oracle_lib import or_seed_bound
    seeds = np.array([123457, 2, 106, 1024], np.int32)  # the planted row is among the seeds, as a draft token would be
    pre = np.array([or_seed_bound(W4, S4, coef, H[m], seeds) for m in range(M)], np.float32)
    ref.ref_screen_1536(ptr(W4), ptr(S4), ptr(coef), ptr(np.ascontiguousarray(H)), M, ptr(pre), ptr(L), ptr(cnt),
                        ptr(surv), lim)
    lists = {f"surv{m}": (np.sort(surv[m, :cnt[m]]) if cnt[m] >= 0 else np.zeros(0, np.int32)) for m in range(M)}
    np.savez_compressed(HERE / "screen_1536.npz", seed=np.int32(7), L=L, cnt=cnt, pre=pre, seeds=seeds,
                        coef_sum=np.float64(coef.astype(np.float64).sum()), **lists)


if __name__ == "__main__":
    if "--screen-only" in sys.argv:
        screen_fixture(reference())
    else:
        main()
