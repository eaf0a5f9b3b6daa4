"""W4G32 / W4A8 CUDA kernels through the C ABI against the CPU oracle, bit for bit.

The oracle (oracle/liboracle.so) is itself pinned to the reference's compiled kernels by
tests/test_oracle_golden.py, so bit-equality here is bit-equality with the reference.  The
north_star tolerance for float GEMV outputs (relative 1e-3) is also asserted explicitly.
"""
import pathlib
import zlib

import numpy as np
import pytest

from oracle_lib import or_quant, or_w4a8, or_w4g32, w4g32_weights

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

GOLD = pathlib.Path(__file__).resolve().parent / "golden"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def ref_layout_to_device(W):
    """numpy restatement of the device layout: per group byte b = t[b] | t[16+b] << 4."""
    N, Kh = W.shape
    t = np.empty((N, 2 * Kh), np.uint8)
    t[:, 0::2] = W & 15
    t[:, 1::2] = W >> 4
    t = t.reshape(N, -1, 32)
    return (t[:, :, :16] | (t[:, :, 16:] << 4)).reshape(N, Kh)


def rel_err(y, ref):
    scale = np.maximum(np.abs(ref), np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    return float(np.max(np.abs(y.astype(np.float64) - ref) / scale))


def test_pack_layout():
    rng = np.random.default_rng(1)
    W, _ = w4g32_weights(rng, 64, 2048)
    Wp = g4.w4_pack(dev(W)).cpu().numpy()
    assert np.array_equal(Wp, ref_layout_to_device(W))


@pytest.mark.parametrize("case", [f"c{i}" for i in range(5)])
def test_golden_fixtures(case):
    d = np.load(GOLD / f"gemm_{case}.npz")
    W, S, X = d["W"], d["S"], d["X"]
    Wp = g4.w4_pack(dev(W))
    Y = g4.w4g32_gemm(Wp, dev(S), dev(X)).cpu().numpy()
    assert np.array_equal(bits(Y), bits(d["Y_w4g32"]))
    q, sx, sm = g4.w4a8_quant(dev(X))
    assert np.array_equal(q.cpu().numpy(), d["q"])
    assert np.array_equal(bits(sx.cpu().numpy()), bits(d["sx"]))
    assert np.array_equal(sm.cpu().numpy(), d["sum"])
    Yi = g4.w4a8_gemm(Wp, dev(S), q, sx, sm).cpu().numpy()
    assert np.array_equal(bits(Yi), bits(d["Y_w4a8"]))


def test_quant_edges():
    d = np.load(GOLD / "quant_edges.npz")
    q, sx, sm = g4.w4a8_quant(dev(d["X"]))
    assert np.array_equal(q.cpu().numpy(), d["q"])
    assert np.array_equal(bits(sx.cpu().numpy()), bits(d["sx"]))
    assert np.array_equal(sm.cpu().numpy(), d["sum"])


# the 8192 x 2048 GEMV; configs[1]: the decoder layer's projection shapes.
CFG1 = {"q": (2048, 2048), "k": (256, 2048), "v": (256, 2048), "o": (2048, 2048),
        "gate_up": (16384, 2048), "down": (2048, 8192)}


@pytest.mark.parametrize("M", [1, 2, 3, 4, 8])
def test_w4g32_cfg0(M):
    rng = np.random.default_rng(100 + M)
    W, S = w4g32_weights(rng, 8192, 2048)
    X = rng.standard_normal((M, 2048), dtype=np.float32)
    Y = g4.w4g32_gemm(g4.w4_pack(dev(W)), dev(S), dev(X)).cpu().numpy()
    ref = or_w4g32(W, S, X)
    assert rel_err(Y, ref) <= 1e-3
    assert np.array_equal(bits(Y), bits(ref))


@pytest.mark.parametrize("N,K", [(16384, 2048), (20011, 2048), (16500, 4096)])
def test_w4g32_tall_variants(N, K, monkeypatch):
    """Tall matrices (the head screen's shape class, N >= 16384) take the tensor-map-fed kernel by
    default; the row-per-thread kernel and the generic CTA-per-rows kernel must give the same
    bits, for M = 1..4, a ragged last row block and an output stride ldy > N."""
    rng = np.random.default_rng(N + K)
    W, S = w4g32_weights(rng, N, K)
    Wp, Sd = g4.w4_pack(dev(W)), dev(S)
    for M in (1, 2, 3, 4):
        X = rng.standard_normal((M, K), dtype=np.float32)
        ref = or_w4g32(W, S, X)
        for variant in (None, "direct", "0"):
            if variant is None:
                monkeypatch.delenv("G4_W4G32_ROWS", raising=False)
            else:
                monkeypatch.setenv("G4_W4G32_ROWS", variant)
            out = torch.full((M, N + 13), -7.0, device="cuda")
            g4.w4g32_gemm(Wp, Sd, dev(X), out=out[:, :N])
            Y = out.cpu().numpy()
            assert np.array_equal(bits(Y[:, :N]), bits(ref)), (M, variant)
            assert np.all(Y[:, N:] == -7.0), (M, variant)
        monkeypatch.delenv("G4_W4G32_ROWS", raising=False)


def test_w4g32_precomputed_gsum_and_ldy():
    rng = np.random.default_rng(7)
    W, S = w4g32_weights(rng, 1000, 4096)
    X = rng.standard_normal((4, 4096), dtype=np.float32)
    Xd = dev(X)
    out = torch.full((4, 1024), -7.0, device="cuda")
    g4.w4g32_gemm(g4.w4_pack(dev(W)), dev(S), Xd, gsum=g4.w4g32_gsum(Xd), out=out[:, :1000])
    Y = out.cpu().numpy()
    assert np.array_equal(bits(Y[:, :1000]), bits(or_w4g32(W, S, X)))
    assert np.all(Y[:, 1000:] == -7.0)


@pytest.mark.parametrize("name", list(CFG1))
@pytest.mark.parametrize("M", [1, 2, 4, 8])
def test_w4a8_cfg1(name, M):
    N, K = CFG1[name]
    rng = np.random.default_rng(zlib.crc32(f"{name}{M}".encode()))
    W, S = w4g32_weights(rng, N, K)
    X = rng.standard_normal((M, K), dtype=np.float32)
    q, sx, sm = g4.w4a8_quant(dev(X))
    qo, sxo, smo = or_quant(X)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(bits(sx.cpu().numpy()), bits(sxo))
    assert np.array_equal(sm.cpu().numpy(), smo)
    Y = g4.w4a8_gemm(g4.w4_pack(dev(W)), dev(S), q, sx, sm).cpu().numpy()
    ref = or_w4a8(W, S, X)
    assert np.array_equal(bits(Y), bits(ref))
    if M in (1, 4):
        Yf = g4.w4g32_gemm(g4.w4_pack(dev(W)), dev(S), dev(X)).cpu().numpy()
        assert np.array_equal(bits(Yf), bits(or_w4g32(W, S, X)))


def test_invalid_shapes_are_rejected():
    x = torch.zeros((9, 64), device="cuda")
    w = torch.zeros((8, 32), dtype=torch.uint8, device="cuda")
    s = torch.zeros((8, 2), dtype=torch.int16, device="cuda")
    with pytest.raises(g4.G4Error):
        g4.w4g32_gemm(w, s, x)  # M = 9 > 8
