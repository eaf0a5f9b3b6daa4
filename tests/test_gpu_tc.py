"""The tensor-core W4A8 GEMM (tcgen05.mma kind::i8 with tensor-memory accumulators, the prefill
path) against the M <= 8 GEMV path and the oracle: integer-exact group dots and the same fp32 chain
per (weight row, activation row), so every output is bit-identical, including ragged last tiles of
activation rows (zero-filled by the tensor-map loads)."""
import numpy as np
import pytest

from oracle_lib import or_w4a8, w4g32_weights

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def gemv_rows(Wp, S, q, sx, sm):
    """The GEMV path, 8 activation rows per call."""
    M = q.shape[0]
    out = []
    for m0 in range(0, M, 8):
        out.append(g4.w4a8_gemm(Wp, S, q[m0:m0 + 8].contiguous(), sx[m0:m0 + 8].contiguous(), sm[m0:m0 + 8].contiguous()))
    return torch.cat(out)


@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (128, 256, 2048), (300, 2560, 2048), (77, 2048, 8192),
                                   (1000, 384, 2048)])
def test_tc_gemm_matches_gemv_path(M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    W, S = w4g32_weights(rng, N, K)
    X = rng.standard_normal((M, K), dtype=np.float32)
    Wp = g4.w4_pack(torch.from_numpy(W).cuda())
    Sd = torch.from_numpy(S).cuda()
    q, sx, sm = g4.w4a8_quant(torch.from_numpy(X).cuda())
    Yt = g4.w4a8_gemm_tc(Wp, Sd, q, sx).cpu().numpy()
    Yg = gemv_rows(Wp, Sd, q, sx, sm).cpu().numpy()
    assert np.array_equal(bits(Yt), bits(Yg))
    if M * N * K <= 128 * 256 * 2048:
        assert np.array_equal(bits(Yt), bits(or_w4a8(W, S, X)))
    assert g4.device_status() == 0
