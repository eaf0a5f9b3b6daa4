"""Row RMS norm (+ W4A8 quantisation) on the GPU against the oracle, bit for bit.

The kernel sums the squares of a row in the reference's 16 ordered partials; a partial whose
elements are bf16-valued with an exponent span of at most 15 is summed as a tree (exact, so equal
to the sequential sum), any other partial by the sequential chain.  The rows below take both paths:
Gaussian bf16 rows (tree), rows with tiny and huge elements (chain), rows that are not bf16-valued
(chain), mixed rows, zeros and subnormals."""
import numpy as np
import pytest

from oracle_lib import bf16_to_f32, bf16_bits, or_quant, or_rmsnorm

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def r16(a):
    return bf16_to_f32(bf16_bits(np.ascontiguousarray(a, np.float32)))


def rows(n, rng):
    g = r16(rng.standard_normal((1, n), dtype=np.float32))
    wide = r16(rng.standard_normal((1, n), dtype=np.float32))
    wide[0, ::7] *= np.float32(2.0 ** -20)  # spans of about 20 binades: sequential chains
    wide[0, 5::11] *= np.float32(2.0 ** 12)
    mixed = g.copy()
    mixed[0, 3] = np.float32(2.0 ** -40)  # one partial (3) takes the chain, the others the tree
    plain = rng.standard_normal((1, n), dtype=np.float32)  # not bf16-valued: every partial chains
    zeros = np.zeros((1, n), np.float32)
    sub = r16(rng.standard_normal((1, n), dtype=np.float32))
    sub[0, ::3] = bf16_to_f32(np.array([0x0001, 0x8003, 0x007F], np.uint16)[rng.integers(0, 3, n // 3 + 1)][: len(sub[0, ::3])])
    small = r16(rng.standard_normal((1, n), dtype=np.float32) * np.float32(1e-30))
    return np.concatenate([g, wide, mixed, plain, zeros, sub, small])


@pytest.mark.parametrize("n", [256, 1536, 2048])
@pytest.mark.parametrize("round_", [0, 1])
def test_rmsnorm_rows_match_oracle(n, round_):
    rng = np.random.default_rng(n + round_)
    X = rows(n, rng)
    w = (np.float32(1.0) + np.float32(0.1) * rng.standard_normal(n, dtype=np.float32)).astype(np.float32)
    Y, q, sx, sm = g4.rmsnorm(dev(X), dev(w), round_=bool(round_), quant=True)
    Yo = or_rmsnorm(X, w, round_)
    assert np.array_equal(bits(Y.cpu().numpy()), bits(Yo))
    qo, sxo, smo = or_quant(Yo)
    assert np.array_equal(q.cpu().numpy(), qo)
    assert np.array_equal(bits(sx.cpu().numpy()), bits(sxo))
    assert np.array_equal(sm.cpu().numpy(), smo)


def test_rmsnorm_without_quantisation_and_many_rows():
    rng = np.random.default_rng(5)
    X = r16(rng.standard_normal((37, 2048), dtype=np.float32) * np.float32(3.0))
    w = rng.standard_normal(2048, dtype=np.float32)
    Y = g4.rmsnorm(dev(X), dev(w))
    assert np.array_equal(bits(Y.cpu().numpy()), bits(or_rmsnorm(X, w, 0)))
