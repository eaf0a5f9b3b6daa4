"""The plain-C oracle against the reference's own compiled kernels (tests/golden fixtures).

Every comparison is bit-exact: the fixtures were produced by oracle/_ref/libg4ref.so, the
reference sources compiled with the reference's build flags (tests/golden/make_golden.py).
"""
import pathlib

import numpy as np
import pytest

from oracle_lib import (bf16_bits, oracle, or_attn, or_calc_thr, or_codebook, or_head_logits, or_pack,
                        or_pick, or_quant, or_screen_build, or_screen_row, or_seed_bound, or_w4a8, or_w4g32,
                        ptr)

GOLD = pathlib.Path(__file__).resolve().parent / "golden"


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("case", [f"c{i}" for i in range(5)])
def test_w4g32_and_w4a8_golden(case):
    d = np.load(GOLD / f"gemm_{case}.npz")
    W, S, X = d["W"], d["S"], d["X"]
    assert np.array_equal(bits(or_w4g32(W, S, X)), bits(d["Y_w4g32"]))
    q, sx, sm = or_quant(X)
    assert np.array_equal(q, d["q"])
    assert np.array_equal(bits(sx), bits(d["sx"]))
    assert np.array_equal(sm, d["sum"])
    assert np.array_equal(bits(or_w4a8(W, S, X)), bits(d["Y_w4a8"]))


def test_quant_edges_golden():
    d = np.load(GOLD / "quant_edges.npz")
    q, sx, sm = or_quant(d["X"])
    assert np.array_equal(q, d["q"])
    assert np.array_equal(bits(sx), bits(d["sx"]))
    assert np.array_equal(sm, d["sum"])


def test_bf16p_pack_and_head_golden():
    d = np.load(GOLD / "bf16p.npz")
    E = d["E"]
    N, K = E.shape
    cb = or_codebook(E)
    assert np.array_equal(cb, d["cb"])
    packed = or_pack(E, cb)
    data, ep, col, dl = packed
    assert np.array_equal(data, d["data"])
    assert np.array_equal(ep, d["exc_ptr"])
    assert np.array_equal(col, d["exc_col"])
    assert np.array_equal(bits(dl), bits(d["exc_delta"]))
    Y = or_head_logits(packed, cb, N, K, d["X"])
    assert np.array_equal(bits(Y), bits(d["Y"]))
    # argmax with the softcap tie rule: lowest index among equal capped bf16 logits
    for m in range(Y.shape[0]):
        r = np.array([oracle().or_r16(float(v)) for v in Y[m]], np.float32)
        caps = np.array([oracle().or_cap(float(v)) for v in r], np.float32)
        mx = r.max()
        want = int(np.nonzero((r >= mx - 2) & (caps == oracle().or_cap(float(mx))))[0][0])
        assert or_pick(Y[m]) == want


def test_pick_tie_rule_lowest_index():
    raw = np.zeros(16, np.float32)
    raw[[3, 9, 12]] = [5.0, 5.0009766, 5.0]  # equal after bf16 rounding (bf16 step at 5 is 1/32)
    assert or_pick(raw) == 3
    raw[3] = 4.0
    assert or_pick(raw) == 9


@pytest.mark.parametrize("case", [f"c{i}" for i in range(4)])
def test_attention_golden(case):
    d = np.load(GOLD / f"attn_{case}.npz")
    out = or_attn(d["K"], d["V"], d["q"], d["pos"], d["lo"], int(d["T"]))
    assert np.array_equal(bits(out), bits(d["out"]))


def test_exp8_gelu_golden():
    d = np.load(GOLD / "exp8_gelu.npz")
    o = oracle()
    x = d["x"]
    e = np.array([o.or_exp8(float(v)) for v in np.minimum(x, 0)], np.float32)
    g = np.array([o.or_gelu(float(v)) for v in x], np.float32)
    assert np.array_equal(bits(e), bits(d["exp8"]))
    assert np.array_equal(bits(g), bits(d["gelu"]))


def test_calc_thr_is_bucket_floor():
    """calc_thr(L) + 0.25 is the lowest z whose capped bf16 value equals cap(r16(L))."""
    o = oracle()
    for L in [0.0, 1.3, 7.77, 25.0, 29.0, -3.0]:
        t = or_calc_thr(L) + 0.25
        assert o.or_cap(o.or_r16(t)) == o.or_cap(o.or_r16(L))


@pytest.mark.slow
def test_screen_against_reference_screen_task():
    """The reference's screen_task at its hard-coded 262144 x 1536 (fixture), against the
    schedule-free restatement: same L per row and the same survivor set."""
    import sys
    sys.path.insert(0, str(GOLD))
    from make_golden import screen_inputs
    d = np.load(GOLD / "screen_1536.npz")
    E, H = screen_inputs(int(d["seed"]))
    W4, S4, coef = or_screen_build(E)
    assert abs(float(coef.astype(np.float64).sum()) - float(d["coef_sum"])) == 0.0
    for m in range(H.shape[0]):
        assert or_seed_bound(W4, S4, coef, H[m], d["seeds"]) == d["pre"][m]
        surv, L = or_screen_row(W4, S4, coef, H[m])
        assert bits(np.float32(L)) == bits(d["L"][m])
        if d["cnt"][m] >= 0:
            assert surv is not None and np.array_equal(surv, d[f"surv{m}"])
    # planted winner: the single survivor is the planted row
    assert list(d["surv0"]) == [123457]
