"""Split-KV decode attention through the C ABI against the oracle (itself pinned to the
reference's attn_task + attn_merge) and the golden fixtures.

Bit-exact except where the merge rescale uses expf: glibc's expf and the correctly rounded exp
used on the GPU differ by one ulp in ~6e-4 of arguments, so the test requires bit equality for
at least 99.9% of outputs and the north_star tolerance (relative 1e-3) for all of them.
"""
import pathlib

import numpy as np
import pytest

from oracle_lib import bf16_bits, or_attn

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

GOLD = pathlib.Path(__file__).resolve().parent / "golden"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check(out, ref):
    out = np.asarray(out, np.float32)
    same = out.view(np.uint32) == ref.view(np.uint32)
    scale = np.maximum(np.abs(ref), np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    rel = float(np.max(np.abs(out.astype(np.float64) - ref) / scale))
    assert rel <= 1e-3, rel
    assert same.mean() >= 0.999, (same.mean(), rel)
    return same.mean()


@pytest.mark.parametrize("case", [f"c{i}" for i in range(4)])
def test_attention_golden(case):
    d = np.load(GOLD / f"attn_{case}.npz")
    out = g4.attn_splitkv(dev(d["K"].view(np.int16)), dev(d["V"].view(np.int16)), dev(d["q"]), d["pos"], d["lo"],
                          T=int(d["T"])).cpu().numpy()
    check(out, d["out"])
    assert g4.device_status() == 0


@pytest.mark.parametrize("ctx", [512, 2048, 6856])
@pytest.mark.parametrize("M", [1, 4])
@pytest.mark.parametrize("sliding", [False, True])
def test_attention_cfg3(ctx, M, sliding):
    rng = np.random.default_rng(ctx * 10 + M + 100 * sliding)
    hd, nh = 256, 8
    Kc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
    Vc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
    q = (rng.standard_normal((M, nh, hd), dtype=np.float32) * np.float32(0.0625)).astype(np.float32)
    pos = np.arange(ctx - M, ctx, dtype=np.int32)
    lo = (np.maximum(0, pos - 511) if sliding else np.zeros(M)).astype(np.int32)
    out = g4.attn_splitkv(dev(Kc.view(np.int16)), dev(Vc.view(np.int16)), dev(q), pos, lo, T=8).cpu().numpy()
    check(out, or_attn(Kc, Vc, q, pos, lo, 8))


def test_attention_ragged_rows_and_tiny_context():
    """Rows with different windows, a context shorter than the chunk count, one key."""
    rng = np.random.default_rng(5)
    hd, nh = 256, 8
    for ctx, pos, lo in [(5, [2, 3, 4], [0, 0, 1]), (1, [0], [0]), (600, [597, 598, 599], [86, 87, 88])]:
        Kc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
        Vc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
        q = rng.standard_normal((len(pos), nh, hd), dtype=np.float32)
        out = g4.attn_splitkv(dev(Kc.view(np.int16)), dev(Vc.view(np.int16)), dev(q), pos, lo, T=8).cpu().numpy()
        check(out, or_attn(Kc, Vc, q, np.array(pos, np.int32), np.array(lo, np.int32), 8))


def test_attention_workspace_too_small():
    q = torch.zeros((1, 8, 256), device="cuda")
    kv = torch.zeros((16, 256), dtype=torch.int16, device="cuda")
    with pytest.raises(g4.G4Error):
        g4.attn_splitkv(kv, kv, q, [15], [0], ws=torch.zeros(4, device="cuda"))


@pytest.mark.parametrize("ctx,M,nh,T", [(9000, 2, 8, 8), (3000, 4, 3, 2), (777, 1, 5, 7), (13000, 1, 8, 8)])
def test_attention_long_chunks_and_odd_head_counts(ctx, M, nh, T):
    """Chunks longer than the statistics kernel's register tile (9,000 keys in 8 chunks; 3,000 in
    2), chunks longer than the chunk kernel serves (13,000 keys: the three-kernel tail), head
    counts that leave (row, head) groups partly empty, and an odd chunk count."""
    rng = np.random.default_rng(ctx + nh)
    hd = 256
    Kc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
    Vc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
    q = (rng.standard_normal((M, nh, hd), dtype=np.float32) * np.float32(0.0625)).astype(np.float32)
    pos = np.arange(ctx - M, ctx, dtype=np.int32)
    lo = np.zeros(M, np.int32)
    out = g4.attn_splitkv(dev(Kc.view(np.int16)), dev(Vc.view(np.int16)), dev(q), pos, lo, T=T).cpu().numpy()
    check(out, or_attn(Kc, Vc, q, pos, lo, T))
    assert g4.device_status() == 0


def test_attention_rejects_unaligned_cache():
    kv = torch.zeros((17, 256), dtype=torch.int16, device="cuda")
    q = torch.zeros((1, 8, 256), device="cuda")
    with pytest.raises(g4.G4Error):
        g4.attn_splitkv(kv.view(-1)[1:].view(-1)[: 16 * 256].view(16, 256), kv, q, [15], [0])
