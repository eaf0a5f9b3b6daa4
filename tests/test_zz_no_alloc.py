"""The allocation-free attention entry point, g4_attn_splitkv_noalloc, through the C ABI.

It exists for callers that cannot give the library device memory: a host application whose own
arena owns every byte of device memory, or a decode thread that must not call cudaMalloc/cudaFree
because those can synchronise the whole device.  Its scratch is a fixed device global inside
libg4.so, shared by every call.  This file is collected last (test_zz_*) so that a failure here
leaves every other test already run; it passes alone in a fresh process as well.
"""
import ctypes

import numpy as np
import pytest

from oracle_lib import bf16_bits

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402


def _inputs(rng, ctx, M, sliding, hd=256, nh=8):
    Kc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
    Vc = bf16_bits(rng.standard_normal((ctx, hd), dtype=np.float32))
    q = (rng.standard_normal((M, nh, hd), dtype=np.float32) * np.float32(0.0625)).astype(np.float32)
    pos = np.arange(ctx - M, ctx, dtype=np.int32)
    lo = (np.maximum(0, pos - 511) if sliding else np.zeros(M)).astype(np.int32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    return dev(Kc.view(np.int16)), dev(Vc.view(np.int16)), dev(q), pos, lo


def _noalloc(Kc, Vc, q, pos, lo, T=8):
    M, nh, hd = q.shape
    out = torch.empty_like(q)
    ia = (ctypes.c_int * 4)(*map(int, pos))
    la = (ctypes.c_int * 4)(*map(int, lo))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = g4.lib().g4_attn_splitkv_noalloc(ctypes.c_void_p(Kc.data_ptr()), ctypes.c_void_p(Vc.data_ptr()),
                                          ctypes.c_void_p(q.data_ptr()), ia, la, M, nh, hd, int(min(lo)),
                                          int(max(pos)), T, ctypes.c_void_p(out.data_ptr()), stream)
    return rc, out


def _close(a, b):
    """The tolerance the attention tests use: relative 1e-3 (here the two paths run the same
    kernels on the same inputs, so the results are also identical)."""
    a = a.cpu().numpy().astype(np.float64)
    b = b.cpu().numpy().astype(np.float64)
    scale = np.maximum(np.abs(b), np.sqrt(np.mean(b ** 2)))
    return float(np.max(np.abs(a - b) / scale))


def test_noalloc_matches_workspace_entry_point_twice():
    rng = np.random.default_rng(2026)
    for ctx, M, sliding in [(6856, 4, False), (700, 3, True)]:  # two calls in a row share the scratch
        Kc, Vc, q, pos, lo = _inputs(rng, ctx, M, sliding)
        rc, out = _noalloc(Kc, Vc, q, pos, lo)
        assert rc == 0, g4.lib().g4_last_error().decode()
        ref = g4.attn_splitkv(Kc, Vc, q, pos, lo, T=8)
        torch.cuda.synchronize()
        assert _close(out, ref) <= 1e-3
        assert torch.equal(out, ref)
    assert g4.device_status() == 0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    rng = np.random.default_rng(1)
    Kc, Vc, q, pos, lo = _inputs(rng, 8200, 1, False)  # 8,200 keys > 8,192
    rc, _ = _noalloc(Kc, Vc, q, pos, lo)
    assert rc == -5
    assert b"exceed the fixed scratch" in g4.lib().g4_last_error()


@pytest.mark.parametrize("hd", [128, 256])
def test_noalloc_at_the_bound_of_its_scratch(hd):
    """The largest call the fixed scratch serves: 8,192 keys (kmax - kmin + 1), M=4, nh=8, T=8,
    for both head widths; identical to the workspace entry point."""
    rng = np.random.default_rng(8192 + hd)
    Kc, Vc, q, pos, lo = _inputs(rng, 8192, 4, False, hd=hd)
    assert int(max(pos)) - int(min(lo)) + 1 == 8192
    rc, out = _noalloc(Kc, Vc, q, pos, lo, T=8)
    assert rc == 0, g4.lib().g4_last_error().decode()
    ref = g4.attn_splitkv(Kc, Vc, q, pos, lo, T=8)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert g4.device_status() == 0


@pytest.mark.parametrize("hd,T", [(256, 9), (512, 8)])
def test_noalloc_rejects_more_chunks_or_wider_heads(hd, T):
    """T = 9 chunks and hd = 512 are valid for the workspace entry point but beyond the fixed
    scratch: G4_ERR_UNSUPPORTED, nothing launched."""
    rng = np.random.default_rng(hd + T)
    Kc, Vc, q, pos, lo = _inputs(rng, 600, 2, False, hd=hd)
    rc, _ = _noalloc(Kc, Vc, q, pos, lo, T=T)
    assert rc == -5
    assert b"exceed the fixed scratch" in g4.lib().g4_last_error()
