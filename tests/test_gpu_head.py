"""Output head on the GPU against the oracle (pinned to the reference's bf16p::pack / rows_tile /
head_task / screen_task by tests/test_oracle_golden.py): codebook, pack bytes, exact logits,
greedy pick with the softcap tie rule, int4 screen build, and the certified screen with
rescoring and fallback.  Argmax indices and survivor sets must be bit-exact (north_star)."""
import pathlib

import numpy as np
import pytest

from oracle_lib import (bf16_bits, bf16_to_f32, or_codebook, or_head_logits, or_pack, or_pick, or_screen_build,
                        or_screen_row)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from g4pkg import g4  # noqa: E402

GOLD = pathlib.Path(__file__).resolve().parent / "golden"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def to_device_layout(W):
    N, Kh = W.shape
    t = np.empty((N, 2 * Kh), np.uint8)
    t[:, 0::2] = W & 15
    t[:, 1::2] = W >> 4
    t = t.reshape(N, -1, 32)
    return (t[:, :, :16] | (t[:, :, 16:] << 4)).reshape(N, Kh)


@pytest.fixture(scope="module", autouse=True)
def _init():
    g4.device_init()


def test_pack_and_logits_golden():
    d = np.load(GOLD / "bf16p.npz")
    E = d["E"]
    N, K = E.shape
    head = g4.PackedHead(dev(E.view(np.int16)))
    assert head.cb_host == bytes(d["cb"])
    assert np.array_equal(head.data.cpu().numpy(), d["data"])
    assert np.array_equal(head.exc_ptr.cpu().numpy(), d["exc_ptr"])
    ne = len(d["exc_col"])
    assert head.n_exc == ne
    assert np.array_equal(head.exc_col.cpu().numpy()[:ne].view(np.uint16), d["exc_col"])
    assert np.array_equal(bits(head.exc_delta.cpu().numpy()[:ne]), bits(d["exc_delta"]))
    Y = head.logits(dev(d["X"])).cpu().numpy()
    assert np.array_equal(bits(Y), bits(d["Y"]))
    idx = g4.head_argmax(dev(Y)).cpu().numpy()
    assert list(idx) == [or_pick(Y[m]) for m in range(Y.shape[0])]


@pytest.mark.parametrize("N", [192, 1000, 4099])
def test_logits_kernel_variants_agree(N, monkeypatch):
    """The tensor-map-fed head GEMV (default), the direct-load one and the staged octet one compute
    the same bits for M = 1..4, including a ragged last block of rows, and match the oracle."""
    rng = np.random.default_rng(N)
    K = 2048
    E = bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    head = g4.PackedHead(dev(E.view(np.int16)))
    packed = (head.data.cpu().numpy(), head.exc_ptr.cpu().numpy(),
              head.exc_col.cpu().numpy()[:head.n_exc].view(np.uint16), head.exc_delta.cpu().numpy()[:head.n_exc])
    for M in (1, 2, 3, 4):
        X = (rng.standard_normal((M, K), dtype=np.float32) / np.float32(45.0)).astype(np.float32)
        Yo = or_head_logits(packed, np.frombuffer(head.cb_host, np.uint8), N, K, X)
        outs = []
        for variant in (None, "direct", "octet"):
            if variant is None:
                monkeypatch.delenv("G4_HEAD_GEMV", raising=False)
            else:
                monkeypatch.setenv("G4_HEAD_GEMV", variant)
            outs.append(head.logits(dev(X)).cpu().numpy())
        monkeypatch.delenv("G4_HEAD_GEMV", raising=False)
        outs.append(head.logits_unpacked(dev(X)).cpu().numpy())
        outs.append(head.logits_nib(dev(X)).cpu().numpy())
        for Y in outs:
            assert np.array_equal(bits(Y), bits(Yo)), M


def test_unpacked_layout():
    """The unpacked copy: each weight as bf16p::pack represents it (codebook exponent), as bf16,
    half h's 16 weights in bytes 32h..32h+31 (octets 0, 2, 1, 3; elements 8o+4h..8o+4h+3)."""
    d = np.load(GOLD / "bf16p.npz")
    head = g4.PackedHead(dev(d["E"].view(np.int16)))
    unp = head.unpacked().cpu().numpy().reshape(-1, 64).view(np.uint16)
    data = np.asarray(d["data"]).reshape(-1, 44)
    cb = np.frombuffer(head.cb_host, np.uint8)
    sm = data[:, :32].astype(np.uint32)
    planes = data[:, 32:44].copy().view(np.uint32)
    e = np.arange(32, dtype=np.uint32)
    codes = ((planes[:, 0:1] >> e) & 1) | (((planes[:, 1:2] >> e) & 1) << 1) | (((planes[:, 2:3] >> e) & 1) << 2)
    ex = cb[codes].astype(np.uint32)
    w = ((sm & 0x80) << 8) | (ex << 7) | (sm & 0x7F)
    order = [8 * o + 4 * h + k for h in range(2) for o in (0, 2, 1, 3) for k in range(4)]
    assert np.array_equal(unp, w[:, order].astype(np.uint16))


def test_nibble_layout():
    """The split-nibble copy: sign/mantissa bytes [N][G/4][2][4][16] (per 4 groups the half-0 parts,
    then the half-1 parts; octets 0, 2, 1, 3, elements 8o+4h..8o+4h+3), then the exponent codes
    [N][G][16] as nibbles (half h's 16 at byte 8h) in the same order."""
    d = np.load(GOLD / "bf16p.npz")
    head = g4.PackedHead(dev(d["E"].view(np.int16)))
    nib = head.nibbled().cpu().numpy()
    data = np.asarray(d["data"]).reshape(-1, 44)
    ng = data.shape[0]
    sm_n = nib[: ng * 32].reshape(ng // 4, 2, 4, 16).transpose(0, 2, 1, 3).reshape(ng, 32)
    cd_n = nib[ng * 32:].reshape(ng, 16)
    planes = data[:, 32:44].copy().view(np.uint32)
    e = np.arange(32, dtype=np.uint32)
    codes = ((planes[:, 0:1] >> e) & 1) | (((planes[:, 1:2] >> e) & 1) << 1) | (((planes[:, 2:3] >> e) & 1) << 2)
    order = [8 * o + 4 * h + k for h in range(2) for o in (0, 2, 1, 3) for k in range(4)]
    assert np.array_equal(sm_n, data[:, :32][:, order])
    c = codes[:, order].astype(np.uint8)
    assert np.array_equal(cd_n, (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8))


def test_pick_tie_rule():
    raw = np.zeros((2, 4096), np.float32)
    raw[0, [70, 900, 3000]] = [5.0, 5.0009766, 5.0]  # equal after bf16 rounding: lowest index wins
    raw[1, [11, 12]] = [-1.0, 7.0]
    raw[1, 4000] = 7.01  # bf16(7.01) == 7.0
    idx = g4.head_argmax(dev(raw)).cpu().numpy()
    assert list(idx) == [or_pick(raw[0]), or_pick(raw[1])] == [70, 12]


@pytest.fixture(scope="module")
def full_head():
    """262144 x 2048 bf16 head ~ N(0, 0.02), packed and screened on the GPU and by the oracle."""
    rng = np.random.default_rng(262144)
    N, K = 262144, 2048
    E = bf16_bits(rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02))
    Ed = dev(E.view(np.int16))
    head = g4.PackedHead(Ed)
    screen = g4.screen_build(Ed)
    torch.cuda.synchronize()
    return E, head, screen, rng, or_screen_build(E)


def test_full_pack_and_screen_build(full_head):
    E, head, screen, _, oscreen = full_head
    cb = or_codebook(E)
    assert head.cb_host == bytes(cb)
    data, ep, col, dl = or_pack(E, cb)
    assert head.n_exc == len(col)
    assert np.array_equal(head.exc_ptr.cpu().numpy(), ep)
    assert np.array_equal(head.data.cpu().numpy(), data)
    W4, S4, coef = oscreen
    assert np.array_equal(screen[0].cpu().numpy(), to_device_layout(W4))
    assert np.array_equal(screen[1].cpu().numpy().view(np.uint16), S4)
    assert np.array_equal(bits(screen[2].cpu().numpy()), bits(coef))


def oracle_logits_full(head, H):
    """The oracle's exact logits of H over every row of the head (OpenMP over rows)."""
    N, K = head.N, head.K
    packed = (head.data.cpu().numpy(), head.exc_ptr.cpu().numpy(),
              head.exc_col.cpu().numpy()[:head.n_exc].view(np.uint16), head.exc_delta.cpu().numpy()[:head.n_exc])
    return or_head_logits(packed, np.frombuffer(head.cb_host, np.uint8), N, K, np.ascontiguousarray(H, np.float32))


def test_screen_random_rows_fall_back_to_exact_argmax(full_head):
    """configs[2] as specified: h ~ N(0,1)/sqrt(2048), M = 4.  Every row survives the bound, so the
    screen falls back to the full exact head, whose argmax must equal the oracle's."""
    E, head, screen, rng, _ = full_head
    N, K = E.shape
    H = (rng.standard_normal((4, K), dtype=np.float32) / np.float32(np.sqrt(K))).astype(np.float32)
    idx, ns = g4.head_screen(screen, head, dev(H))
    idx, ns = idx.cpu().numpy(), ns.cpu().numpy()
    assert list(ns) == [-1, -1, -1, -1]
    Y = head.logits(dev(H)).cpu().numpy()
    Yo = oracle_logits_full(head, H)  # all 262,144 rows
    assert np.array_equal(bits(Y), bits(Yo))
    assert list(idx) == [or_pick(Yo[m]) for m in range(4)]
    assert list(g4.head_argmax(dev(Y)).cpu().numpy()) == list(idx)


def test_screen_planted_winners(full_head):
    """Planted hidden states (h along a head row): the screen keeps few rows, the survivor count
    equals the oracle's, and the winner is the exact-head winner."""
    E, head, screen, rng, (W4, S4, coef) = full_head
    N, K = E.shape
    H = []
    for j, (a, b) in zip([123457, 5], [(24.0, 8.0), (2.4, 7.6)]):
        w = bf16_to_f32(E[j])
        u = w / np.float32(np.linalg.norm(w))
        noise = rng.standard_normal(K, dtype=np.float32) / np.float32(np.sqrt(K))
        H.append((np.float32(a) * u + np.float32(b) * noise).astype(np.float32))
    H = np.stack(H)
    idx, ns = g4.head_screen(screen, head, dev(H))
    idx, ns = idx.cpu().numpy(), ns.cpu().numpy()
    Y = oracle_logits_full(head, H)  # the oracle's logits over all 262,144 rows
    survs = [or_screen_row(W4, S4, coef, H[m])[0] for m in range(2)]
    # the batch falls back as a whole when any row has more than lim survivors (as the reference
    # falls back for the whole verify group when any evaluated row overflows)
    fallback = any(sv is None for sv in survs)
    for m in range(2):
        assert ns[m] == (-1 if fallback else len(survs[m])), (m, ns[m], [None if v is None else len(v) for v in survs])
        assert idx[m] == or_pick(Y[m])
    assert idx[0] == 123457 and survs[0] is not None and list(survs[0]) == [123457]
    # the strong plant alone never falls back: one survivor
    idx1, ns1 = g4.head_screen(screen, head, dev(H[:1]))
    assert int(ns1.cpu()[0]) == 1 and int(idx1.cpu()[0]) == 123457
