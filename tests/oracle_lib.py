"""ctypes bindings for the CPU oracle (test infrastructure only).

``oracle()`` loads oracle/liboracle.so (the plain-C restatement of the reference arithmetic);
``reference()`` loads oracle/_ref/libg4ref.so (the reference's own kernels, compiled from the
reference sources by oracle/Makefile) or returns None when it was not built.
"""
import ctypes
import os
import pathlib

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent.parent
ORACLE_DIR = ROOT / "oracle"

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float


def ptr(a):
    """Raw pointer of a C-contiguous numpy array (or None)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


_SIGS_ORACLE = {
    "or_w4g32_gemm": (None, [_P, _P, _P, _I, _I, _I, _P]),
    "or_w4a8_quant": (None, [_P, _I, _I, _P, _P, _P]),
    "or_w4a8_gemm": (None, [_P, _P, _P, _P, _P, _I, _I, _I, _P]),
    "or_bf16p_codebook": (None, [_P, _I64, _P]),
    "or_bf16p_count": (_I64, [_P, _I, _I, _P, _P]),
    "or_bf16p_pack": (None, [_P, _I, _I, _P, _P, _P, _P, _P]),
    "or_bf16p_gemm": (None, [_P, _P, _P, _P, _P, _I, _I, _P, _I, _P]),
    "or_cap": (_F, [_F]),
    "or_calc_thr": (_F, [_F]),
    "or_head_pick": (_I, [_P, _I]),
    "or_screen_build": (None, [_P, _I, _I, _P, _P, _P]),
    "or_screen_row": (_I, [_P, _P, _P, _I, _I, _P, _P, _I, _I, _P, _P]),
    "or_hnorm": (_F, [_P, _I]),
    "or_seed_bound": (_F, [_P, _P, _P, _I, _P, _P, _I]),
    "or_attn_splitkv": (None, [_P, _P, _I, _I, _I, _P, _P, _P, _I, _I, _I, _P]),
    "or_exp8": (_F, [_F]),
    "or_gelu": (_F, [_F]),
    "or_r16": (_F, [_F]),
    "or_e2e_create": (_P, [_P]),
    "or_e2e_destroy": (None, [_P]),
    "or_e2e_forward": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "or_e2e_draft": (_I, [_P, _I, _P, _I, _I, _P, _P]),
    "or_e2e_generate": (_I, [_P, _P, _I, _I, _P, _P, _P]),
    "or_e2e_generate_trace": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _I]),
    "or_e2e_prefill": (_I, [_P, _P, _I, _P]),
    "or_e2e_prefill_from": (_I, [_P, _P, _I, _I, _P]),
    "or_e2e_history": (_I, [_P, _P, _I, _P, _P]),
    "or_e2e_set_k": (None, [_P, _I]),
    "or_e2e_set_layer_scalar": (None, [_P, _I, ctypes.c_float]),
    "or_e2e_write_checkpoint": (_I, [_P, ctypes.c_char_p, _I]),
    "or_e2e_decode": (_I, [_P, _I, _I, _P, _P, _P, _P, _I]),
    "or_e2e_set_state": (_I, [_P, _P, _P, _I, _P, _I, _P, _I]),
    "or_e2e_set_hooks": (_I, [_P, _P]),
    "or_e2e_gen_bytes": (None, [ctypes.c_ulonglong, ctypes.c_ulonglong, ctypes.c_longlong, _P]),
    "or_e2e_fake_ctx": (None, [_P, _I]),
    "or_rmsnorm": (None, [_P, _P, _I, _I, _P, _I]),
    "or_set_threads": (None, [_I]),
    "or_get_threads": (_I, []),
}

_SIGS_REF = {
    "ref_pool_start": (_I, [_I]),
    "ref_w4g32_gemm": (None, [_P, _P, _P, _I, _I, _I, _P]),
    "ref_w4a8_quant": (None, [_P, _I, _I, _P, _P, _P]),
    "ref_w4a8_gemm": (None, [_P, _P, _P, _I, _I, _I, _P]),
    "ref_bf16p_pack": (_I64, [_P, _I, _I, _P, _P, _P, _P, _P, _I64]),
    "ref_bf16p_gemm": (None, [_P, _I, _I, _P, _P, _I, _P]),
    "ref_attn_splitkv": (None, [_P, _P, _I, _I, _I, _P, _P, _P, _I, _I, _P]),
    "ref_screen_1536": (None, [_P, _P, _P, _P, _I, _P, _P, _P, _P, _I]),
    "ref_gelu8": (None, [_P, _I, _P]),
    "ref_lin_prepare": (_P, [_P, _P, _I, _I]),
    "ref_lin_run": (None, [_P, _P, _I, _P, _I]),
    "ref_head_prepare": (_P, [_P, _I, _I, _P]),
    "ref_head_run": (None, [_P, _P, _I, _P]),
    "ref_attn_tile_run": (None, [_P, _P, _I, _I, _P, _I, _I, _I, _P]),
    "ref_exp8": (None, [_P, _I, _P]),
}


def _load(path, sigs):
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in sigs.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_oracle = None
_ref = None


def oracle():
    global _oracle
    if _oracle is None:
        path = ORACLE_DIR / "liboracle.so"
        if not path.exists():
            raise RuntimeError(f"{path} missing: run `make -C oracle liboracle.so`")
        _oracle = _load(path, _SIGS_ORACLE)
    return _oracle


REF_THREADS = 8


def reference(threads=None):
    """The reference's own kernels, or None when oracle/_ref/libg4ref.so was not built.  The
    reference's thread pool is started on first use with `threads` threads (default: G4_REF_THREADS
    or REF_THREADS, the T = 8 that the parity fixtures use); it cannot be resized afterwards."""
    global _ref
    if _ref is None:
        path = ORACLE_DIR / "_ref" / "libg4ref.so"
        if not path.exists():
            return None
        _ref = _load(path, _SIGS_REF)
        n = threads if threads else int(os.environ.get("G4_REF_THREADS", REF_THREADS))
        _ref.pool_threads = _ref.ref_pool_start(int(n))
    return _ref


# ---------------------------------------------------------------- seeded synthetic inputs
def bf16_bits(x):
    """fp32 -> bf16 bit patterns, round to nearest even (gemma4_engine.cpp:34 without NaNs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def bf16_to_f32(b):
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def w4g32_weights(rng, N, K):
    """configs[0] distribution: int4 q uniform in [-8,7] stored as q+8 nibbles, bf16 scales |N(0,1)|*0.01."""
    t = rng.integers(0, 16, size=(N, K), dtype=np.uint8)
    W = (t[:, 0::2] | (t[:, 1::2] << 4)).astype(np.uint8)
    S = bf16_bits(np.abs(rng.standard_normal((N, K // 32), dtype=np.float32)) * np.float32(0.01))
    return np.ascontiguousarray(W), np.ascontiguousarray(S)


# ---------------------------------------------------------------- oracle wrappers
def or_w4g32(W, S, X):
    M, K = X.shape
    N = W.shape[0]
    Y = np.empty((M, N), np.float32)
    oracle().or_w4g32_gemm(ptr(W), ptr(S), ptr(X), M, N, K, ptr(Y))
    return Y


def or_rmsnorm(X, w, round_):
    X = np.ascontiguousarray(X, np.float32)
    M, n = X.shape
    Y = np.empty((M, n), np.float32)
    w = np.ascontiguousarray(w, np.float32)
    oracle().or_rmsnorm(ptr(X), ptr(w), M, n, ptr(Y), int(round_))
    return Y


def or_quant(X):
    M, K = X.shape
    q = np.empty((M, K), np.int8)
    sx = np.empty((M, K // 32), np.float32)
    sm = np.empty((M, K // 32), np.int32)
    oracle().or_w4a8_quant(ptr(X), M, K, ptr(q), ptr(sx), ptr(sm))
    return q, sx, sm


def or_w4a8(W, S, X):
    M, K = X.shape
    N = W.shape[0]
    q, sx, sm = or_quant(X)
    Y = np.empty((M, N), np.float32)
    oracle().or_w4a8_gemm(ptr(W), ptr(S), ptr(q), ptr(sx), ptr(sm), M, N, K, ptr(Y))
    return Y


def or_codebook(E):
    cb = np.zeros(8, np.uint8)
    oracle().or_bf16p_codebook(ptr(E), E.size, ptr(cb))
    return cb


def or_pack(E, cb):
    N, K = E.shape
    ep = np.zeros(N + 1, np.int64)
    ne = oracle().or_bf16p_count(ptr(E), N, K, ptr(cb), ptr(ep))
    data = np.zeros(N * (K // 32) * 44, np.uint8)
    col = np.zeros(max(ne, 1), np.uint16)
    dl = np.zeros(max(ne, 1), np.float32)
    oracle().or_bf16p_pack(ptr(E), N, K, ptr(cb), ptr(data), ptr(ep), ptr(col), ptr(dl))
    return data, ep, col[:ne], dl[:ne]


def or_head_logits(packed, cb, N, K, X):
    data, ep, col, dl = packed
    M = X.shape[0]
    Y = np.empty((M, N), np.float32)
    col_ = col if col.size else np.zeros(1, np.uint16)
    dl_ = dl if dl.size else np.zeros(1, np.float32)
    oracle().or_bf16p_gemm(ptr(data), ptr(cb), ptr(ep), ptr(col_), ptr(dl_), N, K, ptr(X), M, ptr(Y))
    return Y


def or_pick(raw_row):
    r = np.ascontiguousarray(raw_row, np.float32)
    return oracle().or_head_pick(ptr(r), r.size)


def or_screen_build(E):
    N, K = E.shape
    W4 = np.empty((N, K // 2), np.uint8)
    S4 = np.empty((N, K // 32), np.uint16)
    coef = np.empty(N, np.float32)
    oracle().or_screen_build(ptr(E), N, K, ptr(W4), ptr(S4), ptr(coef))
    return W4, S4, coef


def or_screen_row(W4, S4, coef, h, lim=30000):
    N = W4.shape[0]
    K = h.size
    surv = np.empty(lim, np.int32)
    L = np.zeros(1, np.float32)
    seeds = np.zeros(1, np.int32)
    h = np.ascontiguousarray(h, np.float32)
    c = oracle().or_screen_row(ptr(W4), ptr(S4), ptr(coef), N, K, ptr(h), ptr(seeds), 0, lim, ptr(surv), ptr(L))
    return (surv[:c].copy() if c >= 0 else None), float(L[0])


def or_attn(Kc, Vc, q, pos, lo, T=8):
    """q: [M, nh, hd] fp32; Kc/Vc: [ctx, hd] bf16 bits; returns [M, nh, hd] fp32."""
    M, nh, hd = q.shape
    pos = np.ascontiguousarray(pos, np.int32)
    lo = np.ascontiguousarray(lo, np.int32)
    kmin, kmax = int(lo.min()), int(pos.max())
    out = np.empty((M, nh, hd), np.float32)
    oracle().or_attn_splitkv(ptr(Kc), ptr(Vc), hd, nh, M, ptr(np.ascontiguousarray(q)), ptr(pos), ptr(lo),
                             kmin, kmax, T, ptr(out))
    return out


def or_seed_bound(W4, S4, coef, h, seeds):
    seeds = np.ascontiguousarray(seeds, np.int32)
    h = np.ascontiguousarray(h, np.float32)
    return oracle().or_seed_bound(ptr(W4), ptr(S4), ptr(coef), h.size, ptr(h), ptr(seeds), seeds.size)


def or_calc_thr(L):
    return oracle().or_calc_thr(float(L))


# ---------------------------------------------------------------- end-to-end oracle
class E2EConfig(ctypes.Structure):
    """The oracle's configuration: g4_engine_config's first fields (include/g4.h), then kv_owners,
    mlp_shared, ple, hd_global (head dim of the global layers, 0 = 256) and rope_global_quarter
    (proportional RoPE there)."""
    _fields_ = [(n, ctypes.c_int) for n in ("hidden", "n_layers", "mlp", "vocab", "ctx_max", "prefill_block", "k_draft",
                                            "ngram", "ngram_len", "prefill_int8", "decode_int8", "head_screen",
                                            "screen_lim", "attn_chunks", "att_par", "drafter")] + [
        ("seed", ctypes.c_ulonglong), ("kv_owners", ctypes.c_int), ("mlp_shared", ctypes.c_int),
        ("ple", ctypes.c_int), ("hd_global", ctypes.c_int), ("rope_global_quarter", ctypes.c_int)]  # the oracle's own struct


def e2e_config(**kw):
    c = E2EConfig(hidden=2048, n_layers=30, mlp=8192, vocab=262144, ctx_max=8192, prefill_block=32, k_draft=3, ngram=2,
                  ngram_len=3, prefill_int8=1, decode_int8=1, head_screen=1, screen_lim=30000, attn_chunks=8, att_par=192,
                  drafter=1, seed=20261201)
    for k, v in kw.items():
        setattr(c, k, v)
    return c


class OracleModel:
    def __init__(self, cfg):
        self.cfg = cfg
        self.h = oracle().or_e2e_create(ctypes.byref(cfg))

    def close(self):
        if self.h:
            oracle().or_e2e_destroy(self.h)
            self.h = None

    def forward(self, toks, pos0, want=True, hf=0, int8=True):
        toks = np.ascontiguousarray(toks, np.int32)
        M = toks.size
        G = np.full(M, -1, np.int32)
        hb = np.zeros((M, self.cfg.hidden), np.float32)
        oracle().or_e2e_forward(self.h, ptr(toks), M, pos0, int(want), hf, int(int8), ptr(G), ptr(hb))
        return G, hb

    def draft(self, tok, h, pos, P):
        out = np.zeros(1, np.int32)
        hn = np.zeros(self.cfg.hidden, np.float32)
        oracle().or_e2e_draft(self.h, int(tok), ptr(np.ascontiguousarray(h, np.float32)), pos, P, ptr(out), ptr(hn))
        return int(out[0]), hn

    def fake_ctx(self, n):
        oracle().or_e2e_fake_ctx(self.h, n)

    def generate(self, prompt, n_new, trace=False):
        """run_req: prefill + decode.  With trace, also the per-round records
        {nd, prompt lookup used, drafts[3] (-1 padded), nacc} as an [rounds, 6] array."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_new + 8, np.int32)
        n_out = np.zeros(1, np.int32)
        st = np.zeros(8, np.int32)
        cap = n_new + 8 if trace else 0
        tr = np.full((max(cap, 1), 6), -1, np.int32)
        oracle().or_e2e_generate_trace(self.h, ptr(prompt), prompt.size, n_new, ptr(out), ptr(n_out), ptr(st),
                                       ptr(tr) if trace else None, cap)
        stats = {"rounds": int(st[0]), "ngram_rounds": int(st[1]), "drafted": int(st[2]), "accepted": int(st[3])}
        if trace:
            return out[: n_out[0]].copy(), stats, tr[: stats["rounds"]].copy()
        return out[: n_out[0]].copy(), stats

    def prefill(self, prompt, start=0):
        """start > 0: keep the K/V of positions < start (a prefix of this prompt prefilled earlier)."""
        prompt = np.ascontiguousarray(prompt, np.int32)
        first = np.zeros(1, np.int32)
        assert oracle().or_e2e_prefill_from(self.h, ptr(prompt), prompt.size, int(start), ptr(first)) == 0
        return int(first[0])

    def set_k(self, k):
        oracle().or_e2e_set_k(self.h, int(k))

    def set_layer_scalar(self, layer, value):
        oracle().or_e2e_set_layer_scalar(self.h, int(layer), float(value))

    def write_checkpoint(self, path, packed_u8=False):
        """The model's target weights as a checkpoint in the reference's format (safetensors)."""
        assert oracle().or_e2e_write_checkpoint(self.h, str(path).encode(), int(packed_u8)) == 0

    def history(self):
        """(committed history: prompt + every committed token, last committed position P)."""
        n, P = np.zeros(1, np.int32), np.zeros(1, np.int32)
        oracle().or_e2e_history(self.h, None, 0, ptr(n), ptr(P))
        out = np.zeros(max(1, int(n[0])), np.int32)
        oracle().or_e2e_history(self.h, ptr(out), out.size, ptr(n), ptr(P))
        return out[: n[0]].copy(), int(P[0])

    def decode(self, max_rounds, max_tokens):
        out = np.zeros(max(max_tokens, 1), np.int32)
        n_out = np.zeros(1, np.int32)
        st = np.zeros(8, np.int32)
        oracle().or_e2e_decode(self.h, max_rounds, max_tokens, ptr(out), ptr(n_out), ptr(st), None, 0)
        return out[: n_out[0]].copy(), {"rounds": int(st[0]), "ngram_rounds": int(st[1]), "drafted": int(st[2]),
                                        "accepted": int(st[3])}

    def set_state(self, Kc, Vc, seq, hprev, P):
        """Decode state from another implementation's prefill: K/V [NL, npos, HD] bf16 bits, the
        committed history, the last committed row's hidden and its position."""
        Kc = np.ascontiguousarray(Kc, np.uint16)
        Vc = np.ascontiguousarray(Vc, np.uint16)
        seq = np.ascontiguousarray(seq, np.int32)
        hprev = np.ascontiguousarray(hprev, np.float32)
        rc = oracle().or_e2e_set_state(self.h, ptr(Kc), ptr(Vc), Kc.shape[1], ptr(seq), seq.size, ptr(hprev), int(P))
        if rc:
            raise RuntimeError("or_e2e_set_state rejected the state")

    def use_reference_kernels(self):
        """Route the linears, split-KV attention and exact head through the reference's own compiled
        kernels (oracle/_ref/libg4ref.so, driven by its thread pool).  Returns False when that library
        was not built."""
        ref = reference()
        if ref is None:
            return False
        hooks = (ctypes.c_void_p * 6)(*[ctypes.cast(getattr(ref, n), ctypes.c_void_p).value for n in
                                        ("ref_lin_prepare", "ref_lin_run", "ref_attn_splitkv", "ref_head_prepare",
                                         "ref_head_run", "ref_attn_tile_run")])
        self._hooks = hooks
        return oracle().or_e2e_set_hooks(self.h, ctypes.cast(hooks, ctypes.c_void_p)) == 0


STOP_TOKENS = (1, 106)  # is_stop (gemma4_engine.cpp)


class OracleConversations:
    """run_req's prefix cache (gemma4_engine.cpp:1569-1613) over oracle models, one per conversation
    (each holds its own K/V and history, as a slot does): [model, keys, kv_len, stamp] per
    conversation.  The longest shared prefix picks the conversation, a stored one that shares more
    is switched in, a prompt that shares fewer than min_reuse tokens with every conversation evicts
    the least recently used slot, and the prefill starts at min(shared, n - 1).  new_model() makes
    each conversation's model."""

    def __init__(self, new_model, slots, min_reuse):
        self.min_reuse = min_reuse
        self.active = [new_model(), [], 0, 0]
        self.stored = [[new_model(), [], 0, 0] for _ in range(slots - 1)]
        self.tick = 0

    def close(self):
        for c in [self.active] + self.stored:
            c[0].close()

    def set_k(self, k):
        for c in [self.active] + self.stored:
            c[0].set_k(k)

    @staticmethod
    def _lcp(keys, kv_len, prompt):
        c = 0
        while c < kv_len and c < len(prompt) and c < len(keys) and keys[c] == prompt[c]:
            c += 1
        return c

    def _swap(self, i):
        self.active, self.stored[i] = self.stored[i], self.active

    def request(self, prompt, max_new):
        prompt = [int(t) for t in prompt]
        n = len(prompt)
        common = self._lcp(self.active[1], self.active[2], prompt)
        self.tick += 1
        slot = 0
        if self.stored:
            best, bc = -1, common
            for i, s in enumerate(self.stored):
                c = self._lcp(s[1], s[2], prompt)
                if c > bc:
                    bc, best = c, i
            if best >= 0:
                self.active[3] = self.tick
                self._swap(best)
                slot, common = best + 1, bc
            elif bc < self.min_reuse:
                v = min(range(len(self.stored)), key=lambda i: self.stored[i][3])  # the first oldest
                self.active[3] = self.tick
                self._swap(v)
                self.active[1], self.active[2] = [], 0
                slot, common = v + 1, 0
            self.active[3] = self.tick
        start = min(common, n - 1)
        m = self.active[0]
        first = m.prefill(prompt, start)
        if max_new <= 0:  # prefill only: the prompt is the conversation
            self.active[1], self.active[2] = prompt, n
            return [], start, slot
        out = [first]
        if max_new > 1 and out[0] not in STOP_TOKENS:
            toks, _ = m.decode(1 << 30, max_new - 1)
            out += [int(t) for t in toks]
        for i, t in enumerate(out):
            if t in STOP_TOKENS:
                out = out[: i + 1]
                break
        seq, P = m.history()
        self.active[1] = [int(t) for t in seq[: P + 1]]
        self.active[2] = min(P + 1, len(self.active[1]))
        return out, start, slot


def gen_bytes(seed, tid, n):
    out = np.zeros(n, np.uint8)
    oracle().or_e2e_gen_bytes(seed, tid, n, ptr(out))
    return out


def make_prompt(seed, n, vocab=262144, copy_frac=0.2):
    """configs[4] prompt: Zipf(1.1) token ranks over the vocab (mapped through a fixed permutation),
    with about copy_frac of the positions copied from earlier 8-32-token spans so that prompt lookup
    finds matches.  Deterministic for a seed."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** -1.1
    cdf = np.cumsum(p / p.sum())
    perm = rng.permutation(vocab).astype(np.int32)
    out = np.empty(n, np.int32)
    i = 0
    while i < n:
        if i >= 64 and rng.random() < copy_frac / 20.0 * 1.0:
            L = int(rng.integers(8, 33))
            src = int(rng.integers(0, i - L)) if i - L > 0 else 0
            for k in range(L):
                if i >= n:
                    break
                out[i] = out[src + k]
                i += 1
        else:
            out[i] = perm[min(int(np.searchsorted(cdf, rng.random())), vocab - 1)]
            i += 1
    return out
