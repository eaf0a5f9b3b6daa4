"""Python binding of libg4.so, the C ABI declared in include/g4.h.

This is the host-side mirror of the reference's kernel-header operator surface
(engine/w4g32_avx2.h, engine/w4a8_avx2.h, engine/bf16_exp3_head.h and the engine tasks of
engine/gemma4_engine.cpp): the same operations under the same names, taking torch CUDA tensors
(device memory and the current stream are torch's; the arithmetic is the library's sm_100a
kernels).  There is no CPU fallback: loading fails loudly when libg4.so is missing.
"""
import ctypes
import pathlib

PKG_ROOT = pathlib.Path(__file__).resolve().parent.parent
LIB_PATH = PKG_ROOT / "libg4.so"

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); every entry point of include/g4.h
SIGNATURES = {
    "g4_last_error": (ctypes.c_char_p, []),
    "g4_abi_version": (_I, []),
    "g4_device_status": (_I, [ctypes.POINTER(ctypes.c_uint), _I]),
    "g4_w4_pack": (_I, [_P, _I, _I, _P, _P]),
    "g4_w4g32_gsum": (_I, [_P, _I, _I, _P, _P]),
    "g4_w4g32_gemm": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _I, _P]),
    "g4_w4a8_quant": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "g4_w4a8_gemm": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _I, _P]),
    "g4_w4a8_gemm_tc_ws_bytes": (_SZ, [_I, _I, _I]),
    "g4_w4a8_gemm_tc": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _I, _P, _SZ, _P]),
    "g4_device_init": (_I, []),
    "g4_bf16p_codebook": (_I, [_P, ctypes.c_longlong, _P, _P, _SZ, _P]),
    "g4_bf16p_count": (_I, [_P, _I, _I, _P, _P, _P, _SZ, ctypes.POINTER(ctypes.c_longlong), _P]),
    "g4_bf16p_pack": (_I, [_P, _I, _I, _P, _P, _P, _P, _P, _P]),
    "g4_bf16p_gemm": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _I, _P, _I, _P]),
    "g4_head_argmax": (_I, [_P, _I, _I, _I, _P, _P, _SZ, _P]),
    "g4_rmsnorm": (_I, [_P, _P, _I, _I, _P, _I, _P, _P, _P, _P]),
    "g4_bf16p_unpack": (_I, [_P, _P, _I, _I, _P, _P]),
    "g4_head_screen_shard_bound": (_I, [_P, _P, _P, _I, _I, _P, _I, _I, _P, _P, _SZ, _P]),
    "g4_head_screen_shard_select": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _P, _SZ, _P]),
    "g4_head_screen_shard_pick": (_I, [_I, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "g4_head_screen_dist_ws_bytes": (_SZ, [_I, _I, _I]),
    "g4_bf16p_nib_bytes": (_SZ, [_I, _I]),
    "g4_bf16p_nib_pack": (_I, [_P, _I, _I, _P, _P]),
    "g4_bf16p_nib_gemm": (_I, [_P, _P, _P, _P, _P, _I, _I, _P, _I, _P, _I, _P]),
    "g4_head_screen_dist": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _I, _I, _P, _P, _SZ, _P]),
    "g4_nccl_get_unique_id": (_I, [_P]),
    "g4_nccl_comm_init": (_I, [_P, _I, _I, _P]),
    "g4_nccl_comm_destroy": (_I, [_P]),
    "g4_bf16p_unpacked_gemm": (_I, [_P, _P, _P, _P, _I, _I, _P, _I, _P, _I, _P]),
    "g4_screen_build": (_I, [_P, _I, _I, _P, _P, _P, _P]),
    "g4_head_screen_ws_bytes": (_SZ, [_I, _I, _I]),
    "g4_head_screen": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _SZ, _P]),
    "g4_engine_default_config": (_I, [_P]),
    "g4_engine_create": (_I, [_P, _P]),
    "g4_engine_destroy": (None, [_P]),
    "g4_engine_forward": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P]),
    "g4_engine_draft": (_I, [_P, _I, _P, _I, _I, _P, _P]),
    "g4_engine_generate": (_I, [_P, _P, _I, _I, _P, _P, _P]),
    "g4_engine_fake_ctx": (_I, [_P, _I]),
    "g4_engine_prefill": (_I, [_P, _P, _I, _P]),
    "g4_engine_prefill_from": (_I, [_P, _P, _I, _I, _P]),
    "g4_engine_set_k_draft": (_I, [_P, _I]),
    "g4_engine_request": (_I, [_P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "g4_engine_decode": (_I, [_P, _I, _I, _P, _P, _P]),
    "g4_engine_phase_times": (_I, [_P, _I, _P, _P]),
    "g4_engine_trace": (_I, [_P, _P, _I, _P]),
    "g4_engine_create_shared": (_I, [_P, _P, _P]),
    "g4_checkpoint_open": (_I, [ctypes.c_char_p, ctypes.c_char_p, _P]),
    "g4_checkpoint_close": (None, [_P]),
    "g4_checkpoint_count": (_I, [_P]),
    "g4_checkpoint_tensor": (_I, [_P, ctypes.c_char_p, ctypes.c_char_p, _I, _P, _I, _P, _P]),
    "g4_checkpoint_config": (_I, [_P, _P]),
    "g4_engine_create_from_checkpoint": (_I, [_P, _P, _P]),
    "g4_engine_copy_state": (_I, [_P, _P]),
    "g4_engine_decode_async": (_I, [_P, _I, _I, _P]),
    "g4_engine_decode_wait": (_I, [_P, _P, _P, _P, _P, _P]),
    "g4_engine_time_verify": (_I, [_P, _I, _I, _P]),
    "g4_engine_seg_trace": (_I, [_P, _P, _I, _P]),
    "g4_engine_export_state": (_I, [_P, _I, _P, _P, _P, _I, _P, _P, _P]),
    "g4_attn_splitkv_ws_bytes": (_SZ, [_I, _I, _I, _I, _I, _I]),
    "g4_attn_splitkv": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P, _SZ, _P]),
    "g4_attn_splitkv_noalloc": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _P]),
}


class G4Error(RuntimeError):
    pass


_lib = None


def lib():
    """The loaded libg4.so with argument types set; raises when it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise G4Error(f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                          f"(make -C {PKG_ROOT}); g4 has no CPU fallback")
        lib_ = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib_, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib_
    return _lib


def check(rc, what):
    if rc != 0:
        raise G4Error(f"{what} failed ({rc}): {lib().g4_last_error().decode()}")


def device_status(reset=True):
    """OR of the device status words (bit 0: a bounded device wait gave up)."""
    v = ctypes.c_uint(0)
    check(lib().g4_device_status(ctypes.byref(v), int(reset)), "g4_device_status")
    return v.value


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dev(t, name):
    if not t.is_cuda or not t.is_contiguous():
        raise G4Error(f"{name} must be a contiguous CUDA tensor")
    return t


# ------------------------------------------------------------------ W4G32 / W4A8 operators
def w4_pack(W):
    """Reference W4 layout uint8 [N, K/2] -> device layout (load-time, like w4a8::repack_tiles)."""
    import torch
    _dev(W, "W")
    N, Kh = W.shape
    Wp = torch.empty_like(W)
    check(lib().g4_w4_pack(_ptr(W), N, 2 * Kh, _ptr(Wp), _stream()), "g4_w4_pack")
    return Wp


def w4g32_gsum(X):
    import torch
    _dev(X, "X")
    M, K = X.shape
    gs = torch.empty((M, K // 32), dtype=torch.float32, device=X.device)
    check(lib().g4_w4g32_gsum(_ptr(X), M, K, _ptr(gs), _stream()), "g4_w4g32_gsum")
    return gs


def w4g32_gemm(Wp, S, X, gsum=None, out=None):
    """Y[M, N] = W4G32(Wp, S) @ X[M, K]^T, fp32 order of w4::gemm_rows_tile<MT>."""
    import torch
    for t, n in ((Wp, "Wp"), (S, "S"), (X, "X")):
        _dev(t, n)
    M, K = X.shape
    N = Wp.shape[0]
    Y = out if out is not None else torch.empty((M, N), dtype=torch.float32, device=X.device)
    check(lib().g4_w4g32_gemm(_ptr(Wp), _ptr(S), _ptr(X), _ptr(gsum), M, N, K, _ptr(Y), Y.stride(0), _stream()),
          "g4_w4g32_gemm")
    return Y


def w4a8_gemm_tc(Wp, S, q, sx, out=None):
    """The W4A8 GEMM on the tensor cores (tcgen05 kind::i8) for any M: the same values as
    w4a8_gemm."""
    import torch
    M, K = q.shape
    N = Wp.shape[0]
    Y = out if out is not None else torch.empty((M, N), dtype=torch.float32, device=q.device)
    nb = lib().g4_w4a8_gemm_tc_ws_bytes(M, N, K)
    ws = torch.empty(nb, dtype=torch.uint8, device=q.device)
    for t, n in ((Wp, "Wp"), (S, "S"), (q, "q"), (sx, "sx"), (Y, "Y")):
        _dev(t, n)
    check(lib().g4_w4a8_gemm_tc(_ptr(Wp), _ptr(S), _ptr(q), _ptr(sx), M, N, K, _ptr(Y), N, _ptr(ws), nb, _stream()),
          "g4_w4a8_gemm_tc")
    return Y


def rmsnorm(X, w, round_=False, quant=False):
    """Y = (X * r) * w per row (bf16-rounded when round_), and with quant the W4A8 quantisation of
    Y as (q, sx, sum); r in the order of the reference's rms."""
    import torch
    _dev(X, "X")
    _dev(w, "w")
    M, n = X.shape
    Y = torch.empty((M, n), dtype=torch.float32, device=X.device)
    if quant:
        q = torch.empty((M, n), dtype=torch.int8, device=X.device)
        sx = torch.empty((M, n // 32), dtype=torch.float32, device=X.device)
        sm = torch.empty((M, n // 32), dtype=torch.int32, device=X.device)
    else:
        q = sx = sm = None
    check(lib().g4_rmsnorm(_ptr(X), _ptr(w), M, n, _ptr(Y), int(round_), _ptr(q), _ptr(sx), _ptr(sm), _stream()),
          "g4_rmsnorm")
    return (Y, q, sx, sm) if quant else Y


def w4a8_quant(X):
    """(q int8 [M, K], sx fp32 [M, K/32], sum int32 [M, K/32]) exactly as w4a8::quant."""
    import torch
    _dev(X, "X")
    M, K = X.shape
    q = torch.empty((M, K), dtype=torch.int8, device=X.device)
    sx = torch.empty((M, K // 32), dtype=torch.float32, device=X.device)
    sm = torch.empty((M, K // 32), dtype=torch.int32, device=X.device)
    check(lib().g4_w4a8_quant(_ptr(X), M, K, _ptr(q), _ptr(sx), _ptr(sm), _stream()), "g4_w4a8_quant")
    return q, sx, sm


def w4a8_gemm(Wp, S, q, sx, sm, out=None):
    """Y[M, N] with integer-exact group dots and the fp32 scale chain of w4a8::tile<MT>."""
    import torch
    M, K = q.shape
    N = Wp.shape[0]
    Y = out if out is not None else torch.empty((M, N), dtype=torch.float32, device=q.device)
    check(lib().g4_w4a8_gemm(_ptr(Wp), _ptr(S), _ptr(q), _ptr(sx), _ptr(sm), M, N, K, _ptr(Y), Y.stride(0),
                             _stream()), "g4_w4a8_gemm")
    return Y


# ------------------------------------------------------------------ split-KV attention
def attn_splitkv(Kc, Vc, q, pos, lo, T=8, ws=None, out=None):
    """q [M, nh, hd] fp32 CUDA; Kc/Vc [ctx, hd] int16 (bf16 bits) CUDA; pos/lo host int lists."""
    import torch
    M, nh, hd = q.shape
    pos = list(map(int, pos))
    lo = list(map(int, lo))
    kmin, kmax = min(lo), max(pos)
    need = lib().g4_attn_splitkv_ws_bytes(M, nh, hd, kmin, kmax, T)
    if ws is None:
        ws = torch.empty(need // 4 + 4, dtype=torch.float32, device=q.device)
    out = out if out is not None else torch.empty_like(q)
    ia = (ctypes.c_int * 4)(*pos)
    la = (ctypes.c_int * 4)(*lo)
    check(lib().g4_attn_splitkv(_ptr(Kc), _ptr(Vc), _ptr(q), ia, la, M, nh, hd, kmin, kmax, T, _ptr(out), _ptr(ws),
                                ws.numel() * ws.element_size(), _stream()), "g4_attn_splitkv")
    return out


# ------------------------------------------------------------------ output head
def device_init():
    check(lib().g4_device_init(), "g4_device_init")


class PackedHead:
    """bf16-exp3 packed head on the device (bf16p::Packed): data, codebook, CSR exceptions."""

    def __init__(self, E):
        import torch
        _dev(E, "E")
        N, K = E.shape
        self.N, self.K = N, K
        ws = torch.empty(max(2048, 8 * N), dtype=torch.uint8, device=E.device)
        cb = (ctypes.c_uint8 * 8)()
        check(lib().g4_bf16p_codebook(_ptr(E), E.numel(), cb, _ptr(ws), ws.numel(), _stream()), "g4_bf16p_codebook")
        self.cb_host = bytes(cb)
        self.cb = ctypes.create_string_buffer(self.cb_host, 8)
        self.exc_ptr = torch.empty(N + 1, dtype=torch.int64, device=E.device)
        total = ctypes.c_longlong(0)
        check(lib().g4_bf16p_count(_ptr(E), N, K, self.cb, _ptr(self.exc_ptr), _ptr(ws), ws.numel(), ctypes.byref(total),
                                   _stream()), "g4_bf16p_count")
        self.n_exc = total.value
        self.data = torch.empty(N * (K // 32) * 44, dtype=torch.uint8, device=E.device)
        self.exc_col = torch.empty(max(1, self.n_exc), dtype=torch.int16, device=E.device)
        self.exc_delta = torch.empty(max(1, self.n_exc), dtype=torch.float32, device=E.device)
        check(lib().g4_bf16p_pack(_ptr(E), N, K, self.cb, _ptr(self.data), _ptr(self.exc_ptr), _ptr(self.exc_col),
                                  _ptr(self.exc_delta), _stream()), "g4_bf16p_pack")

    def args(self):
        return (_ptr(self.data), self.cb, _ptr(self.exc_ptr), _ptr(self.exc_col), _ptr(self.exc_delta))

    def logits(self, X, out=None):
        import torch
        M = X.shape[0]
        Y = out if out is not None else torch.empty((M, self.N), dtype=torch.float32, device=X.device)
        check(lib().g4_bf16p_gemm(*self.args(), self.N, self.K, _ptr(X), M, _ptr(Y), Y.stride(0), _stream()),
              "g4_bf16p_gemm")
        return Y

    def unpacked(self):
        """The unpacked copy of the head (g4_bf16p_unpack), made on first use."""
        import torch
        if getattr(self, "_unp", None) is None:
            self._unp = torch.empty(self.N * (self.K // 32) * 64, dtype=torch.uint8, device=self.data.device)
            check(lib().g4_bf16p_unpack(_ptr(self.data), self.cb, self.N, self.K, _ptr(self._unp), _stream()),
                  "g4_bf16p_unpack")
        return self._unp

    def logits_unpacked(self, X, out=None):
        """logits() through the unpacked copy (g4_bf16p_unpacked_gemm): the same values."""
        import torch
        M = X.shape[0]
        Y = out if out is not None else torch.empty((M, self.N), dtype=torch.float32, device=X.device)
        check(lib().g4_bf16p_unpacked_gemm(_ptr(self.unpacked()), _ptr(self.exc_ptr), _ptr(self.exc_col),
                                           _ptr(self.exc_delta), self.N, self.K, _ptr(X), M, _ptr(Y), Y.stride(0),
                                           _stream()), "g4_bf16p_unpacked_gemm")
        return Y


def _nib_methods():
    def nibbled(self):
        """The split-nibble copy of the head (g4_bf16p_nib_pack), made on first use."""
        import torch
        if getattr(self, "_nib", None) is None:
            nb = lib().g4_bf16p_nib_bytes(self.N, self.K)
            self._nib = torch.empty(nb, dtype=torch.uint8, device=self.data.device)
            check(lib().g4_bf16p_nib_pack(_ptr(self.data), self.N, self.K, _ptr(self._nib), _stream()),
                  "g4_bf16p_nib_pack")
        return self._nib

    def logits_nib(self, X, out=None):
        """logits() through the split-nibble copy (g4_bf16p_nib_gemm): the same values."""
        import torch
        M = X.shape[0]
        Y = out if out is not None else torch.empty((M, self.N), dtype=torch.float32, device=X.device)
        check(lib().g4_bf16p_nib_gemm(_ptr(self.nibbled()), self.cb, _ptr(self.exc_ptr), _ptr(self.exc_col),
                                      _ptr(self.exc_delta), self.N, self.K, _ptr(X), M, _ptr(Y), Y.stride(0), _stream()),
              "g4_bf16p_nib_gemm")
        return Y
    PackedHead.nibbled = nibbled
    PackedHead.logits_nib = logits_nib


_nib_methods()


class ScreenShard:
    """One shard of the head for the vocab-parallel screen: rows row0 .. row0 + N of E (bf16 on the
    device), its packed rows, its unpacked copy and its int4 screen copy, and the workspace that
    the three phases share."""

    def __init__(self, E_rows, row0, lim=30000, M=4, unpacked=True):
        import torch
        _dev(E_rows, "E_rows")
        self.N, self.K = E_rows.shape
        self.row0, self.lim, self.M = int(row0), int(lim), int(M)
        self.head = PackedHead(E_rows)
        self.unp = self.head.unpacked() if unpacked and self.K % 64 == 0 else None
        self.screen = screen_build(E_rows)
        nb = lib().g4_head_screen_ws_bytes(self.M, self.N, self.lim)
        self.ws = torch.empty(nb // 4 + 64, dtype=torch.float32, device=E_rows.device)
        self.ws_bytes = self.ws.numel() * 4

    def bound(self, H):
        import torch
        M = H.shape[0]
        L = torch.empty(M, dtype=torch.float32, device=H.device)
        W4, S4, coef = self.screen
        check(lib().g4_head_screen_shard_bound(_ptr(W4), _ptr(S4), _ptr(coef), self.N, self.K, _ptr(H), M, self.lim,
                                               _ptr(L), _ptr(self.ws), self.ws_bytes, _stream()),
              "g4_head_screen_shard_bound")
        return L

    def select(self, H, L):
        import torch
        M = H.shape[0]
        vmax = torch.empty(M, dtype=torch.float32, device=H.device)
        ns = torch.empty(M, dtype=torch.int32, device=H.device)
        h = self.head
        check(lib().g4_head_screen_shard_select(_ptr(self.screen[2]), _ptr(h.data), _ptr(self.unp), h.cb, _ptr(h.exc_ptr),
                                                _ptr(h.exc_col), _ptr(h.exc_delta), self.N, self.K, _ptr(H), M, self.lim,
                                                _ptr(L), _ptr(vmax), _ptr(ns), _ptr(self.ws), self.ws_bytes, _stream()),
              "g4_head_screen_shard_select")
        return vmax, ns

    def pick(self, gmax):
        import torch
        M = gmax.shape[0]
        idx = torch.empty(M, dtype=torch.int32, device=gmax.device)
        check(lib().g4_head_screen_shard_pick(self.N, M, self.lim, self.row0, _ptr(gmax), _ptr(idx), _ptr(self.ws),
                                              self.ws_bytes, _stream()), "g4_head_screen_shard_pick")
        return idx


INT_MAX = 0x7FFFFFFF


class NcclComm:
    """A communicator of the library (g4_nccl_comm_init) over the ranks of a torch.distributed group:
    rank 0's unique id is broadcast through the group."""

    def __init__(self, dist_=None, group=None):
        """dist_ None: a communicator of this process alone (one rank)."""
        import torch
        if dist_ is None:
            uid = torch.zeros(128, dtype=torch.uint8)
            check(lib().g4_nccl_get_unique_id(ctypes.c_void_p(uid.data_ptr())), "g4_nccl_get_unique_id")
            self.h = ctypes.c_void_p()
            check(lib().g4_nccl_comm_init(ctypes.c_void_p(uid.data_ptr()), 1, 0, ctypes.byref(self.h)), "g4_nccl_comm_init")
            self.rank, self.world = 0, 1
            return
        rank, world = dist_.get_rank(group), dist_.get_world_size(group)
        uid = torch.zeros(128, dtype=torch.uint8)
        if rank == 0:
            check(lib().g4_nccl_get_unique_id(ctypes.c_void_p(uid.data_ptr())), "g4_nccl_get_unique_id")
        uid_d = uid.cuda()
        dist_.broadcast(uid_d, src=0, group=group)
        uid = uid_d.cpu()
        self.h = ctypes.c_void_p()
        check(lib().g4_nccl_comm_init(ctypes.c_void_p(uid.data_ptr()), world, rank, ctypes.byref(self.h)),
              "g4_nccl_comm_init")
        self.rank, self.world = rank, world

    def close(self):
        if self.h:
            lib().g4_nccl_comm_destroy(self.h)
            self.h = ctypes.c_void_p()


def screen_dist_native(shard, H, comm, root=0, out=None):
    """The vocab-parallel screen in one library call (g4_head_screen_dist) over a NcclComm."""
    import torch
    M = H.shape[0]
    idx = out if out is not None else torch.empty(M, dtype=torch.int32, device=H.device)
    nb = lib().g4_head_screen_dist_ws_bytes(M, shard.N, shard.lim)
    if getattr(shard, "_dist_ws", None) is None or shard._dist_ws.numel() < nb:
        shard._dist_ws = torch.empty(nb + 256, dtype=torch.uint8, device=H.device)
    ws = shard._dist_ws
    W4, S4, coef = shard.screen
    h = shard.head
    check(lib().g4_head_screen_dist(comm.h, root, _ptr(W4), _ptr(S4), _ptr(coef), _ptr(h.data), _ptr(shard.unp), h.cb,
                                    _ptr(h.exc_ptr), _ptr(h.exc_col), _ptr(h.exc_delta), shard.N, shard.K, shard.row0,
                                    _ptr(H), M, shard.lim, _ptr(idx), _ptr(ws), ws.numel(), _stream()),
          "g4_head_screen_dist")
    return idx


def screen_sharded(shards, H):
    """The vocab-parallel screen with every shard on this process (the reductions done here):
    winners [M] (-1 = none) and survivors per shard [G][M] (-1 = that shard fell back)."""
    import torch
    L = torch.stack([s.bound(H) for s in shards]).max(0).values
    sel = [s.select(H, L) for s in shards]
    gmax = torch.stack([v for v, _ in sel]).max(0).values
    idx = torch.stack([s.pick(gmax) for s in shards]).min(0).values
    idx = torch.where(idx == INT_MAX, torch.full_like(idx, -1), idx)
    return idx, torch.stack([n for _, n in sel])


def screen_shard_dist(shard, H, dist_, group=None, src=0):
    """The vocab-parallel screen with one shard per rank of a torch.distributed group (NCCL over
    NVLink on GPUs): H is broadcast from `src`, then the bound, the candidate max and the winner
    index are all-reduced between the phases.  Returns the winners [M] (-1 = none) on every rank."""
    phases = _ShardPhases(shard)
    return screen_dist(phases, H, dist_, group, src)


class _ShardPhases:
    def __init__(self, shard):
        self.s = shard

    def bound(self, H):
        return self.s.bound(H)

    def select(self, H, L):
        return self.s.select(H, L)[0]

    def pick(self, gmax):
        return self.s.pick(gmax)


def screen_dist(phases, H, dist_, group=None, src=0):
    """The collective skeleton of the vocab-parallel screen over any object with bound / select /
    pick (the device phases on a GPU; a host restatement in the CPU tests)."""
    import torch
    dist_.broadcast(H, src=src, group=group)
    L = phases.bound(H)
    dist_.all_reduce(L, op=dist_.ReduceOp.MAX, group=group)
    vmax = phases.select(H, L)
    dist_.all_reduce(vmax, op=dist_.ReduceOp.MAX, group=group)
    idx = phases.pick(vmax)
    dist_.all_reduce(idx, op=dist_.ReduceOp.MIN, group=group)
    return torch.where(idx == INT_MAX, torch.full_like(idx, -1), idx)


def head_argmax(Y):
    import torch
    M, N = Y.shape
    out = torch.empty(M, dtype=torch.int32, device=Y.device)
    ws = torch.empty(2 * M, dtype=torch.int32, device=Y.device)
    check(lib().g4_head_argmax(_ptr(Y), M, N, Y.stride(0), _ptr(out), _ptr(ws), ws.numel() * 4, _stream()),
          "g4_head_argmax")
    return out


def screen_build(E):
    import torch
    N, K = E.shape
    W4 = torch.empty((N, K // 2), dtype=torch.uint8, device=E.device)
    S4 = torch.empty((N, K // 32), dtype=torch.int16, device=E.device)
    coef = torch.empty(N, dtype=torch.float32, device=E.device)
    check(lib().g4_screen_build(_ptr(E), N, K, _ptr(W4), _ptr(S4), _ptr(coef), _stream()), "g4_screen_build")
    return W4, S4, coef


def head_screen(screen, head, H, lim=30000):
    """Certified screen + rescoring + pick for hidden rows H [M, K]; returns (idx, nsurv)."""
    import torch
    W4, S4, coef = screen
    M, K = H.shape
    need = lib().g4_head_screen_ws_bytes(M, head.N, lim)
    ws = torch.empty(need, dtype=torch.uint8, device=H.device)
    idx = torch.empty(M, dtype=torch.int32, device=H.device)
    ns = torch.empty(M, dtype=torch.int32, device=H.device)
    check(lib().g4_head_screen(_ptr(W4), _ptr(S4), _ptr(coef), *head.args(), head.N, K, _ptr(H), M, lim, _ptr(idx),
                               _ptr(ns), _ptr(ws), need, _stream()), "g4_head_screen")
    return idx, ns


# ------------------------------------------------------------------ speculative decode engine
class EngineConfig(ctypes.Structure):
    """g4_engine_config (include/g4.h)."""
    _fields_ = [(n, ctypes.c_int) for n in ("hidden", "n_layers", "mlp", "vocab", "ctx_max", "prefill_block", "k_draft",
                                            "ngram", "ngram_len", "prefill_int8", "decode_int8", "head_screen",
                                            "screen_lim", "attn_chunks", "att_par", "drafter")] + [
        ("seed", ctypes.c_ulonglong), ("graphs", ctypes.c_int), ("fused_layers", ctypes.c_int),
        ("prefill_tc", ctypes.c_int), ("slots", ctypes.c_int), ("slot_min_reuse", ctypes.c_int),
        ("kv_owners", ctypes.c_int), ("mlp_shared", ctypes.c_int), ("ple", ctypes.c_int)]


class EngineStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("rounds", "ngram_rounds", "drafted", "accepted", "prefill_tokens",
                                            "decode_tokens")] + [("prefill_ms", ctypes.c_double),
                                                                 ("decode_ms", ctypes.c_double),
                                                                 ("decode_gpu_ms", ctypes.c_double)] + [
        (n, ctypes.c_int) for n in ("verify_passes", "verify_rows", "draft_steps")] + [
        ("verify_gpu_ms", ctypes.c_double), ("draft_gpu_ms", ctypes.c_double), ("h2d_bytes", ctypes.c_longlong),
        ("d2h_bytes", ctypes.c_longlong), ("kernel_launches", ctypes.c_longlong), ("head_fallbacks", ctypes.c_int),
        ("screen_skipped", ctypes.c_int), ("ngram_accepted", ctypes.c_int)]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


TOKEN_CB = ctypes.CFUNCTYPE(None, ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_void_p)


class RequestInfo(ctypes.Structure):
    """g4_request_info (include/g4.h)."""
    _fields_ = [(n, ctypes.c_int) for n in ("prompt_tokens", "reused", "slot", "tokens")] + [
        ("prefill_ms", ctypes.c_double), ("decode_ms", ctypes.c_double)] + [
        (n, ctypes.c_int) for n in ("slot_switches", "slot_evictions", "kv_len", "rounds", "ngram_rounds",
                                    "ngram_accepted")]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


def engine_config(**kw):
    c = EngineConfig()
    check(lib().g4_engine_default_config(ctypes.byref(c)), "g4_engine_default_config")
    for k, v in kw.items():
        setattr(c, k, v)
    return c


class Checkpoint:
    """A checkpoint in the reference's format (g4_checkpoint_* in include/g4.h): model.safetensors
    read through the reference's index file (make_index.py's lines) or the safetensors header."""

    def __init__(self, path, index=None):
        self.h = ctypes.c_void_p()
        check(lib().g4_checkpoint_open(str(path).encode(), None if index is None else str(index).encode(),
                                       ctypes.byref(self.h)), "g4_checkpoint_open")

    def close(self):
        if self.h:
            lib().g4_checkpoint_close(self.h)
            self.h = ctypes.c_void_p()

    def __len__(self):
        return lib().g4_checkpoint_count(self.h)

    def tensor(self, name):
        """(dtype, shape, nbytes) of one tensor."""
        dt = ctypes.create_string_buffer(16)
        shape = (ctypes.c_longlong * 8)()
        nd, nb = ctypes.c_int(0), ctypes.c_longlong(0)
        check(lib().g4_checkpoint_tensor(self.h, name.encode(), dt, 16, shape, 8, ctypes.byref(nd), ctypes.byref(nb)),
              "g4_checkpoint_tensor")
        return dt.value.decode(), tuple(shape[i] for i in range(nd.value)), nb.value

    def config(self, cfg=None, **kw):
        """An EngineConfig with the checkpoint's model sizes (g4_checkpoint_config)."""
        cfg = cfg if cfg is not None else engine_config(**kw)
        check(lib().g4_checkpoint_config(self.h, ctypes.byref(cfg)), "g4_checkpoint_config")
        return cfg


class Engine:
    """The speculative greedy-decode engine (g4_engine_* in include/g4.h)."""

    def __init__(self, cfg=None, share=None, checkpoint=None, **kw):
        """share: another Engine whose weights this one uses (an independent request stream);
        checkpoint: a Checkpoint whose target weights the engine loads (its model sizes replace
        the configuration's)."""
        self.cfg = cfg if cfg is not None else engine_config(**kw)
        self.h = ctypes.c_void_p()
        if checkpoint is not None:
            check(lib().g4_engine_create_from_checkpoint(ctypes.byref(self.cfg), checkpoint.h, ctypes.byref(self.h)),
                  "g4_engine_create_from_checkpoint")
            checkpoint.config(self.cfg)
        elif share is not None:
            check(lib().g4_engine_create_shared(ctypes.byref(self.cfg), share.h, ctypes.byref(self.h)),
                  "g4_engine_create_shared")
        else:
            check(lib().g4_engine_create(ctypes.byref(self.cfg), ctypes.byref(self.h)), "g4_engine_create")

    def close(self):
        if self.h:
            lib().g4_engine_destroy(self.h)
            self.h = ctypes.c_void_p()

    def forward(self, toks, pos0, want=True, hf=0, int8=True):
        import numpy as np
        toks = np.ascontiguousarray(toks, np.int32)
        M = toks.size
        G = np.full(M, -1, np.int32)
        hb = np.zeros((M, self.cfg.hidden), np.float32)
        check(lib().g4_engine_forward(self.h, toks.ctypes.data_as(_P), M, pos0, int(want), hf, int(int8),
                                      G.ctypes.data_as(_P), hb.ctypes.data_as(_P)), "g4_engine_forward")
        return G, hb

    def draft(self, tok, h, pos, P):
        import numpy as np
        h = np.ascontiguousarray(h, np.float32)
        out = np.zeros(1, np.int32)
        hn = np.zeros(self.cfg.hidden, np.float32)
        check(lib().g4_engine_draft(self.h, int(tok), h.ctypes.data_as(_P), pos, P, out.ctypes.data_as(_P),
                                    hn.ctypes.data_as(_P)), "g4_engine_draft")
        return int(out[0]), hn

    def fake_ctx(self, n):
        """Fill KV positions [0, n) with the reference's ENGINE_FAKE_CTX values; the next prefill
        starts at position n."""
        check(lib().g4_engine_fake_ctx(self.h, int(n)), "g4_engine_fake_ctx")

    def prefill(self, prompt, start=0):
        """start > 0: keep the K/V of positions < start (g4_engine_prefill_from)."""
        import numpy as np
        prompt = np.ascontiguousarray(prompt, np.int32)
        first = ctypes.c_int(0)
        check(lib().g4_engine_prefill_from(self.h, prompt.ctypes.data_as(_P), prompt.size, int(start),
                                           ctypes.byref(first)), "g4_engine_prefill_from")
        return first.value

    def request(self, prompt, max_new, on_tokens=None):
        """One request through the prefix cache (g4_engine_request): (tokens, info dict).
        on_tokens(list of ints) is called with the tokens as they commit."""
        import numpy as np
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(max(1, int(max_new)), np.int32)
        n = ctypes.c_int(0)
        info = RequestInfo()
        cb = None
        if on_tokens is not None:
            cb = TOKEN_CB(lambda p, k, _u: on_tokens([p[i] for i in range(k)]))
        check(lib().g4_engine_request(self.h, prompt.ctypes.data_as(_P), prompt.size, int(max_new),
                                      out.ctypes.data_as(_P), ctypes.byref(n), ctypes.byref(info),
                                      ctypes.cast(cb, _P) if cb is not None else None, None), "g4_engine_request")
        return out[: n.value].copy(), info.as_dict()

    def decode(self, max_rounds, max_tokens, out=None):
        import numpy as np
        n = ctypes.c_int(0)
        st = EngineStats()
        optr = out.ctypes.data_as(_P) if out is not None else None
        check(lib().g4_engine_decode(self.h, max_rounds, max_tokens, optr, ctypes.byref(n), ctypes.byref(st)),
              "g4_engine_decode")
        return n.value, st.as_dict()

    def trace(self):
        """Per-round records since the prefill as an [rounds, 6] int32 array: {nd, prompt lookup used,
        drafts[3] (-1 padded), nacc}."""
        import numpy as np
        n = ctypes.c_int(0)
        check(lib().g4_engine_trace(self.h, None, 0, ctypes.byref(n)), "g4_engine_trace")
        buf = np.zeros((max(n.value, 1), 6), np.int32)
        check(lib().g4_engine_trace(self.h, buf.ctypes.data_as(_P), n.value, ctypes.byref(n)), "g4_engine_trace")
        return buf[: n.value].copy()

    def seg_trace(self):
        """Stage timestamps (ns) of the last fused verify pass: [launch, CTA (first, last), 24]."""
        import numpy as np
        n = ctypes.c_int(0)
        check(lib().g4_engine_seg_trace(self.h, None, 0, ctypes.byref(n)), "g4_engine_seg_trace")
        buf = np.zeros(n.value, np.uint64)
        check(lib().g4_engine_seg_trace(self.h, buf.ctypes.data_as(_P), n.value, ctypes.byref(n)),
              "g4_engine_seg_trace")
        return buf.reshape(-1, 2, 24)

    def time_verify(self, M, reps=20):
        """Device ms of one verify pass of M rows at the current position (CUDA events)."""
        ms = ctypes.c_double(0)
        check(lib().g4_engine_time_verify(self.h, int(M), int(reps), ctypes.byref(ms)), "g4_engine_time_verify")
        return ms.value

    def export_state(self, npos, kv=True):
        """(K, V [n_layers, npos, 256] uint16 or None, history int32, hprev float32, P)."""
        import numpy as np
        nl = self.cfg.n_layers
        K = np.zeros((nl, npos, 256), np.uint16) if kv else None
        V = np.zeros((nl, npos, 256), np.uint16) if kv else None
        n = ctypes.c_int(0)
        P = ctypes.c_int(0)
        check(lib().g4_engine_export_state(self.h, 0, None, None, None, 0, ctypes.byref(n), None, ctypes.byref(P)),
              "g4_engine_export_state")
        seq = np.zeros(n.value, np.int32)
        h = np.zeros(self.cfg.hidden, np.float32)
        check(lib().g4_engine_export_state(self.h, int(npos) if kv else 0, K.ctypes.data_as(_P) if kv else None,
                                           V.ctypes.data_as(_P) if kv else None, seq.ctypes.data_as(_P), seq.size,
                                           ctypes.byref(n), h.ctypes.data_as(_P), ctypes.byref(P)),
              "g4_engine_export_state")
        return K, V, seq, h, P.value

    def copy_state_from(self, other):
        """Continue other's stream here (KV cache, history, hidden and round state copied)."""
        check(lib().g4_engine_copy_state(self.h, other.h), "g4_engine_copy_state")

    def decode_async(self, max_rounds, max_tokens, start_event=None):
        """Enqueue the rounds of a decode call and return (start_event: a torch.cuda.Event or None)."""
        ev = ctypes.c_void_p(start_event.cuda_event) if start_event is not None else None
        check(lib().g4_engine_decode_async(self.h, max_rounds, max_tokens, ev), "g4_engine_decode_async")

    def decode_wait(self, start_event=None):
        """Complete decode_async: (tokens, stats, device ms since start_event or None)."""
        import numpy as np
        out = np.zeros(self.cfg.ctx_max, np.int32)  # a call commits fewer tokens than the context holds
        n = ctypes.c_int(0)
        st = EngineStats()
        ms = ctypes.c_float(0)
        ev = ctypes.c_void_p(start_event.cuda_event) if start_event is not None else None
        check(lib().g4_engine_decode_wait(self.h, out.ctypes.data_as(_P), ctypes.byref(n), ctypes.byref(st), ev,
                                          ctypes.byref(ms)), "g4_engine_decode_wait")
        return out[: n.value].copy(), st.as_dict(), (ms.value if start_event is not None else None)

    PHASES = ("embed_norm_rope", "linear", "attention", "head", "drafter", "copies")

    def phase_times(self, enable=-1):
        ms = (ctypes.c_double * 6)()
        marks = (ctypes.c_longlong * 6)()
        check(lib().g4_engine_phase_times(self.h, enable, ms, marks), "g4_engine_phase_times")
        return {n: (ms[i], marks[i]) for i, n in enumerate(self.PHASES)}

    def generate(self, prompt, n_new):
        import numpy as np
        prompt = np.ascontiguousarray(prompt, np.int32)
        out = np.zeros(n_new + 8, np.int32)
        n_out = ctypes.c_int(0)
        st = EngineStats()
        check(lib().g4_engine_generate(self.h, prompt.ctypes.data_as(_P), prompt.size, n_new, out.ctypes.data_as(_P),
                                       ctypes.byref(n_out), ctypes.byref(st)), "g4_engine_generate")
        return out[: n_out.value].copy(), st.as_dict()
