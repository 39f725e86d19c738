"""capi -- ctypes access to the C ABI of libattnb.so (include/attnb.h).

The device-pointer entry points (``*_dev``) take raw device addresses and a
CUDA stream; the helpers below accept torch CUDA tensors (torch is used only
for device memory and streams) and enqueue on the current torch stream.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libattnb.so")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_RUNTIME = 2
ERR_CUDA = 3
ERR_DEVICE_TIMEOUT = 4
ERR_OUT_OF_MEMORY = 5

PREC = {None: -1, "default": -1, "3xtf32": 0, "tf32": 1}

# Every symbol include/attnb.h declares.
EXPORTED = [
    "attnb_last_error", "attnb_version", "attnb_stream_status", "attnb_selftest_wait_timeout",
    "attnb_profile_enable", "attnb_profile_read", "attnb_host_alloc", "attnb_host_free",
    "attnb_sgemm", "attnb_gemm_jit", "attnb_sgemm_dev", "attnb_gemm_ex_dev",
    "attnb_gemm_ex_bcast_dev", "attnb_ipc_alloc", "attnb_ipc_free", "attnb_ipc_export", "attnb_ipc_import", "attnb_ipc_close",
    "attnb_linear_dev", "attnb_weight_pack_dev", "attnb_weight_free", "attnb_linear_packed_dev",
    "attnb_attn_step_dense", "attnb_attn_step_dense_dev", "attnb_attn_step_dense_noalloc",
    "attnb_attn_step_dense_bcast_dev", "attnb_peer_barrier_dev",
    "attnb_attn_block_dense", "attnb_attn_block_dense_dev",
    "attnb_attn_block_dense_batched_dev",
    "attnb_mha_block_dense", "attnb_mha_block_dense_dev",
    "attnb_kv_cache_create", "attnb_kv_cache_destroy", "attnb_kv_cache_length",
    "attnb_kv_cache_truncate", "attnb_kv_cache_append", "attnb_kv_cache_step",
    "attnb_kv_cache_step_dev",
]


class Tensor(ctypes.Structure):
    """attnb_tensor / attnb_mtensor: data, H, T, Dh, strideH, strideT, strideDh."""
    _fields_ = [("data", ctypes.c_void_p), ("H", ctypes.c_int), ("T", ctypes.c_int),
                ("Dh", ctypes.c_int), ("strideH", ctypes.c_int64), ("strideT", ctypes.c_int64),
                ("strideDh", ctypes.c_int64)]


class AttnbError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"attnb error {code}: {msg}")
        self.code = code


class AttnbOutOfMemory(AttnbError, MemoryError):
    """ATTNB_ERR_OUT_OF_MEMORY: the device scratch the call needs could not be had."""


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run attn-cpu_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        vp, i, f, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int64
        T = ctypes.POINTER(Tensor)
        L.attnb_last_error.restype = ctypes.c_char_p
        L.attnb_version.restype = ctypes.c_char_p
        L.attnb_stream_status.argtypes = [vp]
        L.attnb_selftest_wait_timeout.argtypes = [i, vp]
        L.attnb_profile_enable.argtypes = [i]
        L.attnb_profile_read.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_double),
                                         ctypes.POINTER(ctypes.c_int)]
        L.attnb_host_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
        L.attnb_host_free.argtypes = [vp]
        L.attnb_sgemm.argtypes = [vp, i, i, vp, i, vp, f, f, i]
        L.attnb_gemm_jit.argtypes = [vp, i, i, vp, i, vp, f, f, i]
        L.attnb_sgemm_dev.argtypes = [vp, i, vp, i, vp, i, i, i, i, f, f, i, vp]
        L.attnb_linear_dev.argtypes = [vp, i, vp, i, vp, vp, i, i, i, i, i, vp]
        L.attnb_gemm_ex_dev.argtypes = [i, i, vp, i, vp, i, vp, vp, i, i, i, i, f, f, i, vp]
        L.attnb_gemm_ex_bcast_dev.argtypes = [i, i, vp, i, vp, i, vp, vp, i,
                                              ctypes.POINTER(vp), i, i, i, i, f, f, i, vp]
        L.attnb_weight_pack_dev.argtypes = [vp, i, i, i, i, ctypes.POINTER(vp), vp]
        L.attnb_weight_free.argtypes = [vp]
        L.attnb_linear_packed_dev.argtypes = [i, vp, i, vp, vp, vp, i, i, ctypes.POINTER(vp), i,
                                              vp]
        L.attnb_ipc_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
        L.attnb_ipc_free.argtypes = [vp]
        L.attnb_ipc_export.argtypes = [vp, vp, ctypes.POINTER(ctypes.c_uint64)]
        L.attnb_ipc_import.argtypes = [vp, ctypes.c_uint64, ctypes.POINTER(vp)]
        L.attnb_ipc_close.argtypes = [vp]
        L.attnb_attn_step_dense.argtypes = [T, T, T, T]
        L.attnb_attn_step_dense_dev.argtypes = [T, T, T, T, vp]
        L.attnb_attn_step_dense_noalloc.argtypes = [T, T, T, T, vp]
        L.attnb_attn_step_dense_bcast_dev.argtypes = [T, T, T, T, ctypes.POINTER(vp), i, vp]
        L.attnb_peer_barrier_dev.argtypes = [vp, ctypes.POINTER(vp), i, i, i, vp]
        L.attnb_attn_block_dense.argtypes = [T, T, T, T, i, i]
        L.attnb_attn_block_dense_dev.argtypes = [T, T, T, T, i, i, vp]
        L.attnb_attn_block_dense_batched_dev.argtypes = [T, T, T, T, i, i64, i64, i64, i64, i, i,
                                                         vp]
        L.attnb_mha_block_dense.argtypes = [vp, i, i, vp, vp, vp, vp, i, i, vp, i]
        L.attnb_mha_block_dense_dev.argtypes = [vp, i, i, i, vp, vp, vp, vp, i, i, vp, i, vp]
        L.attnb_kv_cache_create.argtypes = [i, i, i, ctypes.POINTER(vp)]
        L.attnb_kv_cache_destroy.argtypes = [vp]
        L.attnb_kv_cache_length.argtypes = [vp, ctypes.POINTER(i)]
        L.attnb_kv_cache_truncate.argtypes = [vp, i]
        L.attnb_kv_cache_append.argtypes = [vp, vp, vp, i, vp]
        L.attnb_kv_cache_step.argtypes = [vp, vp, vp, vp, vp]
        L.attnb_kv_cache_step_dev.argtypes = [vp, vp, vp, vp, vp, vp]
        for name in EXPORTED:
            if name not in ("attnb_last_error", "attnb_version"):
                getattr(L, name).restype = ctypes.c_int
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        cls = AttnbOutOfMemory if rc == ERR_OUT_OF_MEMORY else AttnbError
        raise cls(rc, lib().attnb_last_error().decode())


def _stream(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def tensor3(t, as_2d: bool = False) -> Tensor:
    """attnb_tensor view of a float32 CUDA tensor [H,T,Dh] (or [H,Dh] with as_2d)."""
    if as_2d:
        H, Dh = t.shape
        return Tensor(t.data_ptr(), H, 1, Dh, t.stride(0), 0, t.stride(1))
    H, T_, Dh = t.shape
    return Tensor(t.data_ptr(), H, T_, Dh, t.stride(0), t.stride(1), t.stride(2))


def sgemm_dev(A, B, C, alpha=1.0, beta=0.0, precision=None, stream=None) -> None:
    """C = alpha * A @ B + beta * C on 2-D float32 CUDA tensors with unit column stride."""
    M, K = A.shape
    N = B.shape[1]
    check(lib().attnb_sgemm_dev(A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0),
                                C.data_ptr(), C.stride(0), M, N, K, alpha, beta,
                                PREC[precision], _stream(stream)))


def gemm_ex_dev(A, B, C, trans_a=False, trans_b=False, bias=None, alpha=1.0, beta=0.0,
                precision=None, stream=None) -> None:
    """C = alpha * op(A) @ op(B) + beta * C + bias, op(X) = X.T when trans_x.
    A, B, C: 2-D float32 CUDA tensors with unit column stride (A and B may be
    column slices: their row pitch is passed as the leading dimension)."""
    M = A.shape[1] if trans_a else A.shape[0]
    K = A.shape[0] if trans_a else A.shape[1]
    N = B.shape[0] if trans_b else B.shape[1]
    if (B.shape[1] if trans_b else B.shape[0]) != K or tuple(C.shape) != (M, N):
        raise ValueError("gemm_ex_dev: shapes do not match")
    if A.stride(1) != 1 or B.stride(1) != 1 or C.stride(1) != 1:
        raise ValueError("gemm_ex_dev: operands need a unit column stride")
    check(lib().attnb_gemm_ex_dev(int(trans_a), int(trans_b), A.data_ptr(), A.stride(0),
                                  B.data_ptr(), B.stride(0),
                                  bias.data_ptr() if bias is not None else None, C.data_ptr(),
                                  C.stride(0), M, N, K, alpha, beta, PREC[precision],
                                  _stream(stream)))


def gemm_ex_bcast_dev(A, B, C, replicas, trans_a=False, trans_b=False, bias=None, alpha=1.0,
                      beta=0.0, precision=None, stream=None) -> None:
    """gemm_ex_dev that also writes C, element for element, into each address
    in `replicas` (device addresses as ints, same layout and leading dimension
    as C -- e.g. C's rows in the other GPUs' replicas, from ipc_import)."""
    M = A.shape[1] if trans_a else A.shape[0]
    K = A.shape[0] if trans_a else A.shape[1]
    N = B.shape[0] if trans_b else B.shape[1]
    if (B.shape[1] if trans_b else B.shape[0]) != K or tuple(C.shape) != (M, N):
        raise ValueError("gemm_ex_bcast_dev: shapes do not match")
    if A.stride(1) != 1 or B.stride(1) != 1 or C.stride(1) != 1:
        raise ValueError("gemm_ex_bcast_dev: operands need a unit column stride")
    arr = (ctypes.c_void_p * max(1, len(replicas)))(*[int(r) for r in replicas])
    check(lib().attnb_gemm_ex_bcast_dev(int(trans_a), int(trans_b), A.data_ptr(), A.stride(0),
                                        B.data_ptr(), B.stride(0),
                                        bias.data_ptr() if bias is not None else None,
                                        C.data_ptr(), C.stride(0), arr, len(replicas), M, N, K,
                                        alpha, beta, PREC[precision], _stream(stream)))


IPC_HANDLE_BYTES = 64


class _SharedBlock:
    """A device allocation of its own (attnb_ipc_alloc), exposed through the
    CUDA array interface so torch can view it; freed when the last view dies."""

    def __init__(self, shape: tuple):
        n = 1
        for d in shape:
            n *= int(d)
        p = ctypes.c_void_p()
        check(lib().attnb_ipc_alloc(max(4, 4 * n), ctypes.byref(p)))
        self.ptr = p.value
        self.__cuda_array_interface__ = {"shape": tuple(int(d) for d in shape), "typestr": "<f4",
                                         "data": (self.ptr, False), "version": 3,
                                         "strides": None}

    def __del__(self):
        try:
            lib().attnb_ipc_free(self.ptr)
        except Exception:  # interpreter shutdown: the library may be gone
            pass


def shared_empty(shape: tuple):
    """An uninitialised float32 CUDA tensor on the current device in an
    allocation of its own, exportable with ipc_export."""
    import torch

    return torch.as_tensor(_SharedBlock(tuple(shape)), device="cuda")


def ipc_export(t) -> tuple[bytes, int]:
    """(handle, byte offset) of the device allocation holding CUDA tensor `t`,
    for ipc_import in another process of the node."""
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    off = ctypes.c_uint64()
    check(lib().attnb_ipc_export(t.data_ptr(), h, ctypes.byref(off)))
    return h.raw, off.value


def ipc_import(handle: bytes, offset: int) -> int:
    """Device address, in the current device's context, of another process's
    allocation (see ipc_export); release with ipc_close."""
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError("ipc handle must be 64 bytes")
    p = ctypes.c_void_p()
    check(lib().attnb_ipc_import(handle, offset, ctypes.byref(p)))
    return p.value


def ipc_close(ptr: int) -> None:
    check(lib().attnb_ipc_close(ptr))


class PackedWeight:
    """A projection weight W [N, K] (float32 CUDA tensor, unit column stride)
    packed once on the current device for repeated y = x W^T
    (attnb_weight_pack_dev); the packing is enqueued on `stream`."""

    def __init__(self, W, precision=None, stream=None):
        import torch

        if W.dim() != 2 or W.stride(1) != 1 or W.dtype != torch.float32:
            raise ValueError("PackedWeight: W must be 2-D float32 with a unit column stride")
        self.N, self.K = W.shape
        self._h = ctypes.c_void_p()
        check(lib().attnb_weight_pack_dev(W.data_ptr(), W.stride(0), self.N, self.K,
                                          PREC[precision], ctypes.byref(self._h),
                                          _stream(stream)))

    def close(self) -> None:
        if self._h:
            check(lib().attnb_weight_free(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may be gone
            pass


def linear_packed_dev(x, W: PackedWeight, b, y, trans_x=False, replicas=(), stream=None) -> None:
    """y = op(x) @ W^T + b (b may be None), op(x) = x.T when trans_x; y is also
    stored into each address in `replicas` (see gemm_ex_bcast_dev)."""
    M = x.shape[1] if trans_x else x.shape[0]
    K = x.shape[0] if trans_x else x.shape[1]
    if K != W.K or tuple(y.shape) != (M, W.N):
        raise ValueError("linear_packed_dev: shapes do not match")
    if x.stride(1) != 1 or y.stride(1) != 1:
        raise ValueError("linear_packed_dev: operands need a unit column stride")
    if x.dtype != y.dtype or str(x.dtype) != "torch.float32":
        raise ValueError("linear_packed_dev: x and y must be float32")
    arr = (ctypes.c_void_p * max(1, len(replicas)))(*[int(r) for r in replicas])
    check(lib().attnb_linear_packed_dev(int(trans_x), x.data_ptr(), x.stride(0), W._h,
                                        b.data_ptr() if b is not None else None, y.data_ptr(),
                                        y.stride(0), M, arr, len(replicas), _stream(stream)))


def linear_dev(x, W, b, y, precision=None, stream=None) -> None:
    """y = x @ W^T + b (b may be None)."""
    T_, K = x.shape
    N = W.shape[0]
    check(lib().attnb_linear_dev(x.data_ptr(), x.stride(0), W.data_ptr(), W.stride(0),
                                 b.data_ptr() if b is not None else None, y.data_ptr(),
                                 y.stride(0), T_, N, K, PREC[precision], _stream(stream)))


def attn_step_dense_dev(Q, K, V, O, stream=None) -> None:
    q, k, v, o = tensor3(Q, True), tensor3(K), tensor3(V), tensor3(O, True)
    check(lib().attnb_attn_step_dense_dev(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v),
                                          ctypes.byref(o), _stream(stream)))


def attn_step_dense_bcast_dev(Q, K, V, O, replicas, stream=None) -> None:
    """attn_step_dense_dev that also stores O into each address in `replicas`
    (device addresses as ints: O's heads in other GPUs' copies)."""
    q, k, v, o = tensor3(Q, True), tensor3(K), tensor3(V), tensor3(O, True)
    arr = (ctypes.c_void_p * max(1, len(replicas)))(*[int(r) for r in replicas])
    check(lib().attnb_attn_step_dense_bcast_dev(ctypes.byref(q), ctypes.byref(k),
                                                ctypes.byref(v), ctypes.byref(o), arr,
                                                len(replicas), _stream(stream)))


def peer_barrier_dev(flags: int, peer_flags: list, rank: int, limit_us: int = 0,
                     stream=None) -> None:
    """Enqueue the next peer-memory barrier (attnb_peer_barrier_dev): `flags`
    is this rank's array (one epoch per rank, then its barrier count),
    peer_flags[r] rank r's array as mapped here (any value at index `rank`)."""
    n = len(peer_flags)
    arr = (ctypes.c_void_p * n)(*[int(p) if p else None for p in peer_flags])
    check(lib().attnb_peer_barrier_dev(flags, arr, n, rank, limit_us, _stream(stream)))


def attn_step_dense_noalloc(Q, K, V, O, stream=None) -> None:
    """Decode step without any device allocation (fixed 2 MiB scratch shared by
    all calls; see attnb_attn_step_dense_noalloc in include/attnb.h)."""
    q, k, v, o = tensor3(Q, True), tensor3(K), tensor3(V), tensor3(O, True)
    check(lib().attnb_attn_step_dense_noalloc(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v),
                                              ctypes.byref(o), _stream(stream)))


def attn_block_dense_dev(Q, K, V, O, causal=False, precision=None, stream=None) -> None:
    q, k, v, o = tensor3(Q), tensor3(K), tensor3(V), tensor3(O)
    check(lib().attnb_attn_block_dense_dev(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v),
                                           ctypes.byref(o), int(causal), PREC[precision],
                                           _stream(stream)))


def attn_block_dense_batched_dev(Q, K, V, O, causal=False, precision=None, stream=None) -> None:
    """Prefill for independent sequences: Q, O [B, H, L, Dh] and K, V [B, H, T, Dh]
    float32 CUDA views (any strides); the sequences run side by side."""
    if not (Q.dim() == K.dim() == V.dim() == O.dim() == 4):
        raise ValueError("attn_block_dense_batched_dev: 4-D views [B, H, T, Dh] expected")
    B = Q.shape[0]
    if K.shape[0] != B or V.shape[0] != B or O.shape[0] != B:
        raise ValueError("attn_block_dense_batched_dev: batch sizes differ")
    if B == 0:
        return
    q, k, v, o = tensor3(Q[0]), tensor3(K[0]), tensor3(V[0]), tensor3(O[0])
    check(lib().attnb_attn_block_dense_batched_dev(
        ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(o), B, Q.stride(0),
        K.stride(0), V.stride(0), O.stride(0), int(causal), PREC[precision], _stream(stream)))


def mha_block_dense_dev(x, W_in, b_in, W_out, b_out, num_heads, y, causal=False,
                        precision=None, stream=None) -> None:
    """x, y: [batch, T, D] (or [T, D]) contiguous float32 CUDA tensors."""
    if x.dim() == 2:
        batch, (T_, D) = 1, x.shape
    else:
        batch, T_, D = x.shape
    check(lib().attnb_mha_block_dense_dev(x.data_ptr(), batch, T_, D, W_in.data_ptr(),
                                          b_in.data_ptr(), W_out.data_ptr(), b_out.data_ptr(),
                                          num_heads, int(causal), y.data_ptr(), PREC[precision],
                                          _stream(stream)))


def profile_enable(on: bool = True) -> None:
    check(lib().attnb_profile_enable(int(on)))


def profile_read(kernel: str) -> tuple[float, int]:
    """(summed milliseconds, launches) of `kernel` since the last read."""
    ms, n = ctypes.c_double(), ctypes.c_int()
    check(lib().attnb_profile_read(kernel.encode(), ctypes.byref(ms), ctypes.byref(n)))
    return ms.value, n.value


def stream_status(stream=None) -> None:
    check(lib().attnb_stream_status(_stream(stream)))


class KVCacheDev:
    """The resident K/V cache (attnb_kv_cache_*) driven with CUDA tensors.

    K and V stay on the device current at construction, [H, capacity, Dh];
    ``append`` and ``step`` enqueue on ``stream`` (default: torch's current
    stream) and return without synchronising."""

    def __init__(self, H: int, Dh: int, capacity: int):
        self._h = ctypes.c_void_p()
        check(lib().attnb_kv_cache_create(H, Dh, capacity, ctypes.byref(self._h)))
        self.H, self.Dh = H, Dh

    def __len__(self) -> int:
        n = ctypes.c_int()
        check(lib().attnb_kv_cache_length(self._h, ctypes.byref(n)))
        return n.value

    def truncate(self, length: int) -> None:
        check(lib().attnb_kv_cache_truncate(self._h, length))

    def append(self, k, v, stream=None) -> None:
        """k, v: [H, n, Dh] contiguous float32 tensors (CUDA or CPU)."""
        check(lib().attnb_kv_cache_append(self._h, k.data_ptr(), v.data_ptr(), k.shape[1],
                                          _stream(stream)))

    def step(self, q, o, k_new=None, v_new=None, stream=None) -> None:
        """o[H, Dh] = attention of q[H, Dh] over the cache, after appending k_new, v_new."""
        kp = k_new.data_ptr() if k_new is not None else None
        vp_ = v_new.data_ptr() if v_new is not None else None
        check(lib().attnb_kv_cache_step_dev(self._h, q.data_ptr(), kp, vp_, o.data_ptr(),
                                            _stream(stream)))

    def close(self) -> None:
        if self._h:
            check(lib().attnb_kv_cache_destroy(self._h))
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter shutdown: the library may be gone
            pass
