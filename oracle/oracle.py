"""oracle.py -- TEST INFRASTRUCTURE ONLY: ctypes access to the CPU checkers.

Two libraries, both built by ``oracle/Makefile``:

* ``_bin/liboracle.so`` -- the float64 restatement in ``oracle.c`` ("port").
* ``_ref/libattnref.so`` -- the reference's own AVX-512/OpenMP code compiled from
  its sources ("reference"); needs an AVX-512 host.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this module.  It is the checker, never the thing measured or shipped.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_bin", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libattnref.so")

_f = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64
_ll = ctypes.c_longlong


# Source tree of the reference (the directory holding src/ and include/), for
# building _ref/libattnref.so; unset means the reference part is not built.
REF_ENV = "ATTNB_REFERENCE_SRC"


def build(with_reference: bool | None = None) -> None:
    """Compile the checkers: the restatement always, the reference library when
    the environment variable ATTNB_REFERENCE_SRC names its source tree."""
    targets = ["port"]
    ref_dir = os.environ.get(REF_ENV, "")
    if with_reference is None:
        with_reference = bool(ref_dir) and os.path.isdir(os.path.join(ref_dir, "src"))
    if with_reference:
        if not ref_dir:
            raise RuntimeError(f"{REF_ENV} must name the reference's source tree")
        targets += ["ref", f"REF={ref_dir}"]
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def host_has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as fh:
            flags = fh.read()
    except OSError:
        return False
    return all(f in flags for f in ("avx512f", "avx512dq", "avx512bw", "avx512vl"))


_port = None
_ref = None


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_f)


def port_lib():
    global _port
    if _port is None:
        if not os.path.exists(PORT_SO):
            build(with_reference=False)
        lib = ctypes.CDLL(PORT_SO)
        lib.oracle_sgemm.argtypes = [_f, ctypes.c_int, ctypes.c_int, _f, ctypes.c_int, _f,
                                     ctypes.c_float, ctypes.c_float]
        lib.oracle_linear.argtypes = [_f, ctypes.c_int, ctypes.c_int, _f, ctypes.c_int, _f, _f]
        lib.oracle_attn_step.argtypes = ([_f, _i64, _i64, _f, _i64, _i64, _i64, _f, _i64, _i64,
                                          _i64, _f, _i64, _i64] + [ctypes.c_int] * 3)
        lib.oracle_attn_block.argtypes = ([_f, _i64, _i64, _i64] * 3 + [_f, _i64, _i64, _i64]
                                          + [ctypes.c_int] * 5)
        lib.oracle_mha_block.argtypes = [_f, ctypes.c_int, ctypes.c_int, _f, _f, _f, _f,
                                         ctypes.c_int, ctypes.c_int, _f]
        _port = lib
    return _port


def ref_available() -> bool:
    return os.path.exists(REF_SO) and host_has_avx512()


def ref_lib():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError("compiled reference unavailable (not built here or no AVX-512)")
        lib = ctypes.CDLL(REF_SO)
        lib.ref_sgemm.argtypes = [_f, ctypes.c_int, ctypes.c_int, _f, ctypes.c_int, _f,
                                  ctypes.c_float, ctypes.c_float]
        lib.ref_attn_step.argtypes = ([_f, _ll, _ll, _f, _ll, _ll, _ll, _f, _ll, _ll, _ll, _f,
                                       _ll, _ll] + [ctypes.c_int] * 3)
        lib.ref_attn_block.argtypes = ([_f, _ll, _ll, _ll] * 3 + [_f, _ll, _ll, _ll]
                                       + [ctypes.c_int] * 5)
        lib.ref_mha_block.argtypes = [_f, ctypes.c_int, ctypes.c_int, _f, _f, _f, _f,
                                      ctypes.c_int, ctypes.c_int, _f]
        for fn in (lib.ref_sgemm, lib.ref_attn_step, lib.ref_attn_block, lib.ref_mha_block):
            fn.restype = ctypes.c_int
        _ref = lib
    return _ref


def _c32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _strides(a: np.ndarray):
    return [s // a.itemsize for s in a.strides]


# ---------------------------------------------------------------- port (float64)
def sgemm(A, B, alpha=1.0, beta=0.0, C=None):
    A, B = _c32(A), _c32(B)
    M, K = A.shape
    N = B.shape[1]
    out = np.zeros((M, N), np.float32) if C is None else _c32(C).copy()
    port_lib().oracle_sgemm(_ptr(A), M, K, _ptr(B), N, _ptr(out), alpha, beta)
    return out


def sgemm_rows(A, B, rows, alpha=1.0):
    """alpha * A[rows] . B in float64 (numpy), for sampled checks of large GEMMs."""
    A = np.asarray(A)
    return (alpha * (A[rows].astype(np.float64) @ np.asarray(B, np.float64))).astype(np.float32)


def linear_f64(x, W, b=None):
    """y = x . W^T + b in float64 (numpy BLAS), for the projections of sampled
    checks at full size, where the scalar restatement would take minutes."""
    y = np.asarray(x, np.float64) @ np.asarray(W, np.float64).T
    if b is not None:
        y += np.asarray(b, np.float64)
    return y


def linear(x, W, b=None):
    """y = x . W^T + b with x[T,K], W[N,K], b[N] (float64 accumulation)."""
    x, W = _c32(x), _c32(W)
    T, K = x.shape
    N = W.shape[0]
    y = np.empty((T, N), np.float32)
    bb = _c32(b) if b is not None else None
    port_lib().oracle_linear(_ptr(x), T, K, _ptr(W), N, _ptr(bb) if bb is not None else None,
                             _ptr(y))
    return y


def attn_step(Q, K, V):
    """Q[H,Dh], K/V[H,T,Dh] (any strides) -> O[H,Dh]."""
    H, T, Dh = K.shape
    O = np.empty((H, Dh), np.float32)
    q, k, v = _strides(Q), _strides(K), _strides(V)
    port_lib().oracle_attn_step(_ptr_any(Q), q[0], q[1], _ptr_any(K), k[0], k[1], k[2],
                                _ptr_any(V), v[0], v[1], v[2], _ptr(O), Dh, 1, H, T, Dh)
    return O


def attn_block(Q, K, V, causal=False):
    """Q[H,L,Dh], K/V[H,T,Dh] (any strides) -> O[H,L,Dh]."""
    H, L, Dh = Q.shape
    T = K.shape[1]
    O = np.empty((H, L, Dh), np.float32)
    q, k, v = _strides(Q), _strides(K), _strides(V)
    port_lib().oracle_attn_block(_ptr_any(Q), *q, _ptr_any(K), *k, _ptr_any(V), *v, _ptr(O),
                                 L * Dh, Dh, 1, H, L, T, Dh, int(causal))
    return O


def mha_block(x, W_in, b_in, W_out, b_out, num_heads, causal=False):
    x, W_in, b_in, W_out, b_out = map(_c32, (x, W_in, b_in, W_out, b_out))
    T, D = x.shape
    y = np.empty((T, D), np.float32)
    port_lib().oracle_mha_block(_ptr(x), T, D, _ptr(W_in), _ptr(b_in), _ptr(W_out),
                                _ptr(b_out), num_heads, int(causal), _ptr(y))
    return y


def _ptr_any(a: np.ndarray):
    assert a.dtype == np.float32
    return ctypes.cast(a.ctypes.data, _f)


# ---------------------------------------------------------- compiled reference
def ref_sgemm(A, B, alpha=1.0, beta=0.0, C=None):
    A, B = _c32(A), _c32(B)
    M, K = A.shape
    N = B.shape[1]
    out = np.zeros((M, N), np.float32) if C is None else _c32(C).copy()
    rc = ref_lib().ref_sgemm(_ptr(A), M, K, _ptr(B), N, _ptr(out), alpha, beta)
    if rc:
        raise RuntimeError(f"reference sgemm failed ({rc})")
    return out


def ref_attn_step(Q, K, V):
    H, T, Dh = K.shape
    O = np.empty((H, Dh), np.float32)
    q, k, v = _strides(Q), _strides(K), _strides(V)
    rc = ref_lib().ref_attn_step(_ptr_any(Q), q[0], q[1], _ptr_any(K), *k, _ptr_any(V), *v,
                                 _ptr(O), Dh, 1, H, T, Dh)
    if rc:
        raise (ValueError if rc == 1 else RuntimeError)("reference attn_step_dense failed")
    return O


def ref_attn_block(Q, K, V, causal=False):
    H, L, Dh = Q.shape
    T = K.shape[1]
    O = np.empty((H, L, Dh), np.float32)
    q, k, v = _strides(Q), _strides(K), _strides(V)
    rc = ref_lib().ref_attn_block(_ptr_any(Q), *q, _ptr_any(K), *k, _ptr_any(V), *v, _ptr(O),
                                  L * Dh, Dh, 1, H, L, T, Dh, int(causal))
    if rc:
        raise (ValueError if rc == 1 else RuntimeError)("reference attn_block_dense failed")
    return O


def ref_mha_block(x, W_in, b_in, W_out, b_out, num_heads, causal=False):
    x, W_in, b_in, W_out, b_out = map(_c32, (x, W_in, b_in, W_out, b_out))
    T, D = x.shape
    y = np.empty((T, D), np.float32)
    rc = ref_lib().ref_mha_block(_ptr(x), T, D, _ptr(W_in), _ptr(b_in), _ptr(W_out),
                                 _ptr(b_out), num_heads, int(causal), _ptr(y))
    if rc:
        raise (ValueError if rc == 1 else RuntimeError)("reference mha_block_dense failed")
    return y


def rel_err(y, r) -> float:
    """max|y - r| / max|r|: the parity metric (size-independent)."""
    y = np.asarray(y, np.float64)
    r = np.asarray(r, np.float64)
    den = float(np.max(np.abs(r))) if r.size else 0.0
    num = float(np.max(np.abs(y - r))) if r.size else 0.0
    return num / den if den > 0 else num
