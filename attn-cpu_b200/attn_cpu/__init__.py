"""attn_cpu -- drop-in replacement of the reference's ``attn_cpu`` Python package
(python/attn_cpu/__init__.py of the reference), computed on a B200 GPU.

Same functions, argument names and defaults as the reference module:
``mha_block_dense``, ``gemm``, ``gemm_jit``; plus ``attn_step_dense`` and
``attn_block_dense``, which the reference's tests call but its module never
exported, and ``KVCache`` (a device-resident K/V cache for multi-step decode:
``append(k, v)``, ``step(q, k_new=None, v_new=None)``, ``truncate(n)``), which
the reference does not have.  Every function takes and returns NumPy float32 arrays (inputs are
force-cast to C-contiguous float32) and raises ``ValueError`` for shape
problems and ``RuntimeError`` otherwise, like the reference's bindings.

``precision`` (optional, keyword): ``None`` (default: 3xTF32, or TF32 when the
environment variable ATTNB_PRECISION=tf32), ``"3xtf32"`` or ``"tf32"``.

There is no CPU fallback: importing fails if the compiled extension is missing,
and calls fail if no B200 is visible.
"""
from __future__ import annotations

import numpy as np

from ._attn_cpu import (  # noqa: F401  (ImportError here means the extension is not built)
    KVCache,
    attn_block_dense as _attn_block_dense,
    attn_step_dense as _attn_step_dense,
    gemm as _gemm,
    gemm_jit as _gemm_jit,
    mha_block_dense as _mha_block_dense,
    version,
)

_PREC = {None: -1, "default": -1, "3xtf32": 0, "tf32": 1}


def _prec(precision) -> int:
    try:
        return _PREC[precision.lower() if isinstance(precision, str) else precision]
    except KeyError:
        raise ValueError(f"precision must be one of {sorted(k for k in _PREC if k)}") from None


def mha_block_dense(x: np.ndarray, W_in: np.ndarray, b_in: np.ndarray, W_out: np.ndarray,
                    b_out: np.ndarray, num_heads: int, causal: bool = False, *,
                    precision: str | None = None) -> np.ndarray:
    """y[T,D] = MHA(x) with nn.MultiheadAttention packing (W_in [3D,D], b_in [3D],
    W_out [D,D], b_out [D]).  Reference: src/attn_dispatch.cpp:17-133."""
    return _mha_block_dense(x, W_in, b_in, W_out, b_out, num_heads, causal, _prec(precision))


def gemm(A: np.ndarray, B: np.ndarray, alpha: float = 1.0, beta: float = 0.0, *,
         precision: str | None = None) -> np.ndarray:
    """C = alpha * A @ B (+ beta * 0), A [M,K], B [K,N].  Reference: src/gemm.cpp:319-415."""
    return _gemm(A, B, alpha, beta, _prec(precision))


def gemm_jit(A: np.ndarray, B: np.ndarray, alpha: float = 1.0, beta: float = 0.0, *,
             precision: str | None = None) -> np.ndarray:
    """Same function and kernel as :func:`gemm` (reference: src/jit_gemm.cpp:740-754)."""
    return _gemm_jit(A, B, alpha, beta, _prec(precision))


def attn_step_dense(Q: np.ndarray, K: np.ndarray, V: np.ndarray) -> np.ndarray:
    """Decode step: Q [H,Dh], K/V [H,T,Dh] -> O [H,Dh].  Reference: src/attn_dense.cpp:21-73."""
    return _attn_step_dense(Q, K, V)


def attn_block_dense(Q: np.ndarray, K: np.ndarray, V: np.ndarray, causal: bool = False, *,
                     precision: str | None = None) -> np.ndarray:
    """Prefill: Q [H,L,Dh], K/V [H,T,Dh] -> O [H,L,Dh] (causal needs L == T).
    Reference: src/attn_block.cpp:104-241."""
    return _attn_block_dense(Q, K, V, causal, _prec(precision))


__all__ = ["mha_block_dense", "gemm", "gemm_jit", "attn_step_dense", "attn_block_dense",
           "KVCache", "version"]
