"""mha_np -- the reference's NumPy MHA driver (python/attn_cpu/mha_np.py:5-41),
which projects with NumPy and calls ``attn_block_dense`` for the attention.
The reference's module never exported that binding; this package does, so
the driver runs as written."""
from __future__ import annotations

import numpy as np

from . import attn_block_dense


def mha_forward_dense(x, W_in, b_in, W_out, b_out, num_heads, causal=False):
    """x [T,D], W_in [3D,D], b_in [3D], W_out [D,D], b_out [D] -> y [T,D]."""
    T, D = x.shape
    H = num_heads
    if D % H:
        raise ValueError("num_heads must divide D")
    Dh = D // H
    qkv = x @ W_in.T + b_in
    q, k, v = np.split(qkv, 3, axis=1)

    def to_heads(a):
        return np.transpose(a.reshape(T, H, Dh), (1, 0, 2)).astype(np.float32, copy=False)

    O = attn_block_dense(to_heads(q), to_heads(k), to_heads(v), causal=causal)
    O = np.transpose(O, (1, 0, 2)).reshape(T, D)
    return (O @ W_out.T + b_out).astype(np.float32, copy=False)
