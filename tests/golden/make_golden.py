"""Generate the golden fixtures in this directory from the REFERENCE ITSELF.

Runs the reference's own CPU code (compiled from its sources by
oracle/Makefile into oracle/_ref/libattnref.so) on small seeded inputs and
stores inputs + outputs as compressed .npz files.  The GPU parity tests and
the oracle's own pinning test read these files; the reference tree is not
needed at test time.

    python tests/golden/make_golden.py

Cases avoid the one input class where the reference is known to be wrong
(mha_block_dense with Dh == 16, non-causal, T % 16 != 0: unmasked key loads in
include/kernels/attn_dh16_m4_nocausal.h:76-83 and :268-274).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle  # noqa: E402

GEMM_CASES = [  # (M, K, N, alpha, beta)
    (1, 1, 1, 1.0, 0.0), (5, 7, 11, 1.0, 0.0), (33, 65, 129, 1.0, 0.0),
    (127, 255, 63, 1.0, 0.0), (64, 64, 64, 1.0, 0.0), (101, 103, 107, 1.0, 0.0),
    (31, 47, 29, 1.5, 0.5), (16, 8, 40, 0.0, 2.0), (8, 16, 300, -0.75, 0.0),
]
STEP_CASES = [(1, 64, 1), (4, 64, 128), (2, 128, 100), (3, 96, 77), (2, 16, 33)]  # (H, Dh, T)
BLOCK_CASES = [  # (H, L, T, Dh, causal)
    (2, 33, 33, 64, False), (2, 33, 33, 64, True), (2, 64, 100, 32, False),
    (1, 17, 17, 96, True), (1, 70, 70, 128, False),
]
MHA_CASES = [  # (T, D, H, causal)
    (66, 64, 4, True), (64, 64, 2, False), (65, 64, 2, False), (33, 64, 1, False),
    (20, 96, 2, True), (48, 128, 8, False),
]


def main() -> None:
    if not oracle.ref_available():
        raise SystemExit("compiled reference not available: run `make -C oracle`")
    rng = np.random.default_rng(20241201)
    out = {}
    for i, (M, K, N, a, b) in enumerate(GEMM_CASES):
        A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
        B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
        C0 = rng.uniform(-1, 1, (M, N)).astype(np.float32)
        out[f"gemm{i}_A"], out[f"gemm{i}_B"], out[f"gemm{i}_C0"] = A, B, C0
        out[f"gemm{i}_args"] = np.array([M, K, N, a, b], np.float64)
        out[f"gemm{i}_C"] = oracle.ref_sgemm(A, B, a, b, C0 if b != 0 else None)
    for i, (H, Dh, T) in enumerate(STEP_CASES):
        Q = rng.standard_normal((H, Dh), dtype=np.float32)
        K = rng.standard_normal((H, T, Dh), dtype=np.float32)
        V = rng.standard_normal((H, T, Dh), dtype=np.float32)
        out[f"step{i}_Q"], out[f"step{i}_K"], out[f"step{i}_V"] = Q, K, V
        out[f"step{i}_O"] = oracle.ref_attn_step(Q, K, V)
    for i, (H, L, T, Dh, c) in enumerate(BLOCK_CASES):
        Q = rng.standard_normal((H, L, Dh), dtype=np.float32)
        K = rng.standard_normal((H, T, Dh), dtype=np.float32)
        V = rng.standard_normal((H, T, Dh), dtype=np.float32)
        out[f"block{i}_Q"], out[f"block{i}_K"], out[f"block{i}_V"] = Q, K, V
        out[f"block{i}_causal"] = np.array(int(c))
        out[f"block{i}_O"] = oracle.ref_attn_block(Q, K, V, c)
    for i, (T, D, H, c) in enumerate(MHA_CASES):
        x = rng.standard_normal((T, D), dtype=np.float32)
        Wi = (rng.standard_normal((3 * D, D)) / np.sqrt(D)).astype(np.float32)
        bi = (0.1 * rng.standard_normal(3 * D)).astype(np.float32)
        Wo = (rng.standard_normal((D, D)) / np.sqrt(D)).astype(np.float32)
        bo = (0.1 * rng.standard_normal(D)).astype(np.float32)
        for k, v in (("x", x), ("Win", Wi), ("bin", bi), ("Wout", Wo), ("bout", bo)):
            out[f"mha{i}_{k}"] = v
        out[f"mha{i}_args"] = np.array([T, D, H, int(c)])
        out[f"mha{i}_y"] = oracle.ref_mha_block(x, Wi, bi, Wo, bo, H, c)
    path = os.path.join(HERE, "reference_vectors.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
