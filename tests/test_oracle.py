"""The oracle (float64 C restatement) pinned against the reference itself:
the golden vectors the reference produced (tests/golden/make_golden.py) and,
where the compiled reference is present on an AVX-512 host, fresh runs of it."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_err

# fp32 (reference) vs float64 (oracle) orderings differ by a few fp32 ulps.
PIN = 2e-6


def _cases(golden, prefix):
    return sorted({k.split("_")[0] for k in golden.files if k.startswith(prefix)})


def test_gemm_golden(golden):
    for c in _cases(golden, "gemm"):
        M, K, N, a, b = golden[f"{c}_args"]
        C0 = golden[f"{c}_C0"]
        got = oracle.sgemm(golden[f"{c}_A"], golden[f"{c}_B"], a, b, C0 if b != 0 else None)
        assert rel_err(got, golden[f"{c}_C"]) < PIN, c


def test_step_golden(golden):
    for c in _cases(golden, "step"):
        got = oracle.attn_step(golden[f"{c}_Q"], golden[f"{c}_K"], golden[f"{c}_V"])
        assert rel_err(got, golden[f"{c}_O"]) < PIN, c


def test_block_golden(golden):
    for c in _cases(golden, "block"):
        got = oracle.attn_block(golden[f"{c}_Q"], golden[f"{c}_K"], golden[f"{c}_V"],
                                bool(golden[f"{c}_causal"]))
        assert rel_err(got, golden[f"{c}_O"]) < PIN, c


def test_mha_golden(golden):
    for c in _cases(golden, "mha"):
        T, D, H, causal = (int(v) for v in golden[f"{c}_args"])
        got = oracle.mha_block(golden[f"{c}_x"], golden[f"{c}_Win"], golden[f"{c}_bin"],
                               golden[f"{c}_Wout"], golden[f"{c}_bout"], H, bool(causal))
        assert rel_err(got, golden[f"{c}_y"]) < PIN, c


def test_strided_views_match_contiguous():
    rng = np.random.default_rng(3)
    base = rng.standard_normal((5, 40, 2 * 24), dtype=np.float32)
    K = base[:, :, ::2]  # strideDh = 2
    V = base[:, :, 1::2]
    Q = rng.standard_normal((5, 24), dtype=np.float32)
    a = oracle.attn_step(Q, K, V)
    b = oracle.attn_step(Q, np.ascontiguousarray(K), np.ascontiguousarray(V))
    assert np.array_equal(a, b)


needs_ref = pytest.mark.skipif(not oracle.ref_available(),
                               reason="compiled reference not built here or host lacks AVX-512")


@needs_ref
@pytest.mark.parametrize("M,K,N", [(1, 1, 1), (13, 17, 19), (257, 129, 65), (1023, 1025, 1027)])
def test_gemm_vs_reference(M, K, N):
    rng = np.random.default_rng(M * 7 + N)
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((K, N), dtype=np.float32)
    assert rel_err(oracle.sgemm(A, B), oracle.ref_sgemm(A, B)) < 5e-6


@needs_ref
@pytest.mark.parametrize("H,Dh,T", [(1, 64, 1), (4, 64, 128), (8, 64, 1024), (8, 128, 512),
                                    (16, 96, 256)])
def test_step_vs_reference(H, Dh, T):
    """The shapes of the reference's tests/test_attn_step.py:148-157."""
    rng = np.random.default_rng(42)
    Q = rng.standard_normal((H, Dh), dtype=np.float32)
    K = rng.standard_normal((H, T, Dh), dtype=np.float32)
    V = rng.standard_normal((H, T, Dh), dtype=np.float32)
    assert rel_err(oracle.attn_step(Q, K, V), oracle.ref_attn_step(Q, K, V)) < PIN


@needs_ref
@pytest.mark.parametrize("causal", [False, True])
def test_block_vs_reference(causal):
    rng = np.random.default_rng(5)
    Q, K, V = (rng.standard_normal((8, 128, 64), dtype=np.float32) for _ in range(3))
    assert rel_err(oracle.attn_block(Q, K, V, causal), oracle.ref_attn_block(Q, K, V, causal)) < PIN


@needs_ref
@pytest.mark.parametrize("T,D,H,causal", [(65, 128, 4, False), (66, 128, 8, True),
                                          (64, 256, 2, False)])
def test_mha_vs_reference(T, D, H, causal):
    """Cases of the reference's tests/test_mha.py:68-70 (Dh=16 non-causal T=65 is
    the reference's own bug and is covered against the oracle only)."""
    rng = np.random.default_rng(T)
    x = rng.standard_normal((T, D), dtype=np.float32)
    Wi = (rng.standard_normal((3 * D, D)) / np.sqrt(D)).astype(np.float32)
    bi = np.zeros(3 * D, np.float32)
    Wo = (rng.standard_normal((D, D)) / np.sqrt(D)).astype(np.float32)
    bo = np.zeros(D, np.float32)
    assert rel_err(oracle.mha_block(x, Wi, bi, Wo, bo, H, causal),
                   oracle.ref_mha_block(x, Wi, bi, Wo, bo, H, causal)) < PIN


@needs_ref
def test_reference_dh16_tail_bug_is_real():
    """Documents why the Dh=16, non-causal, T%16!=0 case is pinned to the oracle:
    the reference reads keys past T there (include/kernels/attn_dh16_m4_nocausal.h:76-83)."""
    rng = np.random.default_rng(42)
    T, D, H = 65, 128, 8
    x = rng.standard_normal((T, D), dtype=np.float32)
    Wi = (rng.standard_normal((3 * D, D)) / np.sqrt(D)).astype(np.float32)
    Wo = (rng.standard_normal((D, D)) / np.sqrt(D)).astype(np.float32)
    z3, z = np.zeros(3 * D, np.float32), np.zeros(D, np.float32)
    ora = oracle.mha_block(x, Wi, z3, Wo, z, H, False)
    ref = oracle.ref_mha_block(x, Wi, z3, Wo, z, H, False)
    assert rel_err(ref, ora) > 1e-3
