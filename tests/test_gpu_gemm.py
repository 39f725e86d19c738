"""SGEMM (gemm / gemm_jit / sgemm_blocked) on the GPU: the reference's
tests/test_matmul.py shape list (39 shapes, randn inputs, seed 0) with its own
bar (rtol=atol=1e-3 against a matmul) plus the parity bars of this project
against the float64 oracle: 1e-5 (3xTF32) and 2e-3 (TF32)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_3XTF32, TOL_TF32, rel_err

pytestmark = pytest.mark.gpu

SHAPES = [
    (1, 1, 1), (1, 5, 7), (7, 1, 13), (3, 3, 3),
    (5, 7, 11), (13, 17, 19), (31, 47, 29),
    (1, 1024, 1), (1024, 1, 1), (1, 1, 1024), (2, 4096, 3), (4096, 2, 7),
    (33, 65, 129), (127, 255, 63), (257, 129, 65), (123, 456, 789), (111, 222, 333),
    (15, 15, 15), (17, 33, 65), (29, 58, 87), (30, 45, 60), (63, 127, 255),
    (64, 64, 64), (65, 65, 65), (128, 256, 512), (255, 255, 255), (256, 255, 257),
    (512, 513, 514), (1023, 1025, 1027), (999, 1001, 1003),
    (2048, 1280, 960), (2048, 1280, 1920), (4096, 4096, 4096),
    (8192, 8, 16), (16, 8192, 8), (8, 16, 8192),
    (101, 103, 107), (211, 223, 227), (401, 409, 419),
]


def _ref(A, B):
    # float64 oracle; numpy float64 matmul for the largest shapes (same maths).
    if A.shape[0] * A.shape[1] * B.shape[1] > 3e9:
        return (A.astype(np.float64) @ B.astype(np.float64)).astype(np.float32)
    return oracle.sgemm(A, B)


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_gemm_reference_shapes(cuda, M, K, N):
    import attn_cpu

    np.random.seed(0)
    A = np.random.randn(M, K).astype(np.float32)
    B = np.random.randn(K, N).astype(np.float32)
    ref = _ref(A, B)
    out = attn_cpu.gemm(A, B)
    np.testing.assert_allclose(out, ref, rtol=1e-3, atol=1e-3)
    assert rel_err(out, ref) < TOL_3XTF32
    out_tf32 = attn_cpu.gemm(A, B, precision="tf32")
    assert rel_err(out_tf32, ref) < TOL_TF32
    out_jit = attn_cpu.gemm_jit(A, B)
    assert rel_err(out_jit, ref) < TOL_3XTF32


def test_gemm_golden(cuda, golden):
    import attn_cpu
    from attn_cpu import capi
    import ctypes

    for c in sorted({k.split("_")[0] for k in golden.files if k.startswith("gemm")}):
        M, K, N, a, b = golden[f"{c}_args"]
        A, B = golden[f"{c}_A"], golden[f"{c}_B"]
        C = golden[f"{c}_C0"].copy() if b != 0 else np.zeros((int(M), int(N)), np.float32)
        p = lambda x: x.ctypes.data_as(ctypes.c_void_p)
        capi.check(capi.lib().attnb_sgemm(p(A), int(M), int(K), p(B), int(N), p(C), float(a),
                                          float(b), -1))
        assert rel_err(C, golden[f"{c}_C"]) < TOL_3XTF32, c


def test_gemm_alpha_beta_dev(cuda):
    import torch
    from attn_cpu import capi

    g = torch.Generator(device="cuda").manual_seed(1)
    M, K, N = 300, 200, 500
    A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    C0 = torch.rand(M, N, device="cuda", generator=g) * 2 - 1
    C = C0.clone()
    capi.sgemm_dev(A, B, C, alpha=-0.5, beta=1.25)
    capi.stream_status()
    ref = oracle.sgemm(A.cpu().numpy(), B.cpu().numpy(), -0.5, 1.25, C0.cpu().numpy())
    assert rel_err(C.cpu().numpy(), ref) < TOL_3XTF32
    # alpha == 0 only scales C and never reads A or B (src/gemm.cpp:328-336).
    C = C0.clone()
    nan = torch.full_like(A, float("nan"))
    capi.sgemm_dev(nan, B, C, alpha=0.0, beta=2.0)
    assert torch.equal(C, C0 * 2)
    # beta == 0 never reads C.
    C = torch.full_like(C0, float("nan"))
    capi.sgemm_dev(A, B, C, alpha=1.0, beta=0.0)
    assert torch.isfinite(C).all()


def test_gemm_ld_and_unaligned_dev(cuda):
    """Leading dimensions larger than the row and operands off 16-byte alignment."""
    import torch
    from attn_cpu import capi

    g = torch.Generator(device="cuda").manual_seed(2)
    M, K, N = 257, 129, 191
    Abuf = torch.randn(M, K + 3, device="cuda", generator=g)
    Bbuf = torch.randn(K, N + 5, device="cuda", generator=g)
    A, B = Abuf[:, 1:K + 1], Bbuf[:, 2:N + 2]  # misaligned bases, odd pitches
    Cbuf = torch.zeros(M, N + 7, device="cuda")
    C = Cbuf[:, 3:N + 3]
    for prec in (None, "tf32"):
        capi.sgemm_dev(A, B, C, precision=prec)
        ref = oracle.sgemm(A.cpu().numpy(), B.cpu().numpy())
        assert rel_err(C.cpu().numpy(), ref) < (TOL_3XTF32 if prec is None else TOL_TF32)
    assert torch.count_nonzero(Cbuf[:, :3]) == 0 and torch.count_nonzero(Cbuf[:, N + 3:]) == 0


def test_linear_bias_dev(cuda):
    import torch
    from attn_cpu import capi

    g = torch.Generator(device="cuda").manual_seed(4)
    T, K, N = 333, 256, 384
    x = torch.randn(T, K, device="cuda", generator=g)
    W = torch.randn(N, K, device="cuda", generator=g) / 16
    b = torch.randn(N, device="cuda", generator=g)
    y = torch.empty(T, N, device="cuda")
    for prec, tol in ((None, TOL_3XTF32), ("tf32", TOL_TF32)):
        capi.linear_dev(x, W, b, y, precision=prec)
        ref = oracle.linear(x.cpu().numpy(), W.cpu().numpy(), b.cpu().numpy())
        assert rel_err(y.cpu().numpy(), ref) < tol


def test_gemm_1024_config_vs_reference(cuda):
    """SGEMM config: M=N=K=1024, U[-1,1], beta=0, against the compiled reference
    when it runs on this host, else the oracle."""
    import attn_cpu

    rng = np.random.default_rng(0)
    A = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
    B = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
    ref = oracle.ref_sgemm(A, B) if oracle.ref_available() else oracle.sgemm(A, B)
    assert rel_err(attn_cpu.gemm(A, B), ref) < TOL_3XTF32
    assert rel_err(attn_cpu.gemm(A, B, precision="tf32"), ref) < TOL_TF32
