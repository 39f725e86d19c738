"""attnb_gemm_ex_dev (C = alpha * op(A) . op(B) + beta * C + bias, op = none or
transpose) against the float64 oracle: every pair of transpose flags, ragged
sizes, column-slice operands (leading dimension larger than the row), a bias
with beta != 0, and the argument checks.  The entry has no reference
counterpart; the sharded MHA block reads the gathered context through it."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_3XTF32, TOL_TF32, rel_err

pytestmark = pytest.mark.gpu

SHAPES = [(1, 1, 1), (37, 53, 71), (128, 256, 96), (300, 129, 257), (1024, 512, 768)]


@pytest.mark.parametrize("prec", ["3xtf32", "tf32"])
@pytest.mark.parametrize("trans_a", [False, True])
@pytest.mark.parametrize("trans_b", [False, True])
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_gemm_ex_vs_oracle(cuda, M, K, N, trans_a, trans_b, prec):
    import torch
    from attn_cpu import capi

    rng = np.random.default_rng(M * 7 + K * 3 + N)
    A = rng.standard_normal((M, K), dtype=np.float32)
    B = rng.standard_normal((K, N), dtype=np.float32)
    C0 = rng.standard_normal((M, N), dtype=np.float32)
    bias = rng.standard_normal(N, dtype=np.float32)
    alpha, beta = 0.75, 0.5
    ref = alpha * oracle.sgemm(A, B).astype(np.float64) + beta * C0 + bias
    # Operands stored as the flags say, inside wider buffers (ld > row length).
    sa = A.T if trans_a else A
    sb = B.T if trans_b else B
    wa = torch.zeros(sa.shape[0], sa.shape[1] + 5, device="cuda")
    wa[:, 3:3 + sa.shape[1]] = torch.from_numpy(np.ascontiguousarray(sa)).cuda()
    wb = torch.zeros(sb.shape[0], sb.shape[1] + 9, device="cuda")
    wb[:, 1:1 + sb.shape[1]] = torch.from_numpy(np.ascontiguousarray(sb)).cuda()
    C = torch.from_numpy(C0).cuda()
    capi.gemm_ex_dev(wa[:, 3:3 + sa.shape[1]], wb[:, 1:1 + sb.shape[1]], C, trans_a=trans_a,
                     trans_b=trans_b, bias=torch.from_numpy(bias).cuda(), alpha=alpha,
                     beta=beta, precision=prec)
    torch.cuda.synchronize()
    tol = TOL_TF32 if prec == "tf32" else TOL_3XTF32
    assert rel_err(C.cpu().numpy(), ref) < tol


def test_gemm_ex_argument_checks(cuda):
    import ctypes

    from attn_cpu import capi

    L = capi.lib()
    buf = (ctypes.c_float * 64)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    # trans flag out of range
    assert L.attnb_gemm_ex_dev(2, 0, p, 4, p, 4, None, p, 4, 4, 4, 4, 1.0, 0.0, -1, None) != 0
    # lda too small for A^T stored [K, M]
    assert L.attnb_gemm_ex_dev(1, 0, p, 3, p, 4, None, p, 4, 4, 4, 4, 1.0, 0.0, -1, None) != 0
    # empty problem: nothing to do
    assert L.attnb_gemm_ex_dev(0, 0, p, 4, p, 4, None, p, 4, 0, 4, 4, 1.0, 0.0, -1, None) == 0


@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_gemm_ex_empty_inner_dimension(cuda, beta):
    """K == 0: the product is empty, so C = beta * C + bias (beta == 0 does not
    read C, whatever it holds); A and B are not read and may be NULL."""
    import torch
    from attn_cpu import capi

    M, N = 37, 70
    rng = np.random.default_rng(5)
    C0 = rng.standard_normal((M, N), dtype=np.float32)
    bias = rng.standard_normal(N, dtype=np.float32)
    C = torch.from_numpy(C0).cuda()
    if beta == 0.0:
        C.fill_(float("nan"))
    b = torch.from_numpy(bias).cuda()
    rc = capi.lib().attnb_gemm_ex_dev(0, 0, None, 0, None, N, b.data_ptr(), C.data_ptr(), N, M,
                                      N, 0, 1.0, beta, -1,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == capi.OK, capi.lib().attnb_last_error()
    torch.cuda.synchronize()
    ref = beta * C0.astype(np.float64) + bias if beta else np.broadcast_to(bias, (M, N))
    assert np.array_equal(C.cpu().numpy(), ref.astype(np.float32))
    # K < 0 is rejected
    assert capi.lib().attnb_gemm_ex_dev(0, 0, None, 0, None, N, None, C.data_ptr(), N, M, N, -1,
                                        1.0, beta, -1, None) == capi.ERR_INVALID_ARGUMENT
