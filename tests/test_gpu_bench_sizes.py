"""Parity at the sizes bench.py times, in both precisions, on sampled rows and
heads (the float64 oracle cannot redo the whole problems in seconds):

* the attention block, 4 sequences x 2048 tokens, hidden 4096, 32 heads
  (attn::mha_block_dense, src/attn_dispatch.cpp:17-133): rows of y of two
  sequences, against K and V projected in float64, the oracle's attention for
  those query rows and its output projection;
* SGEMM 16384^3 (gemm::sgemm_blocked, src/gemm.cpp:319-415): 32 rows of C,
  first and last tile rows included, which crosses the 3xTF32 kernel's
  accumulator drain at every 256 K steps 64 times;
* prefill [1, 32, 4096, 128] (attn::attn_block_dense, src/attn_block.cpp:104-241):
  the first two heads and the last, on sampled query rows (every key tile).

Bars: max|y - r| / max|r| <= 1e-5 (3xTF32) and 2e-3 (TF32), over the rows checked."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_3XTF32, TOL_TF32, rel_err

pytestmark = pytest.mark.gpu

PRECS = [("3xtf32", TOL_3XTF32), ("tf32", TOL_TF32)]


@pytest.mark.parametrize("prec,tol", PRECS)
def test_attention_block_config_full_size(cuda, prec, tol):
    import torch
    from attn_cpu import capi

    B, T, D, H = 4, 2048, 4096, 32
    Dh = D // H
    g = torch.Generator(device="cuda").manual_seed(44)
    x = torch.randn(B, T, D, device="cuda", generator=g)
    Wi = torch.randn(3 * D, D, device="cuda", generator=g) * 0.02
    Wo = torch.randn(D, D, device="cuda", generator=g) * 0.02
    bi = torch.randn(3 * D, device="cuda", generator=g) * 0.1
    bo = torch.randn(D, device="cuda", generator=g) * 0.1
    y = torch.empty_like(x)
    capi.mha_block_dense_dev(x, Wi, bi, Wo, bo, H, y, False, prec)
    torch.cuda.synchronize()
    capi.stream_status()
    Wi_h, bi_h, Wo_h, bo_h = (t.cpu().numpy() for t in (Wi, bi, Wo, bo))
    rows = np.array([0, 1, 127, 128, 1000, 2046, 2047])
    for b in (0, B - 1):
        xb = x[b].cpu().numpy()
        kv = oracle.linear_f64(xb, Wi_h[D:], bi_h[D:])              # [T, 2D]
        q = oracle.linear_f64(xb[rows], Wi_h[:D], bi_h[:D])         # [r, D]
        heads = lambda a: np.ascontiguousarray(a.reshape(a.shape[0], H, Dh).transpose(1, 0, 2),
                                               dtype=np.float32)
        ctx = oracle.attn_block(heads(q), heads(kv[:, :D]), heads(kv[:, D:]))  # [H, r, Dh]
        ctx = np.ascontiguousarray(ctx.transpose(1, 0, 2).reshape(len(rows), D))
        ref = oracle.linear(ctx, Wo_h, bo_h)
        got = y[b, torch.from_numpy(rows).cuda()].cpu().numpy()
        assert rel_err(got, ref) < tol, (b, rel_err(got, ref))


@pytest.mark.parametrize("prec,tol", PRECS)
def test_sgemm_16384_cubed(cuda, prec, tol):
    import torch
    from attn_cpu import capi

    n = 16384
    g = torch.Generator(device="cuda").manual_seed(45)
    A = torch.rand(n, n, device="cuda", generator=g) * 2 - 1
    B = torch.rand(n, n, device="cuda", generator=g) * 2 - 1
    C = torch.empty(n, n, device="cuda")
    capi.sgemm_dev(A, B, C, precision=prec)
    torch.cuda.synchronize()
    capi.stream_status()
    rng = np.random.default_rng(7)
    rows = np.unique(np.concatenate([[0, 1, 127, 128, 8191, 8192, n - 129, n - 2, n - 1],
                                     rng.integers(0, n, 23)]))
    idx = torch.from_numpy(rows).cuda()
    ref = oracle.sgemm_rows(A[idx].cpu().numpy(), B.cpu().numpy(), slice(None))
    assert rel_err(C[idx].cpu().numpy(), ref) < tol


@pytest.mark.parametrize("prec,tol", PRECS)
def test_prefill_1x32x4096x128(cuda, prec, tol):
    import torch
    from attn_cpu import capi

    H, L, Dh = 32, 4096, 128
    g = torch.Generator(device="cuda").manual_seed(46)
    Q, K, V = (torch.randn(H, L, Dh, device="cuda", generator=g) for _ in range(3))
    O = torch.empty_like(Q)
    capi.attn_block_dense_dev(Q, K, V, O, False, prec)
    torch.cuda.synchronize()
    capi.stream_status()
    rows = np.unique(np.concatenate([np.arange(0, 130), np.arange(130, L, 61), [L - 2, L - 1]]))
    idx = torch.from_numpy(rows).cuda()
    for h in (0, 1, H - 1):
        ref = oracle.attn_block(Q[h:h + 1, idx].cpu().numpy(), K[h:h + 1].cpu().numpy(),
                                V[h:h + 1].cpu().numpy())
        got = O[h:h + 1, idx].cpu().numpy()
        assert rel_err(got, ref) < tol, (h, rel_err(got, ref))
