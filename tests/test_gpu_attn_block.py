"""Prefill attention (attn_block_dense) on the GPU against the oracle and the
reference's golden vectors, causal and not, L != T, strided views."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_3XTF32, TOL_TF32, rel_err

pytestmark = pytest.mark.gpu


def _qkv(H, L, T, Dh, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((H, L, Dh), dtype=np.float32),
            rng.standard_normal((H, T, Dh), dtype=np.float32),
            rng.standard_normal((H, T, Dh), dtype=np.float32))


@pytest.mark.parametrize("H,L,T,Dh,causal", [
    (8, 512, 512, 64, False),    # prefill config [1,8,512,64]
    (8, 512, 512, 64, True),
    (2, 65, 65, 16, False), (2, 66, 66, 16, True), (3, 100, 37, 32, False),
    (4, 128, 128, 128, False), (4, 200, 200, 128, True), (1, 1, 1, 64, False),
    (2, 33, 300, 96, False), (1, 70, 70, 48, True), (2, 129, 129, 64, True),
    (32, 256, 256, 128, False), (2, 300, 300, 32, True), (1, 1000, 1000, 64, False),
    (2, 100, 100, 200, False), (1, 70, 70, 160, True),   # head sizes > 128: CUDA-core kernel
    (6, 300, 300, 64, False), (5, 400, 400, 48, True),   # head counts that 4 does not divide
])
def test_block_vs_oracle(cuda, H, L, T, Dh, causal):
    import attn_cpu

    Q, K, V = _qkv(H, L, T, Dh, L * 31 + T)
    ref = oracle.attn_block(Q, K, V, causal)
    got = attn_cpu.attn_block_dense(Q, K, V, causal=causal)
    assert rel_err(got, ref) < TOL_3XTF32
    got_tf32 = attn_cpu.attn_block_dense(Q, K, V, causal=causal, precision="tf32")
    assert rel_err(got_tf32, ref) < TOL_TF32


def test_block_golden(cuda, golden):
    import attn_cpu

    for c in sorted({k.split("_")[0] for k in golden.files if k.startswith("block")}):
        got = attn_cpu.attn_block_dense(golden[f"{c}_Q"], golden[f"{c}_K"], golden[f"{c}_V"],
                                        causal=bool(golden[f"{c}_causal"]))
        assert rel_err(got, golden[f"{c}_O"]) < TOL_3XTF32, c


def test_block_head_strided_dev(cuda):
    """Q/K/V read in place from a projected [T, 3D] buffer (the MHA layout)."""
    import torch
    from attn_cpu import capi

    T, H, Dh = 256, 4, 64
    D = H * Dh
    g = torch.Generator(device="cuda").manual_seed(3)
    qkv = torch.randn(T, 3 * D, device="cuda", generator=g)
    view = lambda off: qkv[:, off:off + D].reshape(T, H, Dh).permute(1, 0, 2)
    Q, K, V = view(0), view(D), view(2 * D)
    O = torch.empty(T, D, device="cuda")
    Ov = O.view(T, H, Dh).permute(1, 0, 2)
    capi.attn_block_dense_dev(Q, K, V, Ov, causal=True)
    capi.stream_status()
    ref = oracle.attn_block(*(np.ascontiguousarray(t.cpu().numpy()) for t in (Q, K, V)), True)
    assert rel_err(Ov.cpu().numpy(), ref) < TOL_3XTF32


@pytest.mark.parametrize("layout", ["head_strided", "column_strided", "unaligned"])
@pytest.mark.parametrize("T,Dh", [(512, 64), (100, 40), (384, 17)])
def test_block_views_single_tile_dev(cuda, layout, T, Dh):
    """Non-causal calls whose CTAs each hold one key tile (the kernel converts
    the raw operands itself) over views its vector loads cannot take."""
    import torch
    from attn_cpu import capi

    H = 4
    g = torch.Generator(device="cuda").manual_seed(T + Dh)
    if layout == "head_strided":      # [T, 3, H, Dh] buffer, rows 3*H*Dh apart
        qkv = torch.randn(T, 3, H, Dh, device="cuda", generator=g)
        Q, K, V = (qkv[:, i].permute(1, 0, 2) for i in range(3))
    elif layout == "column_strided":  # [H, Dh, T] storage: unit stride along T
        Q, K, V = (torch.randn(H, Dh, T, device="cuda", generator=g).transpose(1, 2)
                   for _ in range(3))
    else:                             # contiguous but 4 bytes off a 16-byte boundary
        flat = torch.randn(3 * H * T * Dh + 1, device="cuda", generator=g)
        Q, K, V = (flat[1 + i * H * T * Dh:1 + (i + 1) * H * T * Dh].view(H, T, Dh)
                   for i in range(3))
    O = torch.empty(H, T, Dh, device="cuda")
    host = [np.ascontiguousarray(t.cpu().numpy()) for t in (Q, K, V)]
    ref = oracle.attn_block(*host, False)
    for prec, tol in (("3xtf32", TOL_3XTF32), ("tf32", TOL_TF32)):
        O.fill_(float("nan"))
        capi.attn_block_dense_dev(Q, K, V, O, False, prec)
        capi.stream_status()
        assert rel_err(O.cpu().numpy(), ref) < tol, prec


def test_mha_np_driver_runs(cuda):
    """The reference's NumPy driver (python/attn_cpu/mha_np.py) now has its binding."""
    from attn_cpu.mha_np import mha_forward_dense

    rng = np.random.default_rng(0)
    T, D, H = 64, 128, 8
    x = rng.standard_normal((T, D), dtype=np.float32)
    Wi = (rng.standard_normal((3 * D, D)) / np.sqrt(D)).astype(np.float32)
    bi = (0.1 * rng.standard_normal(3 * D)).astype(np.float32)
    Wo = (rng.standard_normal((D, D)) / np.sqrt(D)).astype(np.float32)
    bo = (0.1 * rng.standard_normal(D)).astype(np.float32)
    for causal in (False, True):
        y = mha_forward_dense(x, Wi, bi, Wo, bo, H, causal)
        assert rel_err(y, oracle.mha_block(x, Wi, bi, Wo, bo, H, causal)) < 1e-5
