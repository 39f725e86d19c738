"""Decode step (attn_step_dense) on the GPU against the oracle and the
reference's golden vectors.  Plain fp32 FMA on CUDA cores: bar 1e-5."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_FP32, rel_err

pytestmark = pytest.mark.gpu


def _inputs(H, Dh, T, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((H, Dh), dtype=np.float32),
            rng.standard_normal((H, T, Dh), dtype=np.float32),
            rng.standard_normal((H, T, Dh), dtype=np.float32))


@pytest.mark.parametrize("H,Dh,T", [(1, 64, 1), (4, 64, 128), (8, 64, 1024), (8, 128, 512),
                                    (16, 96, 256), (3, 16, 5), (2, 256, 700), (5, 36, 333),
                                    (1, 130, 40), (2, 300, 17)])
def test_step_vs_oracle(cuda, H, Dh, T):
    """Shapes of the reference's tests/test_attn_step.py:148-157 plus tails and
    head sizes that take the generic (non-vector) kernel."""
    import attn_cpu

    Q, K, V = _inputs(H, Dh, T, 42)
    got = attn_cpu.attn_step_dense(Q, K, V)
    assert got.shape == (H, Dh)
    assert rel_err(got, oracle.attn_step(Q, K, V)) < TOL_FP32
    # The reference test's own bar (atol=1e-5, rtol=1e-6 against SDPA).
    np.testing.assert_allclose(got, oracle.attn_step(Q, K, V), atol=1e-5, rtol=1e-6)


def test_step_golden(cuda, golden):
    import attn_cpu

    for c in sorted({k.split("_")[0] for k in golden.files if k.startswith("step")}):
        got = attn_cpu.attn_step_dense(golden[f"{c}_Q"], golden[f"{c}_K"], golden[f"{c}_V"])
        assert rel_err(got, golden[f"{c}_O"]) < TOL_FP32, c


def test_step_strided_views_dev(cuda):
    """Non-contiguous K/V/O views through the device-pointer entry point."""
    import torch
    from attn_cpu import capi

    g = torch.Generator().manual_seed(7)
    H, T, Dh = 6, 300, 64
    base = torch.randn(T, H, 2 * Dh, generator=g)
    K = base[:, :, :Dh].permute(1, 0, 2)         # [H,T,Dh], strides (2Dh, H*2Dh, 1)
    V = base[:, :, Dh:].permute(1, 0, 2)
    Q = torch.randn(H, Dh, generator=g)
    ref = oracle.attn_step(Q.numpy(), np.ascontiguousarray(K.numpy()),
                           np.ascontiguousarray(V.numpy()))
    dK, dV = base.cuda()[:, :, :Dh].permute(1, 0, 2), base.cuda()[:, :, Dh:].permute(1, 0, 2)
    dO = torch.zeros(H, 2 * Dh, device="cuda")[:, ::2]  # strideDh = 2
    capi.attn_step_dense_dev(Q.cuda(), dK, dV, dO)
    capi.stream_status()
    assert rel_err(dO.cpu().numpy(), ref) < TOL_FP32
    # Transposed K (strideDh != 1) takes the generic kernel.
    Kt = dK.contiguous().transpose(1, 2).contiguous().transpose(1, 2)
    dO2 = torch.empty(H, Dh, device="cuda")
    capi.attn_step_dense_dev(Q.cuda(), Kt, dV, dO2)
    assert rel_err(dO2.cpu().numpy(), ref) < TOL_FP32


def test_step_decode_config_full_size(cuda):
    """Decode config at full size: B=8 x H=32 heads, T=4096, Dh=128 (K+V = 1 GiB)."""
    import torch
    from attn_cpu import capi

    g = torch.Generator(device="cuda").manual_seed(11)
    H, T, Dh = 256, 4096, 128
    Q = torch.randn(H, Dh, device="cuda", generator=g)
    K = torch.randn(H, T, Dh, device="cuda", generator=g)
    V = torch.randn(H, T, Dh, device="cuda", generator=g)
    O = torch.empty(H, Dh, device="cuda")
    capi.attn_step_dense_dev(Q, K, V, O)
    capi.stream_status()
    heads = [0, 1, 77, 128, 255]
    ref = oracle.attn_step(Q[heads].cpu().numpy(), K[heads].cpu().numpy(), V[heads].cpu().numpy())
    assert rel_err(O[heads].cpu().numpy(), ref) < TOL_FP32
    # Size-independent property: softmax weights sum to one, so a V of ones
    # gives exactly ones everywhere.
    capi.attn_step_dense_dev(Q, K, torch.ones_like(V), O)
    assert torch.allclose(O, torch.ones_like(O), atol=2e-6)
