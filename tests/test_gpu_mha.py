"""Full MHA block (mha_block_dense) on the GPU: the reference's test_mha.py
cases, the golden vectors, and the attention-block config at reduced T."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_3XTF32, TOL_TF32, rel_err

pytestmark = pytest.mark.gpu


def _weights(D, rng, bias=True):
    Wi = (rng.standard_normal((3 * D, D)) / np.sqrt(D)).astype(np.float32)
    Wo = (rng.standard_normal((D, D)) / np.sqrt(D)).astype(np.float32)
    bi = (0.1 * rng.standard_normal(3 * D)).astype(np.float32) if bias else np.zeros(3 * D, np.float32)
    bo = (0.1 * rng.standard_normal(D)).astype(np.float32) if bias else np.zeros(D, np.float32)
    return Wi, bi, Wo, bo


@pytest.mark.parametrize("T,D,H,causal", [
    (65, 128, 8, False), (66, 128, 8, True),     # tests/test_mha.py:68-70
    (64, 128, 8, False), (64, 128, 8, True),     # tests/test_attn_block.py:34-35
    (1, 64, 4, False), (300, 256, 2, True), (129, 512, 4, False), (77, 96, 3, True),
])
def test_mha_vs_oracle(cuda, T, D, H, causal):
    import attn_cpu

    rng = np.random.default_rng(T * 13 + D)
    x = rng.standard_normal((T, D), dtype=np.float32)
    Wi, bi, Wo, bo = _weights(D, rng)
    ref = oracle.mha_block(x, Wi, bi, Wo, bo, H, causal)
    assert rel_err(attn_cpu.mha_block_dense(x, Wi, bi, Wo, bo, H, causal), ref) < TOL_3XTF32
    y32 = attn_cpu.mha_block_dense(x, Wi, bi, Wo, bo, H, causal, precision="tf32")
    assert rel_err(y32, ref) < TOL_TF32


def test_mha_golden(cuda, golden):
    import attn_cpu

    for c in sorted({k.split("_")[0] for k in golden.files if k.startswith("mha")}):
        T, D, H, causal = (int(v) for v in golden[f"{c}_args"])
        y = attn_cpu.mha_block_dense(golden[f"{c}_x"], golden[f"{c}_Win"], golden[f"{c}_bin"],
                                     golden[f"{c}_Wout"], golden[f"{c}_bout"], H, bool(causal))
        assert rel_err(y, golden[f"{c}_y"]) < TOL_3XTF32, c


def test_mha_runtime_errors(cuda):
    import attn_cpu

    x = np.ones((4, 40), np.float32)
    with pytest.raises(RuntimeError, match="multiple of 16"):
        attn_cpu.mha_block_dense(x, np.ones((120, 40), np.float32), np.ones(120, np.float32),
                                 np.ones((40, 40), np.float32), np.ones(40, np.float32), 4)


def test_mha_block_config_batched_dev(cuda):
    """Attention-block config layout (Dh 128, weights N(0, 0.02^2), batched
    [B, T, D] on device) at hidden 1024 / 8 heads so the float64 oracle stays fast."""
    import torch
    from attn_cpu import capi

    g = torch.Generator(device="cuda").manual_seed(9)
    B, T, D, H = 2, 256, 1024, 8
    x = torch.randn(B, T, D, device="cuda", generator=g)
    Wi = torch.randn(3 * D, D, device="cuda", generator=g) * 0.02
    Wo = torch.randn(D, D, device="cuda", generator=g) * 0.02
    bi = torch.zeros(3 * D, device="cuda")
    bo = torch.zeros(D, device="cuda")
    y = torch.empty_like(x)
    capi.mha_block_dense_dev(x, Wi, bi, Wo, bo, H, y)
    capi.stream_status()
    for b in range(B):
        ref = oracle.mha_block(x[b].cpu().numpy(), Wi.cpu().numpy(), bi.cpu().numpy(),
                               Wo.cpu().numpy(), bo.cpu().numpy(), H, False)
        assert rel_err(y[b].cpu().numpy(), ref) < TOL_3XTF32


def test_mha_tf32_two_query_tile_kernel(cuda):
    """TF32 block with 16 heads x 1280 rows: 160 (head, query tile) pairs, so the
    attention takes the two-query-tile kernel, on the head-strided projections."""
    import attn_cpu

    rng = np.random.default_rng(21)
    T, D, H = 1280, 1024, 16
    x = rng.standard_normal((T, D), dtype=np.float32)
    Wi, bi, Wo, bo = _weights(D, rng)
    ref = oracle.mha_block(x, Wi, bi, Wo, bo, H, False)
    y = attn_cpu.mha_block_dense(x, Wi, bi, Wo, bo, H, False, precision="tf32")
    assert rel_err(y, ref) < TOL_TF32
