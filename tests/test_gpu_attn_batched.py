"""attnb_attn_block_dense_batched_dev (independent sequences at a fixed batch
stride, run side by side on forked streams) against the oracle, sequence by
sequence: head-strided views cut from a packed [B, T, 3 * H * Dh] projection
(the MHA block's layout), an output written transposed ([H * Dh, B * T], the
sharded MHA block's send buffer), more sequences than forks, causal masks,
both precisions, and the argument checks."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_3XTF32, TOL_TF32, rel_err

pytestmark = pytest.mark.gpu

CASES = [
    (3, 4, 300, 64, False),
    (6, 2, 256, 128, True),   # more sequences than the four forks
    (2, 8, 520, 48, False),   # head size padded to 64, ragged tiles
]


@pytest.mark.parametrize("prec", ["3xtf32", "tf32"])
@pytest.mark.parametrize("B,H,T,Dh,causal", CASES)
def test_batched_vs_oracle(cuda, B, H, T, Dh, causal, prec):
    import torch
    from attn_cpu import capi

    rng = np.random.default_rng(B * 100 + H * 10 + Dh)
    qkv = rng.standard_normal((B, T, 3 * H * Dh), dtype=np.float32)
    d = torch.from_numpy(qkv).cuda()

    def heads(p):
        return d[:, :, p * H * Dh:(p + 1) * H * Dh].view(B, T, H, Dh).permute(0, 2, 1, 3)

    outT = torch.full((H * Dh, B * T), 7.0, device="cuda")
    capi.attn_block_dense_batched_dev(heads(0), heads(1), heads(2),
                                      outT.view(H, Dh, B, T).permute(2, 0, 3, 1),
                                      causal=causal, precision=prec)
    torch.cuda.synchronize()
    got = outT.view(H, Dh, B, T).permute(2, 0, 3, 1).cpu().numpy()
    tol = TOL_TF32 if prec == "tf32" else TOL_3XTF32
    for b in range(B):
        q, k, v = (np.ascontiguousarray(
            qkv[b, :, p * H * Dh:(p + 1) * H * Dh].reshape(T, H, Dh).transpose(1, 0, 2))
            for p in range(3))
        assert rel_err(got[b], oracle.attn_block(q, k, v, causal)) < tol, b


def test_batched_argument_checks(cuda):
    import torch
    from attn_cpu import capi

    Q = torch.zeros(2, 2, 16, 32, device="cuda")
    O = torch.zeros(2, 2, 16, 32, device="cuda")
    with pytest.raises(ValueError):
        capi.attn_block_dense_batched_dev(Q, Q[:1], Q, O)
    with pytest.raises(ValueError):
        capi.attn_block_dense_batched_dev(Q[0], Q[0], Q[0], O[0])
    # a shape mismatch inside one sequence is the reference's invalid_argument
    with pytest.raises(capi.AttnbError):
        capi.attn_block_dense_batched_dev(Q, Q[:, :, :, :16], Q, O)
    capi.attn_block_dense_batched_dev(Q[:0], Q[:0], Q[:0], O[:0])  # no sequences
