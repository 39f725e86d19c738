"""1xTF32 prefill on CTA pairs (K3q, attn_pair.cu: one tcgen05.mma.cta_group::2
issues the products of two CTAs' query tiles) against the oracle.  The shapes
have head size 128, 300-320 (head, query tile) pairs (the band where K3q
needs fewer weighted waves of CTAs than K3 and K3p) and eight key tiles or
more, so TF32 calls take it: a ragged key range, an odd query-tile count (the
last pair's second tile is empty), an output view that rules out TMA stores,
and the same calls with K3q turned off (ATTNB_ATTN_CTA_PAIRS=0) in a child
process.  Heads are independent, so the oracle checks three heads of each
call (the first two and the last), which keeps it to seconds."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
from conftest import ROOT, TOL_TF32, rel_err

pytestmark = pytest.mark.gpu

SHAPES = [
    (20, 2048, 1024, 128),  # 16 query tiles per head
    (38, 1024, 1100, 128),  # ragged key range
    (60, 640, 1024, 128),   # five query tiles per head: odd
    (30, 1280, 1024, 96),   # head size 96 does not take K3q (K3p or K3 runs)
]
HEADS = lambda H: [0, 1, H - 1]


def _check(got, Q, K, V):
    hs = HEADS(Q.shape[0])
    ref = oracle.attn_block(Q[hs], K[hs], V[hs], False)
    assert rel_err(got[hs], ref) < TOL_TF32


def _qkv(H, L, T, Dh, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((H, L, Dh), dtype=np.float32),
            rng.standard_normal((H, T, Dh), dtype=np.float32),
            rng.standard_normal((H, T, Dh), dtype=np.float32))


@pytest.mark.parametrize("H,L,T,Dh", SHAPES)
def test_cta_pairs_vs_oracle(cuda, H, L, T, Dh):
    import attn_cpu

    Q, K, V = _qkv(H, L, T, Dh, H * 100 + T)
    _check(attn_cpu.attn_block_dense(Q, K, V, causal=False, precision="tf32"), Q, K, V)


def test_cta_pairs_plain_store_output(cuda):
    """Output rows 129 floats apart: no tensor map, so rows are stored directly."""
    import torch
    from attn_cpu import capi

    H, L, T, Dh = 38, 1024, 1100, 128
    Q, K, V = _qkv(H, L, T, Dh, 5)
    big = torch.full((H, L, Dh + 1), 7.0, device="cuda")
    O = big[:, :, :Dh]
    capi.attn_block_dense_dev(torch.from_numpy(Q).cuda(), torch.from_numpy(K).cuda(),
                              torch.from_numpy(V).cuda(), O, False, "tf32")
    torch.cuda.synchronize()
    _check(O.cpu().numpy(), Q, K, V)
    assert bool((big[:, :, Dh] == 7.0).all())


CHILD = r"""
import json, sys
import numpy as np
sys.path[:0] = [sys.argv[1]]
import attn_cpu
for i, (H, L, T, Dh) in enumerate(json.loads(sys.argv[2])):
    rng = np.random.default_rng(H * 100 + T)
    Q, K, V = (rng.standard_normal((H, n, Dh), dtype=np.float32) for n in (L, T, T))
    np.save(sys.argv[3] + f"/o{i}.npy", attn_cpu.attn_block_dense(Q, K, V, precision="tf32"))
print("done")
"""


def test_cta_pairs_switch_matches(cuda, tmp_path):
    """With K3q off the same calls run K3p or K3; both agree with the oracle
    and with each other."""
    import attn_cpu

    shapes = SHAPES[:2]
    env = dict(os.environ, ATTNB_ATTN_CTA_PAIRS="0")
    out = subprocess.run([sys.executable, "-c", CHILD, os.path.join(ROOT, "attn-cpu_b200"),
                          json.dumps(shapes), str(tmp_path)], env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    for i, (H, L, T, Dh) in enumerate(shapes):
        Q, K, V = _qkv(H, L, T, Dh, H * 100 + T)
        other = np.load(tmp_path / f"o{i}.npy")
        mine = attn_cpu.attn_block_dense(Q, K, V, precision="tf32")
        _check(other, Q, K, V)
        _check(mine, Q, K, V)
        assert rel_err(mine, other) < TOL_TF32
