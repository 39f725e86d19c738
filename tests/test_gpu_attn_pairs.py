"""1xTF32 prefill with two query tiles per CTA (K3p, attn_pp.cu) against the
oracle.  The shapes below have 150-192 (head, query tile) pairs: the key range
is not split, and K3p needs one wave of CTAs where K3 needs two, so TF32 calls
take K3p.  Ragged L and T, odd query-tile counts (the second tile of the last
CTA is empty), causal masks, padded head sizes, an output view that rules out
TMA stores, and the same calls with K3p turned off (ATTNB_ATTN_PAIRS=0) in a
child process."""
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
    (40, 512, 512, 64, False),    # 160 (head, query tile) pairs
    (38, 500, 700, 48, False),    # ragged L and T, head size padded to 64
    (50, 384, 512, 32, False),    # three query tiles per head: odd
    (24, 896, 640, 96, False),    # seven query tiles per head
    (20, 1024, 700, 128, False),
    (24, 1024, 1024, 64, True),
    (50, 384, 384, 128, True),    # three query tiles, causal
    (40, 500, 500, 16, True),     # head size padded to 32, ragged
]


def _qkv(H, L, T, Dh, seed):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((H, L, Dh), dtype=np.float32),
            rng.standard_normal((H, T, Dh), dtype=np.float32),
            rng.standard_normal((H, T, Dh), dtype=np.float32))


@pytest.mark.parametrize("H,L,T,Dh,causal", SHAPES)
def test_pairs_vs_oracle(cuda, H, L, T, Dh, causal):
    import attn_cpu

    Q, K, V = _qkv(H, L, T, Dh, H * 1000 + L)
    ref = oracle.attn_block(Q, K, V, causal)
    got = attn_cpu.attn_block_dense(Q, K, V, causal=causal, precision="tf32")
    assert rel_err(got, ref) < TOL_TF32


def test_pairs_plain_store_output(cuda):
    """Output rows 65 floats apart: no tensor map, so rows are stored directly."""
    import torch
    from attn_cpu import capi

    H, L, T, Dh = 40, 512, 384, 64
    Q, K, V = _qkv(H, L, T, Dh, 7)
    ref = oracle.attn_block(Q, K, V, False)
    big = torch.full((H, L, Dh + 1), 7.0, device="cuda")
    O = big[:, :, :Dh]
    capi.attn_block_dense_dev(torch.from_numpy(Q).cuda(), torch.from_numpy(K).cuda(),
                              torch.from_numpy(V).cuda(), O, False, "tf32")
    torch.cuda.synchronize()
    assert rel_err(O.cpu().numpy(), ref) < TOL_TF32
    assert bool((big[:, :, Dh] == 7.0).all())  # the column between rows is untouched


CHILD = r"""
import json, sys
import numpy as np
sys.path[:0] = [sys.argv[1]]
import attn_cpu
out = {}
for i, (H, L, T, Dh, causal) in enumerate(json.loads(sys.argv[2])):
    rng = np.random.default_rng(H * 1000 + L)
    Q, K, V = (rng.standard_normal((H, n, Dh), dtype=np.float32) for n in (L, T, T))
    np.save(sys.argv[3] + f"/o{i}.npy", attn_cpu.attn_block_dense(Q, K, V, causal=causal,
                                                                   precision="tf32"))
print("done")
"""


def test_pairs_switch_matches(cuda, tmp_path):
    """The same calls with K3p off agree with the oracle too, and differ from
    K3p's results in the last bits (so the switch does change the kernel)."""
    import attn_cpu

    shapes = SHAPES[:3]
    env = dict(os.environ, ATTNB_ATTN_PAIRS="0")
    out = subprocess.run([sys.executable, "-c", CHILD, os.path.join(ROOT, "attn-cpu_b200"),
                          json.dumps(shapes), str(tmp_path)], env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    differs = False
    for i, (H, L, T, Dh, causal) in enumerate(shapes):
        Q, K, V = _qkv(H, L, T, Dh, H * 1000 + L)
        ref = oracle.attn_block(Q, K, V, causal)
        k3 = np.load(tmp_path / f"o{i}.npy")
        k3p = attn_cpu.attn_block_dense(Q, K, V, causal=causal, precision="tf32")
        assert rel_err(k3, ref) < TOL_TF32
        assert rel_err(k3p, ref) < TOL_TF32
        differs |= not np.array_equal(k3, k3p)
    assert differs
