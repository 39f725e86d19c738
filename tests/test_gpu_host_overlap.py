"""Host-pointer prefill calls on page-locked buffers split their heads into
groups whose copies in, attention launches and copies out overlap on three
streams.  A child process lowers the size gate (ATTNB_HOST_OVERLAP_MB) and
asks for three groups (ATTNB_HOST_GROUPS), so that small calls take that path
with ragged groups; every result must match the oracle."""
from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT, TOL_3XTF32, TOL_TF32

pytestmark = pytest.mark.gpu

CHILD = r"""
import json, sys
import numpy as np
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import torch
import attn_cpu, oracle
from attn_cpu import capi

def pinned(a):
    return torch.from_numpy(a).pin_memory().numpy()

cases = [(8, 256, 256, 64, False), (5, 300, 300, 48, True), (4, 128, 1000, 128, False),
         (3, 512, 512, 160, False)]
res = []
for i, (H, L, T, Dh, causal) in enumerate(cases):
    rng = np.random.default_rng(100 + i)
    Q, K, V = (rng.standard_normal((H, n, Dh), dtype=np.float32) for n in (L, T, T))
    r = oracle.attn_block(Q, K, V, causal)
    hq, hk, hv = pinned(Q), pinned(K), pinned(V)
    for prec in ("3xtf32", "tf32"):
        capi.profile_read("attn_tc")
        capi.profile_enable(True)
        o = attn_cpu.attn_block_dense(hq, hk, hv, causal=causal, precision=prec)
        capi.profile_enable(False)
        _, launches = capi.profile_read("attn_tc")
        err = float(np.abs(o - r).max() / np.abs(r).max())
        res.append({"case": [H, L, T, Dh, causal], "prec": prec, "err": err,
                    "launches": launches})
    # The same call on pageable inputs takes the single-launch path.
    o = attn_cpu.attn_block_dense(Q, K, V, causal=causal)
    res.append({"case": [H, L, T, Dh, causal], "prec": "3xtf32-pageable",
                "err": float(np.abs(o - r).max() / np.abs(r).max()), "launches": None})
print(json.dumps(res))
"""


def test_overlapped_host_prefill_matches_oracle(cuda):
    env = dict(os.environ, ATTNB_HOST_OVERLAP_MB="1", ATTNB_HOST_GROUPS="3")
    out = subprocess.run([sys.executable, "-c", CHILD, os.path.join(ROOT, "attn-cpu_b200"),
                          os.path.join(ROOT, "oracle")], env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    res = json.loads(out.stdout.strip().splitlines()[-1])
    assert len(res) == 12
    for r in res:
        tol = TOL_TF32 if r["prec"] == "tf32" else TOL_3XTF32
        assert r["err"] < tol, r
        H, Dh = r["case"][0], r["case"][3]
        if r["launches"] is not None and Dh <= 128:
            # one tcgen05 attention launch per head group (min(3, H) groups)
            assert r["launches"] == min(3, H), r
