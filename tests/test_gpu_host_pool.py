"""Page-locked result memory (attnb_host_alloc / attnb_host_free) and the
Python module's result arrays, which come from it: every call returns its own
buffer, freed buffers are recycled, and a full pool falls back to ordinary
memory with the same results."""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
from conftest import ROOT, TOL_3XTF32, rel_err

pytestmark = pytest.mark.gpu


def test_host_alloc_free_roundtrip(cuda):
    from attn_cpu import capi

    L = capi.lib()
    p = ctypes.c_void_p()
    assert L.attnb_host_alloc(1000, ctypes.byref(p)) == capi.OK and p.value
    buf = (ctypes.c_float * 250).from_address(p.value)
    buf[0], buf[249] = 1.5, -2.0  # the whole request is usable
    assert (buf[0], buf[249]) == (1.5, -2.0)
    assert L.attnb_host_free(p) == capi.OK
    assert L.attnb_host_free(p) == capi.ERR_INVALID_ARGUMENT  # already returned
    assert L.attnb_host_free(ctypes.c_void_p(12345)) == capi.ERR_INVALID_ARGUMENT
    assert L.attnb_host_alloc(0, ctypes.byref(p)) == capi.ERR_INVALID_ARGUMENT
    q = ctypes.c_void_p()
    assert L.attnb_host_alloc(1000, ctypes.byref(q)) == capi.OK and q.value
    assert L.attnb_host_free(q) == capi.OK


def test_result_arrays_are_independent(cuda):
    import attn_cpu

    rng = np.random.default_rng(5)
    Q, K, V = (rng.standard_normal((4, 100, 32), dtype=np.float32) for _ in range(3))
    ref = oracle.attn_block(Q, K, V, False)
    a = attn_cpu.attn_block_dense(Q, K, V)
    b = attn_cpu.attn_block_dense(Q, K, V)
    assert a.ctypes.data != b.ctypes.data and a.flags.owndata is False
    assert a.flags.c_contiguous and a.flags.writeable and a.shape == (4, 100, 32)
    b_copy = b.copy()
    del a
    c = attn_cpu.attn_block_dense(2 * Q, K, V)  # may reuse a's block
    assert np.array_equal(b, b_copy)
    assert rel_err(b, ref) < TOL_3XTF32
    assert rel_err(c, oracle.attn_block(2 * Q, K, V, False)) < TOL_3XTF32


def test_gemm_fresh_result_semantics(cuda):
    import attn_cpu

    rng = np.random.default_rng(6)
    A = rng.standard_normal((33, 17), dtype=np.float32)
    B = rng.standard_normal((17, 9), dtype=np.float32)
    r = oracle.sgemm(A, B)
    for _ in range(3):  # recycled blocks hold old results; beta must not see them
        assert rel_err(attn_cpu.gemm(A, B, beta=2.0), r) < TOL_3XTF32
    assert np.array_equal(attn_cpu.gemm(np.zeros((3, 0), np.float32),
                                        np.zeros((0, 4), np.float32)), np.zeros((3, 4)))
    assert np.isnan(attn_cpu.gemm(A, B, beta=float("inf"))).all()


def test_pool_disabled_falls_back_to_ordinary_memory(cuda):
    code = (
        "import sys, numpy as np; sys.path[:0] = [sys.argv[1], sys.argv[2]]\n"
        "import attn_cpu, oracle\n"
        "rng = np.random.default_rng(7)\n"
        "Q, K, V = (rng.standard_normal((2, 64, 32), dtype=np.float32) for _ in range(3))\n"
        "o = attn_cpu.attn_block_dense(Q, K, V)\n"
        "assert o.flags.owndata, 'expected an ordinary numpy buffer'\n"
        "r = oracle.attn_block(Q, K, V, False)\n"
        "print(float(np.abs(o - r).max() / np.abs(r).max()))\n")
    env = dict(os.environ, ATTNB_PINNED_POOL_MB="0")
    out = subprocess.run([sys.executable, "-c", code, os.path.join(ROOT, "attn-cpu_b200"),
                          os.path.join(ROOT, "oracle")], env=env, capture_output=True,
                         text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    assert float(out.stdout.strip().splitlines()[-1]) < TOL_3XTF32
