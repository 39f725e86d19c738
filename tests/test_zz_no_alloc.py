"""attnb_attn_step_dense_noalloc: the decode step for callers that may not
allocate device memory (a pool or custom allocator that owns the device, a hot
path where allocation is forbidden).  It keeps its split-KV scratch in a fixed
2 MiB device array instead of allocating.  Checked through the C ABI against
the regular device entry point on two calls in a row (the second reuses the
array the first left behind), and for its size limit.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import TOL_FP32, rel_err

pytestmark = pytest.mark.gpu


def _call_noalloc(Q, K, V, O):
    from attn_cpu import capi

    q, k, v, o = capi.tensor3(Q, True), capi.tensor3(K), capi.tensor3(V), capi.tensor3(O, True)
    import torch

    return capi.lib().attnb_attn_step_dense_noalloc(
        ctypes.byref(q), ctypes.byref(k), ctypes.byref(v), ctypes.byref(o),
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_dev_entry_point_twice(cuda):
    import torch
    from attn_cpu import capi

    # The decode config's head shape (T=4096, Dh=128) with 64 heads, few enough
    # that the plan splits each head's keys, so the fixed scratch is used.
    # Different inputs on the two calls: the second must not see the first
    # call's partials.
    H, T, Dh = 64, 4096, 128
    for seed in (1, 2):
        g = torch.Generator(device="cuda").manual_seed(seed)
        Q = torch.randn(H, Dh, device="cuda", generator=g)
        K = torch.randn(H, T, Dh, device="cuda", generator=g)
        V = torch.randn(H, T, Dh, device="cuda", generator=g)
        O_ref = torch.empty(H, Dh, device="cuda")
        O_na = torch.full((H, Dh), float("nan"), device="cuda")
        capi.attn_step_dense_dev(Q, K, V, O_ref)
        rc = _call_noalloc(Q, K, V, O_na)
        assert rc == capi.OK, capi.lib().attnb_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(O_na).all()
        assert rel_err(O_na.cpu().numpy(), O_ref.cpu().numpy()) < TOL_FP32
        # and against the float64 oracle on sampled heads (first, middle, last)
        heads = [0, 1, H // 2, H - 1]
        r = oracle.attn_step(Q[heads].cpu().numpy(), K[heads].cpu().numpy(),
                             V[heads].cpu().numpy())
        assert rel_err(O_na[heads].cpu().numpy(), r) < TOL_FP32


def test_noalloc_small_and_strided(cuda):
    import torch
    from attn_cpu import capi

    g = torch.Generator(device="cuda").manual_seed(3)
    H, T, Dh = 5, 333, 96
    base = torch.randn(T, H, 2 * Dh, device="cuda", generator=g)
    K, V = base[:, :, :Dh].permute(1, 0, 2), base[:, :, Dh:].permute(1, 0, 2)
    Q = torch.randn(H, Dh, device="cuda", generator=g)
    O_ref, O_na = torch.empty(H, Dh, device="cuda"), torch.empty(H, Dh, device="cuda")
    for _ in range(2):
        capi.attn_step_dense_dev(Q, K, V, O_ref)
        assert _call_noalloc(Q, K, V, O_na) == capi.OK
        torch.cuda.synchronize()
        assert rel_err(O_na.cpu().numpy(), O_ref.cpu().numpy()) < TOL_FP32


def test_noalloc_rejects_scratch_beyond_limit(cuda):
    """A plan needing more than the fixed 2 MiB is refused before any work.
    The views overlap inside one small buffer, so every address is valid."""
    import torch
    from attn_cpu import capi

    H, T, Dh = 64, 4096, 2048
    buf = torch.zeros(H + T + Dh, device="cuda")
    K = buf.as_strided((H, T, Dh), (1, 1, 1))
    Q = buf.as_strided((H, Dh), (1, 1))
    O = torch.empty(H, Dh, device="cuda")
    rc = _call_noalloc(Q, K, K, O)
    assert rc == capi.ERR_INVALID_ARGUMENT
    assert b"fixed scratch" in capi.lib().attnb_last_error()
