"""Failure detection on the GPU without a fault: a kernel waits on a barrier
that nothing arrives on; its bounded wait expires (a fraction of a second),
the kernel returns normally and the host reads ATTNB_ERR_DEVICE_TIMEOUT from
the device status word.  The context stays usable afterwards."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_FP32, rel_err

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda):
    import torch
    from attn_cpu import capi

    s = torch.cuda.current_stream().cuda_stream
    capi.stream_status()  # start clean
    assert capi.lib().attnb_selftest_wait_timeout(200000, s) == capi.OK  # 0.2 s
    rc = capi.lib().attnb_stream_status(s)
    assert rc == capi.ERR_DEVICE_TIMEOUT
    assert b"bounded device wait" in capi.lib().attnb_last_error()
    # The status word was cleared and the device still computes correctly.
    capi.stream_status()
    import attn_cpu

    rng = np.random.default_rng(0)
    Q = rng.standard_normal((2, 64), dtype=np.float32)
    K = rng.standard_normal((2, 100, 64), dtype=np.float32)
    V = rng.standard_normal((2, 100, 64), dtype=np.float32)
    assert rel_err(attn_cpu.attn_step_dense(Q, K, V), oracle.attn_step(Q, K, V)) < TOL_FP32


def test_selftest_rejects_bad_limit(cuda):
    from attn_cpu import capi

    assert capi.lib().attnb_selftest_wait_timeout(0, None) == capi.ERR_INVALID_ARGUMENT
