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


# A child process with the device arenas capped at 2 MiB
# (ATTNB_DEVICE_ARENA_CAP_MB, read once at the first allocation): calls that
# need more fail with ATTNB_ERR_OUT_OF_MEMORY before any work is enqueued --
# MemoryError from the Python module and the ctypes layer, std::bad_alloc from
# the C++ drop-in headers, the reference's exception for a failed allocation --
# and calls that fit still run and are correct.
ARENA_CAP_CHILD = r"""
import sys
import numpy as np
import torch
sys.path[:0] = [sys.argv[1], sys.argv[2]]
import attn_cpu, oracle
from attn_cpu import capi
rng = np.random.default_rng(0)
A = rng.uniform(-1, 1, (1024, 1024)).astype(np.float32)
try:
    attn_cpu.gemm(A, A)
    sys.exit("host-pointer gemm past the cap did not fail")
except MemoryError as e:
    assert "arena cap" in capi.lib().attnb_last_error().decode(), e
dA = torch.from_numpy(A).cuda()
dC = torch.empty_like(dA)
try:
    capi.sgemm_dev(dA, dA, dC)
    sys.exit("device-pointer sgemm past the cap did not fail")
except capi.AttnbOutOfMemory as e:
    assert e.code == capi.ERR_OUT_OF_MEMORY
a, b = A[:40, :30].copy(), A[:30, :50].copy()
y = attn_cpu.gemm(a, b)
assert np.max(np.abs(y - oracle.sgemm(a, b))) / np.max(np.abs(oracle.sgemm(a, b))) < 1e-5
print("arena cap ok")
"""

CXX_BAD_ALLOC = r"""
#include <cstdio>
#include <new>
#include <vector>
#include "gemm.h"
int main() {
  std::vector<float> A(1024 * 1024, 0.5f), C(1024 * 1024);
  try { gemm::sgemm_blocked(A.data(), 1024, 1024, A.data(), 1024, C.data()); }
  catch (const std::bad_alloc&) { std::printf("bad_alloc\n"); return 0; }
  return 1;
}
"""


def test_allocation_failure_maps_to_out_of_memory(cuda, tmp_path):
    import os
    import subprocess
    import sys

    from attn_cpu import capi

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, ATTNB_DEVICE_ARENA_CAP_MB="2")
    r = subprocess.run([sys.executable, "-c", ARENA_CAP_CHILD,
                        os.path.join(root, "attn-cpu_b200"), os.path.join(root, "oracle")],
                       capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0 and "arena cap ok" in r.stdout, r.stdout + r.stderr
    src = tmp_path / "bad_alloc.cpp"
    src.write_text(CXX_BAD_ALLOC)
    exe = tmp_path / "bad_alloc"
    pkg = os.path.dirname(capi.LIB_PATH)
    subprocess.run(["/usr/bin/g++", "-std=c++17", "-I", os.path.join(root, "include"), str(src),
                    "-L", pkg, "-lattnb", f"-Wl,-rpath,{pkg}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0 and "bad_alloc" in r.stdout, r.stdout + r.stderr
