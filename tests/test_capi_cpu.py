"""Boundary checks that need no GPU: the C ABI library loads and exports every
symbol include/attnb.h declares, the reference-compatible C++ shims link, and
argument validation raises the reference's exception types and messages
before any device work."""
from __future__ import annotations

import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT

import attn_cpu
from attn_cpu import capi

HEADER = os.path.join(ROOT, "include", "attnb.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(attnb_\w+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    names = declared_symbols()
    assert len(names) >= 13
    lib = capi.lib()
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(capi.EXPORTED)


def test_cxx_shim_symbols_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", capi.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    for sym in ("attn::attn_step_dense(", "attn::attn_block_dense(", "attn::mha_block_dense(",
                "gemm::sgemm_blocked(", "gemm::gemm_blocked_jit("):
        assert sym in out, sym


def test_version():
    assert "sm_100a" in attn_cpu.version()


def test_gemm_shape_errors():
    with pytest.raises(ValueError, match="Inner dim mismatch"):
        attn_cpu.gemm(np.ones((4, 5), np.float32), np.ones((4, 5), np.float32))
    with pytest.raises(ValueError, match="must be 2D"):
        attn_cpu.gemm(np.ones(4, np.float32), np.ones((4, 5), np.float32))


def test_mha_shape_errors():
    x = np.ones((8, 32), np.float32)
    with pytest.raises(ValueError, match=r"W_in shape must be \[3D, D\]"):
        attn_cpu.mha_block_dense(x, np.ones((32, 32), np.float32), np.ones(96, np.float32),
                                 np.ones((32, 32), np.float32), np.ones(32, np.float32), 4)
    with pytest.raises(ValueError, match="num_heads must divide D"):
        attn_cpu.mha_block_dense(x, np.ones((96, 32), np.float32), np.ones(96, np.float32),
                                 np.ones((32, 32), np.float32), np.ones(32, np.float32), 5)


def test_step_validation_matches_reference_messages():
    Q = np.ones((2, 64), np.float32)
    K = np.ones((3, 10, 64), np.float32)
    with pytest.raises(ValueError, match="K/V H must match Q.H"):
        attn_cpu.attn_step_dense(Q, K, K)
    K2 = np.ones((2, 10, 32), np.float32)
    with pytest.raises(ValueError, match="K/V Dh must match Q.Dh"):
        attn_cpu.attn_step_dense(Q, K2, K2)


def test_block_validation_matches_reference_messages():
    Q = np.ones((2, 5, 16), np.float32)
    K = np.ones((2, 7, 16), np.float32)
    with pytest.raises(ValueError, match="causal=true requires L==T"):
        attn_cpu.attn_block_dense(Q, K, K, causal=True)
    with pytest.raises(ValueError, match="Dh mismatch"):
        attn_cpu.attn_block_dense(Q, np.ones((2, 7, 8), np.float32), K)


def test_precision_argument():
    with pytest.raises(ValueError):
        attn_cpu.gemm(np.ones((2, 2), np.float32), np.ones((2, 2), np.float32), precision="fp8")


def test_c_abi_invalid_argument_codes():
    lib = capi.lib()
    t = capi.Tensor(None, 1, 1, 16, 16, 0, 1)
    import ctypes
    rc = lib.attnb_attn_step_dense(ctypes.byref(t), ctypes.byref(t), ctypes.byref(t),
                                   ctypes.byref(t))
    assert rc == capi.ERR_INVALID_ARGUMENT
    assert b"Null data pointer" in lib.attnb_last_error()
    # M, N or K <= 0 returns success without touching anything (src/gemm.cpp:324).
    assert lib.attnb_sgemm(None, 0, 5, None, 5, None, 1.0, 0.0, -1) == capi.OK


CXX_PROGRAM = r"""
#include <cstdio>
#include <stdexcept>
#include "attn.h"
#include "gemm.h"
int main() {
  float q[4] = {0}, k[4] = {0};
  attn::TensorF32 Q{q, 1, 1, 4, 4, 0, 1}, K{k, 2, 1, 4, 4, 4, 1};
  attn::MutableTensorF32 O{q, 1, 4, 4, 1};
  try { attn::attn_step_dense(Q, K, K, O); }
  catch (const std::invalid_argument& e) { std::printf("invalid_argument: %s\n", e.what()); return 0; }
  return 1;
}
"""


def test_cxx_drop_in_headers_compile_and_throw(tmp_path):
    src = tmp_path / "prog.cpp"
    src.write_text(CXX_PROGRAM)
    exe = tmp_path / "prog"
    pkg = os.path.dirname(capi.LIB_PATH)
    subprocess.run(["/usr/bin/g++", "-std=c++17", "-I", os.path.join(ROOT, "include"), str(src),
                    "-L", pkg, "-lattnb", f"-Wl,-rpath,{pkg}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "K/V H must match Q.H" in r.stdout
