"""attnb_gemm_ex_bcast_dev on one GPU: the product goes to C and, element for
element, to every replica.  Here the replicas are other buffers on the same
device (on a node they are the other GPUs' copies, mapped with
attnb_ipc_import), so the epilogue's transposed row stores, ragged edges,
scalar tails and replica count are checked without a second GPU: C against
the float64 oracle, every replica bit-identical to C, and the bytes around
each replica's block untouched.  The entry has no reference counterpart; the
row-sharded SGEMM and the sharded MHA block assemble their outputs with it."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from conftest import TOL_3XTF32, TOL_TF32, rel_err

pytestmark = pytest.mark.gpu

CASES = [
    # M, K, N, trans_a, trans_b, replicas
    (1, 1, 1, False, False, 1),
    (37, 53, 71, False, True, 3),        # ragged tile edges, odd row length
    (300, 129, 256, True, True, 7),      # the MHA block's transposed form, full fan-out
    (1024, 512, 768, False, False, 2),   # several tiles per CTA
    (130, 64, 1030, False, False, 7),    # ldc % 4 != 0: scalar stores
]


@pytest.mark.parametrize("prec", ["3xtf32", "tf32"])
@pytest.mark.parametrize("M,K,N,ta,tb,nrep", CASES)
def test_gemm_bcast_vs_oracle_and_replicas(cuda, M, K, N, ta, tb, nrep, prec):
    import torch
    from attn_cpu import capi

    rng = np.random.default_rng(M + 11 * K + 7 * N + nrep)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    bias = rng.standard_normal(N, dtype=np.float32)
    ref = oracle.sgemm(A, B).astype(np.float64) + bias
    sa = torch.from_numpy(np.ascontiguousarray(A.T if ta else A)).cuda()
    sb = torch.from_numpy(np.ascontiguousarray(B.T if tb else B)).cuda()
    C = torch.full((M, N), float("nan"), device="cuda")
    # Each replica is rows [pad, pad + M) of a larger buffer filled with a
    # sentinel, so stray stores outside the block show.
    pad = 4  # rows; keeps each replica at C's alignment modulo 16 bytes
    sentinel = -12345.0
    reps = [torch.full((M + 2 * pad, N), sentinel, device="cuda") for _ in range(nrep)]
    capi.gemm_ex_bcast_dev(sa, sb, C, [r[pad:pad + M].data_ptr() for r in reps], trans_a=ta,
                           trans_b=tb, bias=torch.from_numpy(bias).cuda(), precision=prec)
    torch.cuda.synchronize()
    c = C.cpu().numpy()
    tol = TOL_TF32 if prec == "tf32" else TOL_3XTF32
    assert rel_err(c, ref) < tol
    for r in reps:
        h = r.cpu().numpy()
        assert np.array_equal(h[pad:pad + M], c)
        assert np.all(h[:pad] == sentinel) and np.all(h[pad + M:] == sentinel)


def test_gemm_bcast_empty_product_and_alpha_zero(cuda):
    """K == 0 gives C = beta * C + bias on C and the replicas; alpha == 0 with
    no bias scales C and copies it."""
    import torch
    from attn_cpu import capi

    M, N = 50, 70
    C0 = torch.randn(M, N, device="cuda")
    bias = torch.randn(N, device="cuda")
    A = torch.zeros(M, 0, device="cuda")
    B = torch.zeros(0, N, device="cuda")
    C = C0.clone()
    reps = [torch.zeros(M, N, device="cuda") for _ in range(2)]
    capi.gemm_ex_bcast_dev(A, B, C, [r.data_ptr() for r in reps], bias=bias, beta=0.5)
    torch.cuda.synchronize()
    want = 0.5 * C0 + bias
    assert torch.allclose(C, want, rtol=1e-6, atol=1e-6)
    for r in reps:
        assert torch.equal(r, C)
    A = torch.randn(M, 20, device="cuda")
    B = torch.randn(20, N, device="cuda")
    C = C0.clone()
    capi.gemm_ex_bcast_dev(A, B, C, [r.data_ptr() for r in reps], alpha=0.0, beta=2.0)
    torch.cuda.synchronize()
    assert torch.allclose(C, 2.0 * C0)
    for r in reps:
        assert torch.equal(r, C)


def test_gemm_bcast_argument_checks(cuda):
    import torch
    from attn_cpu import capi

    L = capi.lib()
    A = torch.randn(8, 8, device="cuda")
    C = torch.zeros(8, 8, device="cuda")
    reps = (ctypes.c_void_p * 8)(*([C.data_ptr()] * 8))
    # more than seven replicas
    assert L.attnb_gemm_ex_bcast_dev(0, 0, A.data_ptr(), 8, A.data_ptr(), 8, None, C.data_ptr(),
                                     8, reps, 8, 8, 8, 8, 1.0, 0.0, -1, None) == capi.ERR_INVALID_ARGUMENT
    # a null replica
    nul = (ctypes.c_void_p * 1)(None)
    assert L.attnb_gemm_ex_bcast_dev(0, 0, A.data_ptr(), 8, A.data_ptr(), 8, None, C.data_ptr(),
                                     8, nul, 1, 8, 8, 8, 1.0, 0.0, -1, None) == capi.ERR_INVALID_ARGUMENT
    # a replica whose alignment modulo 16 bytes differs from C's
    buf = torch.zeros(100, device="cuda")
    odd = (ctypes.c_void_p * 1)(buf.data_ptr() + 4)
    assert L.attnb_gemm_ex_bcast_dev(0, 0, A.data_ptr(), 8, A.data_ptr(), 8, None, C.data_ptr(),
                                     8, odd, 1, 8, 8, 8, 1.0, 0.0, -1, None) == capi.ERR_INVALID_ARGUMENT


def test_ipc_export_of_shared_block(cuda):
    """A shared block is its own allocation (offset 0); a view into it exports
    the same handle with its byte offset; host memory is rejected."""
    import torch
    from attn_cpu import capi

    t = capi.shared_empty((64, 32))
    assert t.is_cuda and t.shape == (64, 32) and t.dtype == torch.float32
    h0, off0 = capi.ipc_export(t)
    h1, off1 = capi.ipc_export(t[5:])
    assert off0 == 0 and off1 == 5 * 32 * 4 and h0 == h1 and len(h0) == 64
    host = (ctypes.c_float * 16)()
    hbuf = ctypes.create_string_buffer(64)
    off = ctypes.c_uint64()
    assert capi.lib().attnb_ipc_export(ctypes.cast(host, ctypes.c_void_p), hbuf,
                                       ctypes.byref(off)) != capi.OK
    del t
    torch.cuda.synchronize()


def test_decode_bcast_vs_oracle_and_replicas(cuda):
    """attnb_attn_step_dense_bcast_dev: O against the oracle, each replica
    bit-identical, for a split plan (merge kernel stores) and a one-range plan
    (copies)."""
    import torch
    from attn_cpu import capi

    for H, T, Dh in ((6, 700, 128), (3, 40, 64)):
        g = torch.Generator(device="cuda").manual_seed(H * T)
        Q = torch.randn(H, Dh, device="cuda", generator=g)
        K = torch.randn(H, T, Dh, device="cuda", generator=g)
        V = torch.randn(H, T, Dh, device="cuda", generator=g)
        O = torch.full((H, Dh), float("nan"), device="cuda")
        reps = [torch.full((H, Dh), -1.0, device="cuda") for _ in range(3)]
        capi.attn_step_dense_bcast_dev(Q, K, V, O, [r.data_ptr() for r in reps])
        torch.cuda.synchronize()
        ref = oracle.attn_step(Q.cpu().numpy(), K.cpu().numpy(), V.cpu().numpy())
        assert rel_err(O.cpu().numpy(), ref) < 1e-5
        for r in reps:
            assert torch.equal(r, O)


def test_peer_barrier_single_gpu(cuda):
    """The peer-memory barrier with both flag arrays on this GPU (rank 0 of
    two): when the other rank's slot already holds the next epoch the kernel
    returns, has advanced its own count and written the epoch into the other
    rank's array; when nothing ever writes the slot, the bounded wait expires
    after 0.2 s, the status word reports ATTNB_ERR_DEVICE_TIMEOUT and the
    context stays usable."""
    import torch
    from attn_cpu import capi

    mine = torch.zeros(3, dtype=torch.int64, device="cuda")   # [slot 0, slot 1, count]
    other = torch.zeros(3, dtype=torch.int64, device="cuda")
    mine[1] = 1  # rank 1 has reached barrier 1
    capi.peer_barrier_dev(mine.data_ptr(), [0, other.data_ptr()], 0)
    capi.stream_status()
    assert mine.tolist() == [0, 1, 1] and other.tolist() == [1, 0, 0]
    capi.peer_barrier_dev(mine.data_ptr(), [0, other.data_ptr()], 0, limit_us=200000)
    with pytest.raises(capi.AttnbError) as e:
        capi.stream_status()
    assert e.value.code == capi.ERR_DEVICE_TIMEOUT
    assert mine.tolist() == [0, 1, 2] and other.tolist() == [2, 0, 0]
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum()) == 8.0
    capi.stream_status()  # cleared


def test_peer_barrier_in_cuda_graph(cuda):
    """The barrier count lives on the device: three replays of a captured
    barrier advance it three times (each replay passing, as the other rank's
    slot is set ahead)."""
    import torch
    from attn_cpu import capi

    mine = torch.zeros(3, dtype=torch.int64, device="cuda")
    other = torch.zeros(3, dtype=torch.int64, device="cuda")
    mine[1] = 100
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        capi.peer_barrier_dev(mine.data_ptr(), [0, other.data_ptr()], 0)  # outside the graph
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            capi.peer_barrier_dev(mine.data_ptr(), [0, other.data_ptr()], 0)
    torch.cuda.synchronize()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    capi.stream_status()
    assert mine[2].item() == 4 and other[0].item() == 4
