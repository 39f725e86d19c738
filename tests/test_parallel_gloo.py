"""Multi-rank partitioning (attn_cpu.parallel) on CPU gloo ranks: the head,
row and column partitions and their all-gathers reassemble exactly what one
device computes.  Local compute is a float64 CPU stand-in so only the
partition/collective logic is under test here; the GPU kernels behind the
default ops are covered by the gpu-marked tests."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from attn_cpu.parallel import (CommInitError, ShardedMHA, attn_block_sharded,
                               attn_step_sharded, gemm_sharded, init_distributed, shard_range)

import oracle


class CPUOps:
    def linear(self, x, W, b, y):
        r = x.double() @ W.double().t()
        if b is not None:
            r = r + b.double()
        y.copy_(r.to(y.dtype))

    def attention(self, q, k, v, o, causal):
        qq = q.detach().numpy().astype(np.float32)
        kk = k.detach().numpy().astype(np.float32)
        vv = v.detach().numpy().astype(np.float32)
        o.copy_(torch.from_numpy(oracle.attn_block(qq, kk, vv, causal)))

    def attention_batched(self, q, k, v, o, causal):
        for b in range(q.shape[0]):
            self.attention(q[b], k[b], v[b], o[b], causal)

    def sgemm(self, A, B, C):
        C.copy_((A.double() @ B.double()).to(C.dtype))

    def decode(self, q, k, v, o):
        o.copy_(torch.from_numpy(oracle.attn_step(q.numpy().astype(np.float32),
                                                  k.numpy().astype(np.float32),
                                                  v.numpy().astype(np.float32))))

    def gemm_ex(self, A, B, C, trans_a, trans_b, bias):
        a = A.double().t() if trans_a else A.double()
        b = B.double().t() if trans_b else B.double()
        r = a @ b
        if bias is not None:
            r = r + bias.double()
        C.copy_(r.to(C.dtype))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        if case[0] == "mha":
            _, B, T, D, H, causal = case
            x = torch.randn(B, T, D, generator=g)
            Wi = torch.randn(3 * D, D, generator=g) / D ** 0.5
            bi = torch.randn(3 * D, generator=g) * 0.1
            Wo = torch.randn(D, D, generator=g) / D ** 0.5
            bo = torch.randn(D, generator=g) * 0.1
            y = ShardedMHA(Wi, bi, Wo, bo, H, causal, ops=CPUOps()).forward(x)
            ref = np.stack([oracle.mha_block(x[b].numpy(), Wi.numpy(), bi.numpy(), Wo.numpy(),
                                             bo.numpy(), H, causal) for b in range(B)])
            err = float(np.max(np.abs(y.numpy() - ref)) / np.max(np.abs(ref)))
        elif case[0] == "gemm":
            _, M, K, N, shard = case
            A = torch.rand(M, K, generator=g) * 2 - 1
            Bm = torch.rand(K, N, generator=g) * 2 - 1
            C = gemm_sharded(A, Bm, ops=CPUOps(), shard=shard)
            ref = oracle.sgemm(A.numpy(), Bm.numpy())
            err = float(np.max(np.abs(C.numpy() - ref)) / np.max(np.abs(ref)))
        elif case[0] == "decode":
            _, H, T, Dh = case
            Q = torch.randn(H, Dh, generator=g)
            # K and V as strided views into one [T, H, 2 Dh] buffer
            kv = torch.randn(T, H, 2 * Dh, generator=g)
            K, V = kv[:, :, :Dh].permute(1, 0, 2), kv[:, :, Dh:].permute(1, 0, 2)
            O = attn_step_sharded(Q, K, V, ops=CPUOps())
            ref = oracle.attn_step(Q.numpy(), np.ascontiguousarray(K.numpy()),
                                   np.ascontiguousarray(V.numpy()))
            err = float(np.max(np.abs(O.numpy() - ref)) / np.max(np.abs(ref)))
        else:
            _, H, L, Dh, causal = case
            Q, K, V = (torch.randn(H, L, Dh, generator=g) for _ in range(3))
            O = attn_block_sharded(Q, K, V, causal, ops=CPUOps())
            ref = oracle.attn_block(Q.numpy(), K.numpy(), V.numpy(), causal)
            err = float(np.max(np.abs(O.numpy() - ref)) / np.max(np.abs(ref)))
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


def _run(world, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    errs = [q.get(timeout=10) for _ in range(world)]
    assert max(e for _, e in errs) < 1e-6, errs


def test_shard_range_covers_everything():
    for n in (0, 1, 7, 32, 33, 4096):
        for w in (1, 2, 3, 8):
            parts = [shard_range(n, r, w) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))
            sizes = [b - a for a, b in parts]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world,case", [
    (2, ("mha", 2, 24, 64, 4, False)),
    (2, ("mha", 1, 17, 48, 3, True)),      # 3 heads over 2 ranks, 17 tokens: ragged
    (3, ("mha", 1, 20, 64, 8, False)),
    (4, ("mha", 2, 16, 32, 2, False)),     # more ranks than heads: two ranks hold none
    (2, ("mha", 2, 1100, 32, 2, False)),   # 2200 tokens, long sequences
])
def test_sharded_mha_gloo(world, case):
    _run(world, case)


@pytest.mark.parametrize("world,case", [
    (2, ("gemm", 37, 29, 41, "rows")),
    (2, ("gemm", 37, 29, 41, "cols")),
    (3, ("gemm", 64, 16, 10, "cols")),
    (3, ("gemm", 3100, 8, 20, "rows")),   # ragged row blocks
])
def test_sharded_gemm_gloo(world, case):
    _run(world, case)


def test_sharded_attention_gloo():
    _run(2, ("attn", 5, 33, 16, True))


@pytest.mark.parametrize("world,case", [
    (2, ("decode", 7, 50, 16)),   # 7 heads over 2 ranks: ragged
    (3, ("decode", 2, 33, 8)),    # more ranks than heads
])
def test_sharded_decode_gloo(world, case):
    _run(world, case)


# ------------------------------------------------------ failure detection
# Failures made on the host (no GPU involved): a rank that never joins the
# process group, and a rank that leaves between steps.

def _init_lonely(port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0", WORLD_SIZE="2")
    import time

    t0 = time.time()
    try:
        init_distributed("gloo", timeout_s=3.0)
        q.put(("joined", time.time() - t0))
    except CommInitError as e:
        q.put(("CommInitError", time.time() - t0, str(e)))


def test_rank_that_never_joins_fails_init_within_timeout():
    """Rank 1 of a world of 2 never starts: rank 0's rendezvous gives up after
    the time limit with CommInitError instead of waiting for good."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_init_lonely, args=(_free_port(), q))
    p.start()
    p.join(timeout=120)
    assert p.exitcode == 0
    res = q.get(timeout=10)
    assert res[0] == "CommInitError", res
    assert res[1] < 60, res


def _leaver(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    init_distributed("gloo", timeout_s=5.0)
    g = torch.Generator().manual_seed(0)
    D, H = 32, 4
    x = torch.randn(1, 8, D, generator=g)
    mha = ShardedMHA(torch.randn(3 * D, D, generator=g), torch.zeros(3 * D),
                     torch.randn(D, D, generator=g), torch.zeros(D), H, ops=CPUOps())
    mha.forward(x)  # step 1 on every rank
    if rank == 1:
        os._exit(3)  # leaves between steps, nothing of its own in flight
    import time

    t0 = time.time()
    try:
        mha.forward(x)  # step 2: the peer is gone
        q.put(("completed", time.time() - t0))
    except RuntimeError as e:
        q.put(("RuntimeError", time.time() - t0, type(e).__name__))


def test_rank_leaving_between_steps_ends_the_next_collective():
    """After a common first step, rank 1 exits; rank 0's next step does not
    hang: its first collective ends with an error within the group's limit."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    res = q.get(timeout=10)
    assert res[0] == "RuntimeError", res
    assert res[1] < 60, res
