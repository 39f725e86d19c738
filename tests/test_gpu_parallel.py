"""Multi-GPU partitions over NCCL (attn_cpu.parallel with the B200 kernels):
two ranks, one per GPU, against the oracle.  Skipped on a single-GPU box; the
same partition logic is covered on CPU gloo ranks by test_parallel_gloo.py."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys

    import torch
    import torch.distributed as dist

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(here, "..", "attn-cpu_b200"))
    sys.path.insert(0, os.path.join(here, "..", "oracle"))
    import oracle
    from attn_cpu import parallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    parallel.init_distributed("nccl", timeout_s=60.0, device=torch.device("cuda", rank),
                              rank=rank, world_size=world)
    try:
        errs = {}
        g = torch.Generator(device="cuda").manual_seed(0)
        D, H, T = 512, 8, 200
        x = torch.randn(2, T, D, device="cuda", generator=g)
        Wi = torch.randn(3 * D, D, device="cuda", generator=g) / D ** 0.5
        bi = torch.randn(3 * D, device="cuda", generator=g) * 0.1
        Wo = torch.randn(D, D, device="cuda", generator=g) / D ** 0.5
        bo = torch.randn(D, device="cuda", generator=g) * 0.1
        y = parallel.ShardedMHA(Wi, bi, Wo, bo, H, causal=True).forward(x)
        ref = oracle.mha_block(x[1].cpu().numpy(), Wi.cpu().numpy(), bi.cpu().numpy(),
                               Wo.cpu().numpy(), bo.cpu().numpy(), H, True)
        errs["mha"] = float(np.max(np.abs(y[1].cpu().numpy() - ref)) / np.max(np.abs(ref)))
        A = torch.rand(300, 257, device="cuda", generator=g) * 2 - 1
        B = torch.rand(257, 513, device="cuda", generator=g) * 2 - 1
        refC = oracle.sgemm(A.cpu().numpy(), B.cpu().numpy())
        for shard in ("rows", "cols"):
            C = parallel.gemm_sharded(A, B, shard=shard)
            errs[shard] = float(np.max(np.abs(C.cpu().numpy() - refC)) / np.max(np.abs(refC)))
        # decode step, 2 x 5 heads (ragged over 2 ranks), T = 700, Dh = 128
        Qd = torch.randn(10, 128, device="cuda", generator=g)
        Kd = torch.randn(10, 700, 128, device="cuda", generator=g)
        Vd = torch.randn(10, 700, 128, device="cuda", generator=g)
        Od = parallel.attn_step_sharded(Qd, Kd, Vd)
        refd = oracle.attn_step(Qd.cpu().numpy(), Kd.cpu().numpy(), Vd.cpu().numpy())
        errs["decode"] = float(np.max(np.abs(Od.cpu().numpy() - refd)) / np.max(np.abs(refd)))
        torch.cuda.synchronize()
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def test_sharded_paths_two_gpus():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    for _ in range(2):
        rank, errs = q.get(timeout=10)
        assert max(errs.values()) < 1e-5, (rank, errs)
