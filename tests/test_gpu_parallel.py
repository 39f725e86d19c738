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
        errs, tols = {}, {}
        g = torch.Generator(device="cuda").manual_seed(0)
        D, H, T = 512, 8, 200
        x = torch.randn(2, T, D, device="cuda", generator=g)
        Wi = torch.randn(3 * D, D, device="cuda", generator=g) / D ** 0.5
        bi = torch.randn(3 * D, device="cuda", generator=g) * 0.1
        Wo = torch.randn(D, D, device="cuda", generator=g) / D ** 0.5
        bo = torch.randn(D, device="cuda", generator=g) * 0.1

        def mha_ref(xb):
            return oracle.mha_block(xb.cpu().numpy(), Wi.cpu().numpy(), bi.cpu().numpy(),
                                    Wo.cpu().numpy(), bo.cpu().numpy(), H, True)

        def rel(a, r):
            return float(np.max(np.abs(a.cpu().numpy() - r)) / np.max(np.abs(r)))

        # Output rows stored into every rank's y by the out-projection kernel
        # (peer memory): two calls in a row on different inputs, so a stale
        # or partial row from the first would show in the second.
        mha = parallel.ShardedMHA(Wi, bi, Wo, bo, H, causal=True)
        assert mha.peer_output
        y = mha.forward(x)
        errs["mha"] = rel(y[1], mha_ref(x[1]))
        x2 = torch.randn(2, T, D, device="cuda", generator=g)
        y2 = mha.forward(x2)
        errs["mha_again"] = rel(y2[0], mha_ref(x2[0]))
        mha.close()
        # The all-gather form of the same block.
        y3 = parallel.ShardedMHA(Wi, bi, Wo, bo, H, causal=True, peer_output=False).forward(x)
        errs["mha_gather"] = rel(y3[1], mha_ref(x[1]))
        # SGEMM rows stored into every rank's C by the GEMM kernel: ragged
        # rows (M = 301 over two ranks), an odd row length (scalar stores),
        # then an aligned shape with the vector stores, each twice.
        for (M_, K_, N_) in ((301, 257, 513), (384, 320, 640)):
            for prec in ("3xtf32", "tf32"):
                sg = parallel.ShardedGemm(M_, N_, ops=parallel.DeviceOps(prec))
                for it in range(2):
                    A_ = torch.rand(M_, K_, device="cuda", generator=g) * 2 - 1
                    B_ = torch.rand(K_, N_, device="cuda", generator=g) * 2 - 1
                    C_ = sg.forward(A_, B_)
                    e = rel(C_, oracle.sgemm(A_.cpu().numpy(), B_.cpu().numpy()))
                    # max|C - r| / max|r| bars: 1e-5 (3xTF32), 2e-3 (TF32)
                    tols[f"gemm_peer_{M_}_{prec}_{it}"] = 1e-5 if prec == "3xtf32" else 2e-3
                    errs[f"gemm_peer_{M_}_{prec}_{it}"] = e
                sg.close()
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
        # Output heads stored into every rank's O by the decode kernels, one
        # peer-memory barrier per step; three steps (the double buffer wraps).
        sd = parallel.ShardedDecode(10, 128)
        for it in range(3):
            Kd2 = torch.randn(10, 700, 128, device="cuda", generator=g)
            Od2 = sd.step(Qd, Kd2, Vd)
            r2 = oracle.attn_step(Qd.cpu().numpy(), Kd2.cpu().numpy(), Vd.cpu().numpy())
            errs[f"decode_peer_{it}"] = rel(Od2, r2)
        sd.close()
        from attn_cpu import capi
        capi.stream_status()  # no bounded wait of the peer barriers expired
        torch.cuda.synchronize()
        q.put((rank, {k: (v, tols.get(k, 1e-5)) for k, v in errs.items()}))
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
        bad = {k: v for k, v in errs.items() if not v[0] < v[1]}
        assert not bad, (rank, bad)
