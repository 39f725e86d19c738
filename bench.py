"""bench.py -- throughput of the B200 hot paths, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload prefill|decode|sgemm|sgemm-large|block] [--precision 3xtf32|tf32]

Default workload (the headline): MHA prefill fp32, batch 1, 8 heads,
seq_q = seq_kv = 512, head_dim 64, Q/K/V ~ N(0,1), scale 1/sqrt(64), no mask,
through attn_block_dense.  A step is one pass of that path over one batch.
At N GPUs (one process per GPU under torchrun) every rank runs its own batch
(batch x heads partition, no collective on the data path): weak scaling,
value = all ranks' FLOPs / the slowest rank's time.

Keys beyond the base contract:
  e2e          the same metric through the public Python API (attn_cpu.*) with
               pinned host inputs: host->device copies, compute and the
               device->host read of the result are inside each timed step;
  roofline     the dominant kernel's algorithmic rate (CUDA events, launching
               stream) against the measured peak in MEASURED_PEAKS.json;
  cpu_baseline the reference's own CPU code (oracle/_ref, compiled from its
               sources) timed on this host on a bounded sample (rank 0, N=1);
  also         the other measured configs (decode GB/s, SGEMM TFLOP/s,
               attention block TFLOP/s) with their own rooflines (N=1 only);
  e2e_resident (decode) the decode step through attn_cpu.KVCache, K/V kept on
               the device: each step moves q and the new token in, o out.

`--impl reference` times the reference's CPU implementation of the headline
path on this host's cores (all threads) and prints its own line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
# Sharded SGEMM and attention block at N > 1: the GEMM kernels store their
# output tiles straight into every GPU's copy (peer memory over NVLink)
# instead of an all-gather after them.  ATTNB_PEER_OUTPUT=0 times the
# all-gather form.
PEER_OUTPUT = os.environ.get("ATTNB_PEER_OUTPUT", "1") != "0"
sys.path.insert(0, os.path.join(ROOT, "attn-cpu_b200"))

# Algorithmic work per call, per workload.
WORKLOADS = {
    "prefill": dict(metric="MHA prefill TFLOP/s", unit="TFLOP/s", H=8, L=512, T=512, Dh=64,
                    desc="MHA prefill fp32 [1,8,512,64] non-causal (attn_block_dense)"),
    "decode": dict(metric="M=1 decode KV-stream GB/s", unit="GB/s", H=256, T=4096, Dh=128,
                   desc="MHA decode step fp32 B=8 x H=32, Dh=128, T=4096 (attn_step_dense)"),
    "sgemm": dict(metric="SGEMM TFLOP/s per GPU", unit="TFLOP/s", M=1024, N=1024, K=1024,
                  desc="SGEMM fp32 1024^3, U[-1,1], beta=0 (gemm)"),
    "sgemm-large": dict(metric="SGEMM TFLOP/s per GPU", unit="TFLOP/s", M=16384, N=16384,
                        K=16384, desc="SGEMM fp32 16384^3, U[-1,1], beta=0 (gemm)"),
    "prefill-large": dict(metric="MHA prefill TFLOP/s", unit="TFLOP/s", H=32, L=4096, T=4096,
                          Dh=128, desc="MHA prefill fp32 [1,32,4096,128] non-causal "
                                       "(attn_block_dense)"),
    "block": dict(metric="attention block TFLOP/s", unit="TFLOP/s", B=4, T=2048, D=4096, H=32,
                  desc="attention block fp32: hidden 4096, 32 heads, Dh 128, batch 4, "
                       "seq 2048 (mha_block_dense)"),
}

# DRAM bytes of each dominant kernel per step (its launches in one step) from
# one-pass ncu captures of dram__bytes_read.sum + dram__bytes_write.sum on the
# same problem; commands and figures in profiles/.  Cold-cache captures.
NCU_TRAFFIC = {
    ("prefill", "3xtf32"): 3.22e6,     # attn_tc, [1,8,512,64]: raw Q/K/V read once
    ("prefill-large", "3xtf32"): 5.00e8,  # attn_tc [1,32,4096,128]: packed K/V re-read via L2
    ("decode", "3xtf32"): 1.0778e9,    # decode: K + V once (1.0737e9) + output, one range a head
    ("decode", "tf32"): 1.0778e9,
    ("sgemm-large", "3xtf32"): 51.15e9,  # gemm_tc 16384^3: packed operands re-read ~12x
    ("block", "3xtf32"): 6.93e9,       # gemm_tc QKV (5.11e9) + output (1.82e9) projections
}


def flops_of(w: str) -> float:
    c = WORKLOADS[w]
    if w.startswith("prefill"):
        return 4.0 * c["H"] * c["L"] * c["T"] * c["Dh"]
    if w == "decode":
        return 4.0 * c["H"] * c["T"] * c["Dh"]
    if w.startswith("sgemm"):
        return 2.0 * c["M"] * c["N"] * c["K"]
    if w == "block":
        B, T, D = c["B"], c["T"], c["D"]
        return B * (2.0 * T * D * 3 * D + 4.0 * T * T * D + 2.0 * T * D * D)
    raise KeyError(w)


def bytes_of(w: str) -> float:
    """Algorithmic HBM bytes of the decode step: K + V once, plus q and o."""
    c = WORKLOADS[w]
    return 4.0 * (2 * c["H"] * c["T"] * c["Dh"] + 2 * c["H"] * c["Dh"])


def load_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "src": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region.
    A timed region shorter than the 100 ms sampling period is bracketed: entry
    waits for a first sample and exit for one more."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < 3.0:
            time.sleep(0.01)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            n0, t0 = len(self.lines), time.time()
            while len(self.lines) <= n0 and time.time() - t0 < 1.0:
                time.sleep(0.01)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ------------------------------------------------------------- helpers
def dist_setup(n_gpus: int):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from attn_cpu import parallel

        torch.cuda.set_device(local)
        parallel.init_distributed("nccl", timeout_s=300.0, device=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def numa_bind(local: int):
    """Restrict this process to the host cores NVML lists as nearest to GPU
    `local`, so page-locked buffers (allocated later, first touched by these
    cores) sit on the GPU's NUMA node and host<->device copies do not cross the
    socket link.  ATTNB_NUMA_BIND=0 turns it off.  Returns (the affinity to
    restore or None, a description for the JSON line)."""
    if os.environ.get("ATTNB_NUMA_BIND", "1") == "0":
        return None, {"bound": False, "why": "ATTNB_NUMA_BIND=0"}
    try:
        import pynvml
        import torch

        prop = torch.cuda.get_device_properties(local)
        bus = f"{prop.pci_domain_id:08x}:{prop.pci_bus_id:02x}:{prop.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = (os.cpu_count() + 63) // 64
        masks = pynvml.nvmlDeviceGetCpuAffinity(h, words)
        near = {w * 64 + b for w, m in enumerate(masks) for b in range(64) if (m >> b) & 1}
        orig = os.sched_getaffinity(0)
        keep = near & orig
        if not keep or keep == orig:
            return None, {"bound": False,
                          "why": f"all {len(orig)} usable cores are near the GPU" if keep
                          else "no usable core is near the GPU"}
        os.sched_setaffinity(0, keep)
        return orig, {"bound": True, "cores": len(keep), "of": len(orig)}
    except Exception as e:  # no NVML or no device: leave the affinity alone
        return None, {"bound": False, "why": type(e).__name__}


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class L2Flusher:
    """Writes a buffer larger than the 126 MB L2 between timed steps.  At
    512 MB the write keeps the GPU busy (~80 us) while the host enqueues the
    step, so the step's events time the device work, not the launch path
    (which the e2e figure includes)."""

    def __init__(self):
        import torch

        self.buf = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    def __call__(self):
        self.buf.fill_(1.0)


def time_device(run, steps: int, warmup: int, world: int, flush: bool):
    """Per-step CUDA-event times (ms) of `run` on the current stream, L2
    flushed between steps outside the events; barrier + sync around."""
    import torch

    fl = L2Flusher() if flush else None
    for _ in range(warmup):
        if fl:
            fl()
        run()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    for i in range(steps):
        if fl:
            fl()
        ev[i][0].record()
        run()
        ev[i][1].record()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


# --------------------------------------------------------- workloads (ours)
def setup_sharded(w: str, precision):
    """One problem partitioned over all ranks (attn_cpu.parallel) with its
    NCCL collectives: heads for prefill / decode / the attention block (the
    block: all-to-all of the context, all-gather of y), row blocks of C for
    SGEMM.  Inputs are identical on every rank (same seed)."""
    import torch

    from attn_cpu import parallel

    c = WORKLOADS[w]
    ops = parallel.DeviceOps(precision)
    g = torch.Generator(device="cuda").manual_seed(1000)
    if w == "prefill":
        Q, K, V = (torch.randn(c["H"], c["L"], c["Dh"], device="cuda", generator=g)
                   for _ in range(3))
        return lambda: parallel.attn_block_sharded(Q, K, V, False, ops=ops)
    if w == "decode":
        Q = torch.randn(c["H"], c["Dh"], device="cuda", generator=g)
        K = torch.randn(c["H"], c["T"], c["Dh"], device="cuda", generator=g)
        V = torch.randn(c["H"], c["T"], c["Dh"], device="cuda", generator=g)
        if PEER_OUTPUT:
            sd = parallel.ShardedDecode(c["H"], c["Dh"], ops=ops)
            return (lambda: sd.step(Q, K, V)), sd.close
        return lambda: parallel.attn_step_sharded(Q, K, V, ops=ops)
    if w.startswith("sgemm"):
        A = torch.rand(c["M"], c["K"], device="cuda", generator=g) * 2 - 1
        B = torch.rand(c["K"], c["N"], device="cuda", generator=g) * 2 - 1
        if PEER_OUTPUT:
            sg = parallel.ShardedGemm(c["M"], c["N"], ops=ops)
            return (lambda: sg.forward(A, B)), sg.close
        return lambda: parallel.gemm_sharded(A, B, ops=ops)
    if w == "block":
        D, H = c["D"], c["H"]
        x = torch.randn(c["B"], c["T"], D, device="cuda", generator=g)
        Wi = torch.randn(3 * D, D, device="cuda", generator=g) * 0.02
        Wo = torch.randn(D, D, device="cuda", generator=g) * 0.02
        mha = parallel.ShardedMHA(Wi, torch.zeros(3 * D, device="cuda"), Wo,
                                  torch.zeros(D, device="cuda"), H, ops=ops,
                                  peer_output=PEER_OUTPUT)
        return (lambda: mha.forward(x)), mha.close
    raise KeyError(f"{w} has no sharded form")


def setup_workload(w: str, rank: int, precision, host: bool = True):
    """Device inputs (seeded per rank) and (run, e2e_run, h2d, d2h, launches);
    with host=False no page-locked host copies are made and e2e_run is None."""
    import numpy as np
    import torch

    import attn_cpu
    from attn_cpu import capi

    c = WORKLOADS[w]
    g = torch.Generator(device="cuda").manual_seed(1000 + rank)
    if w.startswith("prefill"):
        H, L, T, Dh = c["H"], c["L"], c["T"], c["Dh"]
        Q = torch.randn(H, L, Dh, device="cuda", generator=g)
        K = torch.randn(H, T, Dh, device="cuda", generator=g)
        V = torch.randn(H, T, Dh, device="cuda", generator=g)
        O = torch.empty(H, L, Dh, device="cuda")
        run = lambda: capi.attn_block_dense_dev(Q, K, V, O, False, precision)
        e2e = None
        if host:
            hQ, hK, hV = (t.cpu().pin_memory() for t in (Q, K, V))
            nQ, nK, nV = hQ.numpy(), hK.numpy(), hV.numpy()
            e2e = lambda: attn_cpu.attn_block_dense(nQ, nK, nV, precision=precision)
        h2d = 4 * (Q.numel() + K.numel() + V.numel())
        d2h = 4 * O.numel()
        # [1,8,512,64]: one launch (each CTA holds one key tile and loads and
        # splits the raw operands itself); longer sequences: pack + attention.
        return run, e2e, h2d, d2h, 1 if w == "prefill" else 2
    if w == "decode":
        H, T, Dh = c["H"], c["T"], c["Dh"]
        Q = torch.randn(H, Dh, device="cuda", generator=g)
        K = torch.randn(H, T, Dh, device="cuda", generator=g)
        V = torch.randn(H, T, Dh, device="cuda", generator=g)
        O = torch.empty(H, Dh, device="cuda")
        run = lambda: capi.attn_step_dense_dev(Q, K, V, O)
        e2e = None
        if host:
            hQ, hK, hV = (t.cpu().pin_memory() for t in (Q, K, V))
            nQ, nK, nV = hQ.numpy(), hK.numpy(), hV.numpy()
            e2e = lambda: attn_cpu.attn_step_dense(nQ, nK, nV)
        # Launches: the split kernel, plus the split merge when the library's
        # plan (two CTAs per SM over all heads, at least 64 keys a range) cuts
        # a head's keys into more than one range.
        sms = torch.cuda.get_device_properties(0).multi_processor_count
        nsplit = min(max(1, 2 * sms // H), (T + 63) // 64)
        launches = 1 if nsplit == 1 else 2
        return run, e2e, 4 * (Q.numel() + K.numel() + V.numel()), 4 * O.numel(), launches
    if w.startswith("sgemm"):
        M, N, K = c["M"], c["N"], c["K"]
        A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
        B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
        C = torch.empty(M, N, device="cuda")
        run = lambda: capi.sgemm_dev(A, B, C, precision=precision)
        e2e = None
        if host:
            hA, hB = A.cpu().pin_memory(), B.cpu().pin_memory()
            nA, nB = hA.numpy(), hB.numpy()
            e2e = lambda: attn_cpu.gemm(nA, nB, precision=precision)
        # 1xTF32 at 1024^3: one launch (every CTA holds one tile and splits the
        # raw operands itself); otherwise pack + GEMM.
        one = w == "sgemm" and precision == "tf32"
        return run, e2e, 4 * (A.numel() + B.numel()), 4 * C.numel(), 1 if one else 2
    if w == "block":
        Bt, T, D, H = c["B"], c["T"], c["D"], c["H"]
        x = torch.randn(Bt, T, D, device="cuda", generator=g)
        Wi = torch.randn(3 * D, D, device="cuda", generator=g) * 0.02
        Wo = torch.randn(D, D, device="cuda", generator=g) * 0.02
        bi = torch.zeros(3 * D, device="cuda")
        bo = torch.zeros(D, device="cuda")
        y = torch.empty_like(x)
        run = lambda: capi.mha_block_dense_dev(x, Wi, bi, Wo, bo, H, y, False, precision)
        e2e = None
        if host:
            hx = x.cpu().pin_memory()
            hw = [t.cpu().pin_memory().numpy() for t in (Wi, bi, Wo, bo)]
            nx = hx.numpy()
            e2e = lambda: [attn_cpu.mha_block_dense(nx[b], *hw, H, precision=precision)
                           for b in range(Bt)]
        # per sequence (e2e calls the host API once per sequence): x_b and all weights
        h2d = 4 * (x.numel() + Bt * (Wi.numel() + bi.numel() + Wo.numel() + bo.numel()))
        return run, e2e, h2d, 4 * y.numel(), 4 + 2 * Bt  # 2 x (pack + GEMM), B x (pack + attn)
    raise KeyError(w)


# Dominant kernel of each workload (library profiling name) and its
# algorithmic work per step.
def dominant_of(w: str):
    c = WORKLOADS[w]
    if w.startswith("prefill"):
        return "attn_tc", flops_of(w)
    if w == "decode":
        return "decode", bytes_of(w)
    if w.startswith("sgemm"):
        return "gemm_tc", flops_of(w)
    if w == "block":  # QKV and output projections
        B, T, D = c["B"], c["T"], c["D"]
        return "gemm_tc", B * (2.0 * T * D * 3 * D + 2.0 * T * D * D)
    raise KeyError(w)


def roofline_of(w: str, kernel_ms: float, launches: int, peaks: dict, precision) -> dict:
    """Dominant kernel's algorithmic rate: its work per step over its summed
    launch durations per step (CUDA events on the launching stream)."""
    name, work = dominant_of(w)
    traffic = NCU_TRAFFIC.get((w, precision or "3xtf32"))
    base = {"kernel": name, "launches_per_step": launches,
            "kernel_ms_per_step": round(kernel_ms, 5), "traffic": traffic}
    if w == "decode":
        achieved = work / (kernel_ms * 1e-3) / 1e9
        peak = peaks["hbm_gbs"]
        return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4),
                "peak_src": f"{peaks['src']} STREAM-style copy (MEASURED_PEAKS.json hbm_gbs)",
                **base}
    achieved = work / (kernel_ms * 1e-3) / 1e12
    # tcgen05 kind::tf32 issues at half the bf16 rate: the measured cuBLAS bf16
    # burst figure / 2 is the TF32 denominator.
    peak = peaks["bf16_tflops"] / 2
    r = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak, 1),
         "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
         "peak_src": f"{peaks['src']} bf16 burst / 2 (TF32 rate)", **base}
    if (precision or "3xtf32") == "3xtf32":
        # 3xTF32 issues three tf32 products per algorithmic one.
        r["frac_of_3xtf32_cap"] = round(3 * achieved / peak, 4)
    return r


def kernel_time(run, w: str, steps: int, world: int, flush: bool):
    """Per-step summed duration (ms) and launch count of the dominant kernel,
    from the library's CUDA-event hooks over `steps` further steps."""
    import torch

    from attn_cpu import capi

    name, _ = dominant_of(w)
    fl = L2Flusher() if flush else None
    capi.profile_read(name)  # discard anything recorded before
    capi.profile_enable(True)
    try:
        for _ in range(steps):
            if fl:
                fl()
            run()
        torch.cuda.synchronize()
    finally:
        capi.profile_enable(False)
    ms, n = capi.profile_read(name)
    return max_over_ranks(ms / steps, world), n // max(1, steps)


GRAPH_STEPS = 2  # decode steps per CUDA-graph replay (ShardedDecode alternates two buffers)


def graphed(run, reps: int):
    """A CUDA graph of `reps` back-to-back calls of `run` (warmed up first on a
    side stream, so no allocation happens during capture).  Replaying it
    costs the host one launch, so microsecond-scale steps are timed on the
    device rather than behind the host's launch path."""
    import torch

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            run()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            run()
    torch.cuda.synchronize()
    return g


def measure_sharded(w: str, rank: int, world: int, steps: int, warmup: int, precision):
    """Strong scaling: one problem over all ranks, collectives inside the step,
    beside the same problem on one GPU through the single-GPU entry point
    (rank 0 alone, the other ranks waiting at a barrier).  Compact entry."""
    import torch

    from attn_cpu import capi

    flush = w in ("prefill", "sgemm")
    run = setup_sharded(w, precision)
    close = None
    if isinstance(run, tuple):
        run, close = run
    # The decode step is tens of microseconds per rank: its peer-store form
    # (kernels only, no collective) and the one-GPU step are replayed from
    # CUDA graphs of GRAPH_STEPS steps, both alike.
    use_graph = w == "decode" and PEER_OUTPUT
    reps = GRAPH_STEPS if use_graph else 1
    if use_graph:
        run = graphed(run, reps).replay
    times = time_device(run, steps, warmup, world, flush=flush)
    capi.stream_status()
    ms = max_over_ranks(sum(times), world) / (steps * reps)
    del run
    if close is not None:
        close()  # collective: the peer buffers are unmapped on every rank
    torch.cuda.empty_cache()
    ms1 = None
    if rank == 0:
        run1 = setup_workload(w, 0, precision, host=False)[0]
        if use_graph:
            run1 = graphed(run1, reps).replay
        ms1 = sum(time_device(run1, steps, warmup, 1, flush)) / (steps * reps)
        del run1
        torch.cuda.empty_cache()
    barrier(world)
    work = flops_of(w) if w != "decode" else bytes_of(w)
    scale = 1e12 if WORKLOADS[w]["unit"] == "TFLOP/s" else 1e9
    value = work / (ms * 1e-3) / scale
    r = {"w": w, "prec": precision if w != "decode" else "fp32", "scaling": "strong",
         "v": round(value, 2), "u": WORKLOADS[w]["unit"], "ms": round(ms, 4),
         "par": {"prefill": "heads", "decode": "heads", "block": "heads+a2a",
                 "sgemm": "C rows", "sgemm-large": "C rows"}[w]
         + ("" if w == "prefill" else "+peer stores" if PEER_OUTPUT else "+all-gather")
         + f" x{world}"}
    if use_graph:
        r["graph"] = f"{reps} steps per replay"
    if ms1 is not None:
        v1 = work / (ms1 * 1e-3) / scale
        r.update(n1=round(v1, 2), eff=round(value / (world * v1), 3))
    return r


def compact(w: str, res: dict, precision) -> dict:
    """Short form of a secondary measurement for the `also` list: value and
    unit, ms per step, the dominant kernel's CUDA-event time per step and its
    roofline fraction (of the TF32 rate, or of HBM for decode; the dominant
    kernel of each workload is named in dominant_of), e2e and the SM clock."""
    rf = res["roofline"]
    out = {"w": w, "prec": precision if w != "decode" else "fp32", "v": round(res["value"], 1),
           "u": res["unit"], "ms": round(res["ms_per_step"], 4),
           "k_ms": round(rf["kernel_ms_per_step"], 4), "frac": round(rf["frac"], 3)}
    if "frac_of_3xtf32_cap" in rf:
        out["frac3x"] = round(rf["frac_of_3xtf32_cap"], 3)
    if res.get("e2e"):
        out["e2e"] = round(res["e2e"]["value"], 2)
    if res.get("e2e_resident"):
        out["e2e_res"] = round(res["e2e_resident"]["value"], 1)
    clk = res.get("clocks") or {}
    if clk.get("reasons"):  # the SM clock only when something held it down
        out["mhz"] = clk.get("sm_mhz")
        out["why"] = clk["reasons"]
    return out


def measure(w: str, rank: int, world: int, steps: int, warmup: int, precision, peaks,
            with_e2e=True):
    import torch

    run, e2e, h2d, d2h, launches = setup_workload(w, rank, precision, host=with_e2e)
    flush = w in ("prefill", "sgemm")  # the other workloads' inputs exceed L2
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        t0 = time.perf_counter()
        times = time_device(run, steps, warmup, world, flush)
        wall = time.perf_counter() - t0
    from attn_cpu import capi

    capi.stream_status()
    total_ms = max_over_ranks(sum(times), world)
    ms = total_ms / steps
    work = flops_of(w) if w != "decode" else bytes_of(w)
    scale = 1e12 if WORKLOADS[w]["unit"] == "TFLOP/s" else 1e9
    value = world * work / (ms * 1e-3) / scale
    k_ms, k_n = kernel_time(run, w, steps, world, flush)
    res = {"metric": WORKLOADS[w]["metric"], "value": round(value, 3),
           "unit": WORKLOADS[w]["unit"], "ms_per_step": round(ms, 5),
           "roofline": roofline_of(w, k_ms, k_n, peaks, precision),
           "gpu_launches": launches * steps, "l2": "flushed between steps" if flush else
           "inputs larger than L2", "wall_s": round(wall, 3), "clocks": clk.summary()}
    if with_e2e:
        for _ in range(max(1, warmup)):
            e2e()
        barrier(world)
        ts = []
        for _ in range(steps):
            t = time.perf_counter()
            e2e()
            ts.append(time.perf_counter() - t)
        e_ms = max_over_ranks(1e3 * sum(ts) / len(ts), world)
        res["e2e"] = {"value": round(world * work / (e_ms * 1e-3) / scale, 4),
                      "unit": WORKLOADS[w]["unit"], "ms_per_step": round(e_ms, 4),
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
        if w == "decode":
            res["e2e_resident"] = decode_resident_e2e(rank, world, steps, warmup, work, scale)
    del run, e2e
    torch.cuda.empty_cache()
    return res


def decode_resident_e2e(rank: int, world: int, steps: int, warmup: int, work: float,
                        scale: float) -> dict:
    """The decode workload through the resident K/V cache (attn_cpu.KVCache):
    the cache holds T - 1 tokens on the device, and each step (a host call)
    appends the new token's k and v, attends with q and returns o, so only
    q, k_new, v_new go in and o comes out.  The cache is truncated back to
    T - 1 tokens before each step, so every step attends over the same T."""
    import numpy as np
    import torch

    import attn_cpu

    c = WORKLOADS["decode"]
    H, T, Dh = c["H"], c["T"], c["Dh"]
    rng = np.random.default_rng(2000 + rank)
    pin = lambda a: torch.from_numpy(a).pin_memory().numpy()
    K = pin(rng.standard_normal((H, T, Dh), dtype=np.float32))
    V = pin(rng.standard_normal((H, T, Dh), dtype=np.float32))
    q = pin(rng.standard_normal((H, Dh), dtype=np.float32))
    kn, vn = pin(np.ascontiguousarray(K[:, -1])), pin(np.ascontiguousarray(V[:, -1]))
    cache = attn_cpu.KVCache(H, Dh, T)
    cache.append(K[:, :T - 1], V[:, :T - 1])

    def step():
        cache.truncate(T - 1)
        return cache.step(q, kn, vn)

    for _ in range(max(1, warmup)):
        step()
    barrier(world)
    ts = []
    for _ in range(steps):
        t = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t)
    e_ms = max_over_ranks(1e3 * sum(ts) / len(ts), world)
    del cache
    return {"value": round(world * work / (e_ms * 1e-3) / scale, 4),
            "unit": WORKLOADS["decode"]["unit"], "ms_per_step": round(e_ms, 4),
            "h2d_bytes_per_step": 3 * H * Dh * 4, "d2h_bytes_per_step": H * Dh * 4,
            "api": "attn_cpu.KVCache.step (K/V resident on the device)"}


# ----------------------------------------------------- CPU (reference) runs
def cpu_sample(w: str, budget_s: float):
    """Time the reference's CPU code (compiled from its sources) on this host,
    falling back to the float64 restatement when it cannot run here.
    Returns (value, unit, cores, kind, sample description)."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle

    kind = "reference" if oracle.ref_available() else "port"
    cores = int(os.environ.get("OMP_NUM_THREADS") or os.cpu_count() or 1)
    c = WORKLOADS[w]
    rng = np.random.default_rng(0)
    if w == "prefill":
        Q, K, V = (rng.standard_normal((c["H"], c["L"] if i == 0 else c["T"], c["Dh"]),
                                       dtype=np.float32) for i in range(3))
        fn = (lambda: oracle.ref_attn_block(Q, K, V)) if kind == "reference" else \
            (lambda: oracle.attn_block(Q, K, V))
        unit_work, desc = flops_of(w), "full [1,8,512,64] problem per call"
    elif w == "decode":
        H = 32  # bounded sample: 32 of the 256 heads per call
        Q = rng.standard_normal((H, c["Dh"]), dtype=np.float32)
        K = rng.standard_normal((H, c["T"], c["Dh"]), dtype=np.float32)
        V = rng.standard_normal((H, c["T"], c["Dh"]), dtype=np.float32)
        fn = (lambda: oracle.ref_attn_step(Q, K, V)) if kind == "reference" else \
            (lambda: oracle.attn_step(Q, K, V))
        unit_work = 4.0 * (2 * H * c["T"] * c["Dh"] + 2 * H * c["Dh"])
        desc = "32 of 256 heads (T=4096, Dh=128) per call; single-threaded reference function"
        cores = 1
    elif w.startswith("sgemm"):
        n = 1024
        A = rng.uniform(-1, 1, (n, n)).astype(np.float32)
        B = rng.uniform(-1, 1, (n, n)).astype(np.float32)
        fn = (lambda: oracle.ref_sgemm(A, B)) if kind == "reference" else \
            (lambda: oracle.sgemm(A, B))
        unit_work, desc = 2.0 * n ** 3, "1024^3 SGEMM per call"
    else:
        T, D, H = 256, 4096, 32
        x = rng.standard_normal((T, D), dtype=np.float32)
        Wi = (0.02 * rng.standard_normal((3 * D, D))).astype(np.float32)
        Wo = (0.02 * rng.standard_normal((D, D))).astype(np.float32)
        bi, bo = np.zeros(3 * D, np.float32), np.zeros(D, np.float32)
        fn = (lambda: oracle.ref_mha_block(x, Wi, bi, Wo, bo, H)) if kind == "reference" else \
            (lambda: oracle.mha_block(x, Wi, bi, Wo, bo, H))
        unit_work = 2.0 * T * D * 3 * D + 4.0 * T * T * D + 2.0 * T * D * D
        desc = "one sequence of T=256 at hidden 4096 / 32 heads per call; single-threaded"
        cores = 1
    fn()  # warm (the reference picks its unroll once, src/gemm.cpp:272-316)
    n_calls, t0 = 0, time.perf_counter()
    while True:
        fn()
        n_calls += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    per = el / n_calls
    scale = 1e12 if WORKLOADS[w]["unit"] == "TFLOP/s" else 1e9
    return unit_work / per / scale, WORKLOADS[w]["unit"], cores, kind, \
        f"{desc}; {n_calls} calls in {el:.1f} s"


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    w = args.workload
    # All host threads for the reference's OpenMP code: torchrun sets
    # OMP_NUM_THREADS=1 for its workers, and rank 0 runs alone here.  Set
    # before the compiled reference (and its OpenMP runtime) is loaded.
    os.environ["OMP_NUM_THREADS"] = str(len(os.sched_getaffinity(0)) or os.cpu_count() or 1)
    os.environ.setdefault("OMP_PROC_BIND", "close")
    per = max(1.0, args.cpu_seconds / max(1, args.steps))
    vals = []
    kind = cores = sample = unit = None
    for i in range(args.warmup + args.steps):
        v, unit, cores, kind, sample = cpu_sample(w, per if i >= args.warmup else 0.2)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.mean(vals)
    line = {"impl": "reference", "metric": WORKLOADS[w]["metric"], "value": round(value, 5),
            "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_of(w, world),
            "cpu_baseline": {"value": round(value, 5), "unit": unit, "cores": cores,
                             "kind": kind, "sample": sample},
            "e2e": {"value": round(value, 5), "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_of(w: str, world: int) -> dict:
    """The `config` of a line: the same dict in both arms."""
    return {"workload": WORKLOADS[w]["desc"],
            "l2": "flushed between steps" if w in ("prefill", "sgemm") else
                  "inputs larger than L2",
            "parallelism": f"batch-x-heads x{world}", "global_batch": world}


# --------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="prefill")
    ap.add_argument("--precision", choices=["3xtf32", "tf32"], default="3xtf32")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU time budget of the reference measurement")
    ap.add_argument("--no-also", action="store_true", help="skip the secondary configs")
    ap.add_argument("--sharded", default="block,sgemm-large,decode",
                    help="with N>1: also time these workloads (comma list of prefill, decode, "
                         "sgemm, sgemm-large, block) as one problem partitioned over all GPUs, "
                         "in both precisions; empty to skip")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    if args.impl == "reference":
        run_reference_arm(args)
        return

    import torch

    rank, world, local = dist_setup(args.gpus)
    orig_affinity, binding = numa_bind(local)
    peaks = load_peaks()
    prec = args.precision
    head = measure(args.workload, rank, world, args.steps, args.warmup, prec, peaks)
    also = []
    if world == 1 and not args.no_also:
        # The other configs in this run's precision, then the tensor-core
        # configs at scale in the other precision.
        other = "tf32" if prec == "3xtf32" else "3xtf32"
        plan = [(w, prec) for w in ("decode", "sgemm", "sgemm-large", "prefill-large", "block")
                if w != args.workload]
        plan += [(w, other) for w in ("sgemm-large", "prefill-large", "block")]
        for w, pr in plan:
            steps = args.steps if w in ("decode", "sgemm") else max(3, min(args.steps, 5))
            r = measure(w, rank, world, steps, 3, pr, peaks,
                        with_e2e=w in ("decode", "sgemm") and pr == prec)
            also.append(compact(w, r, pr))
    if world > 1 and args.sharded and not args.no_also:
        for w in [x.strip() for x in args.sharded.split(",") if x.strip()]:
            for pr in ((prec,) if w == "decode" else ("3xtf32", "tf32")):
                also.append(measure_sharded(w, rank, world, max(3, min(args.steps, 8)), 3, pr))
    if orig_affinity is not None:
        os.sched_setaffinity(0, orig_affinity)  # the CPU baseline uses every host core
    cpu = None
    if rank == 0 and world == 1:
        v, unit, cores, kind, sample = cpu_sample(args.workload, args.cpu_seconds)
        cpu = {"value": round(v, 5), "unit": unit, "cores": cores, "kind": kind,
               "sample": sample}
    if rank == 0:
        line = {"metric": head["metric"], "value": head["value"], "unit": head["unit"],
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": head["ms_per_step"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "precision": prec, "data": "synthetic (seeded N(0,1) / U[-1,1])",
                "config": config_of(args.workload, world),
                "e2e": head.get("e2e"), "roofline": head["roofline"],
                "gpu_launches": head["gpu_launches"], "clocks": head["clocks"],
                "cpu_baseline": cpu, "host_binding": binding}
        if head.get("e2e_resident"):
            line["e2e_resident"] = head["e2e_resident"]
        line["also"] = also  # last, so the end of the line carries the other configs
        print(json.dumps(line, separators=(",", ":")), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
