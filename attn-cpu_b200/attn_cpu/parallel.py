"""parallel -- the hot paths partitioned over the GPUs of one node.

One process per GPU, torch.distributed (NCCL over NVLink / NVSwitch) for the
collectives.  The reference has no multi-device code at all (its only
parallelism is OpenMP inside one process, src/gemm.cpp:350); the partitions
here follow the work's natural independence:

* attention (prefill and decode): whole heads per rank -- no exchange inside
  the attention itself; an all-gather of the per-head outputs assembles O
  (prefill: attn::attn_block_dense, src/attn_block.cpp:104-241; decode step:
  attn::attn_step_dense, src/attn_dense.cpp:21-73, with the batch and head
  axes flattened into one head axis of B*H);
* the MHA block (attn::mha_block_dense, src/attn_dispatch.cpp:17-133): rank r
  owns heads [h0, h1): it projects only its heads' Q/K/V rows of W_in
  (column-parallel QKV) and runs their attention, writing the context
  transposed, ctx_r^T [hl*Dh, tokens].  Rank s will compute y for a block of
  tokens, so an all-to-all hands it exactly those columns of every rank's
  ctx_r^T: stacked in rank order they are ctx^T [D, tokens_s] for its block
  (1/p of the context per rank, where an all-gather would move all of it).
  Rank s then computes its rows y = ctx W_out^T + b_out from ctx^T read
  transposed (the single-GPU product, same summation order); on NVLink the
  out-projection kernel itself stores those rows into every rank's y
  (peer memory mapped with CUDA IPC), elsewhere an all-gather of the row
  blocks assembles y;
* SGEMM (gemm::sgemm_blocked, src/gemm.cpp:319-415): rank r computes a block
  of C -- a block of rows (A row block x all of B; the all-gather is then
  contiguous) or, as `shard="cols"`, a block of columns (all of A x a column
  block of B, read in place through its leading dimension) followed by an
  all-gather and a permute.  ShardedGemm is the row form without a gather:
  the GEMM kernel stores its tiles into every rank's C over NVLink.

Local compute goes through an `ops` object whose default calls the B200
kernels in libattnb (attn_cpu.capi); tests substitute a CPU implementation to
check the partition and collective logic on gloo ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


class CommInitError(RuntimeError):
    """The process group could not be formed: a rank never joined within the
    time limit, or the rendezvous failed."""


def init_distributed(backend: str = "nccl", timeout_s: float = 300.0, device=None, **kwargs):
    """torch.distributed.init_process_group with a bounded wait.

    Every rank of the job calls this once (RANK / WORLD_SIZE / MASTER_ADDR /
    MASTER_PORT from the environment unless given in ``kwargs``).  If a rank
    never arrives, or the rendezvous store cannot be reached, the others raise
    CommInitError after about ``timeout_s`` seconds instead of waiting for
    good; the same limit bounds every later collective of the group, so a rank
    that leaves between steps ends the others' next collective with an error.
    With ``device`` (a CUDA device) the NCCL communicator is bound to it."""
    import datetime

    opts = dict(kwargs)
    opts["timeout"] = datetime.timedelta(seconds=timeout_s)
    if device is not None:
        opts["device_id"] = device
    try:
        dist.init_process_group(backend, **opts)
    except (RuntimeError, ValueError, OSError) as e:  # DistStoreError etc. derive from these
        raise CommInitError(f"process group ({backend}) could not be formed within "
                            f"{timeout_s:g} s: {e}") from e


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous balanced split of range(n): the first n % world ranks get one more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class DeviceOps:
    """Local compute on the current CUDA device through the C ABI."""

    def __init__(self, precision=None):
        from . import capi

        self.capi = capi
        self.precision = precision

    def linear(self, x, W, b, y):
        self.capi.linear_dev(x, W, b, y, precision=self.precision)

    def attention(self, q, k, v, o, causal):
        self.capi.attn_block_dense_dev(q, k, v, o, causal=causal, precision=self.precision)

    def attention_batched(self, q, k, v, o, causal):
        self.capi.attn_block_dense_batched_dev(q, k, v, o, causal=causal,
                                               precision=self.precision)

    def sgemm(self, A, B, C):
        self.capi.sgemm_dev(A, B, C, precision=self.precision)

    def decode(self, q, k, v, o):
        self.capi.attn_step_dense_dev(q, k, v, o)

    def decode_bcast(self, q, k, v, o, replicas):
        self.capi.attn_step_dense_bcast_dev(q, k, v, o, replicas)

    def pack_weight(self, W):
        """W [N, K] packed once for y = x W^T (in this object's precision)."""
        return self.capi.PackedWeight(W, precision=self.precision)

    def linear_packed(self, x, Wp, b, y, trans_x=False, replicas=()):
        self.capi.linear_packed_dev(x, Wp, b, y, trans_x=trans_x, replicas=replicas)

    def gemm_ex(self, A, B, C, trans_a, trans_b, bias):
        self.capi.gemm_ex_dev(A, B, C, trans_a=trans_a, trans_b=trans_b, bias=bias,
                              precision=self.precision)

    def gemm_ex_bcast(self, A, B, C, replicas, trans_a, trans_b, bias):
        """gemm_ex whose kernel also stores C into the replicas (device
        addresses on other GPUs) as its tiles finish."""
        self.capi.gemm_ex_bcast_dev(A, B, C, replicas, trans_a=trans_a, trans_b=trans_b,
                                    bias=bias, precision=self.precision)


def _world(group):
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def _all_gather_rows(local: torch.Tensor, counts: list[int], group) -> torch.Tensor:
    """Concatenate every rank's `local` [n_r, ...] along dim 0 (ragged n_r)."""
    rank, world = _world(group)
    if world == 1:
        return local
    if len(set(counts)) == 1:
        out = torch.empty((sum(counts),) + tuple(local.shape[1:]), dtype=local.dtype,
                          device=local.device)
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
        return out
    # Ragged blocks: pad every rank's block to the largest, gather, then trim.
    cmax = max(counts)
    tail = tuple(local.shape[1:])
    padded = torch.zeros((cmax,) + tail, dtype=local.dtype, device=local.device)
    padded[:local.shape[0]] = local
    out = torch.empty((world * cmax,) + tail, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, padded, group=group)
    return torch.cat([out[r * cmax:r * cmax + c] for r, c in enumerate(counts)], 0)


def _all_to_all_cols(local: torch.Tensor, row_counts: list[int], group) -> torch.Tensor:
    """Column exchange: ``local`` [n_me, C] holds this rank's rows (n_r rows on
    rank r, ``row_counts``) of a matrix whose columns are split into balanced
    contiguous blocks, block s belonging to rank s.  Returns this rank's
    column block of the whole matrix, [sum(n_r), C_me]: every rank's rows of
    that block, stacked in rank order."""
    rank, world = _world(group)
    if world == 1:
        return local
    n_me, C = local.shape
    cols = [shard_range(C, s, world) for s in range(world)]
    widths = [b - a for a, b in cols]
    if len(set(widths)) == 1:
        # [n_me, world, w] -> [world, n_me, w]: block s contiguous
        send = local.view(n_me, world, widths[0]).transpose(0, 1).contiguous().view(-1)
    else:
        send = torch.cat([local[:, a:b].reshape(-1) for a, b in cols])
    w_me = widths[rank]
    recv = torch.empty(sum(row_counts) * w_me, dtype=local.dtype, device=local.device)
    dist.all_to_all_single(recv, send, output_split_sizes=[n * w_me for n in row_counts],
                           input_split_sizes=[n_me * w for w in widths], group=group)
    return recv.view(sum(row_counts), w_me)


def _peer_capable(ops, group) -> bool:
    """Whether outputs can be broadcast by the kernels' own stores into the
    other GPUs' memory: the B200 ops and an NCCL group of more than one rank."""
    if not hasattr(ops, "gemm_ex_bcast"):
        return False
    rank, world = _world(group)
    return world > 1 and dist.get_backend(group) == "nccl"


def _fence(group, device) -> None:
    """A collective on the current stream (an all-reduce of one word): when it
    completes on a rank, every rank has finished the work it enqueued before
    it, including kernels that stored into this rank's memory."""
    t = torch.zeros(1, dtype=torch.int32, device=device)
    dist.all_reduce(t, group=group)


class PeerReplicas:
    """A float32 buffer of `shape` on every rank of `group`, in a device
    allocation of its own, with the other ranks' buffers mapped into this
    process (CUDA IPC over NVLink / NVSwitch): a kernel on this GPU stores into
    every rank's copy directly.  Collective: every rank constructs it with the
    same shape, and close() is collective too."""

    def __init__(self, shape, group=None, zero: bool = False):
        from . import capi

        self.capi = capi
        self.group = group
        self.rank, self.world = _world(group)
        self.local = capi.shared_empty(tuple(shape))
        if zero:  # ordered before any rank's first store by the gather below
            self.local.zero_()
        mine = capi.ipc_export(self.local)
        entries = [None] * self.world
        dist.all_gather_object(entries, mine, group=group)
        self.peers = []  # (rank, base address of that rank's copy), rank order
        try:
            for r, (h, off) in enumerate(entries):
                if r != self.rank:
                    self.peers.append((r, capi.ipc_import(h, off)))
        except Exception:
            for _, p in self.peers:
                capi.ipc_close(p)
            raise

    def replicas(self, byte_offset: int) -> list[int]:
        """Addresses `byte_offset` bytes into every other rank's copy."""
        return [p + byte_offset for _, p in self.peers]

    def close(self) -> None:
        """Collective: waits until no rank writes any more, then unmaps."""
        if self.peers is None:
            return
        _fence(self.group, self.local.device)
        torch.cuda.current_stream().synchronize()
        for _, p in self.peers:
            self.capi.ipc_close(p)
        self.peers = None


class PeerGroup:
    """Cross-GPU barrier over peer memory for the ranks of `group`
    (attnb_peer_barrier_dev): one small kernel per barrier, a few microseconds,
    where a collective of the communication library costs tens.  Every rank
    calls barrier() at the same points of its stream; work enqueued after a
    barrier on any rank sees every store that any rank enqueued before it
    (including kernel stores into other ranks' memory).  The barrier count
    lives on the device, so steps captured in a CUDA graph replay correctly.
    Waits are bounded: a rank that never arrives shows as
    ATTNB_ERR_DEVICE_TIMEOUT on the others (capi.stream_status).  Collective
    construction and close()."""

    def __init__(self, group=None):
        from . import capi

        self.capi = capi
        self.rank, self.world = _world(group)
        # one uint64 epoch per rank, then this rank's barrier count (two
        # float32 words each), zeroed
        self.flags = PeerReplicas((2 * (self.world + 1),), group, zero=True)
        ptrs = [0] * self.world
        for r, p in self.flags.peers:
            ptrs[r] = p
        ptrs[self.rank] = self.flags.local.data_ptr()  # own slot: not read
        self._ptrs = ptrs

    def barrier(self, limit_us: int = 0) -> None:
        self.capi.peer_barrier_dev(self.flags.local.data_ptr(), self._ptrs, self.rank, limit_us)

    def close(self) -> None:
        self.flags.close()


class ShardedGemm:
    """C = A @ B [M, N] with C's rows partitioned across the ranks of `group`
    and no separate gather: rank r's GEMM kernel stores each finished tile of
    its rows [m0, m1) into C on every rank, over NVLink, while its other tiles
    are still being multiplied (attnb_gemm_ex_bcast_dev).  A and B are the
    same on every rank.  forward() returns this object's C buffer, which the
    next forward overwrites; it is complete on every rank when forward
    returns (stream order).  The summation order of every element is that of
    the single-GPU SGEMM (gemm::sgemm_blocked, src/gemm.cpp:319-415)."""

    def __init__(self, M: int, N: int, group=None, ops=None):
        self.ops = ops if ops is not None else DeviceOps()
        self.group = group
        self.M, self.N = M, N
        self.rank, self.world = _world(group)
        self.m0, self.m1 = shard_range(M, self.rank, self.world)
        self.C = PeerReplicas((M, N), group)
        self.sync = PeerGroup(group)

    def forward(self, A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
        if A.shape[0] != self.M or B.shape[1] != self.N or A.shape[1] != B.shape[0]:
            raise ValueError("ShardedGemm: A must be [M, K] and B [K, N]")
        C = self.C.local
        # No rank may still be reading the previous result when the stores start.
        self.sync.barrier()
        if self.m1 > self.m0:
            self.ops.gemm_ex_bcast(A[self.m0:self.m1], B, C[self.m0:self.m1],
                                   self.C.replicas(self.m0 * self.N * 4), False, False, None)
        self.sync.barrier()  # every rank's rows have landed
        return C

    def close(self) -> None:
        self.C.close()
        self.sync.close()


@dataclass
class _HeadShard:
    h0: int
    h1: int
    W_in: torch.Tensor   # [3 * (h1-h0) * Dh, D]: this rank's Q, K, V rows
    b_in: torch.Tensor


class ShardedMHA:
    """mha_block_dense with heads partitioned across the ranks of `group`.

    W_in is sliced once at construction (the rows of the local heads); every
    rank keeps all of W_out and b_out for its block of y's rows; `forward(x)` takes x [T, D] or
    [B, T, D] (identical on every rank) and returns the full y on every rank.
    """

    def __init__(self, W_in, b_in, W_out, b_out, num_heads: int, causal: bool = False,
                 group=None, ops=None, peer_output=None):
        D = W_in.shape[1]
        if W_in.shape != (3 * D, D) or W_out.shape != (D, D):
            raise ValueError("W_in must be [3D, D] and W_out [D, D]")
        if num_heads <= 0 or D % num_heads:
            raise ValueError("num_heads must divide D")
        self.D, self.H, self.Dh = D, num_heads, D // num_heads
        self.causal = causal
        self.group = group
        self.ops = ops if ops is not None else DeviceOps()
        rank, world = _world(group)
        self.rank, self.world = rank, world
        h0, h1 = shard_range(num_heads, rank, world)
        Dh = self.Dh
        rows = [W_in[p * D + h0 * Dh:p * D + h1 * Dh] for p in range(3)]
        bias = [b_in[p * D + h0 * Dh:p * D + h1 * Dh] for p in range(3)]
        self.shard = _HeadShard(h0, h1, torch.cat(rows, 0).contiguous(),
                                torch.cat(bias, 0).contiguous())
        self.W_out = W_out.contiguous()
        self.b_out = b_out.contiguous()
        self.head_counts = [shard_range(num_heads, r, world)[1] - shard_range(num_heads, r, world)[0]
                            for r in range(world)]
        # Peer output: the out-projection kernel stores y's rows into every
        # rank's y (PeerReplicas per input shape) instead of an all-gather.
        can = _peer_capable(self.ops, group)
        if peer_output and not can:
            raise ValueError("peer_output needs the B200 ops on an NCCL group of >1 rank")
        self.peer_output = can if peer_output is None else bool(peer_output)
        self._y = {}  # (B, T) -> PeerReplicas
        self._sync = PeerGroup(group) if self.peer_output else None
        # The B200 ops pack both projection weights once: the module's weights
        # are fixed at construction (the reference repacks them per call).
        self._packed = None
        if hasattr(self.ops, "pack_weight"):
            self._packed = (self.ops.pack_weight(self.shard.W_in) if h1 > h0 else None,
                            self.ops.pack_weight(self.W_out))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        squeeze = x.dim() == 2
        if squeeze:
            x = x.unsqueeze(0)
        B, T, D = x.shape
        s, Dh = self.shard, self.Dh
        hl = s.h1 - s.h0
        rows = B * T
        x2 = x.reshape(rows, D).contiguous()
        # 1) local heads' [q | k | v] = x W_in_local^T + b_in_local
        qkv = torch.empty(rows, 3 * hl * Dh, dtype=x.dtype, device=x.device)
        if hl and self._packed is not None:
            self.ops.linear_packed(x2, self._packed[0], s.b_in, qkv)
        elif hl:
            self.ops.linear(x2, s.W_in, s.b_in, qkv)
        qkv3 = qkv.view(B, T, 3 * hl * Dh)
        # 2) attention of the local heads, all sequences in one call, written
        #    transposed into the all-gather's send buffer ctx_local^T [hl * Dh, B*T]
        ctxT_local = torch.empty(hl * Dh, rows, dtype=x.dtype, device=x.device)
        if hl:
            def heads(p):  # [B, hl, T, Dh] view of the Q, K or V columns
                return qkv3[:, :, p * hl * Dh:(p + 1) * hl * Dh].view(B, T, hl, Dh).permute(
                    0, 2, 1, 3)
            o = ctxT_local.view(hl, Dh, B, T).permute(2, 0, 3, 1)
            self.ops.attention_batched(heads(0), heads(1), heads(2), o, self.causal)
        # 3) all-to-all: rank s receives columns [r0_s, r1_s) of every rank's
        #    ctx_r^T, which stacked in rank order are ctx^T [D, r1_s - r0_s]
        ctxT_mine = _all_to_all_cols(ctxT_local, [c * Dh for c in self.head_counts], self.group)
        # 4) this rank's rows of y = ctx W_out^T + b_out, reading ctx^T
        #    transposed, then an all-gather of the row blocks
        r0, r1 = shard_range(rows, self.rank, self.world)
        if self.peer_output:
            # The kernel stores y's rows [r0, r1) into every rank's y.  The
            # all-to-all above already ordered these stores after every rank's
            # earlier work (no rank still reads the previous y); the fence
            # after them orders every reader after all ranks' rows.
            yb = self._y.get((B, T))
            if yb is None:
                yb = self._y[(B, T)] = PeerReplicas((rows, D), self.group)
            if r1 > r0 and self._packed is not None:
                self.ops.linear_packed(ctxT_mine, self._packed[1], self.b_out, yb.local[r0:r1],
                                       trans_x=True, replicas=yb.replicas(r0 * D * 4))
            elif r1 > r0:
                self.ops.gemm_ex_bcast(ctxT_mine, self.W_out, yb.local[r0:r1],
                                       yb.replicas(r0 * D * 4), True, True, self.b_out)
            self._sync.barrier()
            y = yb.local.view(B, T, D)
            return y[0] if squeeze else y
        y_rows = torch.empty(r1 - r0, D, dtype=x.dtype, device=x.device)
        if r1 > r0 and self._packed is not None:
            self.ops.linear_packed(ctxT_mine, self._packed[1], self.b_out, y_rows, trans_x=True)
        elif r1 > r0:
            self.ops.gemm_ex(ctxT_mine, self.W_out, y_rows, True, True, self.b_out)
        counts = [shard_range(rows, r, self.world)[1] - shard_range(rows, r, self.world)[0]
                  for r in range(self.world)]
        y = _all_gather_rows(y_rows, counts, self.group).view(B, T, D)
        return y[0] if squeeze else y

    def close(self) -> None:
        """Collective: releases the peer output buffers."""
        for yb in self._y.values():
            yb.close()
        self._y = {}
        if self._sync is not None:
            self._sync.close()
            self._sync = None
        if self._packed is not None:
            for w in self._packed:
                if w is not None:
                    w.close()
            self._packed = None


def gemm_sharded(A: torch.Tensor, B: torch.Tensor, group=None, ops=None,
                 shard: str = "rows") -> torch.Tensor:
    """C = A @ B with C partitioned across the ranks of `group`; returns the full
    C on every rank.  shard="rows": rank r computes rows [m0, m1) of C;
    shard="cols": rank r computes columns [n0, n1) (B's column block is read in
    place through its leading dimension), then an all-gather and a permute."""
    ops = ops if ops is not None else DeviceOps()
    rank, world = _world(group)
    M, K = A.shape
    N = B.shape[1]
    if shard == "rows":
        m0, m1 = shard_range(M, rank, world)
        Cl = torch.empty(m1 - m0, N, dtype=A.dtype, device=A.device)
        if m1 > m0:
            ops.sgemm(A[m0:m1], B, Cl)
        counts = [shard_range(M, r, world)[1] - shard_range(M, r, world)[0] for r in range(world)]
        return _all_gather_rows(Cl, counts, group)
    if shard == "cols":
        n0, n1 = shard_range(N, rank, world)
        Cl = torch.empty(M, n1 - n0, dtype=A.dtype, device=A.device)
        if n1 > n0:
            ops.sgemm(A, B[:, n0:n1], Cl)
        counts = [shard_range(N, r, world)[1] - shard_range(N, r, world)[0] for r in range(world)]
        Ct = _all_gather_rows(Cl.t().contiguous(), counts, group)  # [N, M]
        return Ct.t().contiguous()
    raise ValueError("shard must be 'rows' or 'cols'")


def attn_block_sharded(Q, K, V, causal=False, group=None, ops=None) -> torch.Tensor:
    """attn_block_dense with heads partitioned across ranks; Q/K/V [H, L|T, Dh]
    identical on every rank, returns the full O [H, L, Dh] on every rank."""
    ops = ops if ops is not None else DeviceOps()
    rank, world = _world(group)
    H, L, Dh = Q.shape
    h0, h1 = shard_range(H, rank, world)
    Ol = torch.empty(h1 - h0, L, Dh, dtype=Q.dtype, device=Q.device)
    if h1 > h0:
        ops.attention(Q[h0:h1], K[h0:h1], V[h0:h1], Ol, causal)
    counts = [shard_range(H, r, world)[1] - shard_range(H, r, world)[0] for r in range(world)]
    return _all_gather_rows(Ol, counts, group)


def attn_step_sharded(Q, K, V, group=None, ops=None) -> torch.Tensor:
    """attn_step_dense (one decode step) with heads partitioned across ranks.

    Q [H, Dh] and K / V [H, T, Dh] (batch and heads flattened into H; any
    strides) are the same views on every rank; rank r reads only its heads
    [h0, h1) of K and V, computes O [h1 - h0, Dh], and an all-gather returns
    the full O [H, Dh] on every rank.  The reference's decode step
    (src/attn_dense.cpp:21-73) treats heads independently, so the partition
    changes no arithmetic."""
    ops = ops if ops is not None else DeviceOps()
    rank, world = _world(group)
    H, Dh = Q.shape
    h0, h1 = shard_range(H, rank, world)
    Ol = torch.empty(h1 - h0, Dh, dtype=Q.dtype, device=Q.device)
    if h1 > h0:
        ops.decode(Q[h0:h1], K[h0:h1], V[h0:h1], Ol)
    counts = [shard_range(H, r, world)[1] - shard_range(H, r, world)[0] for r in range(world)]
    return _all_gather_rows(Ol, counts, group)


class ShardedDecode:
    """The decode step (attn::attn_step_dense, src/attn_dense.cpp:21-73) with
    heads partitioned across the ranks of `group` and no separate gather:
    rank r's kernels read only its heads [h0, h1) of K and V and store their
    output heads into O on every rank over NVLink
    (attnb_attn_step_dense_bcast_dev), then one peer-memory barrier
    (PeerGroup) orders every reader after all ranks' heads.  O is double
    buffered, so one barrier per step suffices: step() returns an [H, Dh]
    buffer that stays valid until the step after next.  Q [H, Dh] and K / V
    [H, T, Dh] (batch and heads flattened into H; any strides) are the same
    views on every rank."""

    def __init__(self, H: int, Dh: int, group=None, ops=None):
        self.ops = ops if ops is not None else DeviceOps()
        self.H, self.Dh = H, Dh
        self.rank, self.world = _world(group)
        self.h0, self.h1 = shard_range(H, self.rank, self.world)
        self.O = [PeerReplicas((H, Dh), group) for _ in range(2)]
        self.sync = PeerGroup(group)
        self.n = 0

    def step(self, Q, K, V) -> torch.Tensor:
        if Q.shape != (self.H, self.Dh) or K.shape[0] != self.H or V.shape[0] != self.H:
            raise ValueError("ShardedDecode: Q must be [H, Dh] and K, V [H, T, Dh]")
        ob = self.O[self.n & 1]
        self.n += 1
        h0, h1 = self.h0, self.h1
        if h1 > h0:
            self.ops.decode_bcast(Q[h0:h1], K[h0:h1], V[h0:h1], ob.local[h0:h1],
                                  ob.replicas(h0 * self.Dh * 4))
        self.sync.barrier()
        return ob.local

    def close(self) -> None:
        for ob in self.O:
            ob.close()
        self.sync.close()
