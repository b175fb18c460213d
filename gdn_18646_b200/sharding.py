"""Head and batch sharding of the GDN hot path across the GPUs of one node
(one process per GPU, torch.distributed).

Every (batch, value head) sequence of the gated delta rule is independent
(its fp32 state [dk, dv] never mixes with another), so:

* batch sharding needs no communication at all (each rank owns whole
  sequences and their states) -- the decode path and the weak-scaled
  prefill bench use it;
* head sharding (one long sequence batch, heads split over
  ranks) needs one collective, an all-gather of the bf16 output o so every
  rank holds [B, T, H, dv]; each rank keeps its own fp32 final-state shard.

The reference has no multi-GPU code; this module is new (the all-gather is
NCCL over NVLink on B200, gloo on CPU for tests).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    heads: int           # total value heads H
    h0: int              # first head of this rank
    h1: int              # one past the last head

    @property
    def count(self) -> int:
        return self.h1 - self.h0


def head_shard(H: int, rank: int, world: int, Hqk: int | None = None) -> HeadShard:
    """Contiguous, equal split of H value heads over ``world`` ranks.  With
    grouped value heads (Hqk < H) every rank's heads must map onto whole q/k
    groups, i.e. (H / world) % (H / Hqk) == 0."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} / world {world}")
    if H % world != 0:
        raise ValueError(f"{H} heads do not split evenly over {world} ranks")
    per = H // world
    if Hqk is not None and Hqk != H:
        group = H // Hqk
        if per % group != 0:
            raise ValueError(f"{per} heads per rank cut a q/k group of {group} value heads")
    return HeadShard(rank, world, H, rank * per, (rank + 1) * per)


def batch_shard(B: int, rank: int, world: int) -> slice:
    """Batch rows of ``rank`` when B rows are split as evenly as possible."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} / world {world}")
    base, rem = divmod(B, world)
    start = rank * base + min(rank, rem)
    return slice(start, start + base + (1 if rank < rem else 0))


def shard_heads(x: torch.Tensor, shard: HeadShard, axis: int) -> torch.Tensor:
    """The rank's heads of ``x`` along ``axis`` (contiguous copy)."""
    return x.narrow(axis, shard.h0, shard.count).contiguous()


def gather_heads(o_local: torch.Tensor, shard: HeadShard, group=None) -> torch.Tensor:
    """All-gather [B, T, H/world, dv] shards into [B, T, H, dv] on every rank."""
    import torch.distributed as dist
    world = shard.world
    if world == 1:
        return o_local
    o_local = o_local.contiguous()
    if dist.get_backend(group) == "nccl":
        gathered = torch.empty((world,) + tuple(o_local.shape), dtype=o_local.dtype, device=o_local.device)
        dist.all_gather_into_tensor(gathered, o_local, group=group)
        parts = list(gathered.unbind(0))
    else:
        parts = [torch.empty_like(o_local) for _ in range(world)]
        dist.all_gather(parts, o_local, group=group)
    return torch.cat(parts, dim=2)


def sharded_prefill(q, k, v, A_log, a, b, shard: HeadShard, *, Hqk=None, gather=True, group=None, **kw):
    """Head-sharded prefill (layout [B,T,H,D]): each rank runs the kernel on
    its value heads (and the q/k heads they read), then optionally all-gathers
    o.  Inputs are the FULL tensors; returns (o, state_shard)."""
    from . import ops
    H = v.shape[2]
    Hqk = Hqk or q.shape[2]
    group_sz = H // Hqk
    qs = q.narrow(2, shard.h0 // group_sz, shard.count // group_sz).contiguous()
    ks = k.narrow(2, shard.h0 // group_sz, shard.count // group_sz).contiguous()
    vs = shard_heads(v, shard, 2)
    o, S = ops.prefill(qs, ks, vs, shard_heads(A_log, shard, 0), shard_heads(a, shard, 1),
                       shard_heads(b, shard, 1), layout="bthd", **kw)
    return (gather_heads(o, shard, group) if gather else o), S


# ---------------------------------------------------------------------------
# Head-sharded output projection fused with its reduce-scatter
# ---------------------------------------------------------------------------
def owned_rows(M: int, rank: int, world: int) -> slice:
    """Token rows of the layer output that ``rank`` keeps after the reduce-scatter."""
    if M % world != 0:
        raise ValueError(f"{M} rows do not split evenly over {world} ranks")
    per = M // world
    return slice(rank * per, (rank + 1) * per)


class PeerBuffer:
    """A receive buffer [world, rows, N] bf16 on every rank, and the device
    pointers of all ranks' buffers in this process (CUDA IPC; NVLink peer
    access within a node).  Slot s of rank d's buffer receives rank s's
    partial product for the rows that d owns."""

    def __init__(self, rows: int, N: int, group=None):
        import torch.distributed as dist
        from cuda.bindings import driver as drv
        from cuda.bindings import runtime as rt
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.local = torch.empty(self.world, rows, N, dtype=torch.bfloat16, device="cuda")
        self.flag = torch.zeros(1, device="cuda")
        self._opened = []
        ptr = self.local.data_ptr()
        if self.world == 1:
            self.ptrs = [ptr]
            return
        err, base, _size = drv.cuMemGetAddressRange(ptr)
        if err != drv.CUresult.CUDA_SUCCESS:
            raise RuntimeError(f"cuMemGetAddressRange: {err}")
        offset = ptr - int(base)
        err, handle = rt.cudaIpcGetMemHandle(int(base))
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"cudaIpcGetMemHandle: {err}")
        mine = (bytes(handle.reserved), offset)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self.ptrs = []
        for s, (h, off) in enumerate(everyone):
            if s == self.rank:
                self.ptrs.append(ptr)
                continue
            hh = rt.cudaIpcMemHandle_t()
            hh.reserved = h
            err, peer = rt.cudaIpcOpenMemHandle(hh, rt.cudaIpcMemLazyEnablePeerAccess)
            if err != rt.cudaError_t.cudaSuccess:
                raise RuntimeError(f"cudaIpcOpenMemHandle (rank {s}): {err}")
            self._opened.append(peer)
            self.ptrs.append(int(peer) + off)

    def close(self):
        from cuda.bindings import runtime as rt
        torch.cuda.synchronize()
        for p in self._opened:
            rt.cudaIpcCloseMemHandle(p)
        self._opened = []


def sharded_out_proj(x_local: torch.Tensor, W_local: torch.Tensor, buf: PeerBuffer, out=None) -> torch.Tensor:
    """y[rows owned by this rank] = sum over ranks of x_r W_r^T, with x_local [M, K_r]
    this rank's gated-normed head outputs and W_local [N, K_r] its columns of the
    output projection.  One fused launch computes the partial product and writes
    each tile into its owner's buffer over NVLink (gdn_outproj_rs_fwd); two
    1-element all-reduces order it against the other ranks (the previous call's
    reduction done before slots are overwritten; every rank's tiles landed
    before this reduction)."""
    from . import ops
    import torch.distributed as dist
    if buf.world > 1:
        dist.all_reduce(buf.flag, group=buf.group)
    ops.outproj_rs(x_local, W_local, buf.ptrs, buf.rank, buf.world)
    if buf.world > 1:
        dist.all_reduce(buf.flag, group=buf.group)
    return ops.outproj_reduce(buf.local, out)
