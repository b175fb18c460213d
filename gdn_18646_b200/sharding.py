"""Head and batch sharding of the GDN hot path across the GPUs of one node
(one process per GPU, torch.distributed).

Every (batch, value head) sequence of the gated delta rule is independent
(its fp32 state [dk, dv] never mixes with another), so:

* batch sharding needs no communication at all (each rank owns whole
  sequences and their states) -- the decode path and the weak-scaled
  prefill bench use it;
* head sharding (config 4: one long sequence batch, heads split over ranks)
  needs one collective, an all-gather of the bf16 output o so every rank holds
  o of all heads; each rank keeps its own fp32 final-state shard.  Either NCCL
  after the prefill (``sharded_prefill``) or copy-engine pulls over NVLink
  overlapped with the prefill window by window (``WindowedHeadGather``).

The reference has no multi-GPU code; this module is new (gloo on CPU for tests).
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
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.local = torch.empty(self.world, rows, N, dtype=torch.bfloat16, device="cuda")
        self.flag = torch.zeros(1, device="cuda")
        self.ptrs, self._opened = map_peers(self.local, self.world, self.rank, group)

    def close(self):
        close_peers(self._opened)
        self._opened = []


def map_peers(local: torch.Tensor, world: int, rank: int, group=None):
    """The device pointers of every rank's ``local`` tensor in this process:
    this rank's own, the peers' through CUDA IPC (the allocation's handle and the
    tensor's offset in it, exchanged with all_gather_object).  Collective: every
    rank calls it with its tensor.  Returns (pointers, mappings to close)."""
    import torch.distributed as dist
    from cuda.bindings import driver as drv
    from cuda.bindings import runtime as rt
    ptr = local.data_ptr()
    if world == 1:
        return [ptr], []
    err, base, _size = drv.cuMemGetAddressRange(ptr)
    if err != drv.CUresult.CUDA_SUCCESS:
        raise RuntimeError(f"cuMemGetAddressRange: {err}")
    offset = ptr - int(base)
    err, handle = rt.cudaIpcGetMemHandle(int(base))
    if err != rt.cudaError_t.cudaSuccess:
        raise RuntimeError(f"cudaIpcGetMemHandle: {err}")
    mine = (bytes(handle.reserved), offset)
    everyone = [None] * world
    dist.all_gather_object(everyone, mine, group=group)
    ptrs, opened = [], []
    for s, (h, off) in enumerate(everyone):
        if s == rank:
            ptrs.append(ptr)
            continue
        hh = rt.cudaIpcMemHandle_t()
        hh.reserved = h
        err, peer = rt.cudaIpcOpenMemHandle(hh, rt.cudaIpcMemLazyEnablePeerAccess)
        if err != rt.cudaError_t.cudaSuccess:
            for p in opened:
                rt.cudaIpcCloseMemHandle(p)
            raise RuntimeError(f"cudaIpcOpenMemHandle (rank {s}): {err}")
        opened.append(peer)
        ptrs.append(int(peer) + off)
    return ptrs, opened


def close_peers(opened) -> None:
    """Unmap the IPC mappings ``map_peers`` opened (after the device is idle)."""
    from cuda.bindings import runtime as rt
    torch.cuda.synchronize()
    for p in opened:
        rt.cudaIpcCloseMemHandle(p)


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


# ---------------------------------------------------------------------------
# Head-sharded prefill with the all-gather of o overlapped, token window by window
# ---------------------------------------------------------------------------
CHUNK = 64


def window_plan(T: int, window_tokens: int = 0, ladder: bool = True) -> list[tuple[int, int]]:
    """Token windows (t0, Tw) covering [0, T), every start on a 64-token chunk
    boundary (so the chained windows are bit-identical to one call).  Windows of
    ``window_tokens`` (rounded up to whole chunks; 0 = about T/8); with
    ``ladder`` the last full window is cut into halving ones down to one chunk,
    so the pull that remains after the last prefill is short."""
    if T <= 0:
        raise ValueError(f"T must be positive, got {T}")
    if window_tokens < 0:
        raise ValueError(f"window_tokens must be >= 0, got {window_tokens}")
    nch = (T + CHUNK - 1) // CHUNK
    w = (window_tokens + CHUNK - 1) // CHUNK if window_tokens else max(1, (nch + 7) // 8)
    sizes = [w] * (nch // w) + ([nch % w] if nch % w else [])
    if ladder and sizes:
        last = sizes.pop()
        tail = []
        while last > 1:
            half = last // 2
            tail.append(last - half)
            last = half
        tail.append(last)
        sizes += tail
    out, c0 = [], 0
    for n in sizes:
        t0 = c0 * CHUNK
        out.append((t0, min(T, (c0 + n) * CHUNK) - t0))
        c0 += n
    return out


class WindowedHeadGather:
    """Head-sharded prefill whose all-gather of o overlaps the prefill.

    Every rank holds ``gathered`` [world, B, H_local, T, dv] ("bhtd") or [world,
    B, T, H_local, dv] ("bthd") bf16; the prefill writes this rank's o straight
    into its slot, one token window at a time (gdn_prefill_window_ws, the state
    carried between windows).  After window i is enqueued, a copy stream waits
    for it, takes a 1-element all-reduce (so every rank's window i is in its
    slot) and pulls window i of every peer's slot over NVLink with copy-engine
    transfers (gdn_gather_window), while window i + 1 computes.  A 1-element
    all-reduce at the start of a call keeps a rank from rewriting its slot while
    a peer still pulls the previous call's windows.  The result is the
    gathered buffer itself: valid until the next call."""

    def __init__(self, B: int, T: int, H_local: int, dv: int, layout: str = "bhtd", group=None):
        import torch.distributed as dist
        if layout not in ("bhtd", "bthd"):
            raise ValueError(f"layout must be 'bhtd' or 'bthd', got {layout!r}")
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.layout = layout
        self.B, self.T, self.H, self.dv = B, T, H_local, dv
        shape = (B, H_local, T, dv) if layout == "bhtd" else (B, T, H_local, dv)
        self.gathered = torch.empty((self.world,) + shape, dtype=torch.bfloat16, device="cuda")
        self.flag = torch.zeros(1, device="cuda")
        self.comm = torch.cuda.Stream()
        self.ptrs, self._opened = map_peers(self.gathered, self.world, self.rank, group)

    def close(self) -> None:
        close_peers(self._opened)
        self._opened = []

    def prefill(self, q, k, v, A_log, a, b_logits, *, window_tokens: int = 0, ladder: bool = True, dt_bias=0.0,
                mask=None, state_in=None, state_out=None, scale: float = 0.0):
        """This rank's heads over the whole sequence (q, k, v, gates in the
        buffer's layout), o of all heads gathered.  Returns (gathered, state_out)."""
        import torch.distributed as dist
        from . import _lib, ops
        o_local = self.gathered[self.rank]
        if tuple(v.shape) != tuple(o_local.shape):
            raise ValueError(f"v {tuple(v.shape)} does not match the buffer's slot {tuple(o_local.shape)}")
        dk = q.shape[-1]
        if state_out is None:
            state_out = torch.empty(self.B, self.H, dk, self.dv, dtype=torch.float32, device=q.device)
        plan = window_plan(self.T, window_tokens, ladder)
        wmax = max(tw for _, tw in plan)
        ws = torch.empty(max(1, int(_lib.lib().gdn_prefill_workspace_bytes(self.B, wmax, self.H, dk, self.dv))),
                         dtype=torch.uint8, device=q.device)
        carry = [torch.empty_like(state_out), torch.empty_like(state_out)] if len(plan) > 1 else []
        main = torch.cuda.current_stream()
        if self.world > 1:
            dist.all_reduce(self.flag, group=self.group)
        s_in = state_in
        for i, (t0, tw) in enumerate(plan):
            s_out = state_out if i == len(plan) - 1 else carry[i % 2]
            ops.prefill_window(q, k, v, A_log, a, b_logits, t0, tw, out=o_local, dt_bias=dt_bias, mask=mask,
                               state_in=s_in, state_out=s_out, scale=scale, layout=self.layout, workspace=ws)
            s_in = s_out
            if self.world > 1:
                self.comm.wait_stream(main)
                with torch.cuda.stream(self.comm):
                    dist.all_reduce(self.flag, group=self.group)
                    ops.gather_window(self.gathered, self.ptrs, self.rank, t0, tw, self.layout, stream=self.comm)
        main.wait_stream(self.comm)
        return self.gathered, state_out

    def pull(self, t0: int = 0, Tw: int | None = None) -> None:
        """Only the gather: tokens [t0, t0 + Tw) of every peer's slot into this
        rank's buffer (1-element all-reduce, then the copy-engine pulls), on the
        copy stream, ordered after and before the current stream's work; the
        cost of the transfer that the windowed prefill overlaps."""
        import torch.distributed as dist
        from . import ops
        Tw = self.T - t0 if Tw is None else Tw
        main = torch.cuda.current_stream()
        self.comm.wait_stream(main)
        with torch.cuda.stream(self.comm):
            if self.world > 1:
                dist.all_reduce(self.flag, group=self.group)
                ops.gather_window(self.gathered, self.ptrs, self.rank, t0, Tw, self.layout, stream=self.comm)
        main.wait_stream(self.comm)
