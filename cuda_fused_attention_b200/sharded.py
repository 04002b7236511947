"""Multi-GPU driver: one process per GPU, (batch x heads) slabs split across ranks.

Attention over different (batch, head) slabs is independent (no K/V shared
across heads), so a call over B*H slabs partitions into contiguous slab ranges,
one per rank, and every rank runs the single-GPU kernel on its own range. There
is no collective on the data path. The only collective is the optional gather
of the O slices to one rank (NCCL over NVLink / NVSwitch on GPUs, gloo in the
CPU tests), which callers time separately from the forward pass.

The reference has no multi-GPU code (its docs/project_outline.md:43 lists it as
out of scope); this module is the (batch x heads) sharding BASELINE config 5
asks for.
"""
from dataclasses import dataclass

from . import AttentionShape, launch_attention_sm100


def slab_range(total, rank, world):
    """Contiguous, near-equal [begin, end) ranges of `total` slabs; the first total % world
    ranks take one extra slab."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(total, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


@dataclass(frozen=True)
class SlabShard:
    """This rank's share of a [B, H, N, D] problem."""
    shape: AttentionShape
    rank: int
    world: int

    @property
    def bounds(self):
        return slab_range(self.shape.slabs, self.rank, self.world)

    @property
    def slabs(self):
        begin, end = self.bounds
        return end - begin

    @property
    def max_slabs(self):
        return -(-self.shape.slabs // self.world)

    @property
    def local_shape(self):
        """The shard as a self-contained problem: [slabs, 1, N, D]."""
        return AttentionShape(self.slabs, 1, self.shape.seq_len, self.shape.head_dim)

    @property
    def slab_elems(self):
        return self.shape.seq_len * self.shape.head_dim

    def local_view(self, full):
        """The shard's slabs of a full contiguous [B, H, N, D] tensor (a view, no copy)."""
        begin, end = self.bounds
        return full.reshape(self.shape.slabs, self.slab_elems)[begin:end].reshape(-1)


def forward_local(q_local, k_local, v_local, o_local, shard, causal, stream=None):
    """The per-rank forward: the sm_100a kernel over this rank's slabs (device tensors)."""
    if shard.slabs:
        launch_attention_sm100(q_local, k_local, v_local, o_local, shard.local_shape, causal, stream)


def gather_slabs(o_local, shard, group=None):
    """Collect every rank's O slice on every rank (all_gather); returns the full flat tensor on
    all ranks. When the shards differ in size, slices are padded to the largest so that the
    collective is uniform; every rank must call this, in the same order, like any collective."""
    import torch
    import torch.distributed as dist
    # Moved as raw bytes: bit-exact, and every backend (NCCL, gloo) supports uint8.
    local = o_local.reshape(-1).view(torch.uint8)
    if shard.shape.slabs % shard.world == 0:
        # Equal shards: gather straight from the slice into the output (no padding copy in,
        # no unpadding copy out).
        recv = torch.empty(local.numel() * shard.world, dtype=torch.uint8, device=o_local.device)
        dist.all_gather_into_tensor(recv, local, group=group)
        return recv.view(o_local.dtype)
    item = o_local.element_size()
    pad = shard.max_slabs * shard.slab_elems * item
    send = torch.zeros(pad, dtype=torch.uint8, device=o_local.device)
    send[: local.numel()] = local
    recv = torch.empty(pad * shard.world, dtype=torch.uint8, device=o_local.device)
    dist.all_gather_into_tensor(recv, send, group=group)
    parts = []
    for r in range(shard.world):
        begin, end = slab_range(shard.shape.slabs, r, shard.world)
        parts.append(recv[r * pad: r * pad + (end - begin) * shard.slab_elems * item])
    return torch.cat(parts).view(o_local.dtype)


def time_gather(o_local, shard, iters=5, warmup=2, group=None):
    """Time gather_slabs on its own (it is never inside the forward's timed region): the mean
    time of `iters` gathers after `warmup` untimed ones, max over ranks, with CUDA events on
    the current stream for device tensors and the host clock otherwise. Bandwidths follow the
    NCCL convention for an all-gather: algbw = bytes of the gathered output / time,
    busbw = algbw * (world - 1) / world (what each rank's links carry)."""
    import time
    import torch
    import torch.distributed as dist
    world = shard.world
    on_gpu = o_local.is_cuda
    for _ in range(warmup):
        gather_slabs(o_local, shard, group)
    if dist.is_initialized() and world > 1:
        dist.barrier(group=group, device_ids=[o_local.device.index] if on_gpu else None)
    if on_gpu:
        torch.cuda.synchronize(o_local.device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(iters):
            gather_slabs(o_local, shard, group)
        end.record()
        end.synchronize()
        ms = start.elapsed_time(end) / iters
    else:
        t0 = time.perf_counter()
        for _ in range(iters):
            gather_slabs(o_local, shard, group)
        ms = (time.perf_counter() - t0) * 1e3 / iters
    (ms,) = max_over_ranks([ms], device=o_local.device if on_gpu else None, group=group)
    out_bytes = shard.shape.numel * o_local.element_size()
    algbw = out_bytes / (ms * 1e-3) / 1e9
    even = shard.shape.slabs % world == 0
    return {"ms": ms, "bytes": out_bytes, "algbw_GBps": algbw, "busbw_GBps": algbw * (world - 1) / world,
            "ranks": world, "iters": iters,
            "collective": "all_gather_into_tensor of raw bytes" + (
                ", straight from each rank's slice" if even else
                ", padded to the largest shard, plus the unpadding copy")}


def max_over_ranks(values, device=None, group=None):
    """Element-wise max of a list of floats across ranks (the timing reduction)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.tolist()
