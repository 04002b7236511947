"""Host logic of the multi-GPU driver, as world_size-2 gloo ranks on the CPU.

The per-rank compute here is the CPU oracle standing in for the kernel (these
ranks have no GPU); what is under test is the partition, the gather of the O
slices, the max-over-ranks timing reduction, and that a rank which leaves
early turns into an error on the others instead of a hang.
"""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_slab_range_partitions_exactly():
    from cuda_fused_attention_b200.sharded import slab_range
    for total in (1, 2, 5, 7, 512, 513):
        for world in (1, 2, 3, 4, 8):
            ranges = [slab_range(total, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == total
            for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        slab_range(4, 2, 2)


def _worker(rank, world, port, mode, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    import datetime
    import torch
    import torch.distributed as dist
    import fa_oracle
    from cuda_fused_attention_b200 import AttentionShape
    from cuda_fused_attention_b200.sharded import SlabShard, gather_slabs, max_over_ranks, time_gather

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    shape = AttentionShape(1, 4 if mode == "gather_even" else 5, 70, 64)   # 2+2 or 3+2 slabs
    shard = SlabShard(shape, rank, world)
    q, k, v = fa_oracle.make_inputs(shape.batch, shape.heads, shape.seq_len, shape.head_dim)
    begin, end = shard.bounds
    e = shard.slab_elems
    ql, kl, vl = (x[begin * e:end * e] for x in (q, k, v))
    local = fa_oracle.attention(ql, kl, vl, shard.slabs, 1, shape.seq_len, shape.head_dim, 1)
    bits = torch.from_numpy(np.ascontiguousarray(
        (local.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)).view(np.int16))
    if mode == "leave" and rank == 1:
        dist.destroy_process_group()
        return                      # leaves between steps, never joins the gather
    try:
        if mode == "time":
            stats = time_gather(bits, shard, iters=3, warmup=1)
            if rank == 0:
                import json
                with open(result_path, "w") as fh:
                    json.dump(stats, fh)
            return
        full = gather_slabs(bits, shard)
        (worst,) = max_over_ranks([float(rank + 1)])
        if rank == 0:
            want = fa_oracle.attention(q, k, v, shape.batch, shape.heads, shape.seq_len, shape.head_dim, 1)
            want_bits = (want.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
            ok = np.array_equal(full.numpy().view(np.uint16), want_bits) and worst == float(world)
            with open(result_path, "w") as fh:
                fh.write("ok" if ok else "mismatch")
    except Exception as exc:   # noqa: BLE001 -- the failure mode is the thing under test
        with open(result_path + f".rank{rank}", "w") as fh:
            fh.write(type(exc).__name__)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _spawn(mode, tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    result = str(tmp_path / f"result_{mode}")
    mp.start_processes(_worker, args=(2, port, mode, result), nprocs=2, start_method="spawn", join=True)
    return result


@pytest.mark.parametrize("mode", ["gather", "gather_even"])
def test_gather_and_timing_reduction_two_ranks(tmp_path, mode):
    result = _spawn(mode, tmp_path)
    assert open(result).read() == "ok"


def test_gather_timing_two_ranks(tmp_path):
    """sharded.time_gather, the separately timed O gather that bench.py --gather reports."""
    import json
    stats = json.load(open(_spawn("time", tmp_path)))
    assert stats["ranks"] == 2 and stats["iters"] == 3 and stats["ms"] > 0
    assert stats["bytes"] == 1 * 5 * 70 * 64 * 2
    assert abs(stats["busbw_GBps"] - stats["algbw_GBps"] / 2) < 1e-9


def test_rank_leaving_early_surfaces_as_error(tmp_path):
    result = _spawn("leave", tmp_path)
    # Rank 0's collective ends with an error within the process-group timeout.
    assert os.path.exists(result + ".rank0")
