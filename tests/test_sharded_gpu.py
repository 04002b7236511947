"""The slab-sharded multi-GPU path on real GPUs: one process per GPU, NCCL gather.

Two ranks each run the kernel on their contiguous range of the batch*heads
slabs (no collective on the data path), then gather the O slices with NCCL;
rank 0 requires the gathered output to be bit-identical to a single-GPU run of
the whole problem. Skipped where fewer than two GPUs are visible.
"""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]
    import datetime
    import torch
    import torch.distributed as dist
    import fa_oracle
    from cuda_fused_attention_b200 import AttentionShape, launch_attention_sm100
    from cuda_fused_attention_b200.sharded import SlabShard, forward_local, gather_slabs

    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=device)
    try:
        # 15 slabs: ranges of 8 and 7 (padded gather); 8 slabs: 4 and 4 (direct gather).
        for shape in (AttentionShape(3, 5, 1000, 128), AttentionShape(2, 4, 1000, 128)):
            q, k, v = fa_oracle.make_inputs(shape.batch, shape.heads, shape.seq_len, shape.head_dim)
            full = [torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(device) for x in (q, k, v)]
            shard = SlabShard(shape, rank, world)
            local = [shard.local_view(t).contiguous() for t in full]
            o_local = torch.empty_like(local[0])
            for causal in (False, True):
                forward_local(local[0], local[1], local[2], o_local, shard, causal)
                gathered = gather_slabs(o_local, shard)
                if rank == 0:
                    o_one = torch.empty_like(full[0])
                    launch_attention_sm100(full[0], full[1], full[2], o_one, shape, causal)
                    torch.cuda.synchronize()
                    same = torch.equal(gathered.view(torch.int16), o_one.view(torch.int16))
                    with open(result_path + f".{shape.slabs}.{int(causal)}", "w") as fh:
                        fh.write("ok" if same else "mismatch")
    finally:
        dist.destroy_process_group()


def test_two_gpu_shards_equal_one_gpu(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    result = str(tmp_path / "sharded")
    mp.start_processes(_rank_main, args=(2, _free_port(), result), nprocs=2, start_method="spawn", join=True)
    for slabs in (15, 8):
        for causal in (0, 1):
            assert open(f"{result}.{slabs}.{causal}").read() == "ok"
