"""N-sharding host logic with world_size-2 gloo ranks on CPU: each rank takes its B^T shard, the
shard's D slab (computed here by the CPU oracle standing in for the device kernel) is all-gathered
and reassembled, and the result equals the unsharded D bit for bit. Also checks the max-over-ranks
timing reduction bench.py uses."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, out_path):
    import sys
    for p in (os.path.join(ROOT, "mxfp6-gemm_b200"), os.path.join(ROOT, "oracle")):
        sys.path.insert(0, p)
    from mxfp6_b200.shard import assemble_columns, shard_B
    from mxfp6_b200.synth import make_operands
    from oracle import Oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ops = make_operands(128, 512, 256, kind="codes", seed=3, exp_range=(118, 130))
        Bt_r, sB_r = shard_B(ops.Bt, ops.sB, world, rank)
        orc = Oracle()
        D_r = torch.from_numpy(orc.gemm(ops.A, ops.sA, Bt_r, sB_r, ops.Kp, threads=1))
        gathered = [torch.empty_like(D_r) for _ in range(world)]
        dist.all_gather(gathered, D_r)
        D = assemble_columns(torch.stack(gathered))
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            full = orc.gemm(ops.A, ops.sA, ops.Bt, ops.sB, ops.Kp, threads=1)
            ok = np.array_equal(D.numpy().view(np.uint32), full.view(np.uint32)) and t.item() == world
            with open(out_path, "w") as f:
                f.write("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_column_sharding_with_gloo(tmp_path):
    out = tmp_path / "result.txt"
    port = 29500 + os.getpid() % 1000
    mp.spawn(_worker, args=(2, port, str(out)), nprocs=2, join=True)
    assert out.read_text() == "ok"


def test_shard_range_validation():
    import sys
    sys.path.insert(0, os.path.join(ROOT, "mxfp6-gemm_b200"))
    from mxfp6_b200.shard import assemble_columns, shard_range
    assert shard_range(28672, 8, 7) == (25088, 28672)
    with pytest.raises(ValueError):
        shard_range(28672, 3, 0)
    stacked = np.arange(2 * 3 * 4).reshape(2, 3, 4)
    assert assemble_columns(stacked).tolist() == [[0, 1, 2, 3, 12, 13, 14, 15], [4, 5, 6, 7, 16, 17, 18, 19],
                                                   [8, 9, 10, 11, 20, 21, 22, 23]]
