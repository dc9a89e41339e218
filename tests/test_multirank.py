"""Host logic of the multi-GPU path, run as two gloo ranks on CPU: the batch sharding, the
out-of-band exchange of the collective's id (rank 0 -> all), the max/sum reductions the bench
uses for its device times and the gather of every rank's sampled output rows to rank 0 for the
output check. The NCCL gather of the outputs themselves needs GPUs: bench.py --gpus N checks its
result against the reference runtime on every run ("verify")."""
import os
import socket
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    import bench
    dist = bench.Dist(world)
    try:
        blob = bytes(range(128)) if rank == 0 else None
        got = dist.broadcast_bytes(blob, 128)
        gathered = dist.gather_object({bench.shard(4096, world, rank)[0]: bytes([rank]) * 3})
        results[rank] = {"id": got, "max": dist.max(10.0 + rank), "sum": dist.sum(1.5 * (rank + 1)),
                         "shard": bench.shard(4096, world, rank), "gathered": gathered}
        dist.barrier()
    finally:
        dist.close()


def test_two_gloo_ranks_share_the_id_and_reduce_times():
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_rank_main, args=(world, port, results), nprocs=world, join=True)
        res = dict(results)
    assert res[0]["id"] == res[1]["id"] == bytes(range(128))
    assert res[0]["max"] == res[1]["max"] == 11.0
    assert res[0]["sum"] == res[1]["sum"] == 4.5
    assert [res[r]["shard"] for r in range(world)] == [(0, 2048), (2048, 2048)]
    # the bench's output check: every rank's sampled rows reach rank 0, rank-ordered
    assert res[0]["gathered"] == [{0: b"\0\0\0"}, {2048: b"\1\1\1"}] and res[1]["gathered"] is None


def test_shards_cover_the_global_batch_in_order():
    sys.path.insert(0, str(ROOT))
    import bench
    for world in (1, 2, 4, 8):
        slices = [bench.shard(4096, world, r) for r in range(world)]
        assert slices[0][0] == 0 and all(a[0] + a[1] == b[0] for a, b in zip(slices, slices[1:]))
        assert sum(n for _, n in slices) == 4096
    with pytest.raises(ValueError):
        bench.shard(1000, 3, 0)
