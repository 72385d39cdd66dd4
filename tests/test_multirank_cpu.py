"""World-size-2 tests of the multi-GPU host logic on CPU (gloo backend).

The decode path shards by sequence with no collective on the hot path
(promptboot_b200/shard.py): these tests run two gloo ranks as processes and
check that the ranks' sequence blocks partition the global batch, that each
rank regenerates exactly the prompts and sampler seeds a single process would,
and that the timed duration is the max over ranks.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, per_rank: int, plen: int, out_dir: str):
    import torch
    import torch.distributed as dist
    from promptboot_b200 import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        g = shard.global_sequences(rank, world, per_rank)
        prompts = shard.prompts_for(rank, world, per_rank, plen)
        seeds = np.array([shard.sampling_seed(x) for x in g], dtype=np.int64)
        # Gather every rank's block over gloo (test-only; the bench never gathers).
        gt = torch.from_numpy(g.copy())
        gathered = [torch.empty_like(gt) for _ in range(world)]
        dist.all_gather(gathered, gt)
        shard.barrier(world)
        my_ms = 10.0 + 5.0 * rank          # rank 1 is the slow one
        mx = shard.max_over_ranks(my_ms, world, device="cpu")
        value = shard.aggregate_throughput(per_rank * 4, world, mx)
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), g=g, prompts=prompts, seeds=seeds,
                 gathered=torch.stack(gathered).numpy(), mx=mx, value=value)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_partition_the_batch(tmp_path):
    import torch.multiprocessing as mp
    from promptboot_b200 import shard
    world, per_rank, plen = 2, 6, 16
    mp.start_processes(_worker, args=(world, _free_port(), per_rank, plen, str(tmp_path)),
                       nprocs=world, start_method="spawn", join=True)
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    all_g = np.concatenate([r["g"] for r in res])
    assert sorted(all_g.tolist()) == list(range(world * per_rank))          # a partition
    assert np.array_equal(res[0]["gathered"].reshape(-1), all_g)             # contiguous blocks
    single = np.stack([shard.prompt_for(i, plen) for i in range(world * per_rank)])
    assert np.array_equal(np.concatenate([r["prompts"] for r in res]), single)
    assert np.concatenate([r["seeds"] for r in res]).tolist() == list(range(world * per_rank))
    for r in res:
        assert float(r["mx"]) == 15.0                                        # max over ranks
        assert float(r["value"]) == pytest.approx(per_rank * 4 * world / 0.015)


def test_single_rank_helpers():
    from promptboot_b200 import shard
    assert shard.global_sequences(0, 1, 3).tolist() == [0, 1, 2]
    assert shard.global_sequences(3, 4, 2).tolist() == [6, 7]
    assert shard.max_over_ranks(7.5, 1) == 7.5
    with pytest.raises(ValueError):
        shard.global_sequences(2, 2, 4)
    p = shard.prompt_for(5, 8)
    assert p.dtype == np.uint32 and p.max() < shard.VOCAB_PROMPT
    assert np.array_equal(p, shard.prompt_for(5, 8))
