"""Data-parallel partitioning of independent request streams (one process per
GPU, no collective on the per-token path), checked on CPU: the partition
rules, and two gloo ranks that each compute their own shard and agree on the
whole without exchanging it, plus the bench's max-over-ranks timing."""

import os
import socket

import numpy as np
import pytest

from runtime import dispatch


def workload(n=64, seed=3, shared_fraction=0.25, prefix=16):
    """The multi-stream serving workload in miniature: prompt lengths U[8, 48], a quarter of
    the requests sharing one 16-token prefix."""
    rng = np.random.default_rng(seed)
    common = rng.integers(0, 151936, prefix).tolist()
    prompts = []
    for i in range(n):
        length = int(rng.integers(8, 49))
        ids = rng.integers(0, 151936, length).tolist()
        if i % int(1 / shared_fraction) == 0:
            ids = common + ids[: max(1, length - prefix)]
        prompts.append(ids)
    return prompts


def test_every_request_lands_on_exactly_one_rank():
    prompts = workload()
    for world in (1, 2, 4, 8):
        ranks = dispatch.assign_ranks(prompts, world, 16)
        assert len(ranks) == len(prompts)
        assert all(0 <= r < world for r in ranks)
        shards = [dispatch.shard(prompts, r, world, 16) for r in range(world)]
        merged = sorted(i for s in shards for i in s)
        assert merged == list(range(len(prompts)))


def test_shared_prefix_requests_stay_together():
    prompts = workload()
    ranks = dispatch.assign_ranks(prompts, 2, 16)
    shared = [i for i in range(len(prompts)) if i % 4 == 0]
    assert len({ranks[i] for i in shared}) == 1
    # a group heavier than one rank's share is cut into as few pieces as
    # fit the share (here: 16 of 64 requests, 8 ranks)
    ranks8 = dispatch.assign_ranks(prompts, 8, 16)
    total = sum(dispatch.request_load(p, 16) for p in prompts)
    group = sum(dispatch.request_load(prompts[i], 16) for i in shared)
    assert len({ranks8[i] for i in shared}) == -(-group // int(total / 8))
    # a prompt no longer than the prefix has nothing to reuse: its own group
    assert dispatch.prefix_key(prompts[0][:16], 16, 0) == ("single", 0)


def test_balance_is_within_one_group_of_even():
    prompts = workload(n=512)
    for world in (2, 4, 8):
        ranks = dispatch.assign_ranks(prompts, world, 16)
        loads = np.zeros(world)
        for i, r in enumerate(ranks):
            loads[r] += dispatch.request_load(prompts[i], 16)
        groups = {}
        for i, ids in enumerate(prompts):
            key = dispatch.prefix_key(ids, 16, i)
            groups[key] = groups.get(key, 0) + dispatch.request_load(ids, 16)
        # longest-first greedy: no rank exceeds the mean by more than the
        # largest group
        assert loads.max() <= loads.mean() + max(groups.values())


def test_invalid_arguments():
    with pytest.raises(ValueError):
        dispatch.assign_ranks([[1, 2]], 0, 4)
    with pytest.raises(ValueError):
        dispatch.assign_ranks([[1, 2], [3]], 2, [4])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import sys
    import torch.distributed as dist

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(repo, "hawkpoint-npu-llm_b200"))
    sys.path.insert(0, repo)
    from runtime import dispatch as d
    import bench

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        prompts = workload()
        mine = d.shard(prompts, rank, world, 16)
        load = sum(d.request_load(prompts[i], 16) for i in mine)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        bench.barrier(world)
        slowest = bench.max_over_ranks(float(load), world)
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(repr((mine, gathered, load, slowest)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_on_the_partition(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    port = _free_port()
    mp.start_processes(_rank_main, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    results = [eval((tmp_path / f"rank{r}.txt").read_text()) for r in range(world)]
    shards = [res[0] for res in results]
    for mine, gathered, load, slowest in results:
        assert gathered == shards          # each rank computed the same partition
        assert slowest == max(res[2] for res in results)
    merged = sorted(i for s in shards for i in s)
    assert merged == list(range(len(workload())))
