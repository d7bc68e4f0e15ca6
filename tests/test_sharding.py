"""Request sharding for multi-GPU decode, and the cross-rank maximum, on CPU (gloo)."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from qwenquest_b200.sharding import box_totals, max_over_ranks, request_layer_bytes, shard_requests

# benchmark config 2's shape: long ragged requests and two dense-fallback ones
RAGGED = [70001, 98765, 131000, 65601, 120003, 77777, 101010, 88888, 66666, 130001, 99999, 75000,
          110000, 123456, 1500, 2046]


def test_request_bytes_match_the_roofline_unit():
    # 4,233,216 + 2048 C for a long request, 30,720 + 2052 L for a dense one
    assert request_layer_bytes(32769) == 4_233_216 + 2048 * 512
    assert request_layer_bytes(1500) == 30_720 + 2052 * 1500


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("balance", [False, True])
def test_shards_partition_the_batch(world, balance):
    shards = [shard_requests(RAGGED, r, world, balance=balance) for r in range(world)]
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(RAGGED)))
    for s in shards:
        assert s == sorted(s)
    if not balance:
        sizes = [len(s) for s in shards]
        assert max(sizes) - min(sizes) <= 1
        assert all(s == list(range(s[0], s[0] + len(s))) for s in shards if s)


def test_balanced_shards_even_out_the_bytes():
    world = 4
    loads = [sum(request_layer_bytes(RAGGED[i]) for i in shard_requests(RAGGED, r, world, balance=True))
             for r in range(world)]
    contiguous = [sum(request_layer_bytes(RAGGED[i]) for i in shard_requests(RAGGED, r, world))
                  for r in range(world)]
    assert max(loads) / (sum(loads) / world) < 1.15
    assert max(loads) <= max(contiguous)


def test_rank_out_of_range_is_rejected():
    with pytest.raises(ValueError):
        shard_requests(RAGGED, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        mine = shard_requests(RAGGED, rank, world, balance=True)
        # each rank "times" its shard by its bytes; the box reports the slowest rank
        local = [float(sum(request_layer_bytes(RAGGED[i]) for i in mine)), float(rank)]
        slowest = max_over_ranks(local)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        if rank == 0:
            torch.save({"slowest": slowest, "shards": gathered}, out)
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_and_take_the_slowest(tmp_path):
    world = 2
    out = str(tmp_path / "result.pt")
    mp.spawn(_rank_main, args=(world, _free_port(), out), nprocs=world, join=True)
    res = torch.load(out)
    shards = res["shards"]
    assert sorted(i for s in shards for i in s) == list(range(len(RAGGED)))
    loads = [sum(request_layer_bytes(RAGGED[i]) for i in s) for s in shards]
    assert res["slowest"] == [float(max(loads)), float(world - 1)]


def _box_rank_main(rank: int, world: int, port: int, out: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        # config 4's box: each rank decodes its shard in its own time with its own token count
        res = box_totals([10.0 + rank, 3.0 - rank], [100.0 * (rank + 1)])
        if rank == 0:
            torch.save(res, out)
    finally:
        dist.destroy_process_group()


def test_two_ranks_box_totals(tmp_path):
    out = str(tmp_path / "box.pt")
    mp.spawn(_box_rank_main, args=(2, _free_port(), out), nprocs=2, join=True)
    slowest, totals = torch.load(out)
    assert slowest == [11.0, 3.0] and totals == [300.0]


def test_max_over_ranks_without_a_group_is_the_identity():
    assert max_over_ranks([1.5, -2.0]) == [1.5, -2.0]
