"""Multi-replica host logic on CPU: two gloo ranks shard requests, broadcast weights in place and
gather results (the N > 1 path of the engine has no other exchange)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from climbing_gym_b200 import replica


def test_round_robin_sharding_covers_every_item_once():
    items = [f"req{i}" for i in range(11)]
    shards = [replica.shard_round_robin(items, r, 4) for r in range(4)]
    assert sorted(sum(shards, [])) == sorted(items)
    assert shards[1] == ["req1", "req5", "req9"]
    assert replica.shard_indices(5, 1, 2) == [1, 3]
    with pytest.raises(ValueError):
        replica.shard_round_robin(items, 4, 4)


def test_gather_results_single_rank_is_identity():
    assert replica.gather_results([1, 2, 3], 3, 0, 1) == [1, 2, 3]


class _FakeWeights:
    def __init__(self, tensors):
        self._tensors = tensors

    def tensors(self):
        return self._tensors


class _FakeEngine:
    def __init__(self, tensors):
        self.weights = _FakeWeights(tensors)
        self.policy_version = 0

    def weights_updated(self):
        self.policy_version += 1


def _make_weights(rank: int):
    gen = torch.Generator().manual_seed(100 + rank)
    return [
        torch.randn(2048, 1100, generator=gen).to(torch.bfloat16),  # > 8 MiB: broadcast in place
        torch.randn(64, generator=gen).to(torch.bfloat16),          # small: bucketed
        torch.randn(16, 3, generator=gen).to(torch.bfloat16),
        torch.randint(0, 255, (1000,), generator=gen, dtype=torch.uint8),
        torch.randn(7, generator=gen),
    ]


def _worker(rank: int, world: int, port: int, out_dir: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        weights = _make_weights(rank)
        addresses = [t.data_ptr() for t in weights]
        engine = _FakeEngine(weights)
        # tiny bucket so that the small tensors take more than one bucket
        moved = replica.broadcast_tensors(weights, src=0, bucket_bytes=256)
        assert moved == sum(t.numel() * t.element_size() for t in weights)
        moved_again = replica.broadcast_policy_weights(engine, src=0)
        assert moved_again == moved and engine.policy_version == 1
        assert [t.data_ptr() for t in weights] == addresses, "buffers must be updated in place"
        want = _make_weights(0)
        for got, ref in zip(weights, want):
            assert torch.equal(got, ref), (rank, got.dtype, got.shape)

        requests = list(range(9))
        mine = replica.shard_round_robin(requests, rank, world)
        local = [{"request": r, "tokens": [r, r + 1], "rank": rank} for r in mine]
        merged = replica.gather_results(local, len(requests), rank, world)
        if rank == 0:
            assert [m["request"] for m in merged] == requests
            assert [m["rank"] for m in merged] == [r % world for r in requests]
        else:
            assert merged is None
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_broadcast_in_place_and_gather(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()
