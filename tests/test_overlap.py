"""Rollout / learner overlap on CPU: cohort ordering, snapshot timing and failure draining of
``one_batch_ahead`` (the behaviours the reference pins in tests/test_rollout_overlap.py), and the weight
hand-off between two gloo ranks driven through it."""
import os
import socket
from threading import Event, Lock

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from climbing_gym_b200.overlap import PolicyHandoff, one_batch_ahead


def test_cohorts_stay_ordered_and_snapshots_wait_for_the_drained_collection():
    lock = Lock()
    state = {"active": False, "policy": 0, "engine": None}
    started = [Event() for _ in range(4)]
    consumed, snapshots = [], []

    def snapshot(version):
        with lock:
            assert not state["active"], "the inference copy is overwritten only while no collection runs"
            assert version == state["policy"]
            state["engine"] = version
            snapshots.append(version)

    def collect(index, version):
        with lock:
            assert not state["active"] and state["engine"] == version
            state["active"] = True
        started[index].set()
        with lock:
            assert state["engine"] == version
            state["active"] = False
        return index, version

    def learn(payload, index, cycle):
        if index + 1 < 4:
            assert started[index + 1].wait(timeout=5), "the next cohort collects while this one is learned from"
        assert payload[0] == index and index - payload[1] in (0, 1) and cycle > 0
        consumed.append(payload)
        state["policy"] += 1

    one_batch_ahead(4, collect=collect, snapshot=snapshot, learn=learn)
    assert consumed == [(0, 0), (1, 0), (2, 1), (3, 2)]
    assert snapshots == [0, 0, 1, 2] and state["policy"] == 4


def test_a_failed_collection_stops_learning_at_the_last_complete_cohort():
    learned = []

    def collect(index, version):
        if index == 1:
            raise RuntimeError("collector failed")
        return index

    with pytest.raises(RuntimeError, match="collector failed"):
        one_batch_ahead(3, collect=collect, snapshot=lambda version: None,
                        learn=lambda payload, index, cycle: learned.append(payload))
    assert learned == [0]


def test_a_failed_learner_drains_the_cohort_in_flight():
    next_started, next_finished = Event(), Event()

    def collect(index, version):
        if index == 1:
            next_started.set()
            next_finished.set()
        return index

    def learn(payload, index, cycle):
        assert next_started.wait(timeout=5)
        raise RuntimeError("learner failed")

    with pytest.raises(RuntimeError, match="learner failed"):
        one_batch_ahead(3, collect=collect, snapshot=lambda version: None, learn=learn)
    assert next_finished.is_set()


@pytest.mark.parametrize("count", [0, -1, True, 1.5])
def test_invalid_cohort_counts(count):
    with pytest.raises(ValueError):
        one_batch_ahead(count, collect=None, snapshot=None, learn=None)


class _Weights:
    def __init__(self, tensors):
        self._tensors = tensors

    def tensors(self):
        return self._tensors


class _Engine:
    def __init__(self, tensors):
        self.weights, self.policy_version, self.device = _Weights(tensors), 0, torch.device("cpu")

    def weights_updated(self):
        self.policy_version += 1


def _worker(rank: int, world: int, port: int, out_dir: str):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        weights = [torch.zeros(2048, 1100, dtype=torch.bfloat16), torch.zeros(64)]
        engine = _Engine(weights)
        handoff = PolicyHandoff(engine, src=0)
        seen = []

        def collect(index, version):
            handoff.collector_ready()
            seen.append((index, version, float(weights[1][0])))  # the replica generates with what was handed over
            return index

        def learn(payload, index, cycle):
            if rank == 0:  # the trainer rank's update: every replica must see it one cohort later
                for t in weights:
                    t.fill_(index + 1)

        one_batch_ahead(3, collect=collect, snapshot=handoff, learn=learn)
        assert handoff.versions == [0, 0, 1] and engine.policy_version == 3
        assert handoff.bytes_moved == sum(t.numel() * t.element_size() for t in weights)
        # cohort 0 and 1 run on the initial weights, cohort 2 on the first update (the learner of cohort 1
        # may or may not have finished when cohort 2 was handed its snapshot: lag of at most one update)
        assert [s[:2] for s in seen] == [(0, 0), (1, 0), (2, 1)]
        assert seen[0][2] == 0.0 and seen[2][2] in (1.0, 2.0)
        with open(os.path.join(out_dir, f"ok{rank}"), "w") as f:
            f.write("ok")
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_hand_weights_over_between_cohorts(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    assert (tmp_path / "ok0").exists() and (tmp_path / "ok1").exists()
