"""Rollout / learner overlap: one cohort of rollouts in flight while the learner updates on the previous one.

``one_batch_ahead`` keeps the contract of the reference's scheduler
(src/climbing_gym/rollout/overlap.py:8-34): exactly one cohort is outstanding, cohorts are consumed in
submission order, ``snapshot(version)`` runs on the calling thread and only after the previous collection has
drained, behaviour versions are 0, 0, 1, 2, ... (at most one update of lag), and the producer is drained
before an exception from either callback leaves the function.

``PolicyHandoff`` is the multi-GPU ``snapshot``: the trainer rank's packed bf16 weights are broadcast over
NCCL into every replica's existing buffers on a stream of their own, ordered after the learner's last
optimizer kernel by an event instead of a host synchronisation, so the transfer (2.34 GB for the 1.2B model)
starts the moment the update finishes and overlaps whatever the learner's host thread does next; the
collector's stream waits for the transfer's event before its first kernel. The reference is single-GPU and
copies on the same device (src/climbing_gym/inference/lfm25_engine.py:555-578).
"""
from __future__ import annotations

import queue
import threading
import time
from typing import Any, Callable

import torch


def one_batch_ahead(count: int, *, collect: Callable[[int, int], Any], snapshot: Callable[[int], None],
                    learn: Callable[[Any, int, float], None]) -> None:
    """Run ``count`` cohorts: ``collect(index, version)`` on a producer thread, ``learn(payload, index,
    cycle_start)`` and ``snapshot(version)`` on the calling thread, the next cohort collecting while the
    current one is learned from."""
    if type(count) is not int or count < 1:
        raise ValueError("count must be a positive integer")
    jobs: queue.Queue = queue.Queue()
    done: queue.Queue = queue.Queue()

    def producer():
        while True:
            job = jobs.get()
            if job is None:
                return
            index, version = job
            try:
                done.put((True, collect(index, version)))
            except BaseException as exc:  # handed to the consumer, which re-raises it
                done.put((False, exc))

    worker = threading.Thread(target=producer, name="native-rollout", daemon=True)
    worker.start()
    outstanding = 0
    try:
        started = time.perf_counter()
        snapshot(0)
        jobs.put((0, 0))
        outstanding = 1
        for index in range(count):
            cycle = started if index == 0 else time.perf_counter()
            ok, payload = done.get()
            outstanding = 0
            if not ok:
                raise payload
            if index + 1 < count:
                snapshot(index)  # the collection has drained: the inference copy may be overwritten
                jobs.put((index + 1, index))
                outstanding = 1
            learn(payload, index, cycle)
    finally:
        if outstanding:
            done.get()  # drain the cohort in flight before the caller tears anything down
        jobs.put(None)
        worker.join()


class PolicyHandoff:
    """``snapshot`` callback for ``one_batch_ahead`` over replicas: broadcast the trainer rank's packed
    weights into this replica's engine on a side stream.

    ``learner_stream`` is the stream the optimizer step runs on (the current stream by default); the
    broadcast is ordered after everything enqueued there so far. ``collector_ready()`` must be called on
    the collector's stream (or passed as ``collect``'s first action) before the engine generates."""

    def __init__(self, engine, *, src: int = 0, group=None, learner_stream=None):
        self.engine, self.src, self.group = engine, src, group
        self.device = engine.device
        self.on_gpu = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(device=self.device) if self.on_gpu else None
        self.learner_stream = learner_stream
        self.done = torch.cuda.Event() if self.on_gpu else None
        self.versions: list[int] = []
        self.bytes_moved = 0

    def __call__(self, version: int) -> None:
        from .replica import broadcast_policy_weights

        if self.on_gpu:
            learner = self.learner_stream or torch.cuda.current_stream(self.device)
            self.stream.wait_stream(learner)
            with torch.cuda.stream(self.stream):
                self.bytes_moved = broadcast_policy_weights(self.engine, src=self.src, group=self.group)
                self.done.record(self.stream)
        else:
            self.bytes_moved = broadcast_policy_weights(self.engine, src=self.src, group=self.group)
        self.versions.append(version)

    def collector_ready(self) -> None:
        """Make the current stream wait for the last broadcast (no host synchronisation)."""
        if self.on_gpu:
            torch.cuda.current_stream(self.device).wait_event(self.done)
