#!/usr/bin/env python
"""Rollout throughput of the B200 engine on the headline configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]
    torchrun --nnodes=1 --nproc-per-node N ... bench.py --gpus N ...      (one rank per GPU)

Default workload "fp8-queue2048x256" (the FP8 rollout configuration): LFM2.5-1.2B architecture, random-init
bf16 weights with FP8 W8A8 MLP and e4m3 KV cache, a queue of 2048 requests (prompt lengths lognormal with
median 400 clipped to [32, 4096], output lengths geometric with mean 1500 capped at 4096, enforced as
per-request limits) served by a generation session of 256 live slots, max_model_len 8192, prefill budget
4096 tokens. The session runs continuously; requests are admitted in queue order (the queue wraps) into
slots as they free up. One STEP is a fixed slice of that schedule: 8 scheduling windows, each
``poll(32)`` -> read the finished requests' tokens and log-probs -> release -> admit the next queued
requests into the freed slots (256 decode steps per bench step plus the prefill of the admitted prompts).
Before the warm-up the session is run for 64 untimed windows so that the live set has the age mix of a
session in the middle of its queue (a session that has just been filled has short contexts and no
turnover). ``value`` = tokens generated in the K timed steps / their device time.

Other workloads: "bf16-b64x512" (64 prompts x 512 sampled tokens through ``engine.generate``; one step is
one generate call), "rl-group256x16" (32 prompts x 16 samples per GPU sharing their prompt pages, then
``score_completions`` over every completed sequence; one step is one rollout + scoring, with the NCCL weight
broadcast ahead of it when N > 1), "bf16-long32x1024" / "fp8kv-long32x1024" (long-context stress), "tiny"
and "tiny-queue" (plumbing checks).

Prints ONE JSON line. ``value`` times the steps with prompts resident in HBM; ``e2e`` repeats them with
prompts in pinned host memory (copied to the device inside the timed region) and results read back to the
host. ``roofline`` is the decode step graph: algorithmic bytes (weights + KV history per step) over its
CUDA-event duration against the measured HBM copy bandwidth. ``cpu_baseline`` / ``--impl reference`` time
the reference's own CPU engine (staged by oracle/build_ref.py; the numpy port when it is not staged) on a
bounded sample of the workload. ``--impl reference --reference-device cuda`` runs the reference's own CUDA
engine (Triton + FlashAttention + CUDA graphs) on the same workload on the GPU, the comparator the rollout
target names.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "generated tokens/s"
UNIT = "tokens/s"
DEFAULT_WORKLOAD = "fp8-queue2048x256"

WORKLOADS = {
    # name: (model, batch, prompt_low, prompt_high, new_tokens, graph options)
    "bf16-b64x512": ("1p2b", 64, 64, 1024, 512, {}),
    "fp8-b64x512": ("1p2b", 64, 64, 1024, 512, {"fp8_mlp": True, "fp8_kv": True}),
    "tiny": ("tiny", 8, 8, 64, 32, {}),
    # long-context stress: 32 sequences, prompts of 16-30 K tokens prefilled in 4096-token chunks
    "bf16-long32x1024": ("1p2b", 32, 16384, 30720, 1024, {}),
    "fp8kv-long32x1024": ("1p2b", 32, 16384, 30720, 1024, {"fp8_kv": True}),
}

# DRAM bytes of ONE decode-step replay (dram__bytes_read.sum + dram__bytes_write.sum over its kernels, one
# ncu capture on a small case of the same step) divided by the step's algorithmic bytes at the captured
# sequence lengths. Both grow with the same two terms (weights once, KV history once), so `roofline.traffic`
# scales the full-size algorithmic bytes by this ratio.
DRAM_TRAFFIC_RATIO = {"bf16-b64x512": 1.058, "fp8-queue2048x256": 1.143}

# Continuous batching through a generation session: a queue of requests served by a fixed number of live
# slots; a finished request's slot is refilled from the queue at the next scheduling window.
QUEUE_WORKLOADS = {
    "fp8-queue2048x256": dict(model="1p2b", options={"fp8_mlp": True, "fp8_kv": True}, requests=2048, slots=256,
                              max_model_len=8192, cap=4096, mean_out=1500.0, median=400.0, sigma=0.8, clip=(32, 4096),
                              poll=32, windows_per_step=8, preroll_windows=64),
    "tiny-queue": dict(model="tiny", options={}, requests=24, slots=8, max_model_len=256, cap=32, mean_out=12.0,
                       median=24.0, sigma=0.5, clip=(4, 96), poll=8, windows_per_step=2, preroll_windows=2),
}

# RL group rollout: every prompt is sampled `samples` times; the samples share the prompt's KV pages. After
# the rollout every completed sequence is scored (packed varlen prefill + chunked head).
GROUP_WORKLOADS = {
    "rl-group256x16": dict(model="1p2b", options={"fp8_mlp": True, "fp8_kv": True}, prompts_per_gpu=32, samples=16,
                           prompt_range=(128, 768), mean_out=1200.0, cap=4096, max_model_len=4992, poll=32),
    "tiny-group": dict(model="tiny", options={}, prompts_per_gpu=3, samples=4, prompt_range=(8, 40), mean_out=10.0,
                       cap=24, max_model_len=128, poll=8),
}


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured (MEASURED_PEAKS.json)"
    return 6650.0, "fallback (earlier measurement on this pool)"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index, self.lines, self.proc = gpu_index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu_index)], stdout=subprocess.PIPE, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *_):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, sm_max, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(sm_max) if sm_max else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---- the two implementations behind one small adapter --------------------------------------------------
class Impl:
    """What the workloads need from an engine package: the engine over synthetic weights, its sampling
    configuration class and its prompt flattener. ``ours`` is climbing_gym_b200; ``reference`` is the
    reference's own package staged under oracle/_ref (same public API: that is the drop-in contract)."""

    def __init__(self, name: str):
        self.name = name
        if name == "ours":
            from climbing_gym_b200.config import LFM25SamplingConfig
            from climbing_gym_b200.engine import LFM25Engine, flatten_token_batches
        else:
            from oracle.build_ref import staged_path

            staged = staged_path()
            if staged is None:
                raise RuntimeError("the reference is not staged: run `python oracle/build_ref.py --reference <checkout>`")
            if str(staged) not in sys.path:
                sys.path.insert(0, str(staged))
            from climbing_gym.inference.lfm25_engine import LFM25Engine, LFM25SamplingConfig, flatten_token_batches
        self.Engine, self.Sampling, self.flatten = LFM25Engine, LFM25SamplingConfig, flatten_token_batches

    def build(self, model: str, device, options: dict | None, max_model_len: int, seed: int = 0, dtype=None):
        """Engine over seeded random-init weights of the named architecture; ``options`` are the
        enable_cuda_graphs options (None: leave the engine eager, the reference's CPU path)."""
        import torch
        from climbing_gym_b200 import synthetic

        cfg = synthetic.tiny_config() if model == "tiny" else synthetic.lfm25_1p2b_config()
        dtype = dtype or torch.bfloat16
        if device.type == "cuda":
            state = synthetic.make_state_dict_on_device(cfg, seed, device, dtype)
        else:
            state = {k: torch.from_numpy(v).to(dtype) for k, v in synthetic.make_state_dict_streams(cfg, seed).items()}
        if self.name == "ours":
            engine = self.Engine.from_state_dict(cfg, state, device=device, dtype=dtype, max_model_len=max_model_len)
        else:
            from climbing_gym.inference.lfm25_engine import LFM25PackedWeights
            from climbing_gym.models.lfm2 import LFM2Config

            overrides = {} if device.type == "cuda" else {"attn_backend": "eager"}
            rcfg = LFM2Config.from_dict({**cfg.to_dict(), **overrides})
            weights = LFM25PackedWeights.from_state_dict(rcfg, state, device=device, dtype=dtype)
            engine = self.Engine(weights, max_model_len=max_model_len)
        del state
        if options is not None:
            engine.enable_cuda_graphs(max_graphs=1, **options)
        return engine, cfg


def weight_bytes(engine, options: dict) -> int:
    """Bytes of weights one decode step streams (tied embedding counted once, as the LM head)."""
    total = 0
    fp8 = bool(options.get("fp8_mlp"))
    w = engine.weights
    total += w.lm_head_weight.numel() * w.lm_head_weight.element_size()
    total += w.embedding_norm_weight.numel() * 2
    for layer in w.layers:
        for t in (layer.w13_weight, layer.w2_weight):
            total += t.numel() * (1 if fp8 else t.element_size()) + (t.size(0) * 4 if fp8 else 0)
        total += (layer.operator_norm_weight.numel() + layer.ffn_norm_weight.numel()) * 2
        if layer.attention is not None:
            a = layer.attention
            total += sum(t.numel() * t.element_size() for t in (a.qkv_weight, a.out_weight, a.q_norm_weight, a.k_norm_weight))
        else:
            c = layer.conv
            total += sum(t.numel() * t.element_size() for t in (c.in_weight, c.conv_weight, c.out_weight))
    return total


def kv_bytes_per_token(engine, cfg, options: dict) -> int:
    fp8_kv = bool(options.get("fp8_kv"))
    return engine.weights.num_attention_layers * 2 * cfg.num_key_value_heads * (
        cfg.head_dim * (1 if fp8_kv else 2) + (4 if fp8_kv else 0))


class Ranks:
    """Rank bookkeeping, barrier + synchronize brackets and max-over-ranks device timing."""

    def __init__(self, init_nccl: bool = True):
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.rank, self.world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
        self.local_rank = int(os.environ.get("LOCAL_RANK", 0))
        if not torch.cuda.is_available():
            raise RuntimeError("bench.py needs a CUDA device: the engine has no CPU path")
        torch.cuda.set_device(self.local_rank)
        self.device = torch.device("cuda", self.local_rank)
        if self.world > 1 and init_nccl:
            dist.init_process_group("nccl", device_id=self.device)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def timed(self, fn, steps: int):
        """K calls of fn between barrier + synchronize brackets; CUDA-event time, max over ranks.
        Returns (milliseconds, list of fn's return values)."""
        torch = self.torch
        self.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        results = [fn() for _ in range(steps)]
        end.record()
        self.barrier()
        ms = start.elapsed_time(end)
        if self.world > 1:
            t = torch.tensor([ms], device=self.device)
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, results

    def total(self, value: float) -> float:
        """Sum of a per-rank quantity over all ranks (whole-job aggregate)."""
        if self.world == 1:
            return float(value)
        t = self.torch.tensor([float(value)], device=self.device, dtype=self.torch.float64)
        self.dist.all_reduce(t)
        return float(t.item())

    def finish(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def broadcast_timed(ranks: Ranks, engine) -> dict | None:
    """Policy-weight broadcast from rank 0: the first call (includes NCCL's lazy communicator set-up) and
    the median of three more (what precedes every later rollout)."""
    if ranks.world == 1:
        return None
    from climbing_gym_b200.replica import broadcast_policy_weights

    torch = ranks.torch
    times, moved = [], 0
    for _ in range(4):
        ranks.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        moved = broadcast_policy_weights(engine, src=0)
        end.record()
        ranks.barrier()
        t = torch.tensor([start.elapsed_time(end)], device=ranks.device)
        ranks.dist.all_reduce(t, op=ranks.dist.ReduceOp.MAX)
        times.append(float(t.item()))
    steady = statistics.median(times[1:])
    return {"first_ms": round(times[0], 2), "ms": round(steady, 3), "bytes": int(moved),
            "gb_per_s": round(moved / steady / 1e6, 1), "note": "ms = median of 3 after the first call (max over ranks)"}


# ---- generate-based workloads ------------------------------------------------------------------------
def run_generate(args) -> dict:
    import torch
    from climbing_gym_b200 import _native as nv, synthetic

    ranks = Ranks()
    device, world, rank = ranks.device, ranks.world, ranks.rank
    impl = Impl("ours" if args.impl == "ours" else "reference")
    model, batch, low, high, new_tokens, options = WORKLOADS[args.workload]
    batch = args.batch or batch
    new_tokens = args.new_tokens or new_tokens
    engine, cfg = impl.build(model, device, options, max_model_len=high + new_tokens + 64)
    broadcast = broadcast_timed(ranks, engine) if impl.name == "ours" else None
    prompts = synthetic.uniform_prompts(batch, low, high, cfg.vocab_size, seed=1000 + rank)
    flat_host = impl.flatten(prompts, device="cpu")
    ids_pinned, cu_pinned = flat_host[0].pin_memory(), flat_host[1].pin_memory()
    ids_dev, cu_dev = ids_pinned.to(device), cu_pinned.to(device)
    max_len = flat_host[2]
    sampling = impl.Sampling(temperature=1.0, top_k=0, top_p=1.0, max_new_tokens=new_tokens, seed=0,
                             ignore_eos=True, return_logprobs=True)
    decoder = engine._cuda_decoder
    outputs = {}

    def step_resident():
        outputs["last"] = engine.generate(ids_dev, cu_dev, max_len, repeats=1, sampling=sampling)

    def step_e2e():
        out = engine.generate(ids_pinned.to(device, non_blocking=True), cu_pinned.to(device, non_blocking=True),
                              max_len, repeats=1, sampling=sampling)
        outputs["host"] = (out.token_ids.cpu(), out.logprobs.cpu(), out.lengths.cpu())

    for _ in range(args.warmup):
        step_resident()
    ours = impl.name == "ours"
    launches_before = nv.launch_count() if ours else 0
    if ours:
        decoder.profile_decode, decoder.decode_profile = True, []
    with ClockSampler(ranks.local_rank) as clocks:
        total_ms, _ = ranks.timed(step_resident, args.steps)
    launches = nv.launch_count() - launches_before if ours else None
    decode_ms = decode_replays = 0
    if ours:
        decoder.profile_decode = False
        decode_ms = sum(s.elapsed_time(e) for s, e, _ in decoder.decode_profile)
        decode_replays = sum(n for _, _, n in decoder.decode_profile)
    e2e_ms, _ = ranks.timed(step_e2e, args.steps)
    tokens_per_step = batch * new_tokens
    lengths = outputs["last"].lengths
    if int(lengths.sum()) != tokens_per_step or not bool(torch.isfinite(outputs["last"].logprobs).all()):
        raise RuntimeError("generate returned an incomplete budget or non-finite log-probs")
    value = world * tokens_per_step * args.steps / (total_ms / 1e3)
    e2e_value = world * tokens_per_step * args.steps / (e2e_ms / 1e3)

    # decode roofline: weights + KV history per step (algorithmic bytes), HBM-bound
    roofline = None
    if decode_replays:
        w_bytes = weight_bytes(engine, options)
        kv_tok = kv_bytes_per_token(engine, cfg, options)
        prompt_total = sum(len(p) for p in prompts)
        # replay j (1-based) reads, per row, its prompt plus j generated tokens
        bytes_per_replay = w_bytes + kv_tok * (prompt_total + batch * new_tokens / 2.0)
        peak, peak_source = peaks()
        step_ms = decode_ms / decode_replays
        achieved = bytes_per_replay / (step_ms / 1e3) / 1e9
        ratio = DRAM_TRAFFIC_RATIO.get(args.workload) if not (args.batch or args.new_tokens) else None
        roofline = {"bound": "hbm", "kernel": "decode step graph (all kernels of one token step)",
                    "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "peak_source": peak_source, "traffic": int(ratio * bytes_per_replay) if ratio else None,
                    "traffic_source": ("ncu capture of one replay at short sequences, scaled by algorithmic bytes "
                                       f"(x{ratio})") if ratio else None,
                    "ms_per_launch": round(step_ms, 4),
                    "algorithmic_bytes_per_launch": int(bytes_per_replay), "launches_timed": decode_replays,
                    "decode_share_of_step": round(decode_ms / total_ms, 4)}
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if not options else "bf16+e4m3", "data": "synthetic",
        "config": {"workload": args.workload, "model": model_name(model),
                   "batch_per_gpu": batch, "prompt_lengths": f"uniform[{low},{high}]", "new_tokens": new_tokens,
                   "step": "one engine.generate call over the batch (packed prefill, then new_tokens decode steps)",
                   "sampling": "temperature 1, full support, ignore_eos", "replicas": world,
                   "l2": "working set per decode step (weights + KV) is far larger than the 126 MB L2"},
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": int(ids_pinned.numel() * 8 + cu_pinned.numel() * 4),
                "d2h_bytes_per_step": int(tokens_per_step * 12 + batch * 4), "ms_per_step": round(e2e_ms / args.steps, 3)},
        "gpu_launches": int(launches) if launches is not None else None, "clocks": clocks.summary(), "roofline": roofline,
    }
    if broadcast is not None:
        result["weight_broadcast"] = broadcast
    if not ours:
        result["impl"] = "reference-cuda"
    if world == 1 and ours and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.workload, seconds_budget=args.cpu_seconds)
    ranks.finish()
    return result if rank == 0 else {}


def model_name(model: str) -> str:
    return "LFM2.5-1.2B architecture, random init" if model == "1p2b" else "tiny hybrid"


# ---- continuous batching ------------------------------------------------------------------------------
def queue_requests(name: str, vocab: int, seed: int):
    """Seeded synthetic requests of a queue workload: prompt lengths lognormal around the median and
    clipped, output lengths geometric with the given mean and capped (a per-request length limit
    stands in for the EOS hazard), prompt + output within max_model_len."""
    import numpy as np

    w = QUEUE_WORKLOADS[name]
    rng = np.random.default_rng(seed)
    low, high = w["clip"]
    prompt_lens = np.clip(np.rint(rng.lognormal(np.log(w["median"]), w["sigma"], w["requests"])), low, high).astype(np.int64)
    limits = np.minimum(rng.geometric(1.0 / w["mean_out"], w["requests"]), w["cap"]).astype(np.int64)
    limits = np.maximum(1, np.minimum(limits, w["max_model_len"] - prompt_lens - 1))
    prompts = [rng.integers(3, vocab, size=int(length)).tolist() for length in prompt_lens]
    return prompts, [int(v) for v in limits]


class QueueDriver:
    """Keeps a generation session's slots full from a (wrapping) request queue, one scheduling window at
    a time. Works with this package's session and with the reference's (same admit / poll / release API)."""

    def __init__(self, impl: Impl, session, prompts, limits, device, poll_steps: int, *, ours: bool):
        import torch

        self.torch, self.session, self.device, self.poll_steps, self.ours = torch, session, device, poll_steps, ours
        self.prompts = prompts
        self.samplings = [impl.Sampling(temperature=1.0, top_k=0, top_p=1.0, max_new_tokens=limit, seed=index,
                                        ignore_eos=True, return_logprobs=True) for index, limit in enumerate(limits)]
        self.pinned = [torch.tensor(p, dtype=torch.int64).pin_memory() for p in prompts]
        self.staged = [t.to(device) for t in self.pinned] if ours else None
        self.next_request = 0
        self.slots = session.batch_size
        self.live: dict[int, int] = {}      # slot -> request index
        self.delivered_tokens = 0
        self.delivered_requests = 0
        self.h2d_bytes = self.d2h_bytes = 0
        self.kv_token_steps = 0.0            # sum over decode steps of the live rows' attended tokens
        self.windows = 0

    def _admit(self, slots, host: bool):
        if not slots:
            return
        n = len(self.prompts)
        ids = [(self.next_request + i) % n for i in range(len(slots))]
        self.next_request += len(slots)
        prompts, samplings = [self.prompts[i] for i in ids], [self.samplings[i] for i in ids]
        if self.ours:
            if host:
                device_prompts = [self.pinned[i].to(self.device, non_blocking=True) for i in ids]
                self.h2d_bytes += sum(self.pinned[i].numel() * 8 for i in ids)
            else:
                device_prompts = [self.staged[i] for i in ids]
            self.session.admit(prompts, samplings, slots=slots, device_prompts=device_prompts)
        else:
            self.session.admit(prompts, samplings, slots=slots)  # flattens and copies the ids itself
            self.h2d_bytes += sum(len(p) * 8 for p in prompts)
        self.live.update(zip(slots, ids))

    def fill(self):
        self._admit([s for s in range(self.slots) if s not in self.live], host=False)

    def live_generated(self) -> int:
        """Tokens generated so far by the requests still in their slots."""
        if not self.live:
            return 0
        index = self.torch.tensor(sorted(self.live), device=self.device)
        return int(self.session.lengths[index].sum())

    def _context_tokens(self) -> float:
        index = self.torch.tensor(sorted(self.live), device=self.device)
        return float(self.session.entry.cache.seq_lens[index].sum())

    def window(self, host: bool, *, account_kv: bool = False):
        """poll -> deliver -> release -> refill. ``host``: admitted prompts come from pinned host memory."""
        before = self._context_tokens() + len(self.live) if account_kv else 0.0
        results = self.session.poll(steps=self.poll_steps)
        if account_kv:
            # every live row attends to its context (+ the token it appends) each step; contexts grow by one
            # per step until a row finishes, so the window's sum is the trapezoid between its two ends
            after = self._context_tokens() + len(self.live)
            self.kv_token_steps += self.poll_steps * (before + after) / 2.0
        freed = []
        for result in results:
            n = len(result.token_ids)
            if result.logprobs is None or not all(math.isfinite(v) for v in result.logprobs):
                raise RuntimeError("session returned no or non-finite log-probs")
            self.delivered_tokens += n
            self.delivered_requests += 1
            self.d2h_bytes += n * 12 + 4
            freed.append(result.handle.slot)
            self.session.release(result.handle)
            del self.live[result.handle.slot]
        self.d2h_bytes += self.slots  # the per-poll read of the finish reasons
        self._admit(sorted(freed), host)
        self.windows += 1

    def generated_total(self) -> int:
        return self.delivered_tokens + self.live_generated()


class DeviceQueueDriver(QueueDriver):
    """The same schedule with the slot turnover on the device: the host parks the next prompts of the queue
    (``session.enqueue``: prefill into a spare cache row) and reads results; finished requests leave their
    slots and parked ones enter them inside the decode graph, without a host release / admit between polls."""

    def _occupied(self):
        return self.session.state.queue["slot_requests"] >= 0

    def _park(self, host: bool):
        count = self.session.queue_space()
        if not count:
            return
        n = len(self.prompts)
        ids = [(self.next_request + i) % n for i in range(count)]
        self.next_request += count
        if host:
            device_prompts = [self.pinned[i].to(self.device, non_blocking=True) for i in ids]
            self.h2d_bytes += sum(self.pinned[i].numel() * 8 for i in ids)
        else:
            device_prompts = [self.staged[i] for i in ids]
        self.session.enqueue([self.prompts[i] for i in ids], [self.samplings[i] for i in ids],
                             device_prompts=device_prompts)

    def fill(self):
        self._park(host=False)
        self.session.poll(steps=1)  # the first turnover deals the parked prompts to the empty slots
        self._park(host=False)

    def live_generated(self) -> int:
        return int((self.session.lengths * self._occupied()).sum())

    def window(self, host: bool, *, account_kv: bool = False):
        # The decode steps are launched first; the host then parks the next prompts (metadata, copies and
        # prefill launches queue behind the steps while they run) and only then waits for the poll's reads,
        # which travel on a stream of their own. The queue holds a window's worth of parked prompts and more,
        # so parking with the previous poll's free count never starves the slot turnover.
        context, rows = self.session.last_context
        before = context + rows
        self.session.poll_begin(steps=self.poll_steps)
        self._park(host)
        results = self.session.poll_end()
        if account_kv:
            context, rows = self.session.last_context
            self.kv_token_steps += self.poll_steps * (before + context + rows) / 2.0
        for result in results:
            n = len(result.token_ids)
            if result.logprobs is None or not all(math.isfinite(v) for v in result.logprobs):
                raise RuntimeError("session returned no or non-finite log-probs")
            self.delivered_tokens += n
            self.delivered_requests += 1
            self.d2h_bytes += n * 12 + 4
        self.d2h_bytes += 4 + self.session.state.queue["result_capacity"]  # queue head + the result index
        self.windows += 1


def run_queue(args) -> dict:
    from climbing_gym_b200 import _native as nv

    ranks = Ranks()
    device, world, rank = ranks.device, ranks.world, ranks.rank
    ours = args.impl == "ours"
    impl = Impl("ours" if ours else "reference")
    w = QUEUE_WORKLOADS[args.workload]
    options, slots, poll_steps = w["options"], w["slots"], w["poll"]
    windows_per_step, preroll = w["windows_per_step"], w["preroll_windows"]
    engine, cfg = impl.build(w["model"], device, options, max_model_len=w["max_model_len"])
    broadcast = broadcast_timed(ranks, engine) if ours else None
    prompts, limits = queue_requests(args.workload, cfg.vocab_size, seed=2000 + rank)
    on_device = ours and args.scheduler == "device"
    if on_device:
        session = engine.generation_session(max_batch_size=slots, max_new_tokens=w["cap"], profile_timings=True,
                                            queue_capacity=slots)
        driver = DeviceQueueDriver(impl, session, prompts, limits, device, poll_steps, ours=True)
    else:
        session = engine.generation_session(max_batch_size=slots, max_new_tokens=w["cap"], profile_timings=True)
        driver = QueueDriver(impl, session, prompts, limits, device, poll_steps, ours=ours)
    driver.fill()
    for _ in range(preroll):
        driver.window(host=False)

    def step(host: bool, account_kv: bool = False):
        start = driver.generated_total()
        for _ in range(windows_per_step):
            driver.window(host, account_kv=account_kv)
        return driver.generated_total() - start

    for _ in range(args.warmup):
        step(False)
    launches_before = nv.launch_count() if ours else 0
    timing_before = session.timing_stats()
    with ClockSampler(ranks.local_rank) as clocks:
        total_ms, generated = ranks.timed(lambda: step(False, account_kv=ours), args.steps)
    timing_after = session.timing_stats()
    launches = nv.launch_count() - launches_before if ours else None
    kv_token_steps = driver.kv_token_steps
    driver.h2d_bytes = driver.d2h_bytes = 0
    e2e_ms, generated_e2e = ranks.timed(lambda: step(True), args.steps)
    h2d, d2h = driver.h2d_bytes / args.steps, driver.d2h_bytes / args.steps
    stats = dict(session.stats)
    session.close()
    value = ranks.total(sum(generated)) / (total_ms / 1e3)
    e2e_value = ranks.total(sum(generated_e2e)) / (e2e_ms / 1e3)

    replays = args.steps * windows_per_step * poll_steps
    decode_s = timing_after.get("decode_gpu_seconds", 0.0) - timing_before.get("decode_gpu_seconds", 0.0)
    prefill_s = timing_after.get("prefill_gpu_seconds", 0.0) - timing_before.get("prefill_gpu_seconds", 0.0)
    roofline = None
    if ours and decode_s > 0:
        # decode roofline: every replay streams the weights once and each live row's KV history once
        w_bytes = weight_bytes(engine, options)
        kv_tok = kv_bytes_per_token(engine, cfg, options)
        bytes_per_replay = w_bytes + kv_tok * kv_token_steps / replays
        peak, peak_source = peaks()
        achieved = bytes_per_replay * replays / decode_s / 1e9
        ratio = DRAM_TRAFFIC_RATIO.get(args.workload)
        roofline = {"bound": "hbm", "kernel": f"decode step graph at {slots} slots (all kernels of one token step)",
                    "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                    "peak_source": peak_source, "traffic": int(ratio * bytes_per_replay) if ratio else None,
                    "traffic_source": ("ncu capture of one replay of the same step on a small case, scaled by "
                                       f"algorithmic bytes (x{ratio})") if ratio else None,
                    "ms_per_launch": round(decode_s * 1e3 / replays, 4),
                    "algorithmic_bytes_per_launch": int(bytes_per_replay), "launches_timed": int(replays),
                    "mean_context_tokens_per_row": round(kv_token_steps / replays / slots, 1),
                    "decode_share_of_step": round(decode_s * 1e3 / total_ms, 4),
                    "prefill_share_of_step": round(prefill_s * 1e3 / total_ms, 4)}
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16+e4m3" if options else "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "model": model_name(w["model"]),
                   "requests_per_gpu": w["requests"], "live_slots": slots, "max_model_len": w["max_model_len"],
                   "prompt_lengths": f"lognormal(median {w['median']:g}, sigma {w['sigma']:g}) clipped to {list(w['clip'])}",
                   "output_lengths": f"geometric(mean {w['mean_out']:g}) capped at {w['cap']}, enforced as per-request limits",
                   "step": f"{windows_per_step} scheduling windows of a continuously running session: poll({poll_steps}) -> "
                           "deliver finished requests -> release -> admit the next queued requests into the freed slots "
                           f"({windows_per_step * poll_steps} decode steps + the admitted prompts' prefill)",
                   "scheduler": ("device: finished requests are evicted and parked prompts admitted inside the decode "
                                 "graph; the host launches a window's steps, parks the next prompts behind them and reads results "
                                 "once per window on a stream of its own"
                                 if on_device else "host: release and admit from Python at every window"),
                   "preroll": f"{preroll} untimed windows before the warm-up (age mix of a session in mid-queue)",
                   "options": options, "sampling": "temperature 1, full support", "replicas": world,
                   "tokens_per_step": round(sum(generated) / args.steps, 1),
                   "l2": "working set per decode step (weights + KV) is far larger than the 126 MB L2"},
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "ms_per_step": round(e2e_ms / args.steps, 3)},
        "gpu_launches": int(launches) if launches is not None else None, "clocks": clocks.summary(), "roofline": roofline,
        "session": {"delivered_requests": driver.delivered_requests, "slot_refills": stats.get("slot_refills"),
                    "decode_batches": stats.get("decode_batches")},
    }
    if broadcast is not None:
        result["weight_broadcast"] = broadcast
    if not ours:
        result["impl"] = "reference-cuda"
    if world == 1 and ours and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(args.workload, seconds_budget=args.cpu_seconds)
    ranks.finish()
    return result if rank == 0 else {}


# ---- RL group rollout + scoring -------------------------------------------------------------------------
def run_group(args) -> dict:
    import numpy as np
    from climbing_gym_b200 import _native as nv, synthetic
    from climbing_gym_b200.replica import broadcast_policy_weights

    ranks = Ranks()
    device, world, rank = ranks.device, ranks.world, ranks.rank
    impl = Impl("ours")
    w = GROUP_WORKLOADS[args.workload]
    options, samples, n_prompts = w["options"], w["samples"], w["prompts_per_gpu"]
    slots = n_prompts * samples
    engine, cfg = impl.build(w["model"], device, options, max_model_len=w["max_model_len"])
    engine._cuda_decoder.snapshot_rows = n_prompts
    broadcast = broadcast_timed(ranks, engine)
    low, high = w["prompt_range"]
    prompts = synthetic.uniform_prompts(n_prompts, low, high, cfg.vocab_size, seed=3000 + rank)
    rng = np.random.default_rng(4000 + rank)
    limits = np.minimum(rng.geometric(1.0 / w["mean_out"], slots), w["cap"]).astype(int).tolist()
    phases = {"rollout_ms": 0.0, "scoring_ms": 0.0, "broadcast_ms": 0.0}
    torch = ranks.torch

    def step():
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        marks[0].record()
        if world > 1:
            broadcast_policy_weights(engine, src=0)
        marks[1].record()
        completions: list = [None] * slots
        with engine.generation_session(max_batch_size=slots, max_new_tokens=w["cap"]) as session:
            request_of = {}
            for p, prompt in enumerate(prompts):
                snapshot = session.prefill_snapshot(prompt)
                group = [impl.Sampling(temperature=1.0, max_new_tokens=limits[p * samples + s], seed=p * samples + s,
                                       ignore_eos=True, return_logprobs=True) for s in range(samples)]
                got = session.fork(snapshot, group)
                request_of.update({slot: p * samples + s for s, slot in enumerate(got)})
                session.release_snapshot(snapshot)
            while request_of:
                for result in session.poll(steps=w["poll"]):
                    completions[request_of.pop(result.handle.slot)] = list(result.token_ids)
                    session.release(result.handle)
        marks[2].record()
        scores = engine.score_completions([prompts[i // samples] for i in range(slots)], completions,
                                          max_prefill_tokens=4096)
        marks[3].record()
        marks[3].synchronize()
        if not all(math.isfinite(v) for row in scores for v in row):
            raise RuntimeError("scoring returned non-finite log-probs")
        phases["broadcast_ms"] += marks[0].elapsed_time(marks[1])
        phases["rollout_ms"] += marks[1].elapsed_time(marks[2])
        phases["scoring_ms"] += marks[2].elapsed_time(marks[3])
        return sum(len(c) for c in completions)

    for _ in range(args.warmup):
        step()
    for key in phases:
        phases[key] = 0.0
    launches_before = nv.launch_count()
    with ClockSampler(ranks.local_rank) as clocks:
        total_ms, generated = ranks.timed(step, args.steps)
    launches = nv.launch_count() - launches_before
    value = ranks.total(sum(generated)) / (total_ms / 1e3)
    prompt_tokens = sum(len(p) for p in prompts)
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16+e4m3" if options else "bf16", "data": "synthetic",
        "config": {"workload": args.workload, "model": model_name(w["model"]), "prompts_per_gpu": n_prompts,
                   "samples_per_prompt": samples, "prompt_lengths": f"uniform[{low},{high}]",
                   "output_lengths": f"geometric(mean {w['mean_out']:g}) capped at {w['cap']}, enforced as per-request limits",
                   "step": "weight broadcast (N > 1), group rollout with shared prompt pages (one prefill per prompt, "
                           "its samples forked from the snapshot), then score_completions over every completed sequence",
                   "options": options, "replicas": world, "prompt_tokens": prompt_tokens,
                   "scored_tokens": int(sum(generated) / args.steps)},
        "phases_ms_per_step": {k: round(v / args.steps, 2) for k, v in phases.items()},
        "e2e": None, "gpu_launches": int(launches), "clocks": clocks.summary(), "roofline": None,
    }
    if broadcast is not None:
        result["weight_broadcast"] = broadcast
    ranks.finish()
    return result if rank == 0 else {}


# ---- the reference's CPU engine on a bounded sample -----------------------------------------------------
def cpu_sample(workload: str):
    """Bounded sample of a workload for the host cores: 8 requests, prompts cut to 96 tokens, 24 sampled
    tokens each (the model is the workload's own). Returns (model, prompts, new_tokens, description)."""
    from climbing_gym_b200 import synthetic

    if workload in QUEUE_WORKLOADS:
        model = QUEUE_WORKLOADS[workload]["model"]
        vocab = 4096 if model == "tiny" else 65536
        prompts = [p[:96] for p in queue_requests(workload, vocab, seed=2000)[0][:8]]
        what = "the first 8 requests of the queue, prompts cut to 96 tokens"
    elif workload in GROUP_WORKLOADS:
        model = GROUP_WORKLOADS[workload]["model"]
        vocab = 4096 if model == "tiny" else 65536
        prompts = [p[:96] for p in synthetic.uniform_prompts(8, *GROUP_WORKLOADS[workload]["prompt_range"], vocab, seed=3000)]
        what = "8 prompts of the group workload cut to 96 tokens, one sample each"
    else:
        model, _, low, high, _, _ = WORKLOADS[workload]
        vocab = 4096 if model == "tiny" else 65536
        prompts = [p[:96] for p in synthetic.uniform_prompts(8, low, high, vocab, seed=1000)]
        what = "8 prompts of the batch cut to 96 tokens"
    return model, prompts, 24, what


def host_threads() -> int:
    """Use every host core regardless of what the launcher exported (torchrun sets OMP_NUM_THREADS=1)."""
    import torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    return torch.get_num_threads()


def cpu_baseline(workload: str, *, seconds_budget: float = 25.0, steps: int = 4, warmup: int = 0) -> dict:
    """The reference's own eager CPU engine (fp32, its CPU default) on a bounded sample of the workload;
    the numpy port of it when the reference is not staged. `warmup` untimed passes, then exactly `steps`
    timed passes; the number of sampled tokens per pass is cut down after the first pass if `steps` passes
    would not fit `seconds_budget`."""
    import torch
    from oracle.build_ref import staged_path

    model, prompts, new_tokens, what = cpu_sample(workload)
    threads = host_threads()
    kind = "reference" if staged_path() is not None else "port"
    if kind == "reference":
        impl = Impl("reference")
        engine, _ = impl.build(model, torch.device("cpu"), None, max_model_len=256, dtype=torch.float32)
        flat = impl.flatten(prompts)

        def one_pass(n_new):
            out = engine.generate(*flat, repeats=1, sampling=impl.Sampling(temperature=1.0, max_new_tokens=n_new, seed=0,
                                                                           ignore_eos=True, return_logprobs=True))
            return int(out.lengths.sum())
    else:
        from climbing_gym_b200 import synthetic
        from oracle.lfm25_oracle import OracleConfig, OracleEngine, OracleSampling

        cfg = synthetic.tiny_config() if model == "tiny" else synthetic.lfm25_1p2b_config()
        ocfg = OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, mlp_hidden_size=cfg.mlp_hidden_size,
                            num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                            layer_types=tuple(cfg.layer_types), rope_theta=cfg.rope_theta, norm_eps=cfg.norm_eps,
                            conv_kernel_size=cfg.conv_kernel_size, eos_token_id=cfg.eos_token_id)
        oracle = OracleEngine(ocfg, synthetic.make_state_dict_streams(cfg, seed=0), dtype="fp32", max_model_len=256)

        def one_pass(n_new):
            out = oracle.generate(prompts, 1, OracleSampling(temperature=1.0, max_new_tokens=n_new, seed=0, ignore_eos=True))
            return int(out["lengths"].sum())

    t0 = time.perf_counter()
    one_pass(new_tokens)  # first pass: page in the weights, size the timed passes
    first = time.perf_counter() - t0
    per_pass_budget = seconds_budget / max(1, steps + warmup)
    if first > per_pass_budget:
        new_tokens = max(2, int(new_tokens * per_pass_budget / first))
    for _ in range(warmup):
        one_pass(new_tokens)
    t0 = time.perf_counter()
    done = sum(one_pass(new_tokens) for _ in range(max(1, steps)))
    seconds = time.perf_counter() - t0
    engine_name = ("the reference's LFM25Engine on CPU, fp32, eager attention" if kind == "reference"
                   else "numpy port of the reference's eager engine, fp32")
    return {"value": round(done / seconds, 2), "unit": UNIT, "cores": threads, "host_cores": os.cpu_count(), "kind": kind,
            "sample": f"{max(1, steps)} pass(es) over {what}, {new_tokens} sampled tokens per request; {engine_name}; "
                      f"{seconds:.1f} s", "seconds": round(seconds, 2), "passes": max(1, steps)}


def run_reference(args) -> dict:
    """--impl reference: the reference's own implementation of the path. On the host cores by default (rank 0
    only; the other ranks exit without work); with --reference-device cuda its CUDA engine on the GPU, driven
    through the same workload code as this package's engine."""
    if args.reference_device == "cuda":
        try:
            if args.workload in QUEUE_WORKLOADS:
                return run_queue(args)
            if args.workload in WORKLOADS:
                return run_generate(args)
            raise RuntimeError(f"workload {args.workload} is not wired to the reference's CUDA engine")
        except Exception as exc:  # the line must say why, not die: the caller records it
            if int(os.environ.get("RANK", 0)) != 0:
                return {}
            return {"impl": "reference-cuda", "unavailable": f"{type(exc).__name__}: {str(exc).splitlines()[0][:300]}"}
    if int(os.environ.get("RANK", 0)) != 0:
        return {}
    t0 = time.perf_counter()
    base = cpu_baseline(args.workload, seconds_budget=200.0, steps=args.steps, warmup=args.warmup)
    model = cpu_sample(args.workload)[0]
    return {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(base["seconds"] * 1e3 / base["passes"], 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "model": model_name(model),
                       "step": "one generate pass over the bounded sample named in cpu_baseline.sample",
                       "threads": base["cores"]},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0, "wall_seconds": round(time.perf_counter() - t0, 1)}


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="ours", choices=["ours", "reference"])
    parser.add_argument("--reference-device", default="cpu", choices=["cpu", "cuda"],
                        help="with --impl reference: its CPU engine on a bounded sample (default), or its CUDA engine "
                             "on the full workload on the GPU")
    parser.add_argument("--workload", default=DEFAULT_WORKLOAD,
                        choices=sorted([*WORKLOADS, *QUEUE_WORKLOADS, *GROUP_WORKLOADS]))
    parser.add_argument("--scheduler", default="device", choices=["device", "host"],
                        help="queue workloads: slot turnover inside the decode graph (default) or from the host")
    parser.add_argument("--batch", type=int, default=0, help="override prompts per GPU (generate workloads)")
    parser.add_argument("--new-tokens", type=int, default=0, help="override sampled tokens per prompt (generate workloads)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-seconds", type=float, default=20.0)
    args = parser.parse_args()
    # stdout carries the one JSON line and nothing else: file descriptor 1 is pointed at stderr for the
    # run (NCCL prints its version banner there from C), and the line goes to a duplicate of the real one
    sys.stdout.flush()
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        result = run_reference(args)
    elif args.workload in QUEUE_WORKLOADS:
        result = run_queue(args)
    elif args.workload in GROUP_WORKLOADS:
        result = run_group(args)
    else:
        result = run_generate(args)
    if result:
        print(json.dumps(result), file=json_out, flush=True)


if __name__ == "__main__":
    main()
