#!/usr/bin/env python
"""Rollout throughput of the B200 engine on the headline configuration.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nnodes=1 --nproc-per-node N ... bench.py --gpus N ...      (one rank per GPU)

A "step" is one ``engine.generate`` call over one batch of the workload: packed prefill of the
batch's prompts, then ``new_tokens`` decode steps with sampling and sampled-token log-probs.
Workload (default "bf16-b64x512"): LFM2.5-1.2B architecture, random-init bf16 weights, 64 prompts of
uniform-random ids with lengths uniform in [64, 1024], 512 sampled tokens each (temperature 1,
full support, EOS ignored), CUDA-graph decode. With N > 1 every rank runs its own replica on its
own 64 prompts (weak scaling, no data-path collective); rank 0 broadcasts the policy weights over
NCCL once before the warm-up, as it does before each rollout in training.

Prints ONE JSON line. ``value`` times the steps with inputs resident in HBM; ``e2e`` repeats them
through the public API with pinned-host prompts and a device->host read of tokens, log-probs and
lengths inside the timed region (the reference benchmark's convention). ``roofline`` is the decode
step graph: algorithmic bytes (weights + KV history per step) over its CUDA-event duration against
the measured HBM copy bandwidth. ``cpu_baseline`` times the CPU oracle on a bounded sample.

After the default workload the same process also runs the FP8 rollout configuration once
("fp8-queue2048x256": FP8 W8A8 MLP + e4m3 KV, 2048 queued requests over 256 live slots through a
generation session; one short warm-up pass, one full timed pass) and attaches its numbers as
``fp8_rollout`` (``--fp8-rollout off`` skips it; ``--workload fp8-queue2048x256`` runs it as the
line itself, every step being one pass over the whole queue).
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
DEFAULT_WORKLOAD = "bf16-b64x512"
FP8_ROLLOUT_WORKLOAD = "fp8-queue2048x256"  # also measured (one pass) after the default workload: `fp8_rollout`

WORKLOADS = {
    # name: (model, batch, prompt_low, prompt_high, new_tokens, graph options)
    "bf16-b64x512": ("1p2b", 64, 64, 1024, 512, {}),
    "fp8-b64x512": ("1p2b", 64, 64, 1024, 512, {"fp8_mlp": True, "fp8_kv": True}),
    "tiny": ("tiny", 8, 8, 64, 32, {}),
    # long-context stress: 32 sequences, prompts of 16-30 K tokens prefilled in 4096-token chunks
    "bf16-long32x1024": ("1p2b", 32, 16384, 30720, 1024, {}),
    "fp8kv-long32x1024": ("1p2b", 32, 16384, 30720, 1024, {"fp8_kv": True}),
}

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum over the 139 kernels of ONE decode-step
# replay, one ncu capture) divided by the step's algorithmic bytes at the captured sequence lengths:
# 2.9113 GB measured for 2.7678 GB (profiles/decode_step_bf16_b64_dram_traffic.md). Both grow with the
# same two terms (weights once, KV history once), so `roofline.traffic` scales the full-size
# algorithmic bytes by this ratio.
DRAM_TRAFFIC_RATIO = {"bf16-b64x512": 1.0518}

# Continuous batching through a generation session: a queue of requests served by a fixed number of
# live slots; a finished request's slot is refilled from the queue at the next poll.
#   name: (model, graph options, requests, slots, max_model_len, max output, mean output, prompt
#          median, prompt sigma, prompt clip, poll interval)
QUEUE_WORKLOADS = {
    "fp8-queue2048x256": ("1p2b", {"fp8_mlp": True, "fp8_kv": True}, 2048, 256, 8192, 4096, 1500.0, 400.0, 0.8,
                          (32, 4096), 32),
    "tiny-queue": ("tiny", {}, 24, 8, 256, 32, 12.0, 24.0, 0.5, (4, 96), 8),
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


def build_engine(model: str, device, options: dict, max_model_len: int, seed: int = 0):
    import torch
    from climbing_gym_b200 import synthetic
    from climbing_gym_b200.engine import LFM25Engine

    cfg = synthetic.tiny_config() if model == "tiny" else synthetic.lfm25_1p2b_config()
    state = synthetic.make_state_dict_on_device(cfg, seed, device, torch.bfloat16)
    engine = LFM25Engine.from_state_dict(cfg, state, device=device, dtype=torch.bfloat16, max_model_len=max_model_len)
    del state
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


def run_ours(args) -> dict:
    import torch
    import torch.distributed as dist
    from climbing_gym_b200 import _native as nv, synthetic
    from climbing_gym_b200.config import LFM25SamplingConfig
    from climbing_gym_b200.engine import flatten_token_batches
    from climbing_gym_b200.replica import broadcast_policy_weights

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if not torch.cuda.is_available():
        raise RuntimeError("bench.py needs a CUDA device: the engine has no CPU path")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=device)
    model, batch, low, high, new_tokens, options = WORKLOADS[args.workload]
    batch = args.batch or batch
    new_tokens = args.new_tokens or new_tokens
    engine, cfg = build_engine(model, device, options, max_model_len=high + new_tokens + 64)
    broadcast_ms = None
    if world > 1:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        moved = broadcast_policy_weights(engine, src=0)
        torch.cuda.synchronize()
        broadcast_ms = (time.perf_counter() - t0) * 1e3
    prompts = synthetic.uniform_prompts(batch, low, high, cfg.vocab_size, seed=1000 + rank)
    flat_host = flatten_token_batches(prompts, device="cpu")
    ids_pinned, cu_pinned = flat_host[0].pin_memory(), flat_host[1].pin_memory()
    ids_dev, cu_dev = ids_pinned.to(device), cu_pinned.to(device)
    max_len = flat_host[2]
    sampling = LFM25SamplingConfig(temperature=1.0, top_k=0, top_p=1.0, max_new_tokens=new_tokens, seed=0,
                                   ignore_eos=True, return_logprobs=True)
    decoder = engine._cuda_decoder

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn, steps):
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        barrier()
        ms = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    outputs = {}

    def step_resident():
        outputs["last"] = engine.generate(ids_dev, cu_dev, max_len, repeats=1, sampling=sampling)

    def step_e2e():
        out = engine.generate(ids_pinned.to(device, non_blocking=True), cu_pinned, max_len, repeats=1, sampling=sampling)
        outputs["host"] = (out.token_ids.cpu(), out.logprobs.cpu(), out.lengths.cpu())

    for _ in range(args.warmup):
        step_resident()
    launches_before = nv.launch_count()
    decoder.profile_decode, decoder.decode_profile = True, []
    with ClockSampler(local_rank) as clocks:
        total_ms = timed(step_resident, args.steps)
    decoder.profile_decode = False
    launches = nv.launch_count() - launches_before
    decode_ms = sum(s.elapsed_time(e) for s, e, _ in decoder.decode_profile)
    decode_replays = sum(n for _, _, n in decoder.decode_profile)
    e2e_ms = timed(step_e2e, args.steps)
    tokens_per_step = batch * new_tokens
    lengths = outputs["last"].lengths
    if int(lengths.sum()) != tokens_per_step or not bool(torch.isfinite(outputs["last"].logprobs).all()):
        raise RuntimeError("generate returned an incomplete budget or non-finite log-probs")
    value = world * tokens_per_step * args.steps / (total_ms / 1e3)
    e2e_value = world * tokens_per_step * args.steps / (e2e_ms / 1e3)

    # decode roofline: weights + KV history per step (algorithmic bytes), HBM-bound
    w_bytes = weight_bytes(engine, options)
    n_attn = engine.weights.num_attention_layers
    kv_elem = 1 if options.get("fp8_kv") else 2
    kv_tok = n_attn * 2 * cfg.num_key_value_heads * (cfg.head_dim * kv_elem + (4 if options.get("fp8_kv") else 0))
    prompt_total = sum(len(p) for p in prompts)
    # replay j (1-based) reads, per row, its prompt plus j generated tokens
    kv_bytes_avg = kv_tok * (prompt_total + batch * (new_tokens) / 2.0)
    bytes_per_replay = w_bytes + kv_bytes_avg
    peak, peak_source = peaks()
    roofline = None
    if decode_replays:
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
        "config": {"workload": args.workload, "model": "LFM2.5-1.2B architecture, random init" if model == "1p2b" else "tiny hybrid",
                   "batch_per_gpu": batch, "prompt_lengths": f"uniform[{low},{high}]", "new_tokens": new_tokens,
                   "sampling": "temperature 1, full support, ignore_eos", "replicas": world,
                   "l2": "working set per decode step (weights + KV) is far larger than the 126 MB L2"},
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": int(ids_pinned.numel() * 8 + cu_pinned.numel() * 4),
                "d2h_bytes_per_step": int(tokens_per_step * 12 + batch * 4), "ms_per_step": round(e2e_ms / args.steps, 3)},
        "gpu_launches": int(launches), "clocks": clocks.summary(), "roofline": roofline,
    }
    if broadcast_ms is not None:
        result["weight_broadcast"] = {"ms": round(broadcast_ms, 2), "bytes": int(moved)}
    if args.fp8_rollout == "on" or (args.fp8_rollout == "auto" and args.workload == DEFAULT_WORKLOAD
                                    and not args.batch and not args.new_tokens):
        # the FP8 continuous-batching configuration next to the headline line: one short warm-up pass and
        # one full timed pass of the request queue on the same GPU(s), device-timed like the line itself
        del engine, decoder, ids_dev, cu_dev
        torch.cuda.empty_cache()
        nested = argparse.Namespace(**{**vars(args), "workload": FP8_ROLLOUT_WORKLOAD, "steps": 1, "warmup": 0})
        extra = run_queue(nested, nested=True)
        result["fp8_rollout"] = {key: extra[key] for key in ("value", "unit", "ms_per_step", "dtype", "config", "roofline",
                                                             "gpu_launches", "clocks", "warmup_note")}
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(model, seconds_budget=args.cpu_seconds)
    if world > 1:
        dist.destroy_process_group()
    return result if rank == 0 else {}


def queue_requests(name: str, vocab: int, seed: int):
    """Seeded synthetic requests of a queue workload: prompt lengths lognormal around the median and
    clipped, output lengths geometric with the given mean and capped (a per-request length limit
    stands in for the EOS hazard), prompt + output within max_model_len."""
    import numpy as np

    _, _, n, _, max_len, cap, mean_out, median, sigma, (low, high), _ = QUEUE_WORKLOADS[name]
    rng = np.random.default_rng(seed)
    prompt_lens = np.clip(np.rint(rng.lognormal(np.log(median), sigma, n)), low, high).astype(np.int64)
    limits = np.minimum(rng.geometric(1.0 / mean_out, n), cap).astype(np.int64)
    limits = np.maximum(1, np.minimum(limits, max_len - prompt_lens - 1))
    prompts = [rng.integers(3, vocab, size=int(length)).tolist() for length in prompt_lens]
    return prompts, [int(v) for v in limits]


def run_queue(args, *, nested: bool = False) -> dict:
    """One step = the whole request queue through one generation session. ``nested``: called from another
    workload's run inside its process group - one short warm-up pass over the first slots' worth of requests
    (to capture the graphs and size the buffers), no host-buffer pass, and the result on every rank."""
    import torch
    import torch.distributed as dist
    from climbing_gym_b200 import _native as nv
    from climbing_gym_b200.config import LFM25SamplingConfig
    from climbing_gym_b200.replica import broadcast_policy_weights

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if not torch.cuda.is_available():
        raise RuntimeError("bench.py needs a CUDA device: the engine has no CPU path")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1 and not nested:
        dist.init_process_group("nccl", device_id=device)
    model, options, n_requests, slots, max_len, cap, mean_out, median, sigma, clip, poll_steps = QUEUE_WORKLOADS[args.workload]
    engine, cfg = build_engine(model, device, options, max_model_len=max_len)
    if world > 1:
        broadcast_policy_weights(engine, src=0)
    prompts, limits = queue_requests(args.workload, cfg.vocab_size, seed=2000 + rank)
    staged = [torch.tensor(p, device=device, dtype=torch.int64) for p in prompts]
    queue_samplings = [LFM25SamplingConfig(temperature=1.0, top_k=0, top_p=1.0, max_new_tokens=limit, seed=index,
                                           ignore_eos=True, return_logprobs=True) for index, limit in enumerate(limits)]
    n_queue = n_requests

    def one_pass(on_device: bool, *, short: bool = False) -> dict:
        generated, next_request, live = 0, 0, 0
        n_requests, samplings = n_queue, queue_samplings
        if short:  # warm-up: the first slots' worth of requests, a few tokens each
            n_requests = min(slots, n_queue)
            samplings = [LFM25SamplingConfig(temperature=1.0, max_new_tokens=min(limit, 2 * poll_steps), seed=index,
                                             ignore_eos=True) for index, limit in enumerate(limits[:n_requests])]
        with engine.generation_session(max_batch_size=slots, max_new_tokens=cap, profile_timings=True) as session:
            def admit(count, into=None):
                nonlocal next_request, live
                pick = slice(next_request, next_request + count)
                session.admit(prompts[pick], samplings[pick], slots=into,
                              device_prompts=staged[pick] if on_device else None)
                next_request += count
                live += count

            admit(min(slots, n_requests))
            while live:
                freed = []
                for result in session.poll(steps=poll_steps):
                    generated += len(result.token_ids)
                    if result.logprobs is None or not all(math.isfinite(v) for v in result.logprobs):
                        raise RuntimeError("session returned no or non-finite log-probs")
                    freed.append(result.handle.slot)
                    session.release(result.handle)
                    live -= 1
                refill = min(len(freed), n_requests - next_request)
                if refill:
                    admit(refill, freed[:refill])
            timing = session.timing_stats()
            stats = dict(session.stats)
        return {"generated": generated, "decode_s": timing.get("decode_gpu_seconds", 0.0),
                "prefill_s": timing.get("prefill_gpu_seconds", 0.0), "replays": stats["decode_steps"]}

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(on_device: bool, steps: int):
        barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        passes = [one_pass(on_device) for _ in range(steps)]
        end.record()
        barrier()
        ms = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([ms], device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, passes

    for _ in range(args.warmup):
        one_pass(True)
    if nested:
        one_pass(True, short=True)
    launches_before = nv.launch_count()
    with ClockSampler(local_rank) as clocks:
        total_ms, passes = timed(True, args.steps)
    launches = nv.launch_count() - launches_before
    e2e_ms = timed(False, args.steps)[0] if not nested else total_ms
    expected = sum(limits)
    if any(p["generated"] != expected for p in passes):
        raise RuntimeError("a pass did not deliver every request's output budget")
    value = world * expected * args.steps / (total_ms / 1e3)
    e2e_value = world * expected * args.steps / (e2e_ms / 1e3)

    # decode roofline: every replay streams the weights once and each live row's KV history once
    w_bytes = weight_bytes(engine, options)
    n_attn = engine.weights.num_attention_layers
    fp8_kv = bool(options.get("fp8_kv"))
    kv_tok = n_attn * 2 * cfg.num_key_value_heads * (cfg.head_dim * (1 if fp8_kv else 2) + (4 if fp8_kv else 0))
    kv_tokens = sum((n - 1) * len(p) + (n - 1) * n // 2 for p, n in zip(prompts, limits))  # sum over decode steps of context
    replays = sum(p["replays"] for p in passes) / len(passes)
    decode_s = sum(p["decode_s"] for p in passes) / len(passes)
    bytes_per_replay = w_bytes + kv_tok * kv_tokens / replays
    peak, peak_source = peaks()
    achieved = bytes_per_replay * replays / decode_s / 1e9
    roofline = {"bound": "hbm", "kernel": f"decode step graph at {slots} slots (all kernels of one token step)",
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                "peak_source": peak_source, "traffic": None, "ms_per_launch": round(decode_s * 1e3 / replays, 4),
                "algorithmic_bytes_per_launch": int(bytes_per_replay), "launches_timed": int(replays * len(passes)),
                "decode_share_of_step": round(decode_s * 1e3 * len(passes) / total_ms, 4),
                "prefill_share_of_step": round(sum(p["prefill_s"] for p in passes) * 1e3 / total_ms, 4)}
    prompt_tokens = sum(len(p) for p in prompts)
    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16+e4m3" if options else "bf16", "data": "synthetic",
        "config": {"workload": args.workload,
                   "model": "LFM2.5-1.2B architecture, random init" if model == "1p2b" else "tiny hybrid",
                   "requests_per_gpu": n_requests, "live_slots": slots, "max_model_len": max_len,
                   "prompt_lengths": f"lognormal(median {median:g}, sigma {sigma:g}) clipped to {list(clip)}",
                   "output_lengths": f"geometric(mean {mean_out:g}) capped at {cap}, enforced as per-request limits",
                   "prompt_tokens": prompt_tokens, "output_tokens": expected, "poll_interval": poll_steps,
                   "options": options, "sampling": "temperature 1, full support", "replicas": world,
                   "l2": "working set per decode step (weights + KV) is far larger than the 126 MB L2"},
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": int(prompt_tokens * 8),
                "d2h_bytes_per_step": int(expected * 12 + replays / poll_steps * slots), "ms_per_step": round(e2e_ms / args.steps, 3)},
        "gpu_launches": int(launches), "clocks": clocks.summary(), "roofline": roofline,
    }
    if nested:
        del result["e2e"]
        result["warmup_note"] = "one short pass (first slots' worth of requests, a few tokens each), then one full timed pass"
        return result
    if world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(model, seconds_budget=args.cpu_seconds)
    if world > 1:
        dist.destroy_process_group()
    return result if rank == 0 else {}


def cpu_baseline(model: str, *, seconds_budget: float = 25.0, steps: int = 1, warmup: int = 0) -> dict:
    """The CPU oracle (numpy restatement of the reference's eager engine) on a bounded sample of the
    workload: 8 prompts of 64 tokens, 48 sampled tokens each, fp32 on the host cores. `warmup` untimed
    passes, then up to `steps` timed passes (stops early once `seconds_budget` is spent)."""
    import numpy as np
    from climbing_gym_b200 import synthetic
    from oracle.lfm25_oracle import OracleConfig, OracleEngine, OracleSampling

    cfg = synthetic.tiny_config() if model == "tiny" else synthetic.lfm25_1p2b_config()
    state = synthetic.make_state_dict(cfg, seed=0)
    ocfg = OracleConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size, mlp_hidden_size=cfg.mlp_hidden_size,
                        num_attention_heads=cfg.num_attention_heads, num_key_value_heads=cfg.num_key_value_heads,
                        layer_types=tuple(cfg.layer_types), rope_theta=cfg.rope_theta, norm_eps=cfg.norm_eps,
                        conv_kernel_size=cfg.conv_kernel_size, eos_token_id=cfg.eos_token_id)
    oracle = OracleEngine(ocfg, state, dtype="fp32", max_model_len=256)
    del state
    n_prompts, prompt_len, new_tokens = 8, 64, 48
    prompts = synthetic.uniform_prompts(n_prompts, prompt_len, prompt_len, cfg.vocab_size, seed=7)
    sampling = OracleSampling(temperature=1.0, max_new_tokens=new_tokens, seed=0, ignore_eos=True)
    for _ in range(warmup):
        oracle.generate(prompts, 1, sampling)
    t0 = time.perf_counter()
    done = passes = 0
    for _ in range(max(1, steps)):
        out = oracle.generate(prompts, 1, sampling)
        done += int(out["lengths"].sum())
        passes += 1
        if time.perf_counter() - t0 > seconds_budget:
            break
    seconds = time.perf_counter() - t0
    return {"value": round(done / seconds, 2), "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{passes} pass(es) of {n_prompts} prompts x {prompt_len} tokens, {new_tokens} sampled tokens each, "
                      f"fp32 numpy oracle (multi-threaded BLAS), {seconds:.1f} s", "seconds": round(seconds, 2),
            "passes": passes}


def run_reference(args) -> dict:
    """The reference's CPU implementation of the path, as restated by the oracle port, on host cores."""
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return {}
    model = (QUEUE_WORKLOADS.get(args.workload) or WORKLOADS[args.workload])[0]
    t0 = time.perf_counter()
    # every step is one pass over the bounded sample; a pass takes 10-15 s, so the step count actually
    # timed is capped to keep the whole run within a few minutes (the cap is reported in `sample`)
    base = cpu_baseline(model, seconds_budget=150.0, steps=min(args.steps, 10), warmup=min(args.warmup, 1))
    model_name = model
    return {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(base["seconds"] * 1e3 / base["passes"], 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "model": "LFM2.5-1.2B architecture, random init" if model_name == "1p2b" else "tiny hybrid",
                       "note": "the reference is Python and cannot travel to the GPU box; its CPU engine is timed through "
                               "the numpy port pinned to it by tests/golden (bounded sample of the workload)"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gpu_launches": 0, "wall_seconds": round(time.perf_counter() - t0, 1)}


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=3)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="ours", choices=["ours", "reference"])
    parser.add_argument("--workload", default=DEFAULT_WORKLOAD, choices=sorted([*WORKLOADS, *QUEUE_WORKLOADS]))
    parser.add_argument("--fp8-rollout", default="auto", choices=["auto", "on", "off"],
                        help="append one timed pass of the FP8 continuous-batching queue as `fp8_rollout` "
                             "(auto: with the default workload at its default size)")
    parser.add_argument("--batch", type=int, default=0, help="override prompts per GPU")
    parser.add_argument("--new-tokens", type=int, default=0, help="override sampled tokens per prompt")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-seconds", type=float, default=25.0)
    args = parser.parse_args()
    # stdout carries the one JSON line and nothing else: file descriptor 1 is pointed at stderr for the
    # run (NCCL prints its version banner there from C), and the line goes to a duplicate of the real one
    sys.stdout.flush()
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        result = run_reference(args)
    else:
        result = run_queue(args) if args.workload in QUEUE_WORKLOADS else run_ours(args)
    if result:
        print(json.dumps(result), file=json_out, flush=True)


if __name__ == "__main__":
    main()
