"""Fixed-budget rollout throughput of the B200 engine: the ``climbing-gym benchmark`` command.

Keeps the command line and the report schema of the reference harness
(src/climbing_gym/inference/benchmark.py:23-153) so that ``preflight.validate_preflight``
(src/climbing_gym/preflight.py:62-143) accepts the JSON unchanged: ``engine == "native_lfm25"``,
``config.*`` echoing every flag, ``workload.kind``, ``sampling.*``, ``max_model_len``,
``hardware.name`` and per batch ``median_tokens_per_second``, ``peak_*_bytes`` and
``runs[].{seconds, tokens_per_second, output_tokens}``.

A timed run is one ``engine.generate`` over the batch plus the device->host copies of tokens,
log-probs and lengths; load and warm-up are excluded; every row must deliver its full output budget
(EOS is ignored) with finite log-probs.

Additions: ``--synthetic {tiny,1p2b}`` benchmarks random-init weights of that architecture when no
checkpoint is at hand (prompts are then random ids and traces print ids, not text). This package has
no CPU path, so ``--device`` must be a CUDA device and the decode step always runs as its captured
kernel graph (``--cuda-graphs`` is implied, ``--compile-decode`` is accepted and ignored).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import statistics
import time
from dataclasses import asdict
from datetime import datetime, timezone
from pathlib import Path

import torch

PROMPT_SENTENCE = "Document {index}: Check each arithmetic operation carefully before continuing. "


def build_arg_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    add = parser.add_argument
    add("--model", help="Local checkpoint directory")
    add("--synthetic", choices=["tiny", "1p2b"], help="random-init weights of this architecture instead of --model")
    add("--batches", type=int, nargs="+", default=[1, 32, 128])
    add("--prompt-tokens", type=int, default=128)
    add("--prompts-json", type=Path, help="JSON containing a prompts list of token-ID rows")
    add("--output-tokens", type=int, default=4096)
    add("--max-model-len", type=int)
    add("--device", default="cuda")
    add("--dtype", default="auto", choices=["auto", "bfloat16", "float16", "float32"])
    add("--temperature", type=float, default=1.0)
    add("--top-k", type=int, default=-1, help="-1 disables top-k, matching rollout sampling")
    add("--top-p", type=float, default=1.0)
    add("--repetition-penalty", type=float, default=1.0)
    add("--behavior-topk", type=int, default=0)
    add("--seed", type=int, default=0)
    add("--warmups", type=int, default=1)
    add("--repeats", type=int, default=2)
    for flag in ("--cuda-graphs", "--compile-decode", "--fp8-mlp", "--fp8-kv", "--fp8-lm-head", "--adaptive-batching",
                 "--bf16-weight-packing"):
        add(flag, action="store_true")
    add("--max-prefill-tokens", type=int, default=4096)
    add("--park-gib", type=float, default=0, help="Reserve optimizer-equivalent GPU memory")
    add("--output", type=Path, required=True)
    return parser


def validate_args(parser: argparse.ArgumentParser, args) -> list | None:
    """The reference's argument checks (benchmark.py:66-84); returns the saved prompt rows, if any."""
    positives = (*args.batches, args.prompt_tokens, args.output_tokens, args.warmups, args.repeats, args.max_prefill_tokens)
    if min(positives) <= 0 or args.park_gib < 0:
        parser.error("batch sizes, token counts and repetitions must be positive; parked memory must be nonnegative")
    if bool(args.model) == bool(args.synthetic):
        parser.error("exactly one of --model and --synthetic is required")
    if torch.device(args.device).type != "cuda":
        parser.error("this engine has no CPU path: --device must be a CUDA device")
    if args.top_k == 0 or args.top_k < -1:
        parser.error("--top-k must be -1 or positive")
    if args.prompts_json is None:
        return None
    saved = json.loads(args.prompts_json.read_text())["prompts"]
    if not saved or any(not row or any(type(t) is not int or t < 0 for t in row) for row in saved):
        parser.error("--prompts-json must contain nonempty rows of nonnegative integer token IDs")
    return saved


class _IdTokenizer:
    """Stand-in when benchmarking synthetic weights: text is the list of ids."""

    def __init__(self, vocab: int):
        self.vocab = vocab

    def encode(self, text, add_special_tokens=False):
        digest = hashlib.sha256(text.encode()).digest()
        return [3 + int.from_bytes(digest[i:i + 2], "little") % (self.vocab - 3) for i in range(0, 32, 2)]

    def decode(self, ids, skip_special_tokens=False):
        return " ".join(str(int(i)) for i in ids)


def synthetic_prompts(tokenizer, batch: int, length: int) -> list[list[int]]:
    rows = []
    for index in range(batch):
        ids = tokenizer.encode(PROMPT_SENTENCE.format(index=index), add_special_tokens=False)
        rows.append((ids * (length // len(ids) + 1))[:length])
    return rows


def load_engine(args, context: int):
    from . import synthetic
    from .engine import LFM25Engine
    from .weights import load_tokenizer

    device = torch.device(args.device)
    if args.synthetic:
        cfg = synthetic.tiny_config() if args.synthetic == "tiny" else synthetic.lfm25_1p2b_config()
        dtype = torch.float32 if args.dtype == "float32" else torch.bfloat16
        state = synthetic.make_state_dict_on_device(cfg, args.seed, device, dtype)
        engine = LFM25Engine.from_state_dict(cfg, state, device=device, dtype=dtype, max_model_len=context)
        tokenizer = _IdTokenizer(cfg.vocab_size)
    else:
        engine = LFM25Engine.from_pretrained(args.model, device=device, dtype=args.dtype, max_model_len=context)
        tokenizer = load_tokenizer(args.model)
    engine.enable_cuda_graphs(max_graphs=1, max_prefill_tokens=args.max_prefill_tokens,
                              bf16_weight_packing=args.bf16_weight_packing, fp8_mlp=args.fp8_mlp, fp8_kv=args.fp8_kv,
                              fp8_lm_head=args.fp8_lm_head, adaptive_batching=args.adaptive_batching)
    return engine, tokenizer


def timed_run(engine, flat, sampling, batch: int, output_tokens: int, device) -> tuple[dict, torch.Tensor, torch.Tensor]:
    torch.cuda.synchronize(device)
    start = time.perf_counter()
    output = engine.generate(*flat, repeats=1, sampling=sampling)
    tokens, logprobs, lengths = output.token_ids.cpu(), output.logprobs.cpu(), output.lengths.cpu()
    if output.topk_token_ids is not None:
        output.topk_token_ids.cpu()
        if not bool(torch.isfinite(output.topk_logprobs.cpu()).all()):
            raise RuntimeError("Native rollout returned non-finite sparse behavior logprobs")
    torch.cuda.synchronize(device)
    elapsed = time.perf_counter() - start
    count = int(lengths.sum())
    if count != batch * output_tokens or not bool(torch.isfinite(logprobs).all()):
        raise RuntimeError("Native rollout returned an incomplete budget or non-finite logprobs")
    return {"seconds": elapsed, "output_tokens": count, "tokens_per_second": count / elapsed}, tokens, lengths


def batch_result(batch: int, runs: list[dict], device) -> dict:
    return {"batch_size": batch, "max_num_seqs": batch, "max_inflight_requests": batch, "runs": runs,
            "median_tokens_per_second": statistics.median(r["tokens_per_second"] for r in runs),
            "peak_allocated_bytes": torch.cuda.max_memory_allocated(device) if device.type == "cuda" else None,
            "peak_reserved_bytes": torch.cuda.max_memory_reserved(device) if device.type == "cuda" else None}


def report_header(args, sampling, context: int, saved, device) -> dict:
    return {
        "engine": "native_lfm25", "created_at": datetime.now(timezone.utc).isoformat(),
        "hardware": {"device": str(device),
                     "name": torch.cuda.get_device_name(device) if device.type == "cuda" and torch.cuda.is_available() else "cpu",
                     "torch_version": torch.__version__},
        "workload": {"kind": "representative" if saved else "synthetic",
                     "prompts_sha256": hashlib.sha256(args.prompts_json.read_bytes()).hexdigest() if saved else None,
                     "prompt_lengths": list(map(len, saved)) if saved else [args.prompt_tokens]},
        "config": {k: str(v) if isinstance(v, Path) else v for k, v in vars(args).items()},
        "sampling": asdict(sampling), "max_model_len": context,
        "scheduler": "synchronous fixed batches; no hidden request concurrency cap", "batches": []}


def trace_section(tokenizer, batch: int, row: int, prompt, completion, saved) -> list[str]:
    expected = ("Expected answer: not scored (representative throughput workload)." if saved else
                "Expected answer: not applicable (synthetic throughput workload).")
    return [f"## Batch {batch}, row {row}", "", "Prompt:", "", "```text", tokenizer.decode(prompt, skip_special_tokens=False),
            "```", "", "Complete model response:", "", "```text", tokenizer.decode(completion, skip_special_tokens=False),
            "```", "", expected, f"Outcome: {len(completion)} tokens; sampled log probabilities finite.", ""]


def main(argv=None) -> None:
    from .config import LFM25SamplingConfig
    from .engine import flatten_token_batches

    parser = build_arg_parser()
    args = parser.parse_args(argv)
    saved = validate_args(parser, args)
    args.cuda_graphs = True  # the captured kernel graph is this engine's only decode path
    device = torch.device(args.device)
    context = args.max_model_len or max(args.prompt_tokens, max(map(len, saved)) if saved else 0) + args.output_tokens
    engine, tokenizer = load_engine(args, context)
    parked = torch.empty(int(args.park_gib * 1024 ** 3), device=device, dtype=torch.uint8) if args.park_gib else None
    sampling = LFM25SamplingConfig(max_new_tokens=args.output_tokens, temperature=args.temperature, seed=args.seed,
                                   ignore_eos=True, return_logprobs=True, top_k=0 if args.top_k == -1 else args.top_k,
                                   top_p=args.top_p, repetition_penalty=args.repetition_penalty,
                                   behavior_topk=args.behavior_topk)
    report = report_header(args, sampling, context, saved, device)
    traces = ["# Native throughput traces", "",
              ("Fixed-budget representative task prompts; environment answers are not scored." if saved else
               "Fixed-budget synthetic prompts; expected answer: not applicable (throughput validation)."), ""]
    for batch in args.batches:
        rows = ([saved[i % len(saved)] for i in range(batch)] if saved else
                synthetic_prompts(tokenizer, batch, args.prompt_tokens))
        if any(len(row) + args.output_tokens > context for row in rows):
            parser.error("prompt plus output token budget exceeds --max-model-len")
        flat = flatten_token_batches(rows, device=device)
        for _ in range(args.warmups):
            engine.generate(*flat, repeats=1, sampling=sampling)
        torch.cuda.synchronize(device)
        torch.cuda.reset_peak_memory_stats(device)
        runs = []
        for _ in range(args.repeats):
            run, tokens, lengths = timed_run(engine, flat, sampling, batch, args.output_tokens, device)
            runs.append(run)
        result = batch_result(batch, runs, device)
        report["batches"].append(result)
        for row in range(min(3, batch)):
            traces += trace_section(tokenizer, batch, row, rows[row], tokens[row, 0, :int(lengths[row, 0])].tolist(), saved)
        print(json.dumps(result), flush=True)
        engine.release_inference_buffers()
    args.output.parent.mkdir(parents=True, exist_ok=True)
    args.output.write_text(json.dumps(report, indent=2) + "\n")
    args.output.with_suffix(".md").write_text("\n".join(traces) + "\n")
    del parked


if __name__ == "__main__":
    main()
