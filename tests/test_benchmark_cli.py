"""The benchmark command: flag validation and report schema on CPU (what the reference's preflight
reads, src/climbing_gym/preflight.py:62-143), and one tiny synthetic run on the GPU."""
import json

import pytest
import torch

from climbing_gym_b200 import benchmark
from climbing_gym_b200.config import LFM25SamplingConfig

PREFLIGHT_CONFIG_KEYS = ["model", "device", "output_tokens", "prompts_json", "cuda_graphs", "compile_decode", "fp8_mlp",
                         "fp8_kv", "fp8_lm_head", "adaptive_batching", "bf16_weight_packing", "max_prefill_tokens", "dtype"]
PREFLIGHT_SAMPLING_KEYS = ["return_logprobs", "temperature", "top_k", "top_p", "repetition_penalty", "behavior_topk"]


def parse(*argv):
    parser = benchmark.build_arg_parser()
    return parser, parser.parse_args(list(argv))


def test_reference_flags_are_accepted_with_reference_defaults():
    _, args = parse("--model", "/ckpt", "--output", "r.json")
    assert args.batches == [1, 32, 128] and args.prompt_tokens == 128 and args.output_tokens == 4096
    assert args.top_k == -1 and args.temperature == 1.0 and args.warmups == 1 and args.repeats == 2
    assert args.max_prefill_tokens == 4096 and not args.cuda_graphs and not args.fp8_kv
    _, args = parse("--model", "/ckpt", "--output", "r.json", "--cuda-graphs", "--fp8-mlp", "--fp8-kv", "--fp8-lm-head",
                    "--adaptive-batching", "--bf16-weight-packing", "--compile-decode", "--batches", "64", "256",
                    "--behavior-topk", "8", "--park-gib", "1.5", "--max-model-len", "8192")
    assert args.batches == [64, 256] and args.fp8_mlp and args.fp8_kv and args.behavior_topk == 8 and args.park_gib == 1.5


@pytest.mark.parametrize("argv,message", [
    (["--model", "/m", "--output", "o", "--batches", "0"], "must be positive"),
    (["--model", "/m", "--output", "o", "--park-gib", "-1"], "must be positive"),
    (["--output", "o"], "exactly one of --model and --synthetic"),
    (["--model", "/m", "--synthetic", "tiny", "--output", "o"], "exactly one of --model and --synthetic"),
    (["--model", "/m", "--output", "o", "--device", "cpu"], "no CPU path"),
    (["--model", "/m", "--output", "o", "--top-k", "0"], "--top-k must be -1 or positive"),
])
def test_bad_arguments_are_rejected(argv, message, capsys):
    parser, args = parse(*argv)
    with pytest.raises(SystemExit):
        benchmark.validate_args(parser, args)
    assert message in capsys.readouterr().err


def test_saved_prompts_are_validated(tmp_path, capsys):
    good, bad = tmp_path / "good.json", tmp_path / "bad.json"
    good.write_text(json.dumps({"prompts": [[5, 6, 7], [8]]}))
    bad.write_text(json.dumps({"prompts": [[5, -1]]}))
    parser, args = parse("--model", "/m", "--output", "o", "--prompts-json", str(good))
    assert benchmark.validate_args(parser, args) == [[5, 6, 7], [8]]
    parser, args = parse("--model", "/m", "--output", "o", "--prompts-json", str(bad))
    with pytest.raises(SystemExit):
        benchmark.validate_args(parser, args)
    assert "nonnegative integer token IDs" in capsys.readouterr().err


def test_report_carries_every_key_the_preflight_reads(tmp_path):
    prompts = tmp_path / "p.json"
    prompts.write_text(json.dumps({"prompts": [[1, 2, 3]]}))
    _, args = parse("--model", "/m", "--output", str(tmp_path / "r.json"), "--prompts-json", str(prompts), "--cuda-graphs")
    sampling = LFM25SamplingConfig(max_new_tokens=4, ignore_eos=True)
    report = benchmark.report_header(args, sampling, 132, [[1, 2, 3]], torch.device("cpu"))
    runs = [{"seconds": 2.0, "output_tokens": 8, "tokens_per_second": 4.0},
            {"seconds": 1.0, "output_tokens": 8, "tokens_per_second": 8.0}]
    report["batches"].append(benchmark.batch_result(2, runs, torch.device("cpu")))
    report = json.loads(json.dumps(report))  # must be JSON-serialisable as is
    assert report["engine"] == "native_lfm25" and report["max_model_len"] == 132
    assert all(key in report["config"] for key in PREFLIGHT_CONFIG_KEYS)
    assert all(key in report["sampling"] for key in PREFLIGHT_SAMPLING_KEYS)
    assert report["workload"]["kind"] == "representative" and len(report["workload"]["prompts_sha256"]) == 64
    assert report["workload"]["prompt_lengths"] == [3] and report["hardware"]["name"] == "cpu"
    entry = report["batches"][0]
    assert entry["batch_size"] == 2 and entry["median_tokens_per_second"] == 6.0
    assert {"peak_allocated_bytes", "peak_reserved_bytes", "runs"} <= set(entry)
    assert set(entry["runs"][0]) == {"seconds", "tokens_per_second", "output_tokens"}


def test_synthetic_prompts_have_the_requested_length():
    tokenizer = benchmark._IdTokenizer(4096)
    rows = benchmark.synthetic_prompts(tokenizer, 3, 50)
    assert [len(r) for r in rows] == [50, 50, 50] and rows[0] != rows[1]
    assert all(3 <= t < 4096 for r in rows for t in r)


@pytest.mark.gpu
def test_tiny_synthetic_benchmark_writes_report_and_traces(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    out = tmp_path / "bench" / "report.json"
    benchmark.main(["--synthetic", "tiny", "--batches", "2", "5", "--prompt-tokens", "24", "--output-tokens", "16",
                    "--repeats", "2", "--output", str(out)])
    report = json.loads(out.read_text())
    assert [b["batch_size"] for b in report["batches"]] == [2, 5]
    assert all(run["output_tokens"] == b["batch_size"] * 16 for b in report["batches"] for run in b["runs"])
    assert report["config"]["cuda_graphs"] is True and report["workload"]["kind"] == "synthetic"
    assert report["batches"][0]["peak_allocated_bytes"] > 0
    assert "Outcome: 16 tokens" in out.with_suffix(".md").read_text()
