"""CPU-side checks of the drop-in boundary: the shared library loads, exports every entry point
declared in include/cgym_b200.h, and rejects bad arguments with a message instead of launching."""
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def native():
    from climbing_gym_b200 import _native, build
    build.build()
    _native.load()
    return _native


def declared_entry_points():
    header = (ROOT / "include" / "cgym_b200.h").read_text()
    return sorted(set(re.findall(r"\b(cgym_[a-z0-9_]+)\s*\(", header)))


def test_header_and_binding_list_the_same_entry_points(native):
    declared = declared_entry_points()
    assert declared == native.exported_symbols()
    lib = native.load()
    for name in declared:
        assert hasattr(lib, name), f"{name} is declared but not exported"


def test_every_entry_point_cites_the_reference_or_says_it_has_no_counterpart():
    header = (ROOT / "include" / "cgym_b200.h").read_text()
    blocks = re.split(r"\n(?=/\*)", header)
    for block in blocks:
        names = re.findall(r"\bint (cgym_[a-z0-9_]+)\s*\(", block)
        if not names or names == ["cgym_version"] or "cgym_device_supported" in names:
            continue
        comment = block.split("*/")[0].lower()
        assert re.search(r"\.py:\d+", comment) or "no reference counterpart" in comment or "no counterpart" in comment, names


def test_version_and_argument_validation_without_a_gpu(native):
    lib = native.load()
    assert lib.cgym_version() == 1
    with pytest.raises(native.NativeKernelError, match="bad shape"):
        native.call("cgym_gemm", 1, 1, 1, None, 4, 0, 8, native.BF16, 1, None, 0, None, None)
    with pytest.raises(native.NativeKernelError, match="row width"):
        native.call("cgym_quantize_rows", 1, 1, 1, 2, 40000, native.BF16, None)
    with pytest.raises(native.NativeKernelError, match="head_dim"):
        import ctypes as C
        kv = native.KVLayout(None, None, None, 4, 16, 4, 2, 48, native.BF16)
        native.call("cgym_paged_attention", 1, 1, 1, None, None, C.byref(kv), 0, 1, 4, 1.0, 1, None, native.BF16, 0,
                    None, None)


def test_engine_refuses_to_run_without_cuda():
    import torch
    from climbing_gym_b200 import synthetic
    from climbing_gym_b200.weights import LFM25PackedWeights
    if torch.cuda.is_available():
        pytest.skip("this check is for machines without a GPU")
    from climbing_gym_b200.engine import LFM25Engine
    cfg = synthetic.tiny_config()
    state = {k: torch.from_numpy(v) for k, v in synthetic.make_state_dict(cfg).items()}
    weights = LFM25PackedWeights.from_state_dict(cfg, state, device=torch.device("cpu"), dtype=torch.float32)
    with pytest.raises(RuntimeError, match="no CPU path"):
        LFM25Engine(weights)
