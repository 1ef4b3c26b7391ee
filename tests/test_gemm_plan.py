"""The GEMM launcher's choice of kernel, tile and grid (cgym_gemm_plan: a pure function, no device needed),
pinned on the grids the decode step and the prefill were measured with, and on the one combination that is
closed: no CTA pairs above 256 rows inside a dependent-launch chain."""
import ctypes as C

import pytest

from climbing_gym_b200 import _native as nv

SINGLE, PAIR, PERSISTENT = 0, 1, 2


def plan(m, n, k, *, fp8=False, impl=0, chain=False):
    out = (C.c_int * 6)()
    nv.call("cgym_gemm_plan", m, n, k, int(fp8), impl, int(chain), C.addressof(out))
    kind, un, fm, splits, gx, gy = list(out)
    return dict(kind=kind, un=un, fm=fm, splits=splits, grid=(gx, gy))


@pytest.mark.parametrize("shape,fp8,want", [
    # a 256-row FP8 decode step (inside the captured graph)
    ((256, 16384, 2048), True, dict(kind=SINGLE, un=128, fm=1, splits=1, grid=(128, 2))),   # w13
    ((256, 2048, 8192), True, dict(kind=SINGLE, un=64, fm=1, splits=4, grid=(16, 4))),      # w2
    ((256, 2048, 2048), False, dict(kind=SINGLE, un=64, fm=1, splits=4, grid=(16, 4))),     # out-projections
    ((256, 6144, 2048), False, dict(kind=SINGLE, un=64, fm=1, splits=1, grid=(48, 4))),     # conv in-projection
    ((256, 3072, 2048), False, dict(kind=SINGLE, un=64, fm=1, splits=2, grid=(24, 4))),     # qkv
    ((256, 65536, 2048), False, dict(kind=PAIR, un=256, fm=1, splits=1, grid=(512, 1))),    # LM head
    # a 64-row bf16 decode step
    ((64, 16384, 2048), False, dict(kind=SINGLE, un=64, fm=1, splits=2, grid=(128, 1))),
    ((64, 2048, 8192), False, dict(kind=SINGLE, un=64, fm=1, splits=8, grid=(16, 1))),
    ((64, 2048, 2048), False, dict(kind=SINGLE, un=64, fm=1, splits=8, grid=(16, 1))),
    ((64, 6144, 2048), False, dict(kind=SINGLE, un=64, fm=1, splits=4, grid=(48, 1))),
    ((64, 3072, 2048), False, dict(kind=SINGLE, un=64, fm=1, splits=8, grid=(24, 1))),
    ((64, 65536, 2048), False, dict(kind=SINGLE, un=64, fm=1, splits=1, grid=(512, 1))),
    ((128, 2048, 2048), False, dict(kind=SINGLE, un=128, fm=1, splits=8, grid=(16, 1))),
    ((1, 2048, 2048), False, dict(kind=SINGLE, un=32, fm=1, splits=8, grid=(16, 1))),
    # a 512-row decode step: above 256 rows nothing inside the chain takes CTA pairs
    ((512, 16384, 2048), True, dict(kind=SINGLE, un=256, fm=2, splits=1, grid=(64, 2))),
    ((512, 2048, 2048), False, dict(kind=SINGLE, un=256, fm=1, splits=4, grid=(16, 2))),
    ((512, 65536, 2048), False, dict(kind=SINGLE, un=256, fm=1, splits=1, grid=(512, 2))),
])
def test_plans_inside_a_decode_step(shape, fp8, want):
    assert plan(*shape, fp8=fp8, chain=True) == want


@pytest.mark.parametrize("shape,want", [
    ((4096, 16384, 2048), dict(kind=PERSISTENT, un=256, fm=1, splits=1, grid=(128, 16))),  # w13: 1024 tiles
    ((4096, 6144, 2048), dict(kind=PERSISTENT, un=256, fm=1, splits=1, grid=(48, 16))),    # in-projection: 384 tiles
    ((4096, 3072, 2048), dict(kind=PERSISTENT, un=256, fm=1, splits=1, grid=(24, 16))),    # qkv: 192 tiles
    ((4096, 2048, 2048), dict(kind=PAIR, un=256, fm=1, splits=1, grid=(16, 16))),          # 128 tiles: under two rounds
    ((4096, 2048, 8192), dict(kind=SINGLE, un=256, fm=2, splits=1, grid=(8, 16))),         # w2: K above 4096
    ((512, 16384, 2048), dict(kind=PAIR, un=256, fm=1, splits=1, grid=(128, 2))),          # scoring-sized chunk
    ((300, 2000, 2048), dict(kind=SINGLE, un=256, fm=1, splits=4, grid=(16, 2))),          # N not a multiple of 256
])
def test_plans_of_prefill_and_scoring(shape, want):
    assert plan(*shape, chain=False) == want


def test_forced_forms_and_refusals():
    assert plan(40, 256, 4096, impl=3)["splits"] == 4
    assert plan(256, 256, 512, impl=4)["kind"] == PAIR and plan(256, 256, 512, impl=5)["kind"] == PERSISTENT
    with pytest.raises(nv.NativeKernelError, match="multiple of 256"):
        plan(64, 384, 512, impl=4)
    with pytest.raises(nv.NativeKernelError, match="impl"):
        plan(64, 256, 512, impl=1)
