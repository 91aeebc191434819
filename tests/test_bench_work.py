"""The algorithmic work bench.py divides by measured times to report its rooflines, recomputed here term by term
from the model's shapes (24 layers, d_model 1024, FF 4096, 8 heads of 128, 70-frame left context, 256
subsampling channels, joint 640) at the C3 batch: 256 streams x T = 14 frames from 121-row mel chunks."""

import importlib.util
from pathlib import Path
from types import SimpleNamespace

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


CFG = SimpleNamespace(d_model=1024, ff_dim=4096, sub_channels=256, joint_dim=640, n_layers=24, n_heads=8,
                      left_context=70)
N, T, R = 256, 14, 13


def test_gemm_flops_per_step(bench):
    D, F, M = 1024, 4096, N * T
    per_layer = 2 * M * (2 * F * D) * 2 + 2 * M * 3 * D * D + 2 * M * D * D + 2 * M * 2 * D * D + 2 * M * D * D
    # subsampling: 121 mel rows -> 61 -> 31 -> 16 time rows, 128 bins -> 65 -> 33 -> 17 frequency columns
    sub = N * 31 * 33 * 2 * 256 * 256 + N * 16 * 17 * 2 * 256 * 256 + N * 16 * 2 * (256 * 17) * D
    joint = 2 * M * D * 640
    assert bench.gemm_flops_per_step(N, T, R, CFG) == pytest.approx(24 * per_layer + sub + joint, rel=1e-12)
    assert bench.gemm_flops_per_step(N, T, R, CFG) == pytest.approx(4.234e12, rel=2e-3)


def test_bytes_per_kind(bench):
    b = bench.step_bytes_per_kind(N, T, CFG)
    item = 2 * (2 * 70 * 128 + 3 * T * 128 + T * 128 + 2 * T * 128)    # one (stream, head) of attention, bf16
    assert b["attention"] == 24 * N * 8 * item
    assert b["attention"] / 24 == pytest.approx(117.4e6, rel=1e-3)       # per launch
    assert b["conv"] / 24 == pytest.approx(N * 2 * (T * 2048 + T * 1024 + 2 * 8 * 1024), rel=1e-12)
    rows = N * T
    plain = (1 + 3 * 24) * rows * 6 * 1024                                 # fp32 row in, bf16 row out
    pair = 23 * rows * 10 * 1024 + rows * 8 * 1024                         # + the fp32 row written back
    assert b["norm"] == plain + pair
