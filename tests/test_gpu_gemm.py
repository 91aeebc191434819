"""GEMM kernels through the C ABI (ud_debug_gemm) against a float64 reference of the same bf16/fp32 inputs.

Contract and shapes follow the reference's Tests/DictatorEngineTests/GemmTests.swift: shapes `:34`, fp32
tolerance 1e-4*sqrt(K) + 1e-5 absolute on inputs in [-1, 1) (`:43`), full epilogue (bias, activation, output
scale, residual with scale, `:66-91`). The engine shapes (M = streams x T up to 3584, N in {256, 640, 1024, 2048,
3072, 4096}, K in {256, 1024, 4096, 4352}) exercise both tcgen05 tile widths (BN 128 and 256)."""

import os

import numpy as np
import pytest
import torch

import ud

pytestmark = pytest.mark.gpu

REF_SHAPES = [(1, 1, 1), (1, 1024, 1024), (7, 33, 65), (64, 64, 64), (100, 257, 130), (129, 640, 1024), (3, 4096, 1024)]
TC_SHAPES = [(17, 256, 256), (129, 640, 1024), (200, 3072, 1024), (333, 2048, 1024), (448, 1024, 4352),
             (1024, 4096, 1024), (3584, 1024, 4096), (3584, 4096, 1024),
             # shapes whose tile widths are not 256 (last tiles of 192, 128-wide tiles, 16-column remainders)
             (3584, 1024, 1024), (3584, 640, 1024), (3584, 3072, 1024), (3584, 2048, 1024), (300, 1040, 512),
             (2000, 1040, 256)]


@pytest.fixture(scope="module", params=["bf16", "bf16-1cta", "f32"])
def eng(request):
    """bf16: tcgen05 with 2-CTA pairs where M >= 256 and N % 256 == 0; bf16-1cta: the one-CTA kernel only;
    f32: the FFMA kernels."""
    if request.param == "bf16-1cta":
        os.environ["UD_TC2"] = "0"
    try:
        e = ud.Engine(ud.default_config(n_layers=0, sub_channels=0, joint_dim=0, max_streams=1, max_batch=1,
                                        dtype=ud.DTYPE_F32 if request.param == "f32" else ud.DTYPE_BF16))
    finally:
        os.environ.pop("UD_TC2", None)
    yield e
    e.close()


def _gemm(eng, *args, **kw):
    # The engine works on its own CUDA stream; torch-made operands must be complete before the call.
    torch.cuda.synchronize()
    eng.debug_gemm(*args, **kw)


def _inputs(M, N, K, dt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = (torch.rand(M, K, device="cuda", generator=g) * 2 - 1).to(dt)
    W = (torch.rand(N, K, device="cuda", generator=g) * 2 - 1).to(dt)
    return A.contiguous(), W.contiguous()


@pytest.mark.parametrize("shape", REF_SHAPES + TC_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_plain_gemm(eng, shape):
    M, N, K = shape
    if eng.cfg.dtype == ud.DTYPE_F32 and M * N * K > 2e9:
        pytest.skip("large fp32 shapes exercise the same FFMA kernel")
    dt = torch.bfloat16 if eng.cfg.dtype == ud.DTYPE_BF16 else torch.float32
    A, W = _inputs(M, N, K, dt, 1)
    C = torch.empty(M, N, device="cuda", dtype=torch.float32)
    _gemm(eng, A.data_ptr(), W.data_ptr(), M, N, K, C.data_ptr())
    ref = (A.double() @ W.double().T)
    tol = 1e-4 * K ** 0.5 + 1e-5
    assert (C.double() - ref).abs().max().item() < tol


@pytest.mark.parametrize("shape", [(5, 640, 1024), (129, 1024, 1024), (3584, 4096, 1024), (300, 2048, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("act", [0, 1, 2], ids=["none", "relu", "silu"])
def test_full_epilogue(eng, shape, act):
    M, N, K = shape
    dt = torch.bfloat16 if eng.cfg.dtype == ud.DTYPE_BF16 else torch.float32
    A, W = _inputs(M, N, K, dt, 2)
    g = torch.Generator(device="cuda").manual_seed(3)
    bias = torch.rand(N, device="cuda", generator=g) - 0.5
    R = torch.rand(M, N, device="cuda", generator=g) - 0.5
    C = torch.empty(M, N, device="cuda", dtype=torch.float32)
    _gemm(eng, A.data_ptr(), W.data_ptr(), M, N, K, C.data_ptr(), bias_ptr=bias.data_ptr(), act=act,
                   out_scale=0.5, res_ptr=R.data_ptr(), res_scale=0.75)
    z = A.double() @ W.double().T + bias.double()
    z = torch.relu(z) if act == 1 else (z * torch.sigmoid(z) if act == 2 else z)
    ref = 0.5 * z + 0.75 * R.double()
    assert (C.double() - ref).abs().max().item() < 1e-4 * K ** 0.5 + 1e-5


def test_residual_in_place_and_bf16_output(eng):
    if eng.cfg.dtype != ud.DTYPE_BF16:
        pytest.skip("bf16 output is the bf16 engine's activation path")
    M, N, K = 777, 3072, 1024
    A, W = _inputs(M, N, K, torch.bfloat16, 4)
    X = torch.rand(M, N, device="cuda") - 0.5
    X0 = X.clone()
    _gemm(eng, A.data_ptr(), W.data_ptr(), M, N, K, X.data_ptr(), res_ptr=X.data_ptr())
    ref = A.double() @ W.double().T + X0.double()
    assert (X.double() - ref).abs().max().item() < 1e-4 * K ** 0.5 + 1e-5
    Cb = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    _gemm(eng, A.data_ptr(), W.data_ptr(), M, N, K, Cb.data_ptr(), act=2, out_bf16=True)
    z = A.double() @ W.double().T
    ref = (z * torch.sigmoid(z))
    err = (Cb.double() - ref).abs() / (ref.abs() + 1e-2)
    assert err.max().item() < 1e-2


@pytest.mark.parametrize("shape", [(3584, 1024, 4096), (777, 1024, 1024), (300, 2048, 1024), (2000, 1040, 256)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("act", [0, 2], ids=["none", "silu"])
def test_in_place_residual_equals_separate_residual(eng, shape, act):
    """x += 0.5 * act(A W^T + bias) in place (the encoder's residual form; on the 2-CTA kernel with 256-wide
    tiles an fp32 reduce-add into x) is bit-identical to the same epilogue with a separate residual buffer and
    output (the register epilogue), and within the GEMM tolerance of a float64 reference."""
    M, N, K = shape
    dt = torch.bfloat16 if eng.cfg.dtype == ud.DTYPE_BF16 else torch.float32
    A, W = _inputs(M, N, K, dt, 6)
    g = torch.Generator(device="cuda").manual_seed(7)
    bias = torch.rand(N, device="cuda", generator=g) - 0.5
    X = (torch.rand(M, N, device="cuda", generator=g) - 0.5) * 4
    R = X.clone()
    C = torch.empty(M, N, device="cuda")
    _gemm(eng, A.data_ptr(), W.data_ptr(), M, N, K, C.data_ptr(), bias_ptr=bias.data_ptr(), act=act, out_scale=0.5,
          res_ptr=R.data_ptr())
    _gemm(eng, A.data_ptr(), W.data_ptr(), M, N, K, X.data_ptr(), bias_ptr=bias.data_ptr(), act=act, out_scale=0.5,
          res_ptr=X.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(X, C)
    z = A.double() @ W.double().T + bias.double()
    z = z * torch.sigmoid(z) if act == 2 else z
    assert (X.double() - (0.5 * z + R.double())).abs().max().item() < 1e-4 * K ** 0.5 + 1e-5


def test_repeatable_and_counts_launches(eng):
    M, N, K = 512, 1024, 1024
    dt = torch.bfloat16 if eng.cfg.dtype == ud.DTYPE_BF16 else torch.float32
    A, W = _inputs(M, N, K, dt, 5)
    C1 = torch.empty(M, N, device="cuda")
    C2 = torch.empty(M, N, device="cuda")
    n0 = eng.launch_count()
    _gemm(eng, A.data_ptr(), W.data_ptr(), M, N, K, C1.data_ptr())
    _gemm(eng, A.data_ptr(), W.data_ptr(), M, N, K, C2.data_ptr())
    assert eng.launch_count() == n0 + 2
    assert torch.equal(C1, C2)
