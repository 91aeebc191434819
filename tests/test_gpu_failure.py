"""Failure detection without a GPU fault: a device-side wait on a flag that nothing sets gives up after its limit,
the call returns UD_ERR_DEVICE_TIMEOUT, and the engine (and its CUDA context) stays usable."""

import time

import pytest
import torch

import ud

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_engine_survives():
    e = ud.Engine(ud.default_config(n_layers=0, sub_channels=0, joint_dim=0, max_streams=1, max_batch=1))
    try:
        t0 = time.time()
        with pytest.raises(ud.EngineError) as ei:
            ud.wait_probe(e, 50_000_000)          # 50 ms
        assert ei.value.status == 8
        assert time.time() - t0 < 10
        # the error word was cleared and the context works: a GEMM after the probe is correct
        A = torch.ones(64, 1024, device="cuda", dtype=torch.bfloat16)
        W = torch.ones(256, 1024, device="cuda", dtype=torch.bfloat16)
        C = torch.empty(64, 256, device="cuda")
        torch.cuda.synchronize()
        e.debug_gemm(A.data_ptr(), W.data_ptr(), 64, 256, 1024, C.data_ptr())
        assert torch.all(C == 1024.0)
        e.synchronize()
    finally:
        e.close()
