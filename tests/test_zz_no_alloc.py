"""ud_rnnt_decode_static (scratch in the library's static device block, no allocation in the call) against
ud_rnnt_decode on the same engine: two streams with identical weights and inputs, one decoded through each entry
point, two calls in a row with the decoder state carried between them; plus the size limit, and that a warm call
leaves the device's free memory unchanged. Every decoder kernel is covered: the tensor-core lock-step one
(UD_RNNT_TC=1 puts every batch size on it; by default it takes batches of 20 streams and up), the fp32 lock-step one
(UD_RNNT_TC=0) and one CTA per stream (UD_RNNT_LOCKSTEP=0); the variables are read when the engine is created. Collected last so it also runs after every other GPU test in one process."""

import numpy as np
import pytest
import torch

import ud
from oracle.rnnt import RNNT
from oracle.weights import ModelDims, make_weights, sharpen_joint

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("lockstep,tc", [("1", "1"), ("1", "0"), ("0", "0")], ids=["tensor", "lockstep", "per_stream"])
def test_static_scratch_decode_matches_existing_entry_point(lockstep, tc, monkeypatch):
    monkeypatch.setenv("UD_RNNT_LOCKSTEP", lockstep)
    monkeypatch.setenv("UD_RNNT_TC", tc)
    dims = ModelDims(n_layers=0, sub_channels=0, pred_layers=2)
    sd = sharpen_joint(make_weights(dims, seed=3), dims, 77)
    e = ud.Engine(ud.default_config(n_layers=0, sub_channels=0, pred_layers=2, max_streams=8, max_batch=8,
                                    max_chunk_frames=16,
                                    dtype=ud.DTYPE_F32))
    try:
        e.load_weights(sd)
        f = RNNT(sd, dims).enc_proj(torch.randn(60, dims.d_model, generator=torch.Generator().manual_seed(5))).numpy()
        a, b = e.open(1), e.open(1)
        for chunk in (f[:37], f[37:]):
            ref = e.rnnt_decode(a, chunk)
            got = e.rnnt_decode_static(b, chunk)
            assert got == ref
            assert len(ref) > 0
        # 100 frames of 640 joint features and 10 symbols fill the 256 KiB block; one more is refused.
        big = np.zeros((101, dims.joint_dim), np.float32)
        with pytest.raises(ud.EngineError):
            e.rnnt_decode_static(b, big)
        assert e.rnnt_decode_static(b, big[:100]) == e.rnnt_decode(a, big[:100])
        # A warm call takes no device memory: the device's free bytes are the same before and after.
        c = e.open(1)
        e.rnnt_decode_static(c, f[:20])
        torch.cuda.synchronize(e.device)
        free0 = torch.cuda.mem_get_info(e.device)[0]
        e.rnnt_decode_static(c, f[20:40])
        torch.cuda.synchronize(e.device)
        assert torch.cuda.mem_get_info(e.device)[0] == free0
    finally:
        e.close()
