"""The batched-torch form of the oracle step (oracle.stream_step.BatchEncoder, the CPU baseline at the
benchmark's batch) equals the per-stream oracle step stream by stream: the same projections to fp32 rounding and
the same caches, over a first chunk and two steady chunks of three streams."""

import numpy as np
import torch

from oracle.stream_step import BatchEncoder, Encoder, StreamState, chunk_plan
from oracle.weights import ModelDims, make_weights


def test_batched_oracle_equals_per_stream_oracle():
    dims = ModelDims(n_layers=2)
    sd = make_weights(dims, seed=5)
    enc, benc = Encoder(sd, dims), BatchEncoder(sd, dims)
    R, B = 13, 3
    mels = torch.randn(B, 400, 128, generator=torch.Generator().manual_seed(8))
    sts = [StreamState(dims) for _ in range(B)]
    bsts = [StreamState(dims) for _ in range(B)]
    for start, n, valid, keep_all in list(chunk_plan(400, R))[:3]:
        got = benc.batch_step(bsts, mels[:, start:start + n], n, valid, R)
        for b in range(B):
            ref, keep, *_ = enc.stream_step(sts[b], mels[b, start:start + n], n, valid, keep_all, R)
            assert got.shape[1] == keep
            assert float((got[b] - ref).abs().max() / ref.abs().max()) < 1e-5
            for li in range(dims.n_layers):
                assert torch.allclose(bsts[b].k[li], sts[b].k[li], rtol=1e-5, atol=1e-5)
                assert torch.allclose(bsts[b].conv[li], sts[b].conv[li], rtol=1e-5, atol=1e-5)
            assert (bsts[b].cache_len, bsts[b].step) == (sts[b].cache_len, sts[b].step)
