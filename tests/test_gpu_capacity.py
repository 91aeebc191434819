"""The north star's capacity target on one GPU: 4096 concurrent [70,13] streams in one engine (24 layers, bf16),
every stream stepped in one batched call (M = 57,344 encoder rows per projection, 4096 x 8 attention items, a
page pool of 28,672 pages of 16 frames per layer: about 44 GB of K/V rings). Two steps (the first chunk of 105 mel
rows, then a steady chunk of 121 rows) for all streams; four streams spread over the batch are compared with the
oracle (FastConformer.swift:441-480 restated, the same bf16-rounded GEMM weights) at the bf16 bound, 2e-2
max-relative, and the pool accounting is checked against the per-stream page bound."""

import numpy as np
import pytest
import torch

import ud
from oracle.stream_step import Encoder, StreamState, chunk_plan
from oracle.weights import NEMOTRON, make_weights, round_bf16

pytestmark = pytest.mark.gpu

R, N = 13, 4096
PICK = [0, 1365, 2730, 4095]


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


def test_4096_streams_on_one_gpu():
    sd = make_weights(NEMOTRON, seed=0)
    eng = ud.Engine(ud.default_config(max_streams=N, max_batch=N))
    try:
        eng.load_weights(sd)
        free0, total, esz = eng.pool_info()
        assert total == N * 7 and free0 == total   # 7 pages of 16 frames per stream slot (70 + 16 frames + slack)
        ids = [eng.open(R) for _ in range(N)]
        gen = np.random.default_rng(11)
        mels = gen.standard_normal((N, 226, 128), dtype=np.float32)
        plan = list(chunk_plan(226, R))[:2]
        enc = Encoder(round_bf16(sd), NEMOTRON)
        sts = {s: StreamState(NEMOTRON) for s in PICK}
        for start, rows, valid, keep_all in plan:
            chunks = [mels[s, start:start + rows] for s in range(N)]
            projs, frames, _ = eng.step_batch(ids, chunks, [rows] * N, [valid] * N, [keep_all] * N)
            assert all(f == R + 1 for f in frames)
            for s in PICK:
                ref, keep, *_ = enc.stream_step(sts[s], torch.from_numpy(chunks[s]), rows, valid, keep_all, R)
                assert keep == R + 1
                assert rel(projs[s], ref) < 2e-2, s
        # 28 frames appended per stream: two pages each are mapped
        free1, _, _ = eng.pool_info()
        assert total - free1 == 2 * N
        for s in PICK:
            assert eng.info(ids[s]) == (28, 28, 2)
    finally:
        eng.close()
