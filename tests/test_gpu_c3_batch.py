"""Parity at the benchmark's own batch (configuration C3): 256 streams through the 24-layer bf16 encoder at [70,13],
14 frames per stream and step, so every projection is one GEMM over M = 3584 rows and takes the 2-CTA tcgen05
kernel with its TMA-store (bf16 outputs) and TMA reduce-add (x += s * f(h W^T)) epilogues, the attention and
conv-module grids run 256 streams wide, and the page pool holds 256 streams' rings. The steps run as the bench
runs them: the first two eagerly, later ones as replays of the captured CUDA graph with programmatic dependent
launch between the kernels.

Four steps: the first chunk (105 mel rows), two steady chunks (121 rows), then, after 5% of the streams are
evicted (fresh caches, same ids), a step where the evicted streams take a first chunk next to everyone else's
steady chunk. Eight streams spread over the batch (two of them evicted) are compared with the oracle
(FastConformer.swift:441-480 restated, the same bf16-rounded GEMM weights) at the north star's bf16 bound, 2e-2
max-relative, after every step, and their K, V and conv caches of layers 0 and 23 after the last one."""

import numpy as np
import pytest
import torch

import ud
from oracle.stream_step import Encoder, StreamState, chunk_plan
from oracle.weights import NEMOTRON, make_weights, round_bf16

pytestmark = pytest.mark.gpu

R, N, ROWS = 13, 256, 500
PICK = [0, 37, 74, 111, 148, 185, 222, 255]


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def test_c3_batch_256_streams_24_layers():
    sd = make_weights(NEMOTRON, seed=0)
    eng = ud.Engine(ud.default_config(max_streams=N, max_batch=N))
    try:
        eng.load_weights(sd)
        enc = Encoder(round_bf16(sd), NEMOTRON)
        ids = [eng.open(R) for _ in range(N)]
        mels = np.stack([torch.randn(ROWS, 128, generator=torch.Generator().manual_seed(1000 + s)).numpy()
                         for s in range(N)])
        plan = list(chunk_plan(ROWS, R))
        assert plan[0][1] == 105 and plan[1][1] == 121
        rng = np.random.default_rng(7)
        evict = sorted(set(rng.choice([s for s in range(N) if s not in PICK], size=N // 20 - 2, replace=False).tolist())
                       | {PICK[1], PICK[5]})
        assert len(evict) == N // 20
        pos = {s: 0 for s in range(N)}          # next chunk of each stream
        sts = {s: StreamState(NEMOTRON) for s in PICK}

        def step():
            chunks, rows, vr, ka = [], [], [], []
            for s in range(N):
                start, n, v, keep_all = plan[pos[s]]
                chunks.append(mels[s, start:start + n])
                rows.append(n)
                vr.append(v)
                ka.append(keep_all)
            projs, frames, _ = eng.step_batch(ids, chunks, rows, vr, ka)
            assert all(f == 14 for f in frames)
            out = {}
            for s in PICK:
                ref, keep, *_ = enc.stream_step(sts[s], torch.from_numpy(chunks[s]), rows[s], vr[s], ka[s], R)
                assert frames[s] == keep == 14
                out[s] = rel(projs[s], ref)
            for s in range(N):
                pos[s] += 1
            return out

        for k in range(3):
            errs = step()
            assert max(errs.values()) < 2e-2, (k, errs)
        eng.cache_evict([ids[s] for s in evict])
        for s in evict:
            pos[s] = 0
            if s in sts:
                sts[s] = StreamState(NEMOTRON)
        errs = step()
        assert max(errs.values()) < 2e-2, (3, errs)
        for s in PICK:
            n = sts[s].cache_len
            assert eng.info(ids[s])[0] == n == (14 if s in evict else 56)
            for li in (0, 23):
                k = bf16_bits_to_f32(eng.cache_read(ids[s], li, 0))
                v = bf16_bits_to_f32(eng.cache_read(ids[s], li, 1))
                c = bf16_bits_to_f32(eng.cache_read(ids[s], li, 2))
                assert not k[:70 - n].any() and not v[:70 - n].any()
                assert rel(k[70 - n:], sts[s].k[li, 70 - n:]) < 2e-2, (s, li)
                assert rel(v[70 - n:], sts[s].v[li, 70 - n:]) < 2e-2, (s, li)
                assert rel(c, sts[s].conv[li]) < 2e-2, (s, li)

        # The same batch shape dispatches every projection to the 2-CTA kernel: 8 per layer, the two subsampling
        # pointwise convolutions, the subsampling output and joint.enc, none to the 1-CTA kernel.
        eng.profile(True)
        chunks = [mels[s, plan[pos[s]][0]:plan[pos[s]][0] + plan[pos[s]][1]] for s in range(N)]
        eng.step_batch(ids, chunks, [plan[pos[s]][1] for s in range(N)], [plan[pos[s]][2] for s in range(N)],
                       [False] * N)
        prof = eng.profile_read()
        eng.profile(False)
        assert prof["gemm_tc2"][1] == 24 * 8 + 4, prof
        assert prof["gemm_tc"][1] == 0 and prof["gemm_simt"][1] == 0, prof
    finally:
        eng.close()
