"""Encoder parity on the GPU through the C ABI, against the CPU oracle on identical seeded inputs and weights.

Tolerances: fp32 max-relative 1e-4, bf16 2e-2, where relative = max-abs / max|ref|
(check_spec.py:210-213). The bf16 engine is compared with the oracle run on the same bf16-rounded GEMM
weights, so the bound measures the engine's activation precision. Caches are compared after every step."""

import numpy as np
import pytest
import torch

import ud
from oracle.rnnt import RNNT, DecoderState
from oracle.stream_step import Encoder, StreamState, chunk_plan
from oracle.weights import BLOCK1, NEMOTRON, ModelDims, make_weights, round_bf16

pytestmark = pytest.mark.gpu


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def cache_f32(eng, sid, layer, kind):
    a = eng.cache_read(sid, layer, kind)
    return bf16_bits_to_f32(a) if a.dtype == np.uint16 else a


# ---------------------------------------------------------------- config 1: one block, fp32, [70,0], 200 steps
@pytest.fixture(scope="module")
def block1():
    sd = make_weights(BLOCK1, seed=0)
    eng = ud.Engine(ud.default_config(n_layers=1, sub_channels=0, joint_dim=0, dtype=ud.DTYPE_F32, max_streams=2,
                                      max_batch=2, max_chunk_frames=4))
    eng.load_weights(sd)
    yield eng, sd
    eng.close()


def test_block1_matches_reference_fixture(block1, golden_dir):
    """The first 12 steps against tools/nemotron_ane.py's own outputs (tests/golden/block1_steps.npz)."""
    eng, _ = block1
    g = np.load(golden_dir / "block1_steps.npz")
    sid = eng.open(0)
    for t in range(g["x"].shape[0]):
        out, fr = eng.step(sid, g["x"][t], 1, 1, True)
        assert fr == 1
        assert rel(out, g["out"][t:t + 1]) < 1e-4, t
    n = int(g["cache_len"])
    assert rel(cache_f32(eng, sid, 0, 0)[70 - n:], g["k"]) < 1e-4
    assert rel(cache_f32(eng, sid, 0, 1)[70 - n:], g["v"]) < 1e-4
    assert rel(cache_f32(eng, sid, 0, 2), g["conv"]) < 1e-4
    eng.close_stream(sid)


def test_block1_200_steps_outputs_and_caches(block1):
    eng, sd = block1
    enc = Encoder(sd, BLOCK1)
    st = StreamState(BLOCK1)
    sid = eng.open(0)
    gen = torch.Generator().manual_seed(1)
    worst = 0.0
    for t in range(200):
        x = torch.randn(1, 1024, generator=gen)
        out, fr = eng.step(sid, x.numpy(), 1, 1, True)
        ref = enc.frames_step(st, x)
        worst = max(worst, rel(out, ref))
        assert worst < 1e-4, (t, worst)
        cl, head, step = eng.info(sid)
        assert (cl, head, step) == (st.cache_len, t + 1, t + 1)
        k = cache_f32(eng, sid, 0, 0)
        v = cache_f32(eng, sid, 0, 1)
        c = cache_f32(eng, sid, 0, 2)
        n = st.cache_len
        assert not k[:70 - n].any() and not v[:70 - n].any()   # unfilled slots read as zero
        assert rel(k[70 - n:], st.k[0, 70 - n:]) < 1e-4
        assert rel(v[70 - n:], st.v[0, 70 - n:]) < 1e-4
        assert rel(c, st.conv[0]) < 1e-4
    eng.close_stream(sid)


# ---------------------------------------------------------------- fp32 with subsampling + joint (tight check)
def test_fp32_two_layer_stream_with_subsampling():
    dims = ModelDims(n_layers=2)
    sd = make_weights(dims, seed=0)
    eng = ud.Engine(ud.default_config(n_layers=2, dtype=ud.DTYPE_F32, max_streams=2, max_batch=2))
    eng.load_weights(sd)
    enc = Encoder(sd, dims)
    for R, total, vf in [(1, 57, 57), (13, 369, 360)]:
        st = StreamState(dims)
        sid = eng.open(R)
        mel = torch.randn(total, 128, generator=torch.Generator().manual_seed(R))
        for start, n, valid, keep_all in chunk_plan(total, R, vf):
            chunk = mel[start:start + n]
            proj, frames = eng.step(sid, chunk.numpy(), n, valid, keep_all)
            ref, keep, *_ = enc.stream_step(st, chunk, n, valid, keep_all, R)
            assert frames == keep
            if keep:
                assert rel(proj, ref) < 1e-4
        eng.close_stream(sid)
    eng.close()


# ---------------------------------------------------------------- bf16: the 24-layer encoder at [70,1]
@pytest.fixture(scope="module")
def full24():
    sd = make_weights(NEMOTRON, seed=0)
    eng = ud.Engine(ud.default_config(max_streams=8, max_batch=8))
    eng.load_weights(sd)
    yield eng, sd
    eng.close()


def test_bf16_24_layers_70_1(full24, golden_dir):
    eng, sd = full24
    enc = Encoder(round_bf16(sd), NEMOTRON)
    st = StreamState(NEMOTRON)
    sid = eng.open(1)
    g = np.load(golden_dir / "stream_70_1_l24.npz")
    mel = torch.from_numpy(g["mel"])
    for i, (start, n, valid, keep_all) in enumerate(chunk_plan(mel.shape[0], 1)):
        chunk = mel[start:start + n]
        proj, frames = eng.step(sid, chunk.numpy(), n, valid, keep_all)
        ref, keep, *_ = enc.stream_step(st, chunk, n, valid, keep_all, 1)
        assert frames == keep == int(g[f"s{i}_keep"])
        assert rel(proj, ref) < 2e-2, i
        # and against the reference's own fp32 step (fp32 weights): the same bound holds
        assert rel(proj, g[f"s{i}_proj"]) < 2e-2, i
    for li in (0, 23):
        n = st.cache_len
        assert rel(cache_f32(eng, sid, li, 0)[70 - n:], st.k[li, 70 - n:]) < 2e-2
        assert rel(cache_f32(eng, sid, li, 2), st.conv[li]) < 2e-2
    eng.close_stream(sid)


def test_bf16_batched_ragged_streams_with_decode(full24):
    """Several streams in one batched call, joining at different steps (first chunks of 105 rows next to steady
    chunks of 121 rows), ending with short final chunks (keep_all, validT < T): every stream's projection matches
    the oracle at 2e-2, and the GPU greedy decoder reproduces the CPU decoder run on the GPU's own projections."""
    eng, sd = full24
    R = 13
    enc = Encoder(round_bf16(sd), NEMOTRON)
    dec = RNNT(sd, NEMOTRON)
    lengths = [369, 300, 250, 160]
    valid = [360, 300, 250, 150]
    join = [0, 0, 1, 2]
    ids = [eng.open(R) for _ in lengths]
    mels = [torch.randn(n, 128, generator=torch.Generator().manual_seed(10 + i)) for i, n in enumerate(lengths)]
    plans = [list(chunk_plan(n, R, vf)) for n, vf in zip(lengths, valid)]
    sts = [StreamState(NEMOTRON) for _ in lengths]
    dsts = [DecoderState(NEMOTRON) for _ in lengths]
    steps = max(j + len(p) for j, p in zip(join, plans))
    for k in range(steps):
        act = [i for i in range(len(lengths)) if join[i] <= k < join[i] + len(plans[i])]
        if not act:
            continue
        chunks, rows, vr, ka = [], [], [], []
        for i in act:
            start, n, v, keep_all = plans[i][k - join[i]]
            chunks.append(mels[i][start:start + n].numpy())
            rows.append(n)
            vr.append(v)
            ka.append(keep_all)
        projs, frames, toks = eng.step_batch([ids[i] for i in act], chunks, rows, vr, ka, decode=True)
        for j, i in enumerate(act):
            ref, keep, *_ = enc.stream_step(sts[i], torch.from_numpy(chunks[j]), rows[j], vr[j], ka[j], R)
            assert frames[j] == keep
            if keep:
                assert rel(projs[j], ref) < 2e-2, (k, i)
            cpu_toks = dec.greedy(torch.from_numpy(projs[j]), dsts[i])
            assert toks[j] == cpu_toks, (k, i)
    for sid in ids:
        eng.close_stream(sid)


def test_bf16_long_chunks_next_to_short_ones():
    """Chunks of more than 16 frames (lookahead 30: 31 frames per steady chunk) take the bf16 CUDA-core attention
    kernel instead of the tensor-core one; batched with a lookahead-1 stream in the same call, the batch is ragged
    from 2 to 31 frames. Both streams match the oracle at 2e-2 and their caches stay within the same bound."""
    dims = ModelDims(n_layers=2)
    sd = make_weights(dims, seed=4)
    eng = ud.Engine(ud.default_config(n_layers=2, max_streams=2, max_batch=2, max_chunk_frames=32))
    eng.load_weights(sd)
    enc = Encoder(round_bf16(sd), dims)
    las, lengths = [30, 1], [700, 90]
    ids = [eng.open(r) for r in las]
    mels = [torch.randn(n, 128, generator=torch.Generator().manual_seed(40 + i)) for i, n in enumerate(lengths)]
    plans = [list(chunk_plan(n, r)) for n, r in zip(lengths, las)]
    sts = [StreamState(dims) for _ in las]
    for k in range(max(len(p) for p in plans)):
        act = [i for i in range(2) if k < len(plans[i])]
        chunks, rows, vr, ka = [], [], [], []
        for i in act:
            start, n, v, keep_all = plans[i][k]
            chunks.append(mels[i][start:start + n].numpy())
            rows.append(n)
            vr.append(v)
            ka.append(keep_all)
        projs, frames, _ = eng.step_batch([ids[i] for i in act], chunks, rows, vr, ka)
        for j, i in enumerate(act):
            ref, keep, *_ = enc.stream_step(sts[i], torch.from_numpy(chunks[j]), rows[j], vr[j], ka[j], las[i])
            assert frames[j] == keep
            if keep:
                assert rel(projs[j], ref) < 2e-2, (k, i)
    for i, sid in enumerate(ids):
        n = sts[i].cache_len
        for li in (0, 1):
            assert rel(cache_f32(eng, sid, li, 0)[70 - n:], sts[i].k[li, 70 - n:]) < 2e-2
            assert rel(cache_f32(eng, sid, li, 2), sts[i].conv[li]) < 2e-2
        eng.close_stream(sid)
    eng.close()


def test_protocol_object_matches_batched_path(full24):
    """CudaNemotronEncoder.step (the NemotronEncoder mirror, one stream per call) gives the same result as
    the batched entry point for the same stream history."""
    eng, _ = full24
    sch = ud.NemotronSchedule(lookahead=6)
    a = ud.CudaNemotronEncoder(eng, sch)
    b_id = eng.open(6)
    mel = torch.randn(200, 128, generator=torch.Generator().manual_seed(3)).numpy()
    for start, n, v, keep_all in chunk_plan(200, 6):
        pa, fa = a.step(mel[start:start + n], n, v, keep_all)
        pb, fb, _ = eng.step_batch([b_id], [mel[start:start + n]], [n], [v], [keep_all])
        assert fa == fb[0]
        assert np.array_equal(pa, pb[0])
    a.close()
    eng.close_stream(b_id)


def test_errors_are_statuses_not_crashes(full24):
    eng, _ = full24
    with pytest.raises(ud.EngineError) as ei:
        eng.step(12345, np.zeros((9, 128), np.float32), 9, 9, False)
    assert ei.value.status == 4
    sid = eng.open(1)
    with pytest.raises(ud.EngineError) as ei:
        eng.step(sid, np.zeros((400, 128), np.float32), 400, 400, False)   # beyond max_chunk_frames
    assert ei.value.status == 1
    with pytest.raises(ud.EngineError) as ei:
        eng.step_batch([sid, sid], [np.zeros((9, 128), np.float32)] * 2, [9, 9], [9, 9], [False, False])
    assert ei.value.status == 1
    # the stream is untouched by the rejected calls
    assert eng.info(sid) == (0, 0, 0)
    eng.close_stream(sid)
