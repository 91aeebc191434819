"""The host-side batched streamer (ud_streamer_*, NemotronStreamer.swift:16-163) on the GPU.

  * buffered streams of different lengths: each stream's tokens equal the oracle run stream by stream
    (runBuffered's chunk walk, Encoder.stream_step, then RNNT.greedy with carried state);
  * the same streams fed row by row in random increments (live input) give the same tokens;
  * admission: opening more streams than the engine has slots is refused as a status, and a slot freed by a
    finished stream is reused;
  * a short final tail is zero-extended and masked (end padding, the default) or dropped (end padding off);
  * audio streams (NemotronStreamer.push(samples:) / flush()): the GPU mel frontend feeds the chunk walk; tokens
    equal the oracle pipeline (oracle mel, drainChunks, encoder, greedy), and audio pushed in random sizes gives
    exactly the tokens of the whole utterance pushed at once;
  * emission records (Emission: token, samples seen, compute seconds) and per-stream step wall times: one record
    per token, samples seen = the input received before the emitting step, one wall time per chunk run.
The model is 2 layers with subsampling and a 1-layer prediction net (fp32 engine, 1e-4 tolerance class); the
joint is sharpened so that token choices are decided by clear logit margins."""

import random

import numpy as np
import pytest
import torch

import ud
from oracle.rnnt import RNNT, DecoderState
from oracle.mel import features as mel_features
from oracle.mel import hann_symmetric, slaney_filterbank
from oracle.stream_step import Encoder, StreamState, live_plan
from oracle.weights import ModelDims, make_weights, sharpen_joint

pytestmark = pytest.mark.gpu

R = 6
LENGTHS = [500, 57, 230, 131, 9, 117]   # a stream whose only chunk is its first, a 1-chunk remainder, a 3-row tail


@pytest.fixture(scope="module")
def model():
    dims = ModelDims(n_layers=2)
    sd = sharpen_joint(make_weights(dims, seed=2), dims, 11)
    eng = ud.Engine(ud.default_config(n_layers=2, dtype=ud.DTYPE_F32, max_streams=4, max_batch=4))
    eng.load_weights(sd)
    yield eng, sd, dims
    eng.close()


def _mels():
    return [torch.randn(n, 128, generator=torch.Generator().manual_seed(100 + i)).numpy()
            for i, n in enumerate(LENGTHS)]


def _oracle_tokens(sd, dims, mel: np.ndarray, end_padding: bool = True) -> list[int]:
    enc, dec = Encoder(sd, dims), RNNT(sd, dims)
    st, ds = StreamState(dims), DecoderState(dims)
    toks: list[int] = []
    m = torch.from_numpy(np.ascontiguousarray(mel, np.float32))
    for start, n, valid, keep_all in live_plan(mel.shape[0], R, end_padding):
        rows = torch.zeros(n, m.shape[1])
        rows[:valid] = m[start:start + valid]
        proj, keep, *_ = enc.stream_step(st, rows, n, valid, keep_all, R)
        if keep:
            toks += dec.greedy(proj, ds)
    return toks


def _run(eng, mels, live: bool, seed: int = 0, end_padding: bool = True, pipelined: bool = False) -> list[list[int]]:
    """Admits streams as slots allow (4 of them), feeds them buffered or in random increments, steps until all
    are done; returns tokens per stream in input order."""
    s = ud.Streamer(eng, R, decode=True)
    s.set_end_padding(end_padding)
    s.set_pipelined(pipelined)
    rng = random.Random(seed)
    try:
        pending = list(range(len(mels)))
        active: dict[int, int] = {}        # streamer id -> input index
        fed = [0] * len(mels)
        out: dict[int, list[int]] = {}
        while pending or active:
            while pending and len(active) < 4:
                i = pending.pop(0)
                active[s.open(mels[i])] = i
            for sid, i in active.items():
                if fed[i] < len(mels[i]):
                    n = len(mels[i]) - fed[i] if not live else min(len(mels[i]) - fed[i], rng.randint(1, 80))
                    fed[i] += n
                    s.push(sid, n, last=fed[i] == len(mels[i]))
            s.step()
            done = s.finished()
            for sid in list(active):
                toks, fin = s.tokens(sid)
                assert fin == (sid in done)
                if fin:
                    i = active.pop(sid)
                    em = s.emissions(sid)
                    assert [t for t, _, _ in em] == toks
                    assert all(c > 0 for _, _, c in em)
                    if not live:   # every row was pushed before the first step
                        assert all(ss == 160 * len(mels[i]) for _, ss, _ in em)
                    out[i] = toks
                    s.release(sid)
        return [out[i] for i in range(len(mels))]
    finally:
        s.close()


@pytest.mark.parametrize("end_padding", [True, False])
def test_buffered_streams_match_the_oracle(model, end_padding):
    eng, sd, dims = model
    mels = _mels()
    got = _run(eng, mels, live=False, end_padding=end_padding)
    for i, mel in enumerate(mels):
        assert got[i] == _oracle_tokens(sd, dims, mel, end_padding), i
    assert any(len(t) > 0 for t in got)


def test_live_increments_equal_buffered(model):
    eng, _, _ = model
    mels = _mels()
    assert _run(eng, mels, live=True, seed=3) == _run(eng, mels, live=False)


@pytest.mark.parametrize("live", [False, True], ids=["buffered", "live"])
def test_pipelined_steps_equal_synchronous(model, live):
    """ud_streamer_set_pipelined: every stream's tokens equal the synchronous streamer's (results arrive a step
    later; admission, live feeding and release follow them)."""
    eng, _, _ = model
    mels = _mels()
    assert _run(eng, mels, live=live, seed=4, pipelined=True) == _run(eng, mels, live=live, seed=4)


def test_pipelined_mode_switched_off_mid_stream(model):
    """Leaving the pipelined mode completes the step in flight; the tokens of streams that ran part of their
    chunks pipelined and the rest synchronously equal the all-synchronous run."""
    eng, _, _ = model
    mels = _mels()[:3]
    ref = _run(eng, mels, live=False)
    s = ud.Streamer(eng, R, decode=True)
    try:
        s.set_pipelined(True)
        ids = [s.open(m) for m in mels]
        for sid, m in zip(ids, mels):
            s.push(sid, len(m), last=True)
        s.step()
        s.step()
        s.set_pipelined(False)
        for _ in range(200):
            s.step()
            if all(s.tokens(i)[1] for i in ids):
                break
        assert [s.tokens(i)[0] for i in ids] == ref
    finally:
        s.close()


def test_pipelined_release_of_a_stream_in_flight(model):
    """Releasing a stream whose chunk is in flight completes that step first; the other streams' tokens are
    unchanged, and a stream finished by that completion is reported by the next step."""
    eng, _, _ = model
    mels = _mels()[:3]
    ref = _run(eng, mels, live=False)
    s = ud.Streamer(eng, R, decode=True)
    s.set_pipelined(True)
    try:
        ids = [s.open(m) for m in mels]
        for sid, m in zip(ids, mels):
            s.push(sid, len(m), last=True)
        s.step()                  # step 0 in flight
        s.release(ids[1])         # in that step: it completes first
        out, seen_done = {}, set()
        for _ in range(200):
            s.step()
            seen_done |= set(s.finished())
            for k in (0, 2):
                toks, fin = s.tokens(ids[k])
                if fin:
                    out[k] = toks
            if len(out) == 2:
                break
        assert out[0] == ref[0] and out[2] == ref[2]
        assert {ids[0], ids[2]} <= seen_done
    finally:
        s.close()


def test_admission_is_a_status_and_slots_are_reused(model):
    eng, _, _ = model
    s = ud.Streamer(eng, R, decode=True)
    try:
        mel = np.zeros((60, 128), np.float32)
        ids = [s.open(mel) for _ in range(4)]
        with pytest.raises(ud.EngineError) as ei:
            s.open(mel)
        assert ei.value.status == 5   # pool exhausted
        s.push(ids[0], 60, last=True)
        while not s.tokens(ids[0])[1]:
            s.step()
        s.release(ids[0])
        ids[0] = s.open(mel)          # the finished stream's slot is free again
        with pytest.raises(ud.EngineError):
            s.push(ids[1], 61)        # beyond the stream's buffer
    finally:
        s.close()


def _audio(n, seed):
    g = torch.Generator().manual_seed(seed)
    t = torch.arange(n, dtype=torch.float64) / 16000
    return (0.2 * torch.sin(2 * np.pi * (300 + 40 * seed) * t) + 0.05 * torch.randn(n, generator=g,
                                                                                    dtype=torch.float64)).float().numpy()


def _run_audio(eng, fe, audios, sizes=None, seed=0, pipelined=False):
    s = ud.Streamer(eng, R, decode=True)
    s.set_pipelined(pipelined)
    rng = random.Random(seed)
    try:
        ids = [s.open_audio(fe) for _ in audios]
        pos = [0] * len(audios)
        while any(p < len(a) for p, a in zip(pos, audios)):
            sel = [i for i in range(len(audios)) if pos[i] < len(audios[i])]
            chunks, last = [], []
            for i in sel:
                m = len(audios[i]) - pos[i] if sizes is None else min(len(audios[i]) - pos[i], rng.choice(sizes))
                chunks.append(audios[i][pos[i]:pos[i] + m])
                pos[i] += m
                last.append(pos[i] == len(audios[i]))
            s.push_audio([ids[i] for i in sel], chunks, last)
            s.step()
        for _ in range(64):
            n, _ = s.step()
            if all(s.tokens(i)[1] for i in ids):
                break
        out = []
        for k, i in enumerate(ids):
            toks, fin = s.tokens(i)
            assert fin
            em = s.emissions(i)
            assert [t for t, _, _ in em] == toks
            seen = [ss for _, ss, _ in em]
            assert seen == sorted(seen) and all(0 < x <= len(audios[k]) for x in seen)
            if sizes is None:   # the whole utterance was pushed before the first step
                assert all(x == len(audios[k]) for x in seen)
            out.append((toks, len(s.step_times(i))))
            s.release(i)
        return out
    finally:
        s.close()


def test_audio_streams_match_the_oracle_pipeline(model):
    eng, sd, dims = model
    fb, win = slaney_filterbank(), hann_symmetric()
    fe = ud.MelFrontend(eng, fb.numpy(), win.numpy(), max_streams=4)
    try:
        audios = [_audio(n, i) for i, n in enumerate([16000 * 3 + 77, 9000, 2500])]
        got = _run_audio(eng, fe, audios)
        for i, a in enumerate(audios):
            mel, _ = mel_features(torch.from_numpy(a), fb, win)    # NeMo streaming counts every frame as valid
            assert got[i][0] == _oracle_tokens(sd, dims, mel.numpy()), i
            assert got[i][1] == len(list(live_plan(mel.shape[0], R, True))), i   # one wall time per chunk
        assert any(len(t) > 0 for t, _ in got)
        live = _run_audio(eng, fe, audios, sizes=[1, 160, 333, 1600, 4000], seed=5)
        assert live == got
        assert _run_audio(eng, fe, audios, sizes=[1, 160, 333, 1600, 4000], seed=5, pipelined=True) == got
    finally:
        fe.close()
