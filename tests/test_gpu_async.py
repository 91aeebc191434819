"""Pipelined host-buffer steps (ud_step_batch_async / ud_step_sync) on the GPU.

  * the same stream histories run through ud_step_batch and through ud_step_batch_async give bit-identical
    projections and tokens, with the input given as one pinned block at a fixed stride (direct DMA) and as
    separate per-stream arrays (gathered through the pinned staging buffer);
  * on return, a call has completed the previous step (its outputs are in place); ud_step_sync completes the
    last one;
  * synchronous calls after asynchronous ones see a drained pipeline (same results as an all-synchronous run);
  * a rejected call is a status, and the engine stays usable.
The model is 2 bf16 layers with subsampling, joint and a 1-layer prediction net."""

import numpy as np
import pytest
import torch

import ud
from oracle.stream_step import chunk_plan
from oracle.weights import ModelDims, make_weights, sharpen_joint

pytestmark = pytest.mark.gpu

R = 13
LENGTHS = [369, 300, 250, 160, 121, 105]


@pytest.fixture(scope="module")
def model():
    dims = ModelDims(n_layers=2)
    sd = sharpen_joint(make_weights(dims, seed=5), dims, 11)
    eng = ud.Engine(ud.default_config(n_layers=2, max_streams=16, max_batch=8))
    eng.load_weights(sd)
    yield eng
    eng.close()


def _mels():
    return [torch.randn(n, 128, generator=torch.Generator().manual_seed(300 + i)) for i, n in enumerate(LENGTHS)]


def _steps():
    """Per step: the active streams and their (start, rows, valid, keep_all) (streams end at different steps)."""
    plans = [list(chunk_plan(n, R)) for n in LENGTHS]
    out = []
    for k in range(max(len(p) for p in plans)):
        out.append([(i, plans[i][k]) for i in range(len(LENGTHS)) if k < len(plans[i])])
    return out


def _run_sync(eng, mels):
    ids = [eng.open(R) for _ in LENGTHS]
    res = []
    for act in _steps():
        projs, frames, toks = eng.step_batch([ids[i] for i, _ in act],
                                             [mels[i][st:st + n].numpy() for i, (st, n, v, ka) in act],
                                             [p[1] for _, p in act], [p[2] for _, p in act],
                                             [p[3] for _, p in act], decode=True)
        res.append(([p.copy() for p in projs], frames, toks))
    for sid in ids:
        eng.close_stream(sid)
    return res


def _run_async(eng, mels, pinned_block: bool):
    tm, W, ms = eng.cfg.max_chunk_frames, eng.out_width, eng.cfg.max_symbols
    n_max = len(LENGTHS)
    if pinned_block:
        rows = max(LENGTHS)
        blk = torch.zeros(n_max, rows, 128, pin_memory=True)
        for i, m in enumerate(mels):
            blk[i, :m.shape[0]] = m
        src = blk.numpy()
    outs = [torch.empty(n_max, tm, W, pin_memory=True).numpy() for _ in range(2)]
    toks = [torch.empty(n_max, tm * ms, dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]
    ntoks = [torch.empty(n_max, dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]
    ids = [eng.open(R) for _ in LENGTHS]
    res, pending = [], None

    def collect(p):
        k, act, frames = p
        b = k % 2
        projs = [outs[b][j, :frames[j]].copy() for j in range(len(act))]
        tl = [toks[b][j, :ntoks[b][j]].tolist() for j in range(len(act))]
        res.append((projs, frames, tl))

    for k, act in enumerate(_steps()):
        b = k % 2
        if pinned_block:
            chunks = [src[i, st:st + n] for i, (st, n, v, ka) in act]
        else:
            chunks = [np.ascontiguousarray(mels[i][st:st + n].numpy()) for i, (st, n, v, ka) in act]
        frames = eng.step_batch_async([ids[i] for i, _ in act], chunks, [p[1] for _, p in act],
                                      [p[2] for _, p in act], [p[3] for _, p in act], outs[b], toks[b], ntoks[b])
        if pending is not None:
            collect(pending)          # the previous step is complete once this call has returned
        pending = (k, act, frames)
    eng.step_sync()
    collect(pending)
    for sid in ids:
        eng.close_stream(sid)
    return res


@pytest.mark.parametrize("pinned_block", [True, False], ids=["pinned-block", "gathered"])
def test_async_equals_sync_bit_for_bit(model, pinned_block):
    mels = _mels()
    ref = _run_sync(model, mels)
    got = _run_async(model, mels, pinned_block)
    assert len(got) == len(ref)
    assert any(any(len(t) for t in r[2]) for r in ref)
    for k, ((pg, fg, tg), (pr, fr, tr)) in enumerate(zip(got, ref)):
        assert fg == fr, k
        assert tg == tr, k
        for a, b in zip(pg, pr):
            assert np.array_equal(a, b), k


def test_sync_calls_after_async_ones_drain_the_pipeline(model):
    """Two asynchronous steps, then the rest of the history through ud_step_batch: the same results as an
    all-synchronous run (the synchronous call waits for the outstanding step and its buffers)."""
    mels = _mels()
    ref = _run_sync(model, mels)
    tm, W, ms = model.cfg.max_chunk_frames, model.out_width, model.cfg.max_symbols
    n_max = len(LENGTHS)
    outs = [torch.empty(n_max, tm, W, pin_memory=True).numpy() for _ in range(2)]
    toks = [torch.empty(n_max, tm * ms, dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]
    ntoks = [torch.empty(n_max, dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]
    ids = [model.open(R) for _ in LENGTHS]
    steps = _steps()
    for k, act in enumerate(steps):
        args = ([ids[i] for i, _ in act], [np.ascontiguousarray(mels[i][st:st + n].numpy()) for i, (st, n, v, ka) in act],
                [p[1] for _, p in act], [p[2] for _, p in act], [p[3] for _, p in act])
        if k < 2:
            frames = model.step_batch_async(*args, outs[k], toks[k], ntoks[k])
            assert frames == ref[k][1]
            continue
        if k == 2:   # step 1 is still in flight here; step 0 completed when step 1 was issued
            for j in range(len(steps[0])):
                assert np.array_equal(outs[0][j, :ref[0][1][j]], ref[0][0][j])
        projs, frames, tl = model.step_batch(*args, decode=True)
        if k == 2:
            for j in range(len(steps[1])):
                assert np.array_equal(outs[1][j, :ref[1][1][j]], ref[1][0][j])
                assert toks[1][j, :ntoks[1][j]].tolist() == ref[1][2][j]
        assert frames == ref[k][1] and tl == ref[k][2]
        for a, b in zip(projs, ref[k][0]):
            assert np.array_equal(a, b)
    for sid in ids:
        model.close_stream(sid)


def test_async_projections_only(model):
    """Without token buffers the pipelined step returns the projections alone, equal to ud_step_batch's."""
    mels = _mels()[:2]
    tm, W = model.cfg.max_chunk_frames, model.out_width
    ids_a = [model.open(R) for _ in mels]
    ids_b = [model.open(R) for _ in mels]
    outs = [torch.empty(2, tm, W, pin_memory=True).numpy() for _ in range(2)]
    plans = [list(chunk_plan(len(m), R)) for m in mels]
    steps = min(len(p) for p in plans)
    pending = None
    for k in range(steps):
        chunks = [np.ascontiguousarray(m[p[k][0]:p[k][0] + p[k][1]].numpy()) for m, p in zip(mels, plans)]
        args = ([p[k][1] for p in plans], [p[k][2] for p in plans], [p[k][3] for p in plans])
        projs, frames, _ = model.step_batch(ids_a, chunks, *args)
        fr = model.step_batch_async(ids_b, chunks, *args, outs[k % 2])
        assert fr == frames
        if pending is not None:
            pk, pprojs, pfr = pending
            for j in range(2):
                assert np.array_equal(outs[pk % 2][j, :pfr[j]], pprojs[j])
        pending = (k, [p.copy() for p in projs], frames)
    model.step_sync()
    pk, pprojs, pfr = pending
    for j in range(2):
        assert np.array_equal(outs[pk % 2][j, :pfr[j]], pprojs[j])
    for sid in ids_a + ids_b:
        model.close_stream(sid)


def test_rejected_async_call_is_a_status(model):
    tm, W = model.cfg.max_chunk_frames, model.out_width
    out = torch.empty(1, tm, W, pin_memory=True).numpy()
    model.step_sync()                     # nothing outstanding
    with pytest.raises(ud.EngineError) as ei:
        model.step_batch_async([12345], [np.zeros((105, 128), np.float32)], [105], [105], [False], out)
    assert ei.value.status == 4
    sid = model.open(R)
    frames = model.step_batch_async([sid], [np.zeros((105, 128), np.float32)], [105], [105], [False], out)
    model.step_sync()
    assert frames == [R + 1]
    assert np.isfinite(out[0, :frames[0]]).all()
    model.close_stream(sid)
