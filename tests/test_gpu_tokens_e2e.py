"""Tokens from mel, end to end, under the north star's rule: the bf16 GPU encoder followed by the GPU greedy
decoder must make the decisions of the reference's CPU path (the oracle's fp32 encoder with the unrounded fp32
weights, then its greedy decoder, RNNT.swift:127-151) wherever the oracle's top-2 logit margin exceeds 0.5.

Random N(0, 0.02) weights give logit margins far below 0.5, so the joint is sharpened (joint.enc,
joint.joint_net.2 and the embedding drawn wider by oracle.weights.sharpen_joint with std 0.12, which spreads the
logits of one joint evaluation with a standard deviation of about 9) and the blank logit is raised by 30, which
leaves about a quarter of the joint evaluations blank: frames with several symbols, frames with none.

Every decision of every stream is compared. The GPU's path is followed: at each joint evaluation the oracle's
logits (from its own projection) and the GPU path's logits (the GPU's projection) are computed from the same
decoder state; where the oracle's margin exceeds 0.5 both must choose the same symbol, and the walk continues
with the GPU's choice, so one low-margin decision does not end the comparison. The symbols of that walk must be
exactly the tokens the GPU decoder returned for the step."""

import numpy as np
import pytest
import torch

import ud
from oracle.rnnt import RNNT, DecoderState
from oracle.stream_step import Encoder, StreamState, chunk_plan
from oracle.weights import NEMOTRON, make_weights, sharpen_joint

pytestmark = pytest.mark.gpu

JOINT_STD = 0.12
BLANK_OFFSET = 30.0
MARGIN = 0.5


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


@pytest.fixture(scope="module")
def setup():
    sd = sharpen_joint(make_weights(NEMOTRON, seed=0), NEMOTRON, 77, joint_std=JOINT_STD)
    sd["joint.joint_net.2.bias"] = sd["joint.joint_net.2.bias"].clone()
    sd["joint.joint_net.2.bias"][NEMOTRON.blank] += BLANK_OFFSET
    eng = ud.Engine(ud.default_config(max_streams=16, max_batch=16))
    eng.load_weights(sd)
    yield eng, Encoder(sd, NEMOTRON), RNNT(sd, NEMOTRON)
    eng.close()


def follow(dec, f_ref, f_gpu, st, stats):
    """Greedy walk over one step's kept frames along the GPU's decisions (RNNT.swift:127-151: pending prediction,
    first maximum, at most max_symbols per frame); checks the oracle's high-margin decisions on the way."""
    blank = NEMOTRON.blank
    toks = []
    for t in range(f_gpu.shape[0]):
        emitted = 0
        while emitted < dec.max_symbols:
            if st.pending is None:
                st.pending = dec.predict(st.last_token, st.h, st.c)
            g, ph, pc = st.pending
            lr = dec.joint(f_ref[t], g).numpy()
            lg = dec.joint(f_gpu[t], g).numpy()
            a_ref, a_gpu = int(np.argmax(lr)), int(np.argmax(lg))
            top2 = np.partition(lr, -2)[-2:]
            if top2[1] - top2[0] > MARGIN:
                assert a_gpu == a_ref, (t, a_gpu, a_ref, float(top2[1] - top2[0]))
                stats["compared"] += 1
                stats["tokens"] += int(a_ref != blank)
            else:
                stats["low"] += 1
            if a_gpu == blank:
                break
            toks.append(a_gpu)
            emitted += 1
            st.h, st.c, st.last_token, st.pending = ph, pc, a_gpu, None
    return toks


def run_streams(eng, enc, dec, R, mels):
    """Steps every stream through its whole chunk plan in batched calls with GPU decoding; returns the decision
    counts and the worst projection error."""
    n = len(mels)
    ids = [eng.open(R) for _ in range(n)]
    plans = [list(chunk_plan(m.shape[0], R)) for m in mels]
    sts = [StreamState(NEMOTRON) for _ in range(n)]
    dss = [DecoderState(NEMOTRON) for _ in range(n)]
    stats = {"compared": 0, "tokens": 0, "low": 0}
    worst = 0.0
    for k in range(max(len(p) for p in plans)):
        act = [i for i in range(n) if k < len(plans[i])]
        chunks, rows, vr, ka = [], [], [], []
        for i in act:
            start, r, v, keep_all = plans[i][k]
            chunks.append(mels[i][start:start + r])
            rows.append(r)
            vr.append(v)
            ka.append(keep_all)
        projs, frames, toks = eng.step_batch([ids[i] for i in act], chunks, rows, vr, ka, decode=True)
        for j, i in enumerate(act):
            ref, keep, *_ = enc.stream_step(sts[i], torch.from_numpy(chunks[j]), rows[j], vr[j], ka[j], R)
            assert frames[j] == keep
            if keep:
                worst = max(worst, rel(projs[j], ref))
            walked = follow(dec, ref, torch.from_numpy(np.ascontiguousarray(projs[j])), dss[i], stats)
            assert toks[j] == walked, (k, i)
    for sid in ids:
        eng.close_stream(sid)
    return stats, worst


def test_tokens_batch1_70_1_ten_seconds(setup):
    """Configuration C2's shape: one stream at [70,1] (2 frames per step, the few-row GEMV path), 10 s of mel."""
    eng, enc, dec = setup
    mel = torch.randn(1000, 128, generator=torch.Generator().manual_seed(21)).numpy()
    stats, worst = run_streams(eng, enc, dec, 1, [mel])
    assert worst < 2e-2
    assert stats["tokens"] >= 50 and stats["compared"] >= 4 * stats["low"], stats


def test_tokens_16_streams_70_6(setup):
    """16 streams at [70,6] in one batched call per step (112 encoder rows: the 1-CTA tcgen05 GEMM), lock-step
    GPU decoder; lengths differ, so the last steps are ragged."""
    eng, enc, dec = setup
    mels = [torch.randn(260 + 17 * i, 128, generator=torch.Generator().manual_seed(300 + i)).numpy()
            for i in range(16)]
    stats, worst = run_streams(eng, enc, dec, 6, mels)
    assert worst < 2e-2
    assert stats["tokens"] >= 50 and stats["compared"] >= 4 * stats["low"], stats
