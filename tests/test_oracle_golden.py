"""Pins the CPU oracle against fixtures produced by the reference's own Python code
(tests/golden/make_golden.py runs tools/nemotron_ane.py and reference/nemo/check_spec.py unchanged).

Tolerance: max-abs / max|ref| (check_spec.py:210-213 `rel`) <= 1e-5, the reference's measured fp32
thread-count spread on layer outputs (docs/specs/nemotron.md:300-320). Tokens: identical.
"""

import numpy as np
import pytest
import torch

from oracle.rnnt import RNNT, DecoderState
from oracle.stream_step import Encoder, StreamState, chunk_plan, sub_len
from oracle.weights import BLOCK1, NEMOTRON, ModelDims, make_weights, sharpen_joint


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-30))


def test_block1_steps_match_reference_step(golden_dir):
    g = np.load(golden_dir / "block1_steps.npz")
    enc = Encoder(make_weights(BLOCK1, seed=0), BLOCK1)
    st = StreamState(BLOCK1)
    for t in range(g["x"].shape[0]):
        y = enc.frames_step(st, torch.from_numpy(g["x"][t]))
        assert rel(y, g["out"][t:t + 1]) < 1e-5, t
    n = int(g["cache_len"])
    assert st.cache_len == n
    assert rel(st.k[0, 70 - n:], g["k"]) < 1e-5
    assert rel(st.v[0, 70 - n:], g["v"]) < 1e-5
    assert rel(st.conv[0], g["conv"]) < 1e-5


def test_streaming_equals_offline_chunked_layer(golden_dir):
    """Streaming one chunk of R+1 frames at a time with projected K/V caches reproduces the offline
    layer (check_spec.layer) under NeMo's chunked_limited [70, R] mask, including frames beyond the
    70-frame left context (docs/specs/nemotron.md section 6.4)."""
    g = np.load(golden_dir / "offline_layer.npz")
    R = int(g["lookahead"])
    x = torch.from_numpy(g["x"])
    enc = Encoder(make_weights(BLOCK1, seed=0), BLOCK1)
    st = StreamState(BLOCK1)
    outs = [enc.frames_step(st, x[i:i + R + 1]) for i in range(0, x.shape[0], R + 1)]
    assert rel(torch.cat(outs), g["out"]) < 1e-5


def test_streaming_subsample_equals_offline(golden_dir):
    """Chunks with the 9-row pre-encode cache and 2 dropped frames give the offline subsampling rows
    (check_spec.subsample), as the receptive-field argument in docs/specs/nemotron.md section 6.2 says."""
    g = np.load(golden_dir / "offline_subsample.npz")
    dims = ModelDims(n_layers=0, joint_dim=0)
    enc = Encoder(make_weights(dims, seed=0), dims)
    mel = torch.from_numpy(g["mel"])
    rows = []
    for i, (start, n, valid, _) in enumerate(chunk_plan(mel.shape[0], 1)):
        drop = 0 if i == 0 else 2
        sub = enc.subsample(mel[start:start + n], valid)
        rows.append(sub[drop:])
    got = torch.cat(rows)[: int(g["n"])]
    assert got.shape[0] == int(g["n"])
    assert rel(got, g["pre"]) < 1e-5


@pytest.mark.parametrize("name", ["stream_70_13_l2.npz", "stream_70_1_l24.npz"])
def test_stream_steps_match_reference_step(golden_dir, name):
    g = np.load(golden_dir / name)
    nl = int(g["n_layers"])
    dims = NEMOTRON if nl == 24 else ModelDims(n_layers=nl)
    enc = Encoder(make_weights(dims, seed=0), dims)
    st = StreamState(dims)
    mel = torch.from_numpy(g["mel"])
    R = int(g["lookahead"])
    plan = list(chunk_plan(mel.shape[0], R, int(g["valid_frames"])))
    assert len(plan) == int(g["n_steps"])
    for i, (start, n, valid, keep_all) in enumerate(plan):
        proj, keep, _, T, valid_t = enc.stream_step(st, mel[start:start + n], n, valid, keep_all, R)
        assert (T, valid_t, keep) == (int(g[f"s{i}_T"]), int(g[f"s{i}_valid_t"]), int(g[f"s{i}_keep"]))
        if keep:
            assert rel(proj, g[f"s{i}_proj"]) < 1e-5, i
    n = int(g["cache_len"])
    assert st.cache_len == n
    for li in (0, nl - 1):
        assert rel(st.k[li, 70 - n:], g[f"k_l{li}"]) < 1e-5
        assert rel(st.v[li, 70 - n:], g[f"v_l{li}"]) < 1e-5
        assert rel(st.conv[li], g[f"conv_l{li}"]) < 1e-5


@pytest.mark.parametrize("name", ["greedy_std002.npz", "greedy_std002_blank.npz", "greedy_sharp_joint.npz"])
def test_greedy_matches_check_spec(golden_dir, name):
    g = np.load(golden_dir / name)
    dims = ModelDims(n_layers=0, sub_channels=0, pred_layers=2)
    sd = make_weights(dims, seed=int(g["seed"]), std=float(g["std"]))
    if int(g["sharp_seed"]):
        sd = sharpen_joint(sd, dims, int(g["sharp_seed"]))
    sd["joint.joint_net.2.bias"][dims.blank] += float(g["blank_offset"])
    r = RNNT(sd, dims)
    f = r.enc_proj(torch.from_numpy(g["enc"]))
    # Decoding in two chunks with carried state equals decoding the whole sequence at once.
    st = DecoderState(dims)
    toks = r.greedy(f[:10], st) + r.greedy(f[10:], st)
    assert toks == g["tokens"].tolist()


def test_schedule_lengths():
    # docs/specs/nemotron.md:163-173: [70,1] 9 -> 2 frames, 25 -> 4 (drop 2); [70,6] 49 -> 7, 65 -> 9.
    assert [sub_len(n) for n in (9, 25, 49, 65, 105, 121)] == [2, 4, 7, 9, 14, 16]
