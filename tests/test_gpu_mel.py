"""The log-mel frontend (ud_mel_*, NemoMel.swift:10-161) on the GPU.

  * against reference/nemo/check_spec.py `mel_spec` (fixture made by running it): max-abs / max|ref| <= 1e-4
    (the fp32 tolerance class), frames at or beyond N // 160 exactly 0;
  * against the oracle for edge lengths: no samples, shorter than a window, exact multiples of the hop;
  * live pushes in sizes 1, 37, 160, 999, 3000 (StreamingEquivalenceTests.swift:9-21) give exactly the frames
    of the full utterance, for several streams pushed together;
  * a device-resident batch of utterances equals the utterances one by one;
  * bad calls are statuses."""

import numpy as np
import pytest
import torch

import ud
from oracle.mel import features as mel_oracle
from oracle.mel import hann_symmetric, slaney_filterbank

pytestmark = pytest.mark.gpu


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / (np.abs(b).max() + 1e-30))


@pytest.fixture(scope="module")
def mel():
    eng = ud.Engine(ud.default_config(n_layers=1, dtype=ud.DTYPE_F32, max_streams=2, max_batch=2))
    m = ud.MelFrontend(eng, slaney_filterbank().numpy(), hann_symmetric().numpy(), max_streams=8)
    yield m
    m.close()
    eng.close()


@pytest.mark.parametrize("i", [0, 1, 2])
def test_matches_check_spec(mel, golden_dir, i):
    g = np.load(golden_dir / "mel_spec.npz")
    assert np.array_equal(g["fb"], mel.fb)
    got = mel.features(g[f"audio{i}"])
    ref = g[f"mel{i}"]
    valid = int(g[f"valid{i}"])
    assert got.shape == ref.shape
    assert rel(got, ref) <= 1e-4
    assert np.all(got[valid:] == 0)


@pytest.mark.parametrize("n", [0, 1, 199, 200, 399, 400, 480, 16000, 16000 + 123])
def test_edge_lengths_match_oracle(mel, n):
    a = (torch.randn(n, generator=torch.Generator().manual_seed(n)) * 0.2).numpy()
    ref, valid = mel_oracle(torch.from_numpy(a), torch.from_numpy(mel.fb), hann_symmetric())
    got = mel.features(a)
    assert got.shape == tuple(ref.shape)
    if valid:
        assert rel(got[:valid], ref[:valid].numpy()) <= 1e-4
    assert np.all(got[valid:] == 0)


def test_live_pushes_equal_full_utterance(mel):
    lengths = [16000 + 123, 5000, 333]
    audio = [(torch.randn(n, generator=torch.Generator().manual_seed(7 + n)) * 0.1).numpy() for n in lengths]
    full = [mel.features(a) for a in audio]
    ids = [mel.open() for _ in lengths]
    sizes = [1, 37, 160, 999, 3000]
    pos, got, k = [0] * len(lengths), [[] for _ in lengths], 0
    try:
        while any(p < len(a) for p, a in zip(pos, audio)):
            sel = [i for i in range(len(lengths)) if pos[i] < len(audio[i])]
            chunks = []
            for j, i in enumerate(sel):
                m = min(sizes[(k + j) % 5], len(audio[i]) - pos[i])
                chunks.append(audio[i][pos[i]:pos[i] + m])
                pos[i] += m
            k += 1
            for i, fr in zip(sel, mel.push([ids[i] for i in sel], chunks)):
                got[i].append(fr)
        for i, fr in zip(range(len(lengths)), mel.push(ids, [np.zeros(0, np.float32)] * len(ids),
                                                        finish=[True] * len(ids))):
            got[i].append(fr)
        for i in range(len(lengths)):
            g = np.concatenate(got[i])
            assert g.shape == full[i].shape
            assert np.array_equal(g, full[i]), i
    finally:
        for i in ids:
            mel.close_stream(i)


def test_device_batch_equals_single(mel):
    lengths = [16000, 4321, 0, 800]
    audio = [(torch.randn(n, generator=torch.Generator().manual_seed(50 + n)) * 0.3).numpy() for n in lengths]
    so = np.cumsum([0] + lengths[:-1])
    frames = [n // 160 + 1 for n in lengths]
    ro = np.cumsum([0] + frames[:-1])
    dev = torch.device("cuda", 0)
    a_d = torch.from_numpy(np.concatenate(audio)).to(dev)
    m_d = torch.full((sum(frames), mel.n_mels), -7.0, device=dev)
    torch.cuda.synchronize()   # torch's copies and fill run on its own stream, the frontend on the engine's
    mel.features_device(a_d.data_ptr(), so, lengths, m_d.data_ptr(), ro)
    mel.engine.synchronize()
    got = m_d.cpu().numpy()
    for i, a in enumerate(audio):
        assert np.array_equal(got[ro[i]:ro[i] + frames[i]], mel.features(a)), i


def test_errors_are_statuses(mel):
    sid = mel.open()
    try:
        mel.push([sid], [np.zeros(500, np.float32)], finish=[True])
        with pytest.raises(ud.EngineError):
            mel.push([sid], [np.zeros(10, np.float32)])          # after finish
        with pytest.raises(ud.EngineError):
            mel.push([99], [np.zeros(10, np.float32)])           # unknown stream
    finally:
        mel.close_stream(sid)
    sid = mel.open()
    try:
        with pytest.raises(ud.EngineError):
            mel.push([sid], [np.zeros(16000, np.float32)], cap_frames=3)   # capacity too small
        assert len(mel.push([sid], [np.zeros(0, np.float32)])[0]) == 0     # nothing consumed by the failed call
    finally:
        mel.close_stream(sid)
