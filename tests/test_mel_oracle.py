"""Pins the log-mel oracle (oracle/mel.py) to reference/nemo/check_spec.py `mel_spec` (fixture made by running
it, tests/golden/make_golden.py), and checks the streaming form against the full utterance as the reference's
StreamingEquivalenceTests.testNemoMelStreamEqualsFullUtterance does (push sizes 1, 37, 160, 999, 3000;
max-abs 1e-4)."""

import numpy as np
import pytest
import torch

from oracle.mel import MelStream, features, hann_symmetric, slaney_filterbank


@pytest.mark.parametrize("i", [0, 1, 2])
def test_features_match_check_spec(golden_dir, i):
    g = np.load(golden_dir / "mel_spec.npz")
    m, valid = features(torch.from_numpy(g[f"audio{i}"]), torch.from_numpy(g["fb"]), torch.from_numpy(g["window"]))
    assert valid == int(g[f"valid{i}"])
    ref = g[f"mel{i}"]
    assert m.shape == ref.shape
    assert np.abs(m.numpy() - ref).max() <= 1e-5 * np.abs(ref).max()
    assert np.all(m.numpy()[valid:] == 0)


def test_filterbank_and_window_buffers(golden_dir):
    g = np.load(golden_dir / "mel_spec.npz")
    assert np.array_equal(slaney_filterbank().numpy(), g["fb"])
    assert np.array_equal(hann_symmetric().numpy(), g["window"])
    fb = g["fb"]
    assert fb.shape == (128, 257) and fb.min() >= 0 and np.all(fb.max(1) > 0)


@pytest.mark.parametrize("n", [16000 + 123, 399, 0])
def test_stream_equals_full_utterance(n):
    fb, w = slaney_filterbank(), hann_symmetric()
    a = torch.randn(n, generator=torch.Generator().manual_seed(5)) * 0.1
    full, _ = features(a, fb, w)
    st = MelStream(fb, w)
    got, i, k, sizes = [], 0, 0, [1, 37, 160, 999, 3000]
    while i < n:
        m = min(sizes[k % 5], n - i)
        got.append(st.push(a[i:i + m]))
        i, k = i + m, k + 1
    got.append(st.finish())
    got = torch.cat(got)
    assert got.shape == full.shape
    assert (got - full).abs().max().item() < 1e-4
