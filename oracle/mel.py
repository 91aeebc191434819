"""CPU oracle of the log-mel frontend (test infrastructure only; the product never imports it).

Restates NemoMelFrontend (Sources/DictatorCore/Audio/NemoMel.swift:10-108), NeMo's FilterbankFeatures at
inference, whose spec is docs/specs/nemotron.md:31-55 and whose executable form is
reference/nemo/check_spec.py `mel_spec` (:31-50):
  preemphasis y[0] = x[0], y[n] = x[n] - 0.97 x[n-1]                                    (NemoMel.swift:48-52)
  centred STFT: 256 zeros on both sides, frame t = padded samples [160t, 160t + 512), the 400-tap window
  zero-padded to 512 at taps 56..455                                                    (:54-65, check_spec :35-40)
  power = |X|^2 over the 257 bins (magnitude first, then squared)                       (:93-97, check_spec :41-42)
  mel = fb @ power, log(mel + 2^-24); frames t >= N // 160 are 0                        (:98-107, check_spec :43-49)
and NemoMelStream (NemoMel.swift:110-161): frame t is emitted once sample 160t + 199 exists; `finish` emits the
rest with the right zero padding and the zeroed last frame, so live output equals the full utterance.

The arithmetic is check_spec's (torch fp32, rfft). `slaney_filterbank` restates librosa's published Slaney mel
filterbank (mel scale linear below 1 kHz and logarithmic above, triangles normalised to unit area,
`librosa.filters.mel(norm="slaney", htk=False)`), the construction of the checkpoint's
`preprocessor.featurizer.fb` buffer (docs/specs/nemotron.md:41); `hann_symmetric` is the window buffer's formula.
"""

from __future__ import annotations

import math

import numpy as np
import torch

N_FFT, HOP, WIN, PREEMPH = 512, 160, 400, 0.97
N_BINS = N_FFT // 2 + 1
LOG_GUARD = 2.0 ** -24
WIN_OFF = (N_FFT - WIN) // 2        # 56


def hann_symmetric(n: int = WIN) -> torch.Tensor:
    k = torch.arange(n, dtype=torch.float64)
    return (0.5 - 0.5 * torch.cos(2 * math.pi * k / (n - 1))).to(torch.float32)


def _hz_to_mel(f: np.ndarray) -> np.ndarray:
    f = np.asarray(f, np.float64)
    lin = f / (200.0 / 3)
    log_part = 15.0 + np.log(np.maximum(f, 1e-10) / 1000.0) / (np.log(6.4) / 27.0)
    return np.where(f >= 1000.0, log_part, lin)


def _mel_to_hz(m: np.ndarray) -> np.ndarray:
    m = np.asarray(m, np.float64)
    lin = m * (200.0 / 3)
    log_part = 1000.0 * np.exp((np.log(6.4) / 27.0) * (m - 15.0))
    return np.where(m >= 15.0, log_part, lin)


def slaney_filterbank(n_mels: int = 128, sr: int = 16000, n_fft: int = N_FFT, fmin: float = 0.0,
                      fmax: float = 8000.0) -> torch.Tensor:
    """[n_mels, n_fft // 2 + 1] Slaney-scale, Slaney-normalised triangular filters (float32)."""
    fft_f = np.linspace(0, sr / 2, n_fft // 2 + 1)
    hz = _mel_to_hz(np.linspace(_hz_to_mel(fmin), _hz_to_mel(fmax), n_mels + 2))
    fdiff = np.diff(hz)
    ramps = hz[:, None] - fft_f[None, :]
    lower = -ramps[:-2] / fdiff[:-1, None]
    upper = ramps[2:] / fdiff[1:, None]
    w = np.maximum(0.0, np.minimum(lower, upper))
    w *= (2.0 / (hz[2:] - hz[:-2]))[:, None]
    return torch.from_numpy(w.astype(np.float32))


def _frames_power(y_pad: torch.Tensor, t0: int, T: int, window: torch.Tensor) -> torch.Tensor:
    """Power spectra [T, 257] of frames t0 .. t0+T-1 of the zero-padded preemphasised signal."""
    idx = (torch.arange(T)[:, None] + t0) * HOP + torch.arange(N_FFT)[None, :]
    w = torch.zeros(N_FFT)
    w[WIN_OFF:WIN_OFF + WIN] = window
    X = torch.fft.rfft(y_pad[idx] * w, dim=-1)
    mag = torch.sqrt(X.real ** 2 + X.imag ** 2)
    return mag.pow(2.0)


def features(audio: torch.Tensor, fb: torch.Tensor, window: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Full-utterance log-mel, time-major [N // 160 + 1, n_mels], and the valid frame count N // 160."""
    audio = audio.to(torch.float32)
    n = audio.shape[0]
    T, valid = n // HOP + 1, n // HOP
    if n == 0:
        return torch.zeros(T, fb.shape[0]), valid
    y = torch.cat([audio[:1], audio[1:] - PREEMPH * audio[:-1]])
    y_pad = torch.nn.functional.pad(y, (N_FFT // 2, N_FFT // 2))
    p = _frames_power(y_pad, 0, T, window)
    m = torch.log(p @ fb.T + LOG_GUARD)
    m[valid:] = 0.0
    return m, valid


class MelStream:
    """NemoMelStream: push samples in any sizes; frames come out as soon as their window is complete."""

    def __init__(self, fb: torch.Tensor, window: torch.Tensor):
        self.fb, self.window = fb, window
        self.audio = torch.zeros(0)
        self.frames = 0

    def _emit(self, end: int, valid: int) -> torch.Tensor:
        if end <= self.frames:
            return torch.zeros(0, self.fb.shape[0])
        a = self.audio
        n = a.shape[0]
        y = torch.cat([a[:1], a[1:] - PREEMPH * a[:-1]]) if n else a
        # enough right padding for every emitted frame: frame t reads padded samples up to 160t + 511
        y_pad = torch.nn.functional.pad(y, (N_FFT // 2, max(N_FFT // 2, end * HOP + N_FFT - (n + N_FFT // 2))))
        p = _frames_power(y_pad, self.frames, end - self.frames, self.window)
        m = torch.log(p @ self.fb.T + LOG_GUARD)
        m[max(0, valid - self.frames):] = 0.0
        self.frames = end
        return m

    def push(self, samples: torch.Tensor) -> torch.Tensor:
        self.audio = torch.cat([self.audio, samples.to(torch.float32)])
        n = self.audio.shape[0]
        ready = (n - 200) // HOP + 1 if n >= 200 else 0
        return self._emit(ready, 1 << 62)

    def finish(self) -> torch.Tensor:
        n = self.audio.shape[0]
        return self._emit(n // HOP + 1, n // HOP)
