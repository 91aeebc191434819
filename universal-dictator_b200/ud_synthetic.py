"""Synthetic inputs for benchmarks and examples: seeded random weights under the NeMo checkpoint tensor names,
the model dimensions of the benchmark configurations, and the algorithmic byte count of the cache operations.

Weights: N(0, std) drawn from one torch.Generator(seed) in the checkpoint's tensor order (the state_dict order
of the reference's tensor-name map, docs/specs/nemotron.md:250-282): subsampling (encoder.pre_encode.*), then
per layer the 26 encoder tensors, then the prediction net, joint.pred, joint.enc and joint.joint_net.2.
LayerNorm gains are 1 and biases 0 (they draw nothing); the blank row of the embedding is zero (padding_idx).
The test suite checks that these tensors are identical to the ones its CPU oracle generates."""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch


@dataclass(frozen=True)
class ModelDims:
    """Static model dimensions (the reference's FastConformerConfig, FastConformer.swift:5-38)."""

    n_layers: int = 24
    d_model: int = 1024
    n_heads: int = 8
    ff_dim: int = 4096
    conv_kernel: int = 9
    left_context: int = 70
    sub_channels: int = 256        # 0: no subsampling (frames are fed directly)
    mel_bins: int = 128
    joint_dim: int = 640           # 0: no joint / decoder
    vocab: int = 1025              # 1024 BPE ids + blank (blank = vocab - 1)
    pred_layers: int = 1
    pred_hidden: int = 640

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def sub_freq(self) -> int:
        f = self.mel_bins
        for _ in range(3):
            f = f // 2 + 1
        return f

    @property
    def blank(self) -> int:
        return self.vocab - 1


NEMOTRON = ModelDims()
BLOCK1 = ModelDims(n_layers=1, sub_channels=0, joint_dim=0)


def _names_shapes(dims: ModelDims):
    D, F, H, DK, C = dims.d_model, dims.ff_dim, dims.n_heads, dims.head_dim, dims.sub_channels
    if C:
        p = "encoder.pre_encode."
        for i, sh in ((0, (C, 1, 3, 3)), (2, (C, 1, 3, 3)), (3, (C, C, 1, 1)), (5, (C, 1, 3, 3)), (6, (C, C, 1, 1))):
            yield f"{p}conv.{i}.weight", sh
            yield f"{p}conv.{i}.bias", (C,)
        yield p + "out.weight", (D, C * dims.sub_freq)
        yield p + "out.bias", (D,)
    for li in range(dims.n_layers):
        p = f"encoder.layers.{li}."
        ln = lambda n: ((p + n + ".weight", (D,)), (p + n + ".bias", (D,)))  # noqa: E731
        yield from ln("norm_feed_forward1")
        yield p + "feed_forward1.linear1.weight", (F, D)
        yield p + "feed_forward1.linear2.weight", (D, F)
        yield from ln("norm_self_att")
        for n in ("q", "k", "v", "out", "pos"):
            yield f"{p}self_attn.linear_{n}.weight", (D, D)
        yield p + "self_attn.pos_bias_u", (H, DK)
        yield p + "self_attn.pos_bias_v", (H, DK)
        yield from ln("norm_conv")
        yield p + "conv.pointwise_conv1.weight", (2 * D, D, 1)
        yield p + "conv.depthwise_conv.weight", (D, 1, dims.conv_kernel)
        yield from ln("conv.batch_norm")
        yield p + "conv.pointwise_conv2.weight", (D, D, 1)
        yield from ln("norm_feed_forward2")
        yield p + "feed_forward2.linear1.weight", (F, D)
        yield p + "feed_forward2.linear2.weight", (D, F)
        yield from ln("norm_out")
    if dims.joint_dim:
        Hp, J, V = dims.pred_hidden, dims.joint_dim, dims.vocab
        yield "decoder.prediction.embed.weight", (V, Hp)
        for l in range(dims.pred_layers):
            q = "decoder.prediction.dec_rnn.lstm."
            yield f"{q}weight_ih_l{l}", (4 * Hp, Hp)
            yield f"{q}weight_hh_l{l}", (4 * Hp, Hp)
            yield f"{q}bias_ih_l{l}", (4 * Hp,)
            yield f"{q}bias_hh_l{l}", (4 * Hp,)
        yield "joint.pred.weight", (J, Hp)
        yield "joint.pred.bias", (J,)
        yield "joint.enc.weight", (J, D)
        yield "joint.enc.bias", (J,)
        yield "joint.joint_net.2.weight", (V, J)
        yield "joint.joint_net.2.bias", (V,)


def make_weights(dims: ModelDims = NEMOTRON, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    """Seeded fp32 state dict with checkpoint names (see the module docstring)."""
    g = torch.Generator().manual_seed(seed)
    sd: dict[str, torch.Tensor] = {}
    for name, shape in _names_shapes(dims):
        if ".norm_" in name or ".batch_norm." in name:
            sd[name] = torch.ones(shape) if name.endswith(".weight") else torch.zeros(shape)
        else:
            sd[name] = torch.randn(shape, generator=g, dtype=torch.float32) * std
    if dims.joint_dim:
        sd["decoder.prediction.embed.weight"][dims.blank].zero_()
    return sd


def cache_bytes_per_stream_step(n_layers: int, d: int, elem: int, k: int, left_context: int = 70,
                                conv_rows: int = 8) -> int:
    """Algorithmic HBM bytes of one append + roll + gather of k frames for one stream over all layers: read and
    write the k new K and V rows, read each L-row window and write it out contiguous, write the last min(k, R)
    conv rows, read the k new conv rows and read and write the R-row conv window. The roll moves no data."""
    row = d * elem
    kv = 2 * (k + k + left_context + left_context)
    conv = min(k, conv_rows) + k + conv_rows + conv_rows
    return n_layers * row * (kv + conv)


def hann_window(n: int = 400) -> np.ndarray:
    """Symmetric Hann window (the formula of the checkpoint's preprocessor.featurizer.window buffer)."""
    k = np.arange(n, dtype=np.float64)
    return (0.5 - 0.5 * np.cos(2 * math.pi * k / (n - 1))).astype(np.float32)


def mel_filterbank(n_mels: int = 128, sr: int = 16000, n_fft: int = 512, fmin: float = 0.0,
                   fmax: float = 8000.0) -> np.ndarray:
    """[n_mels, n_fft // 2 + 1] Slaney-scale triangular filters with Slaney (unit-area) normalisation, the
    published construction of the checkpoint's preprocessor.featurizer.fb buffer."""
    def hz_to_mel(f):
        f = np.asarray(f, np.float64)
        return np.where(f >= 1000.0, 15.0 + np.log(np.maximum(f, 1e-10) / 1000.0) / (np.log(6.4) / 27.0),
                        f / (200.0 / 3))

    def mel_to_hz(m):
        m = np.asarray(m, np.float64)
        return np.where(m >= 15.0, 1000.0 * np.exp((np.log(6.4) / 27.0) * (m - 15.0)), m * (200.0 / 3))

    fft_f = np.linspace(0, sr / 2, n_fft // 2 + 1)
    hz = mel_to_hz(np.linspace(hz_to_mel(fmin), hz_to_mel(fmax), n_mels + 2))
    fdiff = np.diff(hz)
    ramps = hz[:, None] - fft_f[None, :]
    w = np.maximum(0.0, np.minimum(-ramps[:-2] / fdiff[:-1, None], ramps[2:] / fdiff[1:, None]))
    w *= (2.0 / (hz[2:] - hz[:-2]))[:, None]
    return w.astype(np.float32)
