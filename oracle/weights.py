"""Seeded random weights under the NeMo checkpoint tensor names (test infrastructure only).

The tensor names and shapes follow the checkpoint's state_dict as listed in the reference's
behavioural spec (`docs/specs/nemotron.md:250-282`, section 8, "Tensor-name map"), in that order:
subsampling (`encoder.pre_encode.*`), then per layer the 26 encoder tensors, then the RNN-T
prediction net (`decoder.prediction.*`), `joint.pred`, `joint.enc` and `joint.joint_net.2`.

Values: N(0, 0.02) drawn from one `torch.Generator().manual_seed(seed)` in that fixed order.
LayerNorm gains are 1 and LayerNorm biases 0 (they draw nothing). The embedding row of the blank id
is zeroed after drawing, as in the checkpoint (`docs/specs/nemotron.md:208`: padding_idx = blank).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class ModelDims:
    """Static model dimensions (reference `FastConformerConfig`, `FastConformer.swift:5-38`)."""

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
# Config 1 of the benchmark: one block, frames in, no subsampling or RNN-T head.
BLOCK1 = ModelDims(n_layers=1, sub_channels=0, joint_dim=0)


def _is_ln(name: str) -> bool:
    return (".norm_" in name) or (".batch_norm." in name)


def tensor_specs(dims: ModelDims) -> list[tuple[str, tuple[int, ...]]]:
    """(name, shape) in checkpoint order for the given dimensions."""
    D, F, H, DK, C = dims.d_model, dims.ff_dim, dims.n_heads, dims.head_dim, dims.sub_channels
    out: list[tuple[str, tuple[int, ...]]] = []
    if C:
        p = "encoder.pre_encode."
        out += [(p + "conv.0.weight", (C, 1, 3, 3)), (p + "conv.0.bias", (C,)),
                (p + "conv.2.weight", (C, 1, 3, 3)), (p + "conv.2.bias", (C,)),
                (p + "conv.3.weight", (C, C, 1, 1)), (p + "conv.3.bias", (C,)),
                (p + "conv.5.weight", (C, 1, 3, 3)), (p + "conv.5.bias", (C,)),
                (p + "conv.6.weight", (C, C, 1, 1)), (p + "conv.6.bias", (C,)),
                (p + "out.weight", (D, C * dims.sub_freq)), (p + "out.bias", (D,))]
    for li in range(dims.n_layers):
        p = f"encoder.layers.{li}."
        out += [(p + "norm_feed_forward1.weight", (D,)), (p + "norm_feed_forward1.bias", (D,)),
                (p + "feed_forward1.linear1.weight", (F, D)), (p + "feed_forward1.linear2.weight", (D, F)),
                (p + "norm_self_att.weight", (D,)), (p + "norm_self_att.bias", (D,)),
                (p + "self_attn.linear_q.weight", (D, D)), (p + "self_attn.linear_k.weight", (D, D)),
                (p + "self_attn.linear_v.weight", (D, D)), (p + "self_attn.linear_out.weight", (D, D)),
                (p + "self_attn.linear_pos.weight", (D, D)),
                (p + "self_attn.pos_bias_u", (H, DK)), (p + "self_attn.pos_bias_v", (H, DK)),
                (p + "norm_conv.weight", (D,)), (p + "norm_conv.bias", (D,)),
                (p + "conv.pointwise_conv1.weight", (2 * D, D, 1)),
                (p + "conv.depthwise_conv.weight", (D, 1, dims.conv_kernel)),
                (p + "conv.batch_norm.weight", (D,)), (p + "conv.batch_norm.bias", (D,)),
                (p + "conv.pointwise_conv2.weight", (D, D, 1)),
                (p + "norm_feed_forward2.weight", (D,)), (p + "norm_feed_forward2.bias", (D,)),
                (p + "feed_forward2.linear1.weight", (F, D)), (p + "feed_forward2.linear2.weight", (D, F)),
                (p + "norm_out.weight", (D,)), (p + "norm_out.bias", (D,))]
    if dims.joint_dim:
        Hp, J, V = dims.pred_hidden, dims.joint_dim, dims.vocab
        out.append(("decoder.prediction.embed.weight", (V, Hp)))
        for l in range(dims.pred_layers):
            q = "decoder.prediction.dec_rnn.lstm."
            out += [(q + f"weight_ih_l{l}", (4 * Hp, Hp)), (q + f"weight_hh_l{l}", (4 * Hp, Hp)),
                    (q + f"bias_ih_l{l}", (4 * Hp,)), (q + f"bias_hh_l{l}", (4 * Hp,))]
        out += [("joint.pred.weight", (J, Hp)), ("joint.pred.bias", (J,)),
                ("joint.enc.weight", (J, D)), ("joint.enc.bias", (J,)),
                ("joint.joint_net.2.weight", (V, J)), ("joint.joint_net.2.bias", (V,))]
    return out


def make_weights(dims: ModelDims = NEMOTRON, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    """Seeded fp32 state dict with checkpoint names (see module docstring)."""
    g = torch.Generator().manual_seed(seed)
    sd: dict[str, torch.Tensor] = {}
    for name, shape in tensor_specs(dims):
        if _is_ln(name):
            sd[name] = torch.ones(shape) if name.endswith(".weight") else torch.zeros(shape)
        else:
            sd[name] = torch.randn(shape, generator=g, dtype=torch.float32) * std
    if dims.joint_dim:
        sd["decoder.prediction.embed.weight"][dims.blank].zero_()
    return sd


def round_bf16(sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """The weights as the bf16 engine stores them: GEMM operands rounded to bf16 (round to nearest
    even), everything else kept fp32. Used so bf16 parity measures activation precision only."""
    out = {}
    for k, v in sd.items():
        gemm = (k.endswith("linear1.weight") or k.endswith("linear2.weight") or ".linear_" in k
                or "pointwise_conv" in k or k in ("encoder.pre_encode.conv.3.weight", "encoder.pre_encode.conv.6.weight",
                                                  "encoder.pre_encode.out.weight", "joint.enc.weight"))
        if gemm and "linear_pos" not in k:
            out[k] = v.to(torch.bfloat16).to(torch.float32)
        else:
            out[k] = v
    return out


def sharpen_joint(sd: dict[str, torch.Tensor], dims: ModelDims, seed: int, joint_std: float = 0.25,
                  embed_std: float = 1.0) -> dict[str, torch.Tensor]:
    """Test-weight variant with a sharp joint: joint.enc and joint.joint_net.2 drawn with `joint_std` and the
    embedding with `embed_std` (blank row zero) from their own generator, the LSTM left at its small init.
    Logit margins are then large (well above 0.5) while the prediction recurrence stays well conditioned."""
    g = torch.Generator().manual_seed(seed)
    out = dict(sd)
    out["joint.joint_net.2.weight"] = torch.randn(dims.vocab, dims.joint_dim, generator=g) * joint_std
    out["joint.enc.weight"] = torch.randn(dims.joint_dim, dims.d_model, generator=g) * joint_std
    emb = torch.randn(dims.vocab, dims.pred_hidden, generator=g) * embed_std
    emb[dims.blank] = 0
    out["decoder.prediction.embed.weight"] = emb
    return out
