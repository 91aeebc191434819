"""CPU restatement (fp32, torch) of the cache-aware streaming FastConformer encoder step.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA library and the timed CPU baseline, never a
product path.

What it restates (reference paths are relative to the reference project root):
  * chunk schedule            Sources/DictatorCore/Nemotron/NemotronSchedule.swift:7-16
  * protocol step             Sources/DictatorEngine/Models/Nemotron.swift:74-91 (drop 2 after the first
                              chunk, keep = keepAll ? validT : min(validT, R + 1), joint.enc on kept rows)
  * streaming step            Sources/DictatorEngine/Models/FastConformer.swift:441-480 (key ranges
                              [L - cacheLen, L + validT), cache roll = last L K/V rows and last K-1 conv
                              rows, cacheLen = min(cacheLen + T, L))
  * causal dw-striding subsampling with per-stage time masks
                              tools/nemotron_ane.py:73-83, FastConformer.swift:219-250
  * macaron conformer layer   tools/nemotron_ane.py:85-119, FastConformer.swift:262-321
  * rel-pos attention         Sources/DictatorEngine/Metal/20_conformer.metal:140-219 (masked keys get
                              probability exactly 0; an empty key range gives a zero output, as NeMo's
                              `a[mask] = 0`, docs/specs/nemotron.md:120)
  * position tables           tools/nemotron_ane.py:41-46, 62-68; FastConformer.swift:147-178
The reference oracle `tools/nemotron_ane.py` masks keys with an additive -1e4 bias instead of ranges;
the two agree whenever at least one key is visible, which `tests/golden/` pins.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .weights import NEMOTRON, ModelDims


def next_len(t: int) -> int:
    """Causal stride-2 conv output length, k=3, pad (2, 1): FastConformer.swift:215 (`nextLen`)."""
    return t // 2 + 1


def sub_len(t: int) -> int:
    for _ in range(3):
        t = next_len(t)
    return t


@dataclass(frozen=True)
class Schedule:
    """NemotronSchedule.swift:7-16."""

    lookahead: int
    left_context: int = 70
    pre_encode_cache: int = 9
    drop_extra: int = 2

    @property
    def first_chunk(self) -> int:
        return 1 + 8 * self.lookahead

    @property
    def chunk(self) -> int:
        return 8 + 8 * self.lookahead

    @property
    def out_frames(self) -> int:
        return self.lookahead + 1


def sinusoid(pos: float, d: int) -> torch.Tensor:
    """NeMo RelPositionalEncoding row for relative position `pos`, fp32 (nemotron_ane.py:41-46)."""
    div = torch.exp(torch.arange(0, d, 2, dtype=torch.float32) * -(math.log(10000.0) / d))
    pe = torch.zeros(d)
    pe[0::2] = torch.sin(pos * div)
    pe[1::2] = torch.cos(pos * div)
    return pe


def sinusoid_table(rel_lo: int, rel_hi: int, d: int) -> torch.Tensor:
    """Rows for relative positions rel_lo..rel_hi (inclusive), ascending."""
    return torch.stack([sinusoid(float(r), d) for r in range(rel_lo, rel_hi + 1)])


class StreamState:
    """Per-stream caches (FastConformer.swift:406-435): projected K and V of the last L frames per layer,
    the last K-1 depthwise-conv inputs per layer (time-major), cacheLen and the step counter."""

    def __init__(self, dims: ModelDims = NEMOTRON):
        L, D, NL = dims.left_context, dims.d_model, dims.n_layers
        self.k = torch.zeros(NL, L, D)
        self.v = torch.zeros(NL, L, D)
        self.conv = torch.zeros(NL, dims.conv_kernel - 1, D)
        self.cache_len = 0
        self.step = 0


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), w, b, 1e-5)


def relpos_attention(q, k, v, ptab, rel_lo, u, vb, lo, hi):
    """Transformer-XL attention over keys [lo, hi) (20_conformer.metal:140-219).

    q [T, D]; k, v [Tk, D]; ptab [n_rel, D] projected position rows for rel = rel_lo + row;
    rel(i, j) = (Tk - T) + i - j. Returns [T, D]."""
    T, D = q.shape
    Tk = k.shape[0]
    H, DK = u.shape
    out = torch.zeros(T, D)
    lo, hi = max(lo, 0), min(hi, Tk)
    if hi <= lo:
        return out
    qh = q.view(T, H, DK).transpose(0, 1)
    kh = k[lo:hi].view(hi - lo, H, DK).transpose(0, 1)
    vh = v[lo:hi].view(hi - lo, H, DK).transpose(0, 1)
    ac = (qh + u[:, None, :]) @ kh.transpose(1, 2)                                   # [H, T, n]
    i = torch.arange(T)[:, None]
    j = torch.arange(lo, hi)[None, :]
    rel = (Tk - T) + i - j - rel_lo                                                   # [T, n]
    pg = ptab[rel].view(T, hi - lo, H, DK).permute(2, 0, 1, 3)                        # [H, T, n, DK]
    bd = ((qh + vb[:, None, :])[:, :, None, :] * pg).sum(-1)
    p = torch.softmax((ac + bd) / math.sqrt(DK), dim=-1)
    return (p @ vh).transpose(0, 1).reshape(T, D)


class Encoder:
    """fp32 CPU encoder over a state dict with checkpoint names."""

    def __init__(self, sd: dict[str, torch.Tensor], dims: ModelDims = NEMOTRON):
        self.sd = {k: v.float() for k, v in sd.items()}
        self.dims = dims
        self._ptab: dict[tuple[int, int], tuple[torch.Tensor, int]] = {}

    def w(self, name: str) -> torch.Tensor:
        return self.sd[name]

    # ------------------------------------------------------------------ subsampling
    def subsample(self, mel: torch.Tensor, valid_rows: int) -> torch.Tensor:
        """mel [Tin, mel_bins] -> [sub_len(Tin), D]; rows at or beyond each stage's valid length are
        zeroed (nemotron_ane.py:73-83 masks m0..m3; FastConformer.swift:219-250)."""
        dims = self.dims
        C = dims.sub_channels
        p = "encoder.pre_encode."
        v1 = next_len(valid_rows)
        v2 = next_len(v1)
        v3 = next_len(v2)

        def mask(x, n):
            x = x.clone()
            x[:, :, max(n, 0):, :] = 0
            return x

        x = mask(mel[None, None].float(), valid_rows)
        x = mask(F.relu(F.conv2d(F.pad(x, (2, 1, 2, 1)), self.w(p + "conv.0.weight"), self.w(p + "conv.0.bias"), stride=2)), v1)
        x = F.conv2d(F.pad(x, (2, 1, 2, 1)), self.w(p + "conv.2.weight"), self.w(p + "conv.2.bias"), stride=2, groups=C)
        x = mask(F.relu(F.conv2d(x, self.w(p + "conv.3.weight"), self.w(p + "conv.3.bias"))), v2)
        x = F.conv2d(F.pad(x, (2, 1, 2, 1)), self.w(p + "conv.5.weight"), self.w(p + "conv.5.bias"), stride=2, groups=C)
        x = mask(F.relu(F.conv2d(x, self.w(p + "conv.6.weight"), self.w(p + "conv.6.bias"))), v3)
        _, c, t, f = x.shape
        x = x.permute(0, 2, 1, 3).reshape(t, c * f)            # channel-major flatten: index c*F3 + f
        return F.linear(x, self.w(p + "out.weight"), self.w(p + "out.bias"))

    # ------------------------------------------------------------------ position tables
    def pos_table(self, li: int, T: int) -> tuple[torch.Tensor, int]:
        """Projected rows P = sinusoid(rel) . W_pos^T for rel in [-(T-1), L+T-1] (nemotron_ane.py:62-68)."""
        key = (li, T)
        if key not in self._ptab:
            L, D = self.dims.left_context, self.dims.d_model
            lo = -(T - 1)
            pe = sinusoid_table(lo, L + T - 1, D)
            P = pe @ self.w(f"encoder.layers.{li}.self_attn.linear_pos.weight").T
            self._ptab[key] = (P, lo)
        return self._ptab[key]

    # ------------------------------------------------------------------ layers
    def layers(self, x: torch.Tensor, valid_t: int, st: StreamState) -> torch.Tensor:
        """All conformer layers over this chunk's frames x [T, D]; updates st.k/v/conv in place (not
        cache_len / step). Keys are [L cached ; T new], visible range [L - cacheLen, L + validT)."""
        dims = self.dims
        L, D, K = dims.left_context, dims.d_model, dims.conv_kernel
        T = x.shape[0]
        x = x.float()
        lo, hi = L - st.cache_len, L + valid_t
        for li in range(dims.n_layers):
            p = f"encoder.layers.{li}."
            w = lambda n: self.w(p + n)  # noqa: E731
            h = layer_norm(x, w("norm_feed_forward1.weight"), w("norm_feed_forward1.bias"))
            x = x + 0.5 * F.linear(F.silu(F.linear(h, w("feed_forward1.linear1.weight"))), w("feed_forward1.linear2.weight"))
            h = layer_norm(x, w("norm_self_att.weight"), w("norm_self_att.bias"))
            q = F.linear(h, w("self_attn.linear_q.weight"))
            k = torch.cat([st.k[li], F.linear(h, w("self_attn.linear_k.weight"))], 0)
            v = torch.cat([st.v[li], F.linear(h, w("self_attn.linear_v.weight"))], 0)
            ptab, rel_lo = self.pos_table(li, T)
            att = relpos_attention(q, k, v, ptab, rel_lo, w("self_attn.pos_bias_u"), w("self_attn.pos_bias_v"), lo, hi)
            x = x + F.linear(att, w("self_attn.linear_out.weight"))
            h = layer_norm(x, w("norm_conv.weight"), w("norm_conv.bias"))
            g = F.glu(F.linear(h, w("conv.pointwise_conv1.weight")[:, :, 0]), dim=-1)
            g[valid_t:] = 0                                       # pad mask on the GLU output
            ci = torch.cat([st.conv[li], g], 0)                   # [K-1+T, D]
            dw = w("conv.depthwise_conv.weight")[:, 0, :]         # [D, K], tap K-1 = current frame
            y = torch.stack([(ci[t:t + K] * dw.T).sum(0) for t in range(T)], 0)
            y = F.silu(layer_norm(y, w("conv.batch_norm.weight"), w("conv.batch_norm.bias")))
            x = x + F.linear(y, w("conv.pointwise_conv2.weight")[:, :, 0])
            h = layer_norm(x, w("norm_feed_forward2.weight"), w("norm_feed_forward2.bias"))
            x = x + 0.5 * F.linear(F.silu(F.linear(h, w("feed_forward2.linear1.weight"))), w("feed_forward2.linear2.weight"))
            x = layer_norm(x, w("norm_out.weight"), w("norm_out.bias"))
            st.k[li] = k[T:]
            st.v[li] = v[T:]
            st.conv[li] = ci[T:]
        return x

    # ------------------------------------------------------------------ protocol-level steps
    def frames_step(self, st: StreamState, x: torch.Tensor, valid_t: int | None = None) -> torch.Tensor:
        """Layers-only streaming step over frames x [T, D] (the single-block configuration)."""
        T = x.shape[0]
        vt = T if valid_t is None else valid_t
        out = self.layers(x, vt, st)
        st.cache_len = min(st.cache_len + T, self.dims.left_context)
        st.step += 1
        return out

    def stream_step(self, st: StreamState, mel: torch.Tensor, n_rows: int, valid_rows: int, keep_all: bool,
                    lookahead: int):
        """One NemotronEncoder.step (Nemotron.swift:74-91 over FastConformer.swift:441-480).
        Returns (proj [keep, J], keep, encoder output [T, D], T, validT)."""
        drop = 0 if st.step == 0 else 2
        Tsub = sub_len(n_rows)
        T = Tsub - drop
        valid_t = max(0, min(sub_len(valid_rows) - drop, T))
        sub = self.subsample(mel[:n_rows], valid_rows)
        out = self.frames_step(st, sub[drop:drop + T], valid_t)
        keep = valid_t if keep_all else min(valid_t, lookahead + 1)
        proj = F.linear(out[:keep], self.w("joint.enc.weight"), self.w("joint.enc.bias"))
        return proj, keep, out, T, valid_t


class BatchEncoder(Encoder):
    """The same step for many streams at once, vectorised over the streams (a batched-torch form of
    Encoder.stream_step, for the CPU baseline at the benchmark's batch). Every stream of a call must share the
    chunk geometry: n_rows, valid_rows, the step counter (first chunk or not) and cacheLen, as the benchmark's
    synchronous streams do. The arithmetic is stream_step's: the per-stream products become batched ones."""

    def batch_step(self, sts: list[StreamState], mel: torch.Tensor, n_rows: int, valid_rows: int,
                   lookahead: int) -> torch.Tensor:
        """mel [B, n_rows, mel_bins] -> projections [B, keep, J]; every state advances one chunk."""
        dims = self.dims
        B = len(sts)
        st0 = sts[0]
        assert all(st.step == st0.step and st.cache_len == st0.cache_len for st in sts)
        drop = 0 if st0.step == 0 else 2
        T = sub_len(n_rows) - drop
        valid_t = max(0, min(sub_len(valid_rows) - drop, T))
        x = self.subsample_batch(mel[:, :n_rows], valid_rows)[:, drop:drop + T]
        L, D, K = dims.left_context, dims.d_model, dims.conv_kernel
        H, DK = dims.n_heads, dims.head_dim
        lo, hi = L - st0.cache_len, L + valid_t
        for li in range(dims.n_layers):
            p = f"encoder.layers.{li}."
            w = lambda n: self.w(p + n)  # noqa: E731
            h = layer_norm(x, w("norm_feed_forward1.weight"), w("norm_feed_forward1.bias"))
            x = x + 0.5 * F.linear(F.silu(F.linear(h, w("feed_forward1.linear1.weight"))), w("feed_forward1.linear2.weight"))
            h = layer_norm(x, w("norm_self_att.weight"), w("norm_self_att.bias"))
            q = F.linear(h, w("self_attn.linear_q.weight"))
            k = torch.cat([torch.stack([st.k[li] for st in sts]), F.linear(h, w("self_attn.linear_k.weight"))], 1)
            v = torch.cat([torch.stack([st.v[li] for st in sts]), F.linear(h, w("self_attn.linear_v.weight"))], 1)
            att = torch.zeros(B, T, D)
            if hi > lo:
                ptab, rel_lo = self.pos_table(li, T)
                u, vb = w("self_attn.pos_bias_u"), w("self_attn.pos_bias_v")
                qh = q.view(B, T, H, DK).transpose(1, 2)                                 # [B, H, T, DK]
                kh = k[:, lo:hi].reshape(B, hi - lo, H, DK).transpose(1, 2)
                vh = v[:, lo:hi].reshape(B, hi - lo, H, DK).transpose(1, 2)
                ac = (qh + u[None, :, None, :]) @ kh.transpose(2, 3)                     # [B, H, T, n]
                i = torch.arange(T)[:, None]
                j = torch.arange(lo, hi)[None, :]
                rel = L + i - j - rel_lo
                pg = ptab[rel].view(T, hi - lo, H, DK).permute(2, 0, 1, 3)               # [H, T, n, DK]
                bd = torch.einsum("bhtd,htnd->bhtn", qh + vb[None, :, None, :], pg)
                pr = torch.softmax((ac + bd) / math.sqrt(DK), dim=-1)
                att = (pr @ vh).transpose(1, 2).reshape(B, T, D)
            x = x + F.linear(att, w("self_attn.linear_out.weight"))
            h = layer_norm(x, w("norm_conv.weight"), w("norm_conv.bias"))
            g = F.glu(F.linear(h, w("conv.pointwise_conv1.weight")[:, :, 0]), dim=-1)
            g[:, valid_t:] = 0
            ci = torch.cat([torch.stack([st.conv[li] for st in sts]), g], 1)           # [B, K-1+T, D]
            dw = w("conv.depthwise_conv.weight")[:, 0, :]                               # [D, K]
            y = (ci.unfold(1, K, 1) * dw[None, None]).sum(-1)                           # [B, T, D]
            y = F.silu(layer_norm(y, w("conv.batch_norm.weight"), w("conv.batch_norm.bias")))
            x = x + F.linear(y, w("conv.pointwise_conv2.weight")[:, :, 0])
            h = layer_norm(x, w("norm_feed_forward2.weight"), w("norm_feed_forward2.bias"))
            x = x + 0.5 * F.linear(F.silu(F.linear(h, w("feed_forward2.linear1.weight"))), w("feed_forward2.linear2.weight"))
            x = layer_norm(x, w("norm_out.weight"), w("norm_out.bias"))
            for b, st in enumerate(sts):
                st.k[li] = k[b, T:]
                st.v[li] = v[b, T:]
                st.conv[li] = ci[b, T:]
        for st in sts:
            st.cache_len = min(st.cache_len + T, L)
            st.step += 1
        keep = min(valid_t, lookahead + 1)
        return F.linear(x[:, :keep], self.w("joint.enc.weight"), self.w("joint.enc.bias"))

    def subsample_batch(self, mel: torch.Tensor, valid_rows: int) -> torch.Tensor:
        """Encoder.subsample over a batch mel [B, Tin, mel_bins] -> [B, sub_len(Tin), D], one valid length."""
        C = self.dims.sub_channels
        p = "encoder.pre_encode."
        v1 = next_len(valid_rows)
        v2 = next_len(v1)
        v3 = next_len(v2)

        def mask(x, n):
            x = x.clone()
            x[:, :, max(n, 0):, :] = 0
            return x

        x = mask(mel[:, None].float(), valid_rows)
        x = mask(F.relu(F.conv2d(F.pad(x, (2, 1, 2, 1)), self.w(p + "conv.0.weight"), self.w(p + "conv.0.bias"), stride=2)), v1)
        x = F.conv2d(F.pad(x, (2, 1, 2, 1)), self.w(p + "conv.2.weight"), self.w(p + "conv.2.bias"), stride=2, groups=C)
        x = mask(F.relu(F.conv2d(x, self.w(p + "conv.3.weight"), self.w(p + "conv.3.bias"))), v2)
        x = F.conv2d(F.pad(x, (2, 1, 2, 1)), self.w(p + "conv.5.weight"), self.w(p + "conv.5.bias"), stride=2, groups=C)
        x = mask(F.relu(F.conv2d(x, self.w(p + "conv.6.weight"), self.w(p + "conv.6.bias"))), v3)
        b, c, t, f = x.shape
        x = x.permute(0, 2, 1, 3).reshape(b, t, c * f)
        return F.linear(x, self.w(p + "out.weight"), self.w(p + "out.bias"))


def drain_next(lookahead: int, idx: int, have: int, final: bool, end_padding: bool):
    """One iteration of NemotronStreamer.drainChunks (NemotronStreamer.swift:109-154), the live chunk walk, for a
    stream that has consumed mel rows up to `idx` of the `have` it holds: returns None to wait (final False) or
    when the stream has ended (final True), else (cache_start, rows, pad_rows, keep_all, next_idx). A full chunk
    runs as soon as its rows exist; at the end a tail shorter than the minimum chunk (8 rows, 1 for a first
    chunk) is zero-extended to it and masked when `end_padding` (the reference's default), else dropped."""
    sch = Schedule(lookahead)
    first = idx == 0
    size = sch.first_chunk if first else sch.chunk
    end = idx + size
    if end > have and not final:
        return None
    chunk_len = min(end, have) - idx
    min_len = 1 if first else 8
    if chunk_len <= 0 or (chunk_len < min_len and not (final and end_padding)):
        return None
    cache_start = idx if first else max(0, idx - sch.pre_encode_cache)
    rows = min(end, have) - cache_start
    pad = max(0, min_len - chunk_len)
    is_last = final and end >= have
    return cache_start, rows, pad, (pad > 0) or is_last, end


def live_plan(total_rows: int, lookahead: int, end_padding: bool = True):
    """drainChunks over a complete mel buffer: yields (row_start, n_rows, valid_rows, keep_all), n_rows including
    the zero rows of a padded tail. Without end padding it equals runBuffered's walk (chunk_plan)."""
    idx = 0
    while True:
        c = drain_next(lookahead, idx, total_rows, True, end_padding)
        if c is None:
            return
        start, rows, pad, keep, idx = c
        yield start, rows + pad, rows, keep
        if keep:
            return


def chunk_plan(total_rows: int, lookahead: int, valid_frames: int | None = None):
    """NemotronStreamer.runBuffered's chunk walk (NemotronStreamer.swift:70-91) over a full mel
    buffer of `total_rows` rows: yields (row_start, n_rows, valid_rows, keep_all)."""
    sch = Schedule(lookahead)
    vf = total_rows if valid_frames is None else valid_frames
    idx = 0
    while idx < total_rows:
        first = idx == 0
        size = sch.first_chunk if first else sch.chunk
        end = min(idx + size, total_rows)
        chunk_len = end - idx
        if chunk_len < (1 if first else 8):
            return
        cache_start = idx if first else max(0, idx - sch.pre_encode_cache)
        added = idx - cache_start
        rows = added + chunk_len
        valid = max(0, min(vf - idx + added, rows))
        idx += size
        yield cache_start, rows, valid, idx >= total_rows
