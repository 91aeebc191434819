"""CPU restatement (fp32) of the RNN-T prediction net, joint and greedy decoding.

TEST INFRASTRUCTURE ONLY (checker and CPU baseline).

Reference: Sources/DictatorCore/Decoding/RNNT.swift
  * predict        :73-114  embed(token) (blank -> zeros), per LSTM layer gates = W_ih x + W_hh h + (b_ih + b_hh),
                            gate order i, f, g, o; c' = s(f) c + s(i) tanh(g); h' = s(o) tanh(c'); then joint.pred
  * jointLogits    :117-123 logits = W_out relu(f + g) + b_out
  * greedy         :127-151 per frame up to max_symbols emissions; blank advances the frame; the prediction
                            output for the last token is cached (`pending`) and committed only on emission;
                            state (h, c, lastToken, pending) carries across chunks
The same loop is `greedy` in reference/nemo/check_spec.py:176-207 (two LSTM layers hard-coded there;
RNNT.swift:40-48 loops over however many layers exist, as this restatement does).
"""

from __future__ import annotations

import numpy as np
import torch

from .weights import ModelDims


class DecoderState:
    def __init__(self, dims: ModelDims):
        self.h = torch.zeros(dims.pred_layers, dims.pred_hidden)
        self.c = torch.zeros(dims.pred_layers, dims.pred_hidden)
        self.last_token = dims.blank
        self.pending = None          # (g [J], h, c) for last_token, not yet committed


class RNNT:
    def __init__(self, sd: dict[str, torch.Tensor], dims: ModelDims, max_symbols: int = 10):
        self.dims = dims
        self.max_symbols = max_symbols
        q = "decoder.prediction."
        self.embed = sd[q + "embed.weight"].float()
        self.lstm = [(sd[q + f"dec_rnn.lstm.weight_ih_l{l}"].float(), sd[q + f"dec_rnn.lstm.weight_hh_l{l}"].float(),
                      (sd[q + f"dec_rnn.lstm.bias_ih_l{l}"] + sd[q + f"dec_rnn.lstm.bias_hh_l{l}"]).float())
                     for l in range(dims.pred_layers)]
        self.pred_w, self.pred_b = sd["joint.pred.weight"].float(), sd["joint.pred.bias"].float()
        self.out_w, self.out_b = sd["joint.joint_net.2.weight"].float(), sd["joint.joint_net.2.bias"].float()
        self.enc_w, self.enc_b = sd["joint.enc.weight"].float(), sd["joint.enc.bias"].float()

    def predict(self, token: int, h: torch.Tensor, c: torch.Tensor):
        Hp = self.dims.pred_hidden
        x = self.embed[token] if token != self.dims.blank else torch.zeros(Hp)
        nh, nc = h.clone(), c.clone()
        for l, (wi, wh, b) in enumerate(self.lstm):
            gates = wi @ x + wh @ h[l] + b
            i_, f_, g_, o_ = gates.split(Hp)
            nc[l] = torch.sigmoid(f_) * c[l] + torch.sigmoid(i_) * torch.tanh(g_)
            nh[l] = torch.sigmoid(o_) * torch.tanh(nc[l])
            x = nh[l]
        return self.pred_w @ x + self.pred_b, nh, nc

    def joint(self, f: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
        return self.out_w @ torch.relu(f + g) + self.out_b

    def enc_proj(self, enc: torch.Tensor) -> torch.Tensor:
        return enc @ self.enc_w.T + self.enc_b

    def greedy(self, f: torch.Tensor, st: DecoderState, trace: list | None = None) -> list[int]:
        """Greedy decode of projected frames f [T, J]; returns emitted ids. If `trace` is a list, one
        (frame, chosen id, top-1 minus top-2 logit margin) tuple is appended per joint evaluation."""
        blank = self.dims.blank
        toks: list[int] = []
        for t in range(f.shape[0]):
            emitted = 0
            while emitted < self.max_symbols:
                if st.pending is None:
                    st.pending = self.predict(st.last_token, st.h, st.c)
                g, ph, pc = st.pending
                logits = self.joint(f[t], g).numpy()
                best = int(np.argmax(logits))                 # first maximum, as RNNT.swift:138-140
                if trace is not None:
                    top2 = np.partition(logits, -2)[-2:]
                    trace.append((t, best, float(top2[1] - top2[0])))
                if best == blank:
                    break
                toks.append(best)
                emitted += 1
                st.h, st.c, st.last_token, st.pending = ph, pc, best, None
        return toks
