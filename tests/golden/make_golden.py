"""Generates the golden fixtures in this directory by running the reference's OWN Python code.

Run in a container that has the reference checkout (it is read, never written):
    python tests/golden/make_golden.py --reference <path to the reference checkout>

Reference code used, imported unchanged:
  * tools/nemotron_ane.py  `Step` (`:49-119`): the reference's torch CPU restatement of the cache-aware
    streaming step (subsampling + conformer layers + joint.enc), driven here with its own masks
    (m0..m3, fmask, kbias) built as its docstring (`:11-19`) and NemotronANE.swift:98-108 describe.
    Its caches come back as fp16 (`:119`); the fixtures keep them fp32 by making `Tensor.half` the
    identity while `Step.layers` runs (no other change).
  * reference/nemo/check_spec.py `subsample` (`:53-82`), `rel_pos_table` / `att_mask` (`:85-107`),
    `layer` (`:122-173`) and `greedy` (`:176-207`): the offline spec re-implementation. Its module
    imports `common`, which would create directories under the reference root; a stub module with the
    three names it imports is installed in `sys.modules` first.

Inputs are seeded (torch.Generator) and the weights come from oracle.weights.make_weights, so every
fixture stores what it needs: inputs, outputs and the seeds/dims used.
"""

from __future__ import annotations

import argparse
import math
import contextlib
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle.weights import BLOCK1, NEMOTRON, ModelDims, make_weights, sharpen_joint  # noqa: E402
from oracle.stream_step import chunk_plan, next_len, sub_len  # noqa: E402


def import_reference(ref: Path):
    sys.path.insert(0, str(ref / "tools"))
    import nemotron_ane  # noqa: F401

    stub = types.ModuleType("common")
    stub.DATA = Path("/nonexistent")
    stub.load_model = lambda *a, **k: None
    stub.set_threads = lambda *a, **k: None
    sys.modules["common"] = stub
    sys.path.insert(0, str(ref / "reference" / "nemo"))
    import check_spec  # noqa: F401

    return sys.modules["nemotron_ane"], sys.modules["check_spec"]


@contextlib.contextmanager
def fp32_caches():
    orig = torch.Tensor.half
    torch.Tensor.half = lambda self: self
    try:
        yield
    finally:
        torch.Tensor.half = orig


def kbias(L, cache_len, valid_t, T):
    b = torch.full((L + T,), -1e4)
    b[L - cache_len:L + valid_t] = 0
    return b


def ref_stream(na, sd, dims: ModelDims, mel: torch.Tensor, lookahead: int, valid_frames: int, nlayers: int):
    """Drives nemotron_ane.Step chunk by chunk over the runBuffered plan; returns per-step records."""
    L, D, K = dims.left_context, dims.d_model, dims.conv_kernel
    kc = torch.zeros(nlayers, L, D)
    vc = torch.zeros(nlayers, L, D)
    cc = torch.zeros(nlayers, K - 1, D)
    cache_len, step = 0, 0
    steps = {}
    recs = []
    for start, rows, valid, keep_all in chunk_plan(mel.shape[0], lookahead, valid_frames):
        drop = 0 if step == 0 else 2
        key = (rows, drop)
        if key not in steps:
            steps[key] = na.Step(sd, rows, drop, nlayers).eval()
        s = steps[key]
        T = s.T
        v1 = next_len(valid)
        v2 = next_len(v1)
        v3 = next_len(v2)
        valid_t = max(0, min(sub_len(valid) - drop, T))
        m0 = (torch.arange(rows) < valid).float()
        m1 = (torch.arange(s.T1) < v1).float()
        m2 = (torch.arange(s.T2) < v2).float()
        m3 = (torch.arange(s.T3) < v3).float()
        fmask = (torch.arange(T) < valid_t).float()
        with torch.no_grad(), fp32_caches():
            x = s.subsample(mel[start:start + rows], m0, m1, m2, m3)
            proj, kc, vc, cc = s.layers(x, fmask, kbias(L, cache_len, valid_t, T), kc, vc, cc)
        keep = valid_t if keep_all else min(valid_t, lookahead + 1)
        recs.append(dict(start=start, rows=rows, valid=valid, keep_all=int(keep_all), T=T, valid_t=valid_t,
                         keep=keep, proj=proj[:keep].numpy().copy(), proj_all=proj.numpy().copy()))
        cache_len = min(cache_len + T, L)
        step += 1
    return recs, kc, vc, cc, cache_len


def gen_stream(na, ref_dims: ModelDims, lookahead: int, total_rows: int, valid_frames: int, name: str,
               keep_layers=(0, -1)):
    sd = make_weights(ref_dims, seed=0)
    g = torch.Generator().manual_seed(1)
    mel = torch.randn(total_rows, ref_dims.mel_bins, generator=g)
    recs, kc, vc, cc, cache_len = ref_stream(na, sd, ref_dims, mel, lookahead, valid_frames, ref_dims.n_layers)
    out = dict(mel=mel.numpy(), lookahead=lookahead, valid_frames=valid_frames, n_layers=ref_dims.n_layers,
               cache_len=cache_len, n_steps=len(recs))
    for i, r in enumerate(recs):
        for k, v in r.items():
            out[f"s{i}_{k}"] = np.asarray(v)
    for li in keep_layers:
        lidx = li % ref_dims.n_layers
        out[f"k_l{lidx}"] = kc[lidx, ref_dims.left_context - cache_len:].numpy()
        out[f"v_l{lidx}"] = vc[lidx, ref_dims.left_context - cache_len:].numpy()
        out[f"conv_l{lidx}"] = cc[lidx].numpy()
    np.savez_compressed(HERE / name, **out)
    print(f"wrote {name}: {len(recs)} steps, T={[r['T'] for r in recs]}, keep={[r['keep'] for r in recs]}")


def gen_block1(na, n_steps=12):
    """Config-1 shape: one block, T = 1 ([70,0]), frames in. joint.enc = identity so Step's projection
    returns the block output unchanged."""
    dims = BLOCK1
    sd = make_weights(dims, seed=0)
    sd["joint.enc.weight"] = torch.eye(dims.d_model)
    sd["joint.enc.bias"] = torch.zeros(dims.d_model)
    s = na.Step(sd, 1, 0, 1).eval()
    assert s.T == 1
    L, D = dims.left_context, dims.d_model
    g = torch.Generator().manual_seed(1)
    xs = torch.randn(n_steps, 1, D, generator=g)
    kc, vc, cc = torch.zeros(1, L, D), torch.zeros(1, L, D), torch.zeros(1, dims.conv_kernel - 1, D)
    outs = []
    cache_len = 0
    for t in range(n_steps):
        with torch.no_grad(), fp32_caches():
            y, kc, vc, cc = s.layers(xs[t], torch.ones(1), kbias(L, cache_len, 1, 1), kc, vc, cc)
        outs.append(y.numpy().copy())
        cache_len = min(cache_len + 1, L)
    np.savez_compressed(HERE / "block1_steps.npz", x=xs.numpy(), out=np.concatenate(outs), cache_len=cache_len,
                        k=kc[0, L - cache_len:].numpy(), v=vc[0, L - cache_len:].numpy(), conv=cc[0].numpy())
    print(f"wrote block1_steps.npz: {n_steps} steps")


def gen_offline_layer(cs, T=96, lookahead=1):
    """check_spec.layer over a whole sequence with the chunked_limited [70, R] mask: the offline golden
    that streaming (one chunk of R+1 frames at a time, projected K/V caches) must reproduce."""
    dims = BLOCK1
    sd = make_weights(dims, seed=0)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(T, dims.d_model, generator=g)
    pe = cs.rel_pos_table(T)
    mask = cs.att_mask(T, [dims.left_context, lookahead], "chunked_limited")
    cfg = dict(causal=True, conv_norm="layer")
    with torch.no_grad():
        out = cs.layer(x, pe, mask, sd, 0, cfg)
    np.savez_compressed(HERE / "offline_layer.npz", x=x.numpy(), out=out.numpy(), lookahead=lookahead)
    print(f"wrote offline_layer.npz: T={T}")


def gen_offline_subsample(cs, rows=81):
    dims = ModelDims(n_layers=0, joint_dim=0)
    sd = make_weights(dims, seed=0)
    g = torch.Generator().manual_seed(7)
    mel = torch.randn(rows, dims.mel_bins, generator=g)
    with torch.no_grad():
        pre, n = cs.subsample(mel.T.contiguous(), rows, sd, True)
    np.savez_compressed(HERE / "offline_subsample.npz", mel=mel.numpy(), pre=pre.numpy(), n=n)
    print(f"wrote offline_subsample.npz: rows={rows} -> {n}")


def gen_greedy(cs, seed, std, T, name, blank_offset=0.0, sharp_seed=0):
    """check_spec.greedy over seeded frames. `blank_offset` is added to the blank logit's bias so that
    blank wins some decisions (with plain random weights every frame emits the 10-symbol maximum);
    `sharp_seed` > 0 swaps in a sharp joint (oracle.weights.sharpen_joint) for large logit margins."""
    dims = ModelDims(n_layers=0, sub_channels=0, pred_layers=2)     # check_spec.greedy hard-codes 2 layers
    sd = make_weights(dims, seed=seed, std=std)
    if sharp_seed:
        sd = sharpen_joint(sd, dims, sharp_seed)
    sd["joint.joint_net.2.bias"][dims.blank] += blank_offset
    g = torch.Generator().manual_seed(seed + 100)
    enc = torch.randn(T, dims.d_model, generator=g)
    with torch.no_grad():
        toks = cs.greedy(enc, sd, max_symbols=10, blank=dims.blank)
    np.savez_compressed(HERE / name, enc=enc.numpy(), tokens=np.asarray(toks, np.int32), seed=seed, std=std,
                        blank_offset=blank_offset, sharp_seed=sharp_seed)
    print(f"wrote {name}: {len(toks)} tokens over {T} frames")


def gen_mel(cs):
    """check_spec.mel_spec (the nemotron frontend, normalize=False) over seeded audio: a tone plus noise of
    16000 + 123 samples, a length that is a multiple of the hop, and one shorter than a window. The filterbank
    is oracle.mel.slaney_filterbank and the window oracle.mel.hann_symmetric; both are stored."""
    from oracle.mel import hann_symmetric, slaney_filterbank

    fb, win = slaney_filterbank(), hann_symmetric()
    out = {"fb": fb.numpy(), "window": win.numpy()}
    g = torch.Generator().manual_seed(21)
    for i, n in enumerate([16000 + 123, 4800, 333]):
        t = torch.arange(n, dtype=torch.float64) / 16000
        a = (0.3 * torch.sin(2 * math.pi * 440 * t) + 0.05 * torch.randn(n, generator=g, dtype=torch.float64))
        a = a.to(torch.float32)
        with torch.no_grad():
            m, t_valid = cs.mel_spec(a, fb, win, normalize=False)
        out[f"audio{i}"] = a.numpy()
        out[f"mel{i}"] = m.T.contiguous().numpy()      # time-major [T, 128]
        out[f"valid{i}"] = np.int64(t_valid)
    np.savez_compressed(HERE / "mel_spec.npz", **out)
    print("wrote mel_spec.npz")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    torch.set_num_threads(8)
    na, cs = import_reference(args.reference)
    gen_block1(na)
    gen_offline_layer(cs)
    gen_offline_subsample(cs)
    gen_mel(cs)
    gen_greedy(cs, seed=0, std=0.02, T=24, name="greedy_std002.npz")
    gen_greedy(cs, seed=0, std=0.02, T=24, name="greedy_std002_blank.npz", blank_offset=0.5)
    gen_greedy(cs, seed=3, std=0.02, T=24, name="greedy_sharp_joint.npz", blank_offset=100.0, sharp_seed=77)
    # [70,13] with two layers: first chunk 105 rows (T=14, no drop), steady 121 rows (T=14 after dropping 2),
    # and a short final chunk with fewer valid rows than rows (keep_all, validT < T).
    gen_stream(na, ModelDims(n_layers=2), lookahead=13, total_rows=369, valid_frames=360, name="stream_70_13_l2.npz")
    # The full 24-layer encoder at [70,1] over four chunks.
    gen_stream(na, NEMOTRON, lookahead=1, total_rows=57, valid_frames=57, name="stream_70_1_l24.npz")


if __name__ == "__main__":
    main()
