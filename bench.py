#!/usr/bin/env python
"""Benchmark: stream-steps/s of the cache-aware streaming 24-layer FastConformer encoder step on B200.

Workload (configuration C3 of the benchmark): per GPU, 256 synchronous streams at attention context [70,13]
(T = 14 encoder frames per step from 121-row mel chunks, 105 rows for a stream's first chunk), bf16, the encoder
step of the reference's NemotronStreamer.step: subsampling, 24 conformer layers over the paged K/V / conv caches
and the joint encoder projection (`--decode` adds greedy RNN-T decoding of the kept frames with carried decoder
state).
Synthetic data: each stream's 30 s of N(0,1) 128-bin mel (seed = stream id); weights N(0, 0.02), seed 0.
One bench "step" = one batched step of all streams on a GPU; `value` = streams x steps x GPUs / max-over-ranks
device time. Scaling is weak (256 streams per GPU); GPUs share nothing (no collectives on the data path).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--streams S] [--lookahead R]
    torchrun --nproc-per-node N bench.py --gpus N ...

Rank 0 prints one JSON line. `--impl reference` times the CPU restatement of the reference's own step
(oracle/, the reference being Swift/Metal plus a torch CPU restatement that cannot run on the GPU host) on
all host cores, one stream-step per bench step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "universal-dictator_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "stream-steps/s (24-layer enc step)"
UNIT = "stream-steps/s"
L_CTX, MEL, TOTAL_ROWS = 70, 128, 3000          # 30 s of mel at 100 fps


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d["bf16_tflops_sustained"], "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def rank_streams(n: int, rank: int) -> list[int]:
    """Global ids of the n streams rank `rank` owns: disjoint across ranks (streams are sharded, nothing is
    shared), so each rank's synthetic input differs."""
    return [rank * n + s for s in range(n)]


def max_over_ranks(value: float, dist, device) -> float:
    """The slowest rank's time: every rank contributes its own device time, all receive the maximum."""
    if dist is None:
        return value
    t = torch.tensor([value], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(units_per_rank: int, steps: int, world: int, t_max_ms: float) -> float:
    """Units processed by all ranks per second of the slowest rank's time."""
    return units_per_rank * steps * world / (t_max_ms / 1e3)


def chunk_schedule(R: int, total_rows: int):
    """The live chunk walk (NemotronStreamer.swift:109-154) over a whole utterance: (start, rows) per step,
    first chunk 1+8R rows, then 9 pre-encode rows + 8+8R new rows; only full chunks."""
    first, chunk = 1 + 8 * R, 8 + 8 * R
    out = [(0, first)]
    idx = first
    while idx + chunk <= total_rows:
        out.append((idx - 9, 9 + chunk))
        idx += chunk
    return out


class ClockSampler:
    """Samples SM clock, power and clock-event reasons with NVML every 10 ms during the timed region."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x10: "sync_boost"}

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz, self.ok = [], set(), None, False
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            pass
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def gemm_flops_per_step(n: int, T: int, R: int, cfg) -> float:
    """Algorithmic FLOPs of the step's tensor-core GEMMs: per layer the FF (2 x 2 x 4096 x 1024), QKV (3 x 1024^2),
    output (1024^2), pointwise conv (2048 x 1024 + 1024^2) projections over M = n*T rows, the subsampling
    pointwise and output GEMMs over their rows, and the joint encoder projection."""
    D, F, C, J, NL = cfg.d_model, cfg.ff_dim, cfg.sub_channels, cfg.joint_dim, cfg.n_layers
    M = n * T
    layers = NL * M * 2 * (2 * F * D + 3 * D * D + D * D + 2 * D * D + D * D + 2 * F * D)
    nxt = lambda t: t // 2 + 1  # noqa: E731
    rows = 9 + 8 + 8 * R
    T1, T2, T3 = nxt(rows), nxt(nxt(rows)), nxt(nxt(nxt(rows)))
    F1, F2, F3 = nxt(MEL), nxt(nxt(MEL)), nxt(nxt(nxt(MEL)))
    sub = n * T2 * F2 * 2 * C * C + n * T3 * F3 * 2 * C * C + n * T3 * 2 * (C * F3) * D
    joint = M * 2 * D * J
    return float(layers + sub + joint)


def step_bytes_per_kind(n: int, T: int, cfg) -> dict:
    """Algorithmic HBM bytes per step of the bandwidth-bound kernels (bf16 activations and caches, fp32 residual):
    attention per (stream, head) the cached K and V window (L rows each), the chunk's Q, K and V rows, the output
    and the K/V append; the conv module per stream T pointwise-conv rows in (2 D), T rows out, the 8-row ring read
    and written; LayerNorm per row the fp32 row read and the bf16 row written (the fused pair also writes the fp32
    row back), for the layer's norms (norm_ff1 once, then per layer norm_att, norm_conv, norm_ff2 and the fused
    norm_out + next norm_ff1, the last layer's norm_out alone)."""
    D, NL, L, H = cfg.d_model, cfg.n_layers, cfg.left_context, cfg.n_heads
    dk = D // H
    attn = NL * n * H * 2 * (2 * L * dk + 3 * T * dk + T * dk + 2 * T * dk)
    conv = NL * n * 2 * (T * 2 * D + T * D + 2 * 8 * D)
    rows = n * T
    ln_plain = (1 + 3 * NL) * rows * (4 * D + 2 * D)
    ln_pair = (NL - 1) * rows * (4 * D + 4 * D + 2 * D) + rows * (4 * D + 4 * D)
    return {"attention": float(attn), "conv": float(conv), "norm": float(ln_plain + ln_pair)}


def weight_bytes(cfg) -> float:
    """bf16 bytes of every GEMM operand a step reads: 24 layers x 24.12 M, the subsampling pointwise and output
    projections, and joint.enc."""
    D, F, C, J, NL = cfg.d_model, cfg.ff_dim, cfg.sub_channels, cfg.joint_dim, cfg.n_layers
    F3 = ((MEL // 2 + 1) // 2 + 1) // 2 + 1
    layer = 2 * F * D * 2 + 3 * D * D + D * D + 2 * D * D + D * D
    return 2.0 * (NL * layer + 2 * C * C + C * F3 * D + D * J)


def cpu_baseline(sd, R: int, budget_s: float = 12.0, max_steps: int = 40):
    """The CPU restatement of the reference's step (fp32, batch 1, all host threads) on a bounded sample of
    the same workload: one stream's consecutive chunks. Returns (stream-steps/s, threads, sample text)."""
    from oracle.rnnt import RNNT, DecoderState
    from oracle.stream_step import Encoder, StreamState
    from oracle.weights import NEMOTRON

    torch.set_num_threads(os.cpu_count() or 1)
    enc = Encoder(sd, NEMOTRON)
    dec = RNNT(sd, NEMOTRON)
    st, ds = StreamState(NEMOTRON), DecoderState(NEMOTRON)
    mel = torch.randn(TOTAL_ROWS, MEL, generator=torch.Generator().manual_seed(0))
    sched = chunk_schedule(R, TOTAL_ROWS)
    n = 0
    with torch.inference_mode():
        proj, *_ = enc.stream_step(st, mel[0:sched[0][1]], sched[0][1], sched[0][1], False, R)  # warm-up
        t0 = time.perf_counter()
        while n < max_steps and (time.perf_counter() - t0) < budget_s:
            start, rows = sched[1 + n % (len(sched) - 1)]
            proj, *_ = enc.stream_step(st, mel[start:start + rows], rows, rows, False, R)
            dec.greedy(proj, ds)
            n += 1
        dt = time.perf_counter() - t0
    return n / dt, torch.get_num_threads(), f"{n} consecutive stream-steps of one stream ({dt:.1f} s), [70,{R}], fp32, 24 layers + joint + greedy"


def cpu_baseline_batched(sd, R: int, n: int):
    """The batched-torch form of the same CPU step (oracle BatchEncoder: one vectorised step for all n streams,
    fp32, all host threads): a first chunk for every stream (untimed), then one timed steady chunk of all n.
    Returns (stream-steps/s, threads, sample text)."""
    from oracle.stream_step import BatchEncoder, StreamState
    from oracle.weights import NEMOTRON

    torch.set_num_threads(os.cpu_count() or 1)
    benc = BatchEncoder(sd, NEMOTRON)
    sts = [StreamState(NEMOTRON) for _ in range(n)]
    first, chunk = 1 + 8 * R, 9 + 8 + 8 * R
    mel = torch.randn(n, first + chunk, MEL, generator=torch.Generator().manual_seed(0))
    with torch.inference_mode():
        benc.batch_step(sts, mel[:, :first], first, first, R)
        t0 = time.perf_counter()
        benc.batch_step(sts, mel[:, first - 9:first - 9 + chunk], chunk, chunk, R)
        dt = time.perf_counter() - t0
    return n / dt, torch.get_num_threads(), (f"one steady chunk of all {n} streams in one batched step ({dt:.1f} s), "
                                             f"[70,{R}], fp32, 24 layers + joint (oracle BatchEncoder)")


def run_reference(args, world, rank):
    """Reference arm: rank 0 times the CPU restatement; other ranks exit without work."""
    if rank != 0:
        return None
    from oracle.rnnt import RNNT, DecoderState
    from oracle.stream_step import Encoder, StreamState
    from oracle.weights import NEMOTRON, make_weights

    R = args.lookahead
    sd = make_weights(NEMOTRON, seed=0)
    torch.set_num_threads(os.cpu_count() or 1)
    enc, dec = Encoder(sd, NEMOTRON), RNNT(sd, NEMOTRON)
    st, ds = StreamState(NEMOTRON), DecoderState(NEMOTRON)
    mel = torch.randn(TOTAL_ROWS, MEL, generator=torch.Generator().manual_seed(0))
    sched = chunk_schedule(R, TOTAL_ROWS)

    def one(i):
        start, rows = sched[i % len(sched)]
        if i % len(sched) == 0:
            st.__init__(NEMOTRON)
            ds.__init__(NEMOTRON)
        proj, *_ = enc.stream_step(st, mel[start:start + rows], rows, rows, False, R)
        dec.greedy(proj, ds)

    with torch.inference_mode():
        for i in range(args.warmup):
            one(i)
        t0 = time.perf_counter()
        for i in range(args.warmup, args.warmup + args.steps):
            one(i)
        dt = time.perf_counter() - t0
    v = args.steps / dt
    cores = torch.get_num_threads()
    return {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args),
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": f"one stream-step per bench step ({args.steps} timed), batch 1, fp32, torch "
                                       f"{torch.__version__}, CPU restatement of tools/nemotron_ane.py Step + RNN-T greedy"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def workload_config(args):
    if args.workload == "c2":
        return {"workload": f"C2: one stream, [70,{args.lookahead}] (T={args.lookahead + 1}, "
                            f"{9 + 8 + 8 * args.lookahead}-row mel chunks), subsampling + 24-layer FastConformer + "
                            "joint.enc + RNN-T greedy (1-layer LSTM 640), 10 s of mel",
                "streams_per_gpu": 1, "lookahead": args.lookahead, "n_layers": 24, "d_model": 1024, "decode": True,
                "blank_offset": args.blank_offset,
                "l2": "weights (1.16 GB) larger than L2, read by every step",
                "parallelism": f"stream-sharded x{args.gpus}, no collectives"}
    return {"workload": f"C3: {args.streams} synchronous streams/GPU, [70,{args.lookahead}] (T={args.lookahead + 1}, "
                        f"{9 + 8 + 8 * args.lookahead}-row mel chunks), subsampling + 24-layer FastConformer + joint.enc"
                        + (" + RNN-T greedy" if args.decode else ""),
            "streams_per_gpu": args.streams, "lookahead": args.lookahead, "n_layers": 24, "d_model": 1024,
            "cache": "paged rings, 16-frame pages", "decode": args.decode,
            "mel_rows_per_stream": TOTAL_ROWS if args.streams <= 1024 else 1000,
            "l2": "inputs larger than L2 (1.16 GB of weights and the per-stream caches stream through each step)",
            "parallelism": f"stream-sharded x{args.gpus}, no collectives"}


def measure_cache_ops(B: int, k: int, steps: int, warmup: int, world: int, rank: int, local: int, dist) -> dict:
    """Config 5: the cache-op microbenchmark on this rank's GPU. Per step, for B streams and all 24 layers: append k
    new frames of projected K and V plus conv rows after each stream's head, roll (metadata), gather every
    stream's 70-frame K/V window and 8 conv rows into contiguous buffers, then evict and refill 5% of the streams.
    Stream ids are a fresh random permutation every step. GB/s = algorithmic bytes / device time (CUDA events on
    the engine stream, max over ranks), bytes counted per stream from its cacheLen: the k new K/V rows read and
    written, the valid window rows read and all L window rows written out, the conv rows (k read, min(k, 8)
    written into the ring, 8 read and 8 written out), plus the conv-ring reset of each evicted stream."""
    import ud
    from ud_synthetic import cache_bytes_per_stream_step as bytes_per_stream_step

    NL, D, L = 24, 1024, 70
    dev = torch.device("cuda", local)
    cfg = ud.default_config(n_layers=NL, sub_channels=0, joint_dim=0, max_streams=B, max_batch=B,
                            max_chunk_frames=max(k, 2))
    eng = ud.Engine(cfg, device=local)
    ids = [eng.open(0) for _ in range(B)]
    gen = torch.Generator(device=dev).manual_seed(rank)
    kv_new = torch.randn(B, NL, 2, k, D, device=dev, generator=gen).to(torch.bfloat16)
    cv_new = torch.randn(B, NL, k, D, device=dev, generator=gen).to(torch.bfloat16)
    kv_out = torch.empty(B, NL, 2, L, D, device=dev, dtype=torch.bfloat16)
    cv_out = torch.empty(B, NL, 8, D, device=dev, dtype=torch.bfloat16)
    torch.cuda.synchronize(dev)
    rng = np.random.default_rng(rank)
    stream = torch.cuda.ExternalStream(eng.cuda_stream(), device=dev)
    cache_len = np.zeros(B, np.int64)          # host mirror of each stream's cacheLen (bytes are counted from it)
    row = D * 2

    def step():
        perm = [int(i) for i in rng.permutation(ids)]
        eng.cache_append(perm, k, kv_new.data_ptr(), cv_new.data_ptr())
        eng.cache_roll(perm, k)
        eng.cache_gather(perm, kv_out.data_ptr(), cv_out.data_ptr())
        np.minimum(cache_len + k, L, out=cache_len)
        nbytes = NL * row * (B * (2 * (2 * k + L) + k + min(k, 8) + 16) + 2 * int(cache_len.sum()))
        ev = rng.choice(ids, size=max(1, B // 20), replace=False)
        eng.cache_evict([int(i) for i in ev])
        cache_len[ev] = 0
        return nbytes + len(ev) * NL * 8 * row

    for _ in range(warmup):
        step()
    eng.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = eng.launch_count()
    total_bytes = 0
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(steps):
            total_bytes += step()
        e1.record(stream)
        e1.synchronize()
    launches = eng.launch_count() - l0
    ms = e0.elapsed_time(e1)
    t = max_over_ranks(ms, dist, dev)
    eng.close()
    del kv_new, cv_new, kv_out, cv_out
    torch.cuda.empty_cache()
    gbs = total_bytes * world / (t / 1e3) / 1e9
    hbm, _, _, src = peaks()
    return {"value": gbs, "unit": "GB/s", "ms_per_step": t / steps, "steps": steps, "warmup": warmup,
            "streams_per_gpu": B, "k": k, "bytes_per_step": total_bytes / steps,
            "full_window_bytes_per_stream_step": bytes_per_stream_step(NL, D, 2, k), "gpu_launches": launches,
            "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": hbm, "unit": "GB/s",
                         "frac": gbs / world / hbm, "traffic": None,
                         "note": f"per GPU; peak = {src} HBM copy"},
            "clocks": clk.summary()}


def run_cache_bench(args, world, rank, local):
    """Config 5 as its own bench line (`--workload c5`): cache-op HBM GB/s of all ranks."""
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    B, k = args.cache_streams, args.cache_k
    r = measure_cache_ops(B, k, args.steps, args.warmup, world, rank, local, dist)
    if rank == 0:
        print(json.dumps({"metric": "cache-op HBM GB/s (append+roll+gather, 24 layers)", "value": r["value"],
                          "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": f"C5: {B} streams/GPU, k={k} frames/step, 24 layers x 70 x 1024 K/V "
                                                 "rings + 8-row conv rings, random permutation, 5% evict+refill",
                                     "bytes_per_step": r["bytes_per_step"],
                                     "full_window_bytes_per_stream_step": r["full_window_bytes_per_stream_step"],
                                     "l2": "rings and outputs larger than L2"},
                          "gpu_launches": r["gpu_launches"], "roofline": r["roofline"], "clocks": r["clocks"]}),
              flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_mel_bench(args, world, rank, local):
    """Log-mel frontend (ud_mel_*): per step, `--mel-streams` utterances of `--mel-seconds` of seeded audio
    (0.1 N(0,1) plus a 440 Hz tone), resident in HBM, through one ud_mel_features_device call. value = mel frames
    of all ranks per second (CUDA events on the engine stream, max over ranks); the roofline counts each audio
    sample read once and each mel row written once. e2e: the same audio through live pushes (ud_mel_push_batch,
    host samples in, host frames out), one push of the whole utterance per stream and step. The CPU baseline is
    the oracle (check_spec's torch fp32 arithmetic) on one utterance."""
    import ud
    from ud_synthetic import hann_window, mel_filterbank

    B, secs, sr = args.mel_streams, args.mel_seconds, 16000
    n = int(secs * sr)
    T = n // 160 + 1
    if args.impl == "reference":
        if rank != 0:
            return
        from oracle.mel import features

        torch.set_num_threads(os.cpu_count() or 1)
        fb, win = torch.from_numpy(mel_filterbank()), torch.from_numpy(hann_window())
        a = torch.randn(n, generator=torch.Generator().manual_seed(0)) * 0.1
        features(a, fb, win)
        ts = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            features(a, fb, win)
            ts.append(time.perf_counter() - t0)
        v = T / statistics.median(ts)
        print(json.dumps({"metric": "mel frames/s (log-mel frontend)", "value": v, "unit": "frames/s", "impl": "reference",
                          "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                          "config": {"workload": f"one utterance of {secs} s per step (of {B} per GPU step)"},
                          "cpu_baseline": {"value": v, "unit": "frames/s", "cores": torch.get_num_threads(),
                                           "kind": "port", "sample": f"{args.steps} utterances of {secs} s"},
                          "e2e": {"value": v, "unit": "frames/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
              flush=True)
        return
    dev = torch.device("cuda", local)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    eng = ud.Engine(ud.default_config(n_layers=1, sub_channels=0, joint_dim=0, max_streams=1, max_batch=1),
                    device=local)
    fe = ud.MelFrontend(eng, mel_filterbank(), hann_window(), max_streams=B)
    g = torch.Generator(device=dev).manual_seed(rank)
    t = torch.arange(n, device=dev, dtype=torch.float32) / sr
    audio = (torch.randn(B, n, device=dev, generator=g) * 0.1 + 0.3 * torch.sin(2 * math.pi * 440 * t)).contiguous()
    mel = torch.empty(B * T, fe.n_mels, device=dev)
    so = np.arange(B, dtype=np.int64) * n
    ro = np.arange(B, dtype=np.int64) * T
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(eng.cuda_stream(), device=dev)
    for _ in range(args.warmup):
        fe.features_device(audio.data_ptr(), so, [n] * B, mel.data_ptr(), ro)
    eng.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            fe.features_device(audio.data_ptr(), so, [n] * B, mel.data_ptr(), ro)
        e1.record(stream)
        e1.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1), dist, dev) / args.steps
    frames = B * T * world
    value = frames / (ms / 1e3)
    nbytes = B * (4 * n + 4 * fe.n_mels * T)
    gbs = nbytes / (ms / 1e3) / 1e9
    hbm, _, _, src = peaks()
    # e2e: live pushes from host memory, frames back to host memory.
    e2e = None
    if not args.no_e2e:
        host = audio.cpu().numpy()
        ids = [fe.open() for _ in range(B)]
        reps = max(1, min(args.steps, 5))
        t0 = time.perf_counter()
        for _ in range(reps):
            fe.push(ids, [host[i] for i in range(B)], finish=[True] * B, cap_frames=T)
            for i in ids:
                fe.close_stream(i)
            ids = [fe.open() for _ in range(B)]
        dt = (time.perf_counter() - t0) / reps
        for i in ids:
            fe.close_stream(i)
        e2e = {"value": B * T * world / max_over_ranks(dt, dist, dev), "unit": "frames/s",
               "h2d_bytes_per_step": 4 * B * n, "d2h_bytes_per_step": 4 * B * T * fe.n_mels,
               "timing": "host wall clock, ud_mel_push_batch of every stream's whole utterance (finish)"}
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        from oracle.mel import features

        torch.set_num_threads(os.cpu_count() or 1)
        a = audio[0].cpu()
        fb, win = torch.from_numpy(mel_filterbank()), torch.from_numpy(hann_window())
        features(a, fb, win)
        t0 = time.perf_counter()
        k = 0
        while k < 20 and time.perf_counter() - t0 < 10:
            features(a, fb, win)
            k += 1
        dt = (time.perf_counter() - t0) / k
        cpu = {"value": T / dt, "unit": "frames/s", "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{k} utterances of {secs} s through the oracle (torch fp32 rfft)"}
    if rank == 0:
        print(json.dumps({"metric": "mel frames/s (log-mel frontend)", "value": value, "unit": "frames/s",
                          "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                          "data": "synthetic",
                          "config": {"workload": f"{B} utterances/GPU of {secs} s (16 kHz) per step, 128 mel bins",
                                     "l2": "audio and mel larger than L2", "frames_per_step": B * T,
                                     "parallelism": f"utterance-sharded x{world}, no collectives"},
                          "e2e": e2e, "gpu_launches": args.steps,
                          "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                                       "frac": gbs / hbm, "traffic": None, "kernel": "mel_kernel",
                                       "note": f"audio read once + mel written once per step / step time; peak = "
                                               f"{src} HBM copy"},
                          "cpu_baseline": cpu, "cpu_baseline_batched": cpu_b, "clocks": clk.summary()}), flush=True)
    fe.close()
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_streamer_bench(args, world, rank, local):
    """Config 4: concurrent streams through the host-side streamer (ud_streamer_*, NemotronStreamer's chunk walk)
    at [70,6], `--c4-streams` slots per GPU (512 = 4096 over 8 GPUs). Streams arrive as a Poisson process of
    200/s per GPU in audio time (a step advances every stream by one 0.56 s chunk), last U[2 s, 60 s], wait in a
    queue for a free slot, and leave when their final chunk (keepAll) has run; greedy RNN-T decoding runs on
    every kept frame with each stream's carried decoder state. Each stream's mel is a window of a seeded N(0,1)
    host pool, all of it available at admission. The streamer is pipelined (ud_streamer_set_pipelined: a step's
    host-side chunk gathering and copies overlap the previous step's device work; `--c4-sync` for synchronous
    steps). Timing is the host wall clock around the streamer steps (host rows in, tokens out), max over ranks;
    value = stream-steps of all ranks per second."""
    import ud
    from ud_synthetic import NEMOTRON, make_weights

    R, slots, fps = 6, args.c4_streams, 100
    chunk_s = (8 + 8 * R) / fps
    dev = torch.device("cuda", local)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    cfg = ud.default_config(max_streams=slots, max_batch=slots, max_chunk_frames=16,
                            **({"n_layers": args.layers} if args.layers else {}))
    eng = ud.Engine(cfg, device=local)
    sd = make_weights(NEMOTRON, seed=0)
    if args.layers:   # the first args.layers encoder layers
        sd = {k: v for k, v in sd.items() if ".layers." not in k or int(k.split(".layers.")[1].split(".")[0]) < args.layers}
    sd["joint.joint_net.2.bias"][NEMOTRON.blank] += args.blank_offset
    eng.load_weights(sd)
    st = ud.Streamer(eng, R, decode=True)
    st.set_pipelined(not args.c4_sync)
    rng = np.random.default_rng(1000 + rank)
    pool = np.random.default_rng(rank).standard_normal((64 * 60 * fps, MEL), dtype=np.float32)
    queue: list[int] = []          # lengths in rows of waiting streams
    active: dict[int, int] = {}    # streamer id -> rows
    stats = {"steps": 0, "admitted": 0, "finished": 0, "tokens": 0}

    def step():
        queue.extend(int(rng.uniform(2, 60) * fps) for _ in range(rng.poisson(200 * chunk_s)))
        while queue and len(active) < slots:
            n = queue.pop(0)
            off = int(rng.integers(0, pool.shape[0] - n))
            sid = st.open(pool[off:off + n])
            st.push(sid, n, last=True)
            active[sid] = n
            stats["admitted"] += 1
        n_stepped, n_done = st.step()
        if n_done:
            for sid in st.finished():
                stats["tokens"] += len(st.tokens(sid)[0])
                st.release(sid)
                del active[sid]
                stats["finished"] += 1
        return n_stepped

    for _ in range(args.warmup):
        step()
    eng.synchronize()
    if dist:
        dist.barrier()
    total = 0
    l0 = eng.launch_count()
    with ClockSampler(local) as clk:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            total += step()
        dt = time.perf_counter() - t0
    launches = eng.launch_count() - l0
    t_max = max_over_ranks(dt * 1e3, dist, dev)
    # Where the device time goes: 3 more steps with per-kind CUDA-event timing (eager launches, no graphs).
    eng.profile(True)
    for _ in range(3):
        step()
    eng.synchronize()
    prof = eng.profile_read()
    eng.profile(False)
    all_steps = total
    if dist:
        tt = torch.tensor([float(total)], device=dev, dtype=torch.float64)
        dist.all_reduce(tt)
        all_steps = int(tt.item())
    value = all_steps / (t_max / 1e3)
    if rank == 0:
        print(json.dumps({"metric": METRIC + " [C4 streamer]", "value": value, "unit": UNIT, "n_gpus": world,
                          "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_max / args.steps,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                          "data": "synthetic",
                          "config": {"workload": f"C4: {slots} stream slots/GPU, [70,6] (T=7, 65-row chunks), Poisson "
                                                 "arrivals 200/s/GPU, lengths U[2 s, 60 s], greedy RNN-T per stream",
                                     "blank_offset": args.blank_offset,
                                     "stream_steps_per_step": all_steps / max(1, args.steps) / world,
                                     "admitted": stats["admitted"], "finished": stats["finished"],
                                     "tokens": stats["tokens"], "queue": len(queue),
                                     "timing": "host wall clock, " + ("synchronous" if args.c4_sync else "pipelined") +
                                               " streamer steps (host mel in, tokens out)",
                                     "parallelism": f"stream-sharded x{world}, no collectives"},
                          "gpu_launches": launches,
                          "kernel_ms_per_step": {k: round(v[0] / 3, 4) for k, v in prof.items() if v[1]},
                          "clocks": clk.summary()}), flush=True)
    st.close()
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


GEMM_SHAPES = [  # (name, N, K, activation, residual, bf16 output): one encoder layer's projections
    ("ff.up", 4096, 1024, 2, False, True), ("ff.down", 1024, 4096, 0, True, False),
    ("attn.qkv", 3072, 1024, 0, False, True), ("attn.out", 1024, 1024, 0, True, False),
    ("conv.pw1", 2048, 1024, 0, False, True), ("conv.pw2", 1024, 1024, 0, True, False)]


def run_gemm_bench(args, local):
    """The tcgen05 GEMM alone on one encoder layer's projection shapes, M = streams x (lookahead + 1) rows, with
    each shape's epilogue (SiLU, residual, output type). Every call reads one of 24 weight copies in turn, as
    the 24 layers do, so weights stream from HBM; device time per launch comes from the engine's per-launch
    CUDA events. One JSON line: total FLOPs / total device time, with per-shape TFLOP/s and, for context,
    cuBLAS's time for the same product (torch.matmul back to back, no epilogue)."""
    import ud

    dev = torch.device("cuda", local)
    torch.cuda.set_device(local)
    M = args.streams * (args.lookahead + 1)
    eng = ud.Engine(ud.default_config(n_layers=0, sub_channels=0, joint_dim=0, max_streams=1, max_batch=1),
                    device=local)
    gen = torch.Generator(device=dev).manual_seed(0)
    _, peak, _, src = peaks()   # kernels timed alone: the burst bf16 figure
    per_shape, tot_flop, tot_ms, launches = {}, 0.0, 0.0, 0
    for name, N, K, act, res, obf in GEMM_SHAPES:
        A = (torch.randn(M, K, device=dev, generator=gen) * 0.5).bfloat16()
        Ws = [(torch.randn(N, K, device=dev, generator=gen) * 0.03).bfloat16() for _ in range(24)]
        R = torch.randn(M, N, device=dev, generator=gen) if res else None
        # residual shapes in place (x += s * f(h W^T)), as the encoder runs them
        out = R if res else torch.empty(M, N, device=dev, dtype=torch.bfloat16 if obf else torch.float32)
        torch.cuda.synchronize()

        def call(i):
            eng.debug_gemm(A.data_ptr(), Ws[i % 24].data_ptr(), M, N, K, out.data_ptr(), act=act,
                           res_ptr=R.data_ptr() if res else None, out_bf16=obf)

        for i in range(args.warmup):
            call(i)
        eng.profile(True)
        for i in range(args.steps):
            call(i)
        prof = eng.profile_read()
        eng.profile(False)
        ms = prof["gemm_tc"][0] + prof["gemm_tc2"][0]
        n = prof["gemm_tc"][1] + prof["gemm_tc2"][1]
        if n != args.steps:
            raise RuntimeError(f"{name}: {n} tensor-core GEMM launches for {args.steps} calls")
        flop = 2.0 * M * N * K * args.steps
        # For context only: cuBLAS (torch.matmul, bf16 output, no epilogue) on the same operands.
        ref_out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        for i in range(args.warmup):
            torch.matmul(A, Ws[i % 24].t(), out=ref_out)
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        c0.record()
        for i in range(args.steps):
            torch.matmul(A, Ws[i % 24].t(), out=ref_out)
        c1.record()
        c1.synchronize()
        cublas_ms = c0.elapsed_time(c1)
        per_shape[f"{name} {M}x{N}x{K}"] = {"us": ms * 1e3 / n, "tflops": flop / (ms / 1e3) / 1e12,
                                            "cublas_us": cublas_ms * 1e3 / args.steps,
                                            "cublas_tflops": flop / (cublas_ms / 1e3) / 1e12}
        del ref_out
        tot_flop += flop
        tot_ms += ms
        launches += n
        del A, Ws, R, out
    achieved = tot_flop / (tot_ms / 1e3) / 1e12
    print(json.dumps({"metric": "GEMM TFLOP/s (encoder layer shapes)", "value": achieved, "unit": "TFLOP/s",
                      "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": tot_ms / args.steps, "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": f"GEMM: one layer's six projections at M={M}, 24 weight copies each",
                                 "engine": "2-CTA tcgen05" if os.environ.get("UD_TC2", "1") != "0" else "1-CTA tcgen05",
                                 "l2": "weights larger than L2 across the 24 copies"},
                      "gpu_launches": launches, "per_shape": per_shape,
                      "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                                   "frac": achieved / peak, "traffic": None, "note": f"peak = {src} burst bf16"}}), flush=True)
    eng.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--streams", type=int, default=256)
    ap.add_argument("--lookahead", type=int, default=13)
    ap.add_argument("--layers", type=int, default=0,
                    help="c4: encoder layers (0: the model's 24). Fewer layers keep a profile of the RNN-T decoder "
                         "small on the device; not a benchmark configuration")
    ap.add_argument("--decode", action="store_true",
                    help="also run greedy RNN-T decoding in each step (configs 2 and 4; C3 is the encoder step)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cache-ops", action="store_true", help="c3: skip the cache-op (C5) sub-measurement")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5", "gemm", "mel"], default="c3",
                    help="c3: the encoder step (default); c2: one stream at [70,1] with RNN-T decoding (latency); "
                         "c4: concurrent streams through the host-side streamer; c5: the cache-op microbenchmark; "
                         "gemm: the tensor-core GEMM on one layer's shapes; mel: the log-mel frontend")
    ap.add_argument("--mel-streams", type=int, default=512, help="mel: utterances per GPU step")
    ap.add_argument("--mel-seconds", type=float, default=10.0, help="mel: seconds of audio per utterance")
    ap.add_argument("--c4-streams", type=int, default=512, help="c4: stream slots per GPU")
    ap.add_argument("--c4-sync", action="store_true", help="c4: synchronous streamer steps instead of pipelined")
    ap.add_argument("--blank-offset", type=float, default=1.0,
                    help="c2/c4: added to the joint's blank bias. With N(0,0.02) weights greedy decoding emits the "
                         "10-symbol maximum on every frame below about 0.5 and no symbol from 1.0 up; 1.0 (the "
                         "default) costs one joint evaluation per frame, 0 is the worst case")
    ap.add_argument("--cache-streams", type=int, default=1024, help="c5: streams per GPU")
    ap.add_argument("--cache-k", type=int, default=14, help="c5: frames appended per stream per step")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload == "c2":
        args.streams, args.lookahead, args.decode = 1, 1, True

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.workload == "c5":
        run_cache_bench(args, world, rank, local)
        return
    if args.workload == "mel":
        run_mel_bench(args, world, rank, local)
        return
    if args.workload == "c4":
        run_streamer_bench(args, world, rank, local)
        return
    if args.workload == "gemm":
        if rank == 0:
            run_gemm_bench(args, local)
        return
    if args.impl == "reference":
        res = run_reference(args, world, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    import ud
    from ud_synthetic import NEMOTRON, make_weights

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    R, n = args.lookahead, args.streams
    T = R + 1
    cfg = ud.default_config(max_streams=n, max_batch=n, max_chunk_frames=max(16, T))
    eng = ud.Engine(cfg, device=local)
    sd = make_weights(NEMOTRON, seed=0)
    if args.workload == "c2":
        sd["joint.joint_net.2.bias"][NEMOTRON.blank] += args.blank_offset
    eng.load_weights(sd)
    ids = [eng.open(R) for _ in range(n)]

    dev = torch.device("cuda", local)
    # 30 s of mel per stream; above 1024 streams per GPU 10 s (still 8 steps before an utterance ends), which keeps
    # the device input and its pinned host copy near 2 GB each.
    total_rows = 1000 if args.workload == "c2" or n > 1024 else TOTAL_ROWS
    mel = torch.empty(n, total_rows, MEL, device=dev)
    for s, gid in enumerate(rank_streams(n, rank)):
        mel[s].normal_(generator=torch.Generator(device=dev).manual_seed(gid))
    tm, J, ms = cfg.max_chunk_frames, cfg.joint_dim, cfg.max_symbols
    proj = torch.empty(n, tm, J, device=dev)
    toks = torch.empty(n, tm * ms, device=dev, dtype=torch.int32)
    ntok = torch.empty(n, device=dev, dtype=torch.int32)
    torch.cuda.synchronize()
    sched = chunk_schedule(R, total_rows)
    decode = args.decode
    state = {"i": 0}

    def step():
        c = state["i"] % len(sched)
        if c == 0 and state["i"] > 0:
            eng.cache_evict(ids)           # the utterance ended: fresh caches and decoder state, same slots
        start, rows = sched[c]
        eng.step_batch_device(ids, mel.data_ptr() + start * MEL * 4, total_rows, [rows] * n, [rows] * n, [False] * n,
                              proj.data_ptr(), toks.data_ptr() if decode else None, ntok.data_ptr() if decode else None)
        state["i"] += 1

    stream = torch.cuda.ExternalStream(eng.cuda_stream(), device=dev)
    for _ in range(args.warmup):
        step()
    eng.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    l0 = eng.launch_count()
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        ev1.synchronize()
    eng.synchronize()
    launches = eng.launch_count() - l0
    ms_dev = ev0.elapsed_time(ev1)
    t_max = max_over_ranks(ms_dev, dist, dev)
    if dist:
        dist.barrier()
    value = whole_job_rate(n, args.steps, world, t_max)

    # Kernel attribution (outside the timed region): per-class device time over two more steps.
    eng.profile(True)
    for _ in range(2):
        step()
    prof = eng.profile_read()
    eng.profile(False)
    hbm, bf16_burst, bf16_sus, src = peaks()
    tc_ms = (prof["gemm_tc"][0] + prof["gemm_tc2"][0]) / 2
    tc_launches = (prof["gemm_tc"][1] + prof["gemm_tc2"][1]) / 2
    flops = gemm_flops_per_step(n, T, R, cfg)
    achieved = flops / (tc_ms / 1e3) / 1e12 if tc_ms > 0 else None
    # The same kernels inside the graph-replayed step (outside the timed region): each 2-CTA GEMM, TMA attention,
    # LayerNorm and conv-module launch stamps the global timer when its first CTA passes the grid-dependency wait
    # and when its last CTA's work ends; the step's graph and programmatic dependent launch are as in the timed
    # region. Five steps: the first runs eagerly, the second captures the timer graph, the last three replay it and
    # are averaged.
    graph_mode, kernel_graph = None, None
    eng.graph_timers(True)
    g_runs = []
    for i in range(5):
        step()
        if i >= 2:
            g_runs.append(eng.graph_timers_read())
    eng.graph_timers(False)
    kernel_roof_graph = None
    if g_runs and g_runs[-1]["gemm_tc2"][1] > 0:
        kernel_graph = {k: round(sum(r[k][0] for r in g_runs) / len(g_runs), 4) for k in g_runs[-1] if g_runs[-1][k][1]}
        kbytes = step_bytes_per_kind(n, T, cfg)
        kernel_roof_graph = {k: {"bytes_per_step": kbytes[k], "gbs": kbytes[k] / (kernel_graph[k] / 1e3) / 1e9,
                                 "frac": kbytes[k] / (kernel_graph[k] / 1e3) / 1e9 / hbm}
                             for k in kbytes if kernel_graph.get(k)}
        g_ms = kernel_graph["gemm_tc2"]
        g_ach = flops / (g_ms / 1e3) / 1e12
        graph_mode = {"achieved": g_ach, "frac": g_ach / bf16_sus, "gemm_ms_per_step": g_ms,
                      "launches_per_step": g_runs[-1]["gemm_tc2"][1],
                      "note": "algorithmic GEMM FLOPs per step / summed (last CTA finish - first CTA past the "
                              "grid-dependency wait) of the 2-CTA GEMM launches, global-timer stamps in the "
                              "graph-replayed step, mean of 3 steps outside the timed region"
                              + ("; the layer stack runs as two halves on two streams here, so overlapping "
                                 "launches are counted twice and this is a lower bound" if n * T >= 8192 else "")}
    traffic, traffic_of = None, None
    tfile = ROOT / "profiles" / "gemm_tc_c3_traffic.txt"
    if tfile.exists():
        for line in tfile.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                traffic = float(line.split(":")[1])
            elif line.startswith("kernel:"):
                traffic_of = line.split(":", 1)[1].strip()

    # End to end through the host-buffer API (pinned host mel in, projections + tokens out to pinned host
    # buffers), wall clock: pipelined ud_step_batch_async calls (step k+1's input copy and step k's output copy
    # overlap the compute; every step's copies are inside the timed region), and for reference the synchronous
    # ud_step_batch.
    e2e = None
    if not args.no_e2e:
        hmel = torch.empty(n, total_rows, MEL, pin_memory=True)
        hmel.copy_(mel.cpu())
        hnp = hmel.numpy()
        outs = [torch.empty(n, tm, J, pin_memory=True).numpy() for _ in range(2)]
        touts = [torch.empty(n, tm * ms, dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]
        nouts = [torch.empty(n, dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]
        state_h = {"i": 0}

        def step_host(pipelined: bool):
            c = state_h["i"] % len(sched)
            if c == 0:
                eng.cache_evict(ids)
            start, rows = sched[c]
            chunks = [hnp[s, start:start + rows] for s in range(n)]
            if pipelined:
                b = state_h["i"] % 2
                eng.step_batch_async(ids, chunks, [rows] * n, [rows] * n, [False] * n, outs[b],
                                     touts[b] if decode else None, nouts[b] if decode else None)
            else:
                eng.step_batch(ids, chunks, [rows] * n, [rows] * n, [False] * n, decode=decode)
            state_h["i"] += 1
            return rows

        def timed(pipelined: bool) -> tuple[float, int]:
            state_h["i"] = 0
            # The step's CUDA graph is captured at the second sighting of a batch shape and staging buffer;
            # the pipelined calls alternate two buffers, so four warm-up steps capture both.
            for _ in range(max(args.warmup, 4) if pipelined else args.warmup):
                step_host(pipelined)
            eng.step_sync()
            if dist:
                dist.barrier()
            t0 = time.perf_counter()
            rows_sum = 0
            for _ in range(args.steps):
                rows_sum += step_host(pipelined)
            eng.step_sync()
            return max_over_ranks(time.perf_counter() - t0, dist, dev), rows_sum

        dt_sync, _ = timed(False)
        dt, rows_sum = timed(True)
        h2d = rows_sum / args.steps * MEL * 4 * n
        d2h = n * tm * J * 4 + ((n * tm * ms * 4 + n * 4) if decode else 0)
        e2e = {"value": whole_job_rate(n, args.steps, world, dt * 1e3), "unit": UNIT, "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h),
               "timing": "host wall clock, pipelined ud_step_batch_async calls from and to pinned host buffers",
               "synchronous_value": whole_job_rate(n, args.steps, world, dt_sync * 1e3)}

    # The metric's second half, cache-op HBM GB/s, in the same run: configuration C5 at 1024 streams per GPU and
    # k = 14, on an engine of its own (every rank takes part; time is the max over ranks).
    cache_ops = None
    if args.workload == "c3" and not args.no_cache_ops:
        cache_ops = measure_cache_ops(1024, 14, 10, 3, world, rank, local, dist)
        cache_ops["metric"] = "cache-op HBM GB/s (append+roll+gather, 24 layers)"
        cache_ops["workload"] = ("C5: 1024 streams/GPU, k=14 frames/step, 24 layers x 70 x 1024 K/V rings + 8-row "
                                 "conv rings, random permutation, 5% evict+refill")

    # Capacity against real time: one step advances every stream by one chunk of 8 + 8R mel rows (10 ms each).
    free_pages, total_pages, esz = eng.pool_info()
    chunk_ms = (8 + 8 * R) * 10.0
    step_ms = t_max / args.steps
    capacity = {"streams_per_gpu": n, "realtime_budget_ms": chunk_ms, "ms_per_step": step_ms,
                "realtime_factor": chunk_ms / step_ms,
                "realtime_streams_at_this_step_time": int(n * chunk_ms / step_ms),
                "cache_pool_bytes": int(2 * cfg.n_layers * total_pages * cfg.page_frames * cfg.d_model * esz +
                                        cfg.n_layers * n * (cfg.conv_kernel - 1) * cfg.d_model * esz),
                "note": "per-stream step time falls as the batch grows (the weights are read once per step), so "
                        "streams x budget / step time underestimates the streams one GPU keeps in real time"}

    cpu = cpu_b = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_baseline(sd, R)
        cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
        if args.workload == "c3" and n <= 512:
            v, cores, sample = cpu_baseline_batched(sd, R, n)
            cpu_b = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}

    roof_gemv = None
    if n * T <= 16:   # few rows: the projections run as GEMVs over the whole weight set (HBM-bound)
        simt_ms = prof["gemm_simt"][0] / 2
        wbytes = weight_bytes(cfg)
        gbs = wbytes / (simt_ms / 1e3) / 1e9 if simt_ms > 0 else None
        roof_gemv = {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": (gbs / hbm) if gbs else None, "traffic": None, "kernel": "gemm_simt (GEMV)",
                     "note": f"weight bytes per step ({wbytes / 1e9:.3f} GB bf16) / summed GEMV time per step, CUDA "
                             f"events on the engine stream; peak = {src} HBM copy"}
    if rank == 0:
        res = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
               "warmup": args.warmup, "ms_per_step": t_max / args.steps, "higher_is_better": True, "scaling": "weak",
               "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": workload_config(args),
               "e2e": e2e, "gpu_launches": launches,
               "roofline": roof_gemv or {"bound": "tensor", "achieved": achieved, "peak": bf16_sus, "unit": "TFLOP/s",
                            "frac": (achieved / bf16_sus) if achieved else None, "traffic": traffic,
                            "kernel": "gemm_tc (tcgen05)",
                            "traffic_of": (f"{traffic_of}: dram__bytes_read.sum + dram__bytes_write.sum from one ncu "
                                           "capture (profiles/gemm_tc_c3_traffic.txt)") if traffic_of else None,
                            "note": f"algorithmic GEMM FLOPs per step / summed tcgen05 GEMM time per step "
                                    f"({tc_launches:.0f} launches), CUDA events on the engine stream; peak = "
                                    f"{src} sustained bf16",
                            "graph_mode": graph_mode},
               "kernel_ms_per_step": {k: round(v[0] / 2, 4) for k, v in prof.items() if v[1]},
               "kernel_ms_per_step_graph": kernel_graph,
               "kernel_roofline_graph": kernel_roof_graph,
               "kernel_attribution_graph": ("the same kinds in the graph-replayed step, as in the timed region: per "
                                            "launch, last CTA end - first CTA past the grid-dependency wait "
                                            "(global-timer stamps), summed per kind, mean of 3 steps outside the "
                                            "timed region; subsampling and the joint projection are not stamped"),
               "kernel_attribution": ("two extra steps outside the timed region, launched eagerly (no CUDA graph, no "
                                      "programmatic dependent launch) with CUDA events around every launch: "
                                      f"{sum(v[0] for v in prof.values()) / 2:.3f} ms per step summed over the "
                                      f"kernels, against {t_max / args.steps:.3f} ms for the graph-replayed step in "
                                      "the timed region; each launch's time includes its own ramp and tail, which "
                                      "the graph overlaps with its neighbours, so roofline.achieved is a lower bound"),
               "cache_ops": cache_ops, "capacity": capacity,
               "cpu_baseline": cpu, "cpu_baseline_batched": cpu_b, "clocks": clk.summary()}
        print(json.dumps(res), flush=True)

    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
