"""CUDA-graph replay of the steady step gives bit-identical results to eager launches (same engine code,
same inputs), across shape changes (first chunk, steady chunks, a short final chunk) and across the two
batched entry points."""

import os
import time

import numpy as np
import pytest
import torch

import ud
from oracle.stream_step import chunk_plan
from oracle.weights import ModelDims, make_weights

pytestmark = pytest.mark.gpu


def _run(graphs: bool, sd, dims, n=3, env=None, timers=False):
    env = dict(env or {}, UD_GRAPHS="1" if graphs else "0")
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        e = ud.Engine(ud.default_config(n_layers=dims.n_layers, max_streams=max(4, n), max_batch=max(4, n)))
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    e.load_weights(sd)
    if timers:
        e.graph_timers(True)
    readings = []
    ids = [e.open(13) for _ in range(n)]
    mels = [torch.randn(400, 128, generator=torch.Generator().manual_seed(20 + i)).numpy() for i in range(n)]
    plans = [list(chunk_plan(400, 13, 400 - 7 * (i % 3))) for i in range(n)]
    outs = []
    for k in range(max(len(p) for p in plans)):
        act = [i for i in range(n) if k < len(plans[i])]
        chunks = [mels[i][plans[i][k][0]:plans[i][k][0] + plans[i][k][1]] for i in act]
        t0 = time.perf_counter()
        projs, frames, toks = e.step_batch([ids[i] for i in act], chunks, [plans[i][k][1] for i in act],
                                           [plans[i][k][2] for i in act], [plans[i][k][3] for i in act], decode=True)
        wall_ms = (time.perf_counter() - t0) * 1e3
        outs.append(([p.copy() for p in projs], frames, toks))
        if timers:
            readings.append((min(plans[i][k][1] for i in act), wall_ms, e.graph_timers_read()))
    e.close()
    return (outs, readings) if timers else outs


def test_graph_replay_is_bit_identical():
    dims = ModelDims(n_layers=3)
    sd = make_weights(dims, seed=0)
    eager = _run(False, sd, dims)
    graph = _run(True, sd, dims)
    assert len(eager) == len(graph)
    for (pa, fa, ta), (pb, fb, tb) in zip(eager, graph):
        assert fa == fb and ta == tb
        for x, y in zip(pa, pb):
            assert np.array_equal(x, y)


def test_graph_replay_bit_identical_at_two_cta_batch():
    """20 streams x 14 frames = 280 rows: the 2-CTA GEMMs (a partial last row block of 24 rows, TMA-store and
    TMA reduce-add epilogues) give the same bits eagerly and replayed from the captured graph."""
    dims = ModelDims(n_layers=2)
    sd = make_weights(dims, seed=1)
    eager = _run(False, sd, dims, n=20)
    graph = _run(True, sd, dims, n=20)
    for (pa, fa, ta), (pb, fb, tb) in zip(eager, graph):
        assert fa == fb and ta == tb
        for x, y in zip(pa, pb):
            assert np.array_equal(x, y)


def test_graph_mode_timers_leave_results_unchanged():
    """The graph-mode kernel timers (ud_graph_timers: global-timer stamps in every 2-CTA GEMM, TMA attention,
    LayerNorm and conv-module launch, the steps captured in graphs of their own) give the same bits as graph replay
    without them. At 20 streams x 14 frames every step's launches of those kinds are timed (per layer 8 projections,
    one attention, one conv module, 4 LayerNorms) and the summed time of all of them is positive and below the
    step's wall time. (The short final chunks run too few rows for the 2-CTA GEMMs and are left out.)"""
    dims = ModelDims(n_layers=2)
    sd = make_weights(dims, seed=1)
    plain = _run(True, sd, dims, n=20)
    timed, readings = _run(True, sd, dims, n=20, timers=True)
    for (pa, fa, ta), (pb, fb, tb) in zip(plain, timed):
        assert fa == fb and ta == tb
        for x, y in zip(pa, pb):
            assert np.array_equal(x, y)
    full = [r for r in readings if r[0] >= 105]   # first (105 mel rows) and steady (121) chunks of all 20 streams
    assert len(full) >= 3
    for rows, wall_ms, kinds in full:
        assert kinds["gemm_tc2"][1] >= 2 * 8, kinds
        assert kinds["attention"][1] == 2 and kinds["conv"][1] == 2, kinds
        assert kinds["norm"][1] >= 2 * 4, kinds
        assert all(ms > 0.0 for ms, _ in kinds.values()), kinds
        assert sum(ms for ms, _ in kinds.values()) < wall_ms, (kinds, wall_ms)


def test_tma_attention_matches_one_cta_per_stream_head_kernel():
    """The persistent TMA-fed attention kernel and the one-CTA-per-(stream, head) kernel stage the same bf16 rows
    and run the same fragment arithmetic: a 2-layer engine gives the same bits with either (UD_ATTN_TMA=0 selects
    the latter), over first, steady and short final chunks of 20 streams."""
    dims = ModelDims(n_layers=2)
    sd = make_weights(dims, seed=2)
    a = _run(True, sd, dims, n=20)
    b = _run(True, sd, dims, n=20, env={"UD_ATTN_TMA": "0"})
    for (pa, fa, ta), (pb, fb, tb) in zip(a, b):
        assert fa == fb and ta == tb
        for x, y in zip(pa, pb):
            assert np.array_equal(x, y)


def test_two_stream_halves_are_bit_identical_to_one_stream():
    """Large batches run the layer stack as two halves on two streams (their LayerNorms and tail CTAs share SMs
    with the other half's GEMMs; by default from 8192 rows, UD_SPLIT=<rows> sets the threshold). Every row's
    arithmetic is the same as on one stream (UD_SPLIT=0): 80 streams (1,120 rows per steady chunk) with the
    threshold at 1024 rows give the same bits, replayed from graphs and eager."""
    dims = ModelDims(n_layers=2)
    sd = make_weights(dims, seed=3)
    one = _run(True, sd, dims, n=80, env={"UD_SPLIT": "0"})
    for graphs in (True, False):
        two = _run(graphs, sd, dims, n=80, env={"UD_SPLIT": "1024"})
        assert len(one) == len(two)
        for (pa, fa, ta), (pb, fb, tb) in zip(one, two):
            assert fa == fb and ta == tb
            for x, y in zip(pa, pb):
                assert np.array_equal(x, y)
