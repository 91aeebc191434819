"""CUDA-graph replay of the steady step gives bit-identical results to eager launches (same engine code,
same inputs), across shape changes (first chunk, steady chunks, a short final chunk) and across the two
batched entry points."""

import os

import numpy as np
import pytest
import torch

import ud
from oracle.stream_step import chunk_plan
from oracle.weights import ModelDims, make_weights

pytestmark = pytest.mark.gpu


def _run(graphs: bool, sd, dims):
    os.environ["UD_GRAPHS"] = "1" if graphs else "0"
    try:
        e = ud.Engine(ud.default_config(n_layers=dims.n_layers, max_streams=4, max_batch=4))
    finally:
        os.environ.pop("UD_GRAPHS", None)
    e.load_weights(sd)
    ids = [e.open(13) for _ in range(3)]
    mels = [torch.randn(400, 128, generator=torch.Generator().manual_seed(20 + i)).numpy() for i in range(3)]
    plans = [list(chunk_plan(400, 13, 400 - 7 * i)) for i in range(3)]
    outs = []
    for k in range(max(len(p) for p in plans)):
        act = [i for i in range(3) if k < len(plans[i])]
        chunks = [mels[i][plans[i][k][0]:plans[i][k][0] + plans[i][k][1]] for i in act]
        projs, frames, toks = e.step_batch([ids[i] for i in act], chunks, [plans[i][k][1] for i in act],
                                           [plans[i][k][2] for i in act], [plans[i][k][3] for i in act], decode=True)
        outs.append((projs, frames, toks))
    e.close()
    return outs


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
