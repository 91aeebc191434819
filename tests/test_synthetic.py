"""The package's synthetic-input module (used by the benchmark) generates exactly what the CPU oracle
generates: the same tensors under the same names for every model shape the tests and benchmarks use, and the
same algorithmic byte count for the cache operations."""

import pytest
import torch

import ud_synthetic as syn
from oracle import cache_ring
from oracle import mel as om
from oracle import weights as ow


@pytest.mark.parametrize("dims", [ow.BLOCK1, ow.ModelDims(n_layers=2), ow.ModelDims(n_layers=0, sub_channels=0,
                                                                                     pred_layers=2)],
                         ids=["block1", "two_layers", "rnnt_only"])
def test_weights_identical(dims):
    a = ow.make_weights(dims, seed=3)
    b = syn.make_weights(syn.ModelDims(**dims.__dict__), seed=3)
    assert list(a) == list(b)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def test_full_model_names_and_dims():
    assert syn.NEMOTRON == syn.ModelDims(**ow.NEMOTRON.__dict__)
    assert [n for n, _ in syn._names_shapes(syn.NEMOTRON)] == [n for n, _ in ow.tensor_specs(ow.NEMOTRON)]


@pytest.mark.parametrize("k", [1, 2, 7, 14])
def test_cache_bytes_identical(k):
    assert syn.cache_bytes_per_stream_step(24, 1024, 2, k) == cache_ring.bytes_per_stream_step(24, 1024, 2, k)


def test_mel_buffers_identical():
    assert (syn.mel_filterbank() == om.slaney_filterbank().numpy()).all()
    assert (syn.hann_window() == om.hann_symmetric().numpy()).all()
