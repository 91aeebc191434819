"""The safetensors weight loader (ud_load_safetensors; SafeTensorsHeader / widenToFloats,
Sources/DictatorCore/Weights/WeightSource.swift:10-56) on the GPU.

  * an F32 file with every tensor of a 2-layer model, plus tensors the engine does not use and a __metadata__
    entry, loads to an engine whose streaming steps are bit-identical to one loaded from the same tensors
    through ud_load_weights;
  * BF16 and F16 files (matrices in the 16-bit type, vectors in F32, as exported checkpoints mix them) equal
    engines loaded with the tensors rounded to that type: the loader widens 16-bit values exactly;
  * tensors of other dtypes (integer counters) are skipped; a missing tensor, a bad header and a missing file are
    statuses."""

import json
import struct

import numpy as np
import pytest
import torch
from safetensors.numpy import save_file

import ud
from oracle.stream_step import chunk_plan
from oracle.weights import ModelDims, make_weights

pytestmark = pytest.mark.gpu

DIMS = ModelDims(n_layers=2)


def _cfg():
    return ud.default_config(n_layers=2, max_streams=2, max_batch=2)


def _steps(eng, n_rows=121, lookahead=1):
    """Three streaming steps of one stream; the projections of each."""
    sid = eng.open(lookahead)
    mel = torch.randn(n_rows, 128, generator=torch.Generator().manual_seed(9)).numpy()
    out = []
    for start, n, v, ka in chunk_plan(n_rows, lookahead):
        proj, fr = eng.step(sid, mel[start:start + n], n, v, ka)
        out.append(proj.copy())
        if len(out) == 3:
            break
    eng.close_stream(sid)
    return out


def _engine(load):
    e = ud.Engine(_cfg())
    load(e)
    return e


def _np_dict(sd):
    return {k: v.detach().cpu().float().numpy() for k, v in sd.items()}


def _write_bf16_file(path, sd):
    """safetensors with matrices BF16 and vectors F32 (the format written by hand: numpy has no bfloat16)."""
    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for k, v in sd.items():
        t = v.detach().cpu().float()
        if t.dim() >= 2:
            raw = t.to(torch.bfloat16).view(torch.int16).numpy().tobytes()
            dt = "BF16"
        else:
            raw = t.numpy().astype(np.float32).tobytes()
            dt = "F32"
        header[k] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


@pytest.fixture(scope="module")
def sd():
    return make_weights(DIMS, seed=3)


@pytest.fixture(scope="module")
def reference(sd):
    e = _engine(lambda e: e.load_weights(sd))
    out = _steps(e)
    e.close()
    return out


def test_f32_file_equals_load_weights(tmp_path, sd, reference):
    d = _np_dict(sd)
    d["preprocessor.featurizer.window"] = np.hanning(400).astype(np.float32)   # not used by the engine
    d["decoder.unused_extra"] = np.zeros((3, 5), np.float32)
    d["encoder.layers.0.conv.batch_norm.num_batches_tracked"] = np.array(7, np.int64)   # skipped (not a float)
    p = tmp_path / "model_f32.safetensors"
    save_file(d, str(p), metadata={"source": "test"})
    e = _engine(lambda e: e.load_safetensors(p))
    got = _steps(e)
    e.close()
    for a, b in zip(got, reference):
        assert np.array_equal(a, b)


def test_bf16_file_equals_rounded_weights(tmp_path, sd):
    p = tmp_path / "model_bf16.safetensors"
    _write_bf16_file(p, sd)
    rounded = {k: (v.to(torch.bfloat16).float() if v.dim() >= 2 else v) for k, v in sd.items()}
    e1 = _engine(lambda e: e.load_safetensors(p))
    e2 = _engine(lambda e: e.load_weights(rounded))
    a, b = _steps(e1), _steps(e2)
    e1.close()
    e2.close()
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_f16_file_equals_rounded_weights(tmp_path, sd):
    d = {k: (v.detach().cpu().half().numpy() if v.dim() >= 2 else v.detach().cpu().float().numpy())
         for k, v in sd.items()}
    p = tmp_path / "model_f16.safetensors"
    save_file(d, str(p))
    rounded = {k: (v.half().float() if v.dim() >= 2 else v) for k, v in sd.items()}
    e1 = _engine(lambda e: e.load_safetensors(p))
    e2 = _engine(lambda e: e.load_weights(rounded))
    a, b = _steps(e1), _steps(e2)
    e1.close()
    e2.close()
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_loader_errors_are_statuses(tmp_path, sd):
    d = _np_dict(sd)
    missing = dict(d)
    del missing["encoder.layers.1.feed_forward2.linear2.weight"]
    p = tmp_path / "missing.safetensors"
    save_file(missing, str(p))
    e = ud.Engine(_cfg())
    with pytest.raises(ud.EngineError) as ei:
        e.load_safetensors(p)
    assert ei.value.status == 6   # UD_ERR_WEIGHTS
    e.close()

    bad = tmp_path / "bad.safetensors"
    bad.write_bytes(struct.pack("<Q", 12) + b"{not json!!}")
    e = ud.Engine(_cfg())
    with pytest.raises(ud.EngineError) as ei:
        e.load_safetensors(bad)
    assert ei.value.status == 9   # UD_ERR_IO
    neg = tmp_path / "neg.safetensors"
    h = b'{"a":{"dtype":"F32","shape":[1],"data_offsets":[-4,0]}}'
    neg.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 4)
    with pytest.raises(ud.EngineError) as ei:
        e.load_safetensors(neg)
    assert ei.value.status == 9
    with pytest.raises(ud.EngineError) as ei:
        e.load_safetensors(tmp_path / "does_not_exist.safetensors")
    assert ei.value.status == 9
    q = tmp_path / "ints.safetensors"
    save_file({"some.int.tensor": np.arange(6, dtype=np.int64)}, str(q))
    with pytest.raises(ud.EngineError) as ei:
        e.load_safetensors(q)
    assert ei.value.status == 6   # nothing the engine can read
    e.close()
