"""The C-ABI library: it loads, exports every symbol include/ud.h declares (and only those), and fails loudly
(an error status with a message, never a crash or a silent CPU path) where no CUDA device is present."""

import re
import subprocess
from pathlib import Path

import pytest

import ud

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "ud.h").read_text()
    return sorted(set(re.findall(r"^UD_API\s+[\w\s\*]*?\b(ud_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_binding_symbols():
    assert header_symbols() == sorted(ud.ABI_SYMBOLS)


def test_library_exports_exactly_the_header():
    lib = ud.LIB_PATH
    assert lib.exists(), "libud.so must be built in-tree (universal-dictator_b200/build.py)"
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True, text=True, check=True).stdout
    exported = sorted({m.group(1) for m in re.finditer(r"\sT\s(ud_\w+)$", out, flags=re.M)})
    assert exported == header_symbols()


def test_loads_and_binds_every_symbol():
    L = ud.lib()
    for name in ud.ABI_SYMBOLS:
        assert getattr(L, name) is not None


def test_config_defaults_are_nemotron():
    c = ud.default_config()
    assert (c.n_layers, c.d_model, c.n_heads, c.ff_dim, c.conv_kernel, c.left_context) == (24, 1024, 8, 4096, 9, 70)
    assert (c.sub_channels, c.mel_bins, c.joint_dim, c.vocab, c.pred_hidden, c.max_symbols) == (256, 128, 640, 1025, 640, 10)
    assert c.dtype == ud.DTYPE_BF16 and c.page_frames == 16


def test_status_strings():
    L = ud.lib()
    assert L.ud_status_string(0) == b"ok"
    assert L.ud_status_string(8) == b"device wait expired"


def test_invalid_config_is_rejected_before_touching_a_device():
    with pytest.raises(ud.EngineError) as ei:
        ud.Engine(ud.default_config(conv_kernel=7))
    assert ei.value.status == 10 and "conv_kernel" in str(ei.value)
    with pytest.raises(ud.EngineError) as ei:
        ud.Engine(ud.default_config(max_chunk_frames=64))
    assert ei.value.status == 1


def test_no_device_fails_loudly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(ud.EngineError) as ei:
        ud.Engine(ud.default_config())
    assert ei.value.status == 2
    assert "device" in str(ei.value).lower()


def test_null_handles_are_statuses_not_crashes():
    """Entry points given a NULL engine / streamer / frontend / decoder return a status (no device needed)."""
    import ctypes as C

    L = ud.lib()
    out = (C.c_float * 16)()
    frames = (C.c_int * 1)()
    ids = (C.c_int32 * 1)(0)
    rows = (C.c_int * 1)(9)
    mel = (C.POINTER(C.c_float) * 1)(C.cast(out, C.POINTER(C.c_float)))
    assert L.ud_step_batch_async(None, 1, ids, mel, rows, rows, rows, out, frames, None, None) == 1
    assert L.ud_step_sync(None) == 1
    assert L.ud_synchronize(None) == 1
    assert L.ud_streamer_set_pipelined(None, 1) == 1
    n = C.c_int()
    assert L.ud_streamer_emissions(None, 0, None, None, None, 0, C.byref(n)) == 4
    assert L.ud_streamer_step_times(None, 0, None, 0, C.byref(n)) == 4
    assert L.ud_detok_decode(None, None, 0, None, 0, C.byref(C.c_size_t())) == 1
