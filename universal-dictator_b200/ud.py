"""ctypes binding of libud.so (include/ud.h), mirroring the reference's encoder protocol.

The reference's host side is Swift:
    protocol NemotronEncoder { var schedule: NemotronSchedule; func step(mel:nRows:validRows:keepAll:) throws
                               -> (proj: [Float], frames: Int) }      Sources/DictatorCore/Nemotron/NemotronStreamer.swift:6-12
    struct NemotronSchedule                                           Sources/DictatorCore/Nemotron/NemotronSchedule.swift:7-16
    enum EngineError: Error                                           Sources/DictatorCore/Errors.swift:3-10
This module exposes the same names and argument meanings over the C ABI: `CudaNemotronEncoder.step`
returns (proj [frames, joint_dim] float32, frames) and raises `EngineError` where the Swift code throws.
`Engine` adds the batched path, the cache operations and the RNN-T decoder.

The library is loaded from this directory (libud.so, built by build.py); there is no fallback: if the
library or a CUDA device is missing, construction raises.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path
from typing import Mapping, Sequence

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "libud.so"

UD_OK = 0
STATUS = {0: "ok", 1: "invalid argument", 2: "CUDA error", 3: "out of memory", 4: "no such stream",
          5: "pool exhausted", 6: "weights error", 7: "not ready", 8: "device wait expired", 9: "I/O error",
          10: "unsupported"}
DTYPE_F32, DTYPE_BF16 = 0, 1
KINDS = ["gemm_tc", "gemm_simt", "attention", "conv", "norm", "subsample", "rnnt", "cache", "other", "gemm_tc2"]

# Every symbol include/ud.h declares (the test suite checks the library exports exactly these).
ABI_SYMBOLS = [
    "ud_config_default", "ud_init", "ud_shutdown", "ud_load_weights", "ud_load_safetensors", "ud_stream_open",
    "ud_stream_close", "ud_stream_step", "ud_step_batch", "ud_step_batch_async", "ud_step_sync",
    "ud_step_batch_device", "ud_rnnt_decode",
    "ud_rnnt_decode_static",
    "ud_cache_append", "ud_cache_roll", "ud_cache_gather", "ud_cache_evict", "ud_cache_read", "ud_stream_info",
    "ud_get_cuda_stream", "ud_pool_info", "ud_synchronize", "ud_launch_count", "ud_debug_gemm",
    "ud_debug_wait_probe", "ud_profile_enable", "ud_profile_read", "ud_graph_timers", "ud_graph_timers_read",
    "ud_last_error",
    "ud_status_string", "ud_get_config", "ud_chunk_next", "ud_streamer_create", "ud_streamer_destroy",
    "ud_streamer_open", "ud_streamer_push", "ud_streamer_step", "ud_streamer_finished", "ud_streamer_tokens",
    "ud_streamer_release", "ud_streamer_emissions", "ud_streamer_step_times", "ud_streamer_set_end_padding",
    "ud_streamer_set_pipelined", "ud_streamer_open_audio", "ud_streamer_push_audio", "ud_mel_create", "ud_mel_destroy", "ud_mel_features", "ud_mel_features_device",
    "ud_mel_stream_open", "ud_mel_stream_close", "ud_mel_push_batch", "ud_detok_create", "ud_detok_create_file",
    "ud_detok_destroy", "ud_detok_size", "ud_detok_decode",
]


class EngineError(RuntimeError):
    """A non-OK ud_status (the Swift EngineError / GPU failure of the reference)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "n_layers", "d_model", "n_heads", "ff_dim", "conv_kernel", "left_context", "sub_channels", "mel_bins",
        "joint_dim", "vocab", "pred_layers", "pred_hidden", "max_symbols", "dtype", "max_streams", "max_batch",
        "max_chunk_frames", "page_frames", "n_pages")]


class Weight(C.Structure):
    _fields_ = [("name", C.c_char_p), ("data", C.POINTER(C.c_float)), ("ndim", C.c_int), ("shape", C.c_int64 * 4)]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: build it with universal-dictator_b200/build.py")
        L = C.CDLL(str(LIB_PATH))
        P, I, F, VP = C.POINTER, C.c_int, C.c_float, C.c_void_p
        eng = C.c_void_p
        sig = {
            "ud_config_default": (None, [P(Config)]),
            "ud_init": (I, [P(Config), I, P(eng)]),
            "ud_shutdown": (I, [eng]),
            "ud_load_weights": (I, [eng, P(Weight), I]),
            "ud_load_safetensors": (I, [eng, C.c_char_p]),
            "ud_stream_open": (I, [eng, I, P(C.c_int32)]),
            "ud_stream_close": (I, [eng, C.c_int32]),
            "ud_stream_step": (I, [eng, C.c_int32, P(F), I, I, I, P(F), P(I)]),
            "ud_step_batch": (I, [eng, I, P(C.c_int32), P(P(F)), P(I), P(I), P(I), P(F), P(I), P(C.c_int32), P(I)]),
            "ud_step_batch_async": (I, [eng, I, P(C.c_int32), P(P(F)), P(I), P(I), P(I), P(F), P(I), P(C.c_int32),
                                        P(I)]),
            "ud_step_sync": (I, [eng]),
            "ud_step_batch_device": (I, [eng, I, P(C.c_int32), VP, I, P(I), P(I), P(I), VP, P(I), VP, VP]),
            "ud_rnnt_decode": (I, [eng, C.c_int32, P(F), I, P(C.c_int32), P(I)]),
            "ud_rnnt_decode_static": (I, [eng, C.c_int32, P(F), I, P(C.c_int32), P(I)]),
            "ud_cache_append": (I, [eng, I, P(C.c_int32), I, VP, VP]),
            "ud_cache_roll": (I, [eng, I, P(C.c_int32), I]),
            "ud_cache_gather": (I, [eng, I, P(C.c_int32), VP, VP]),
            "ud_cache_evict": (I, [eng, I, P(C.c_int32)]),
            "ud_cache_read": (I, [eng, C.c_int32, I, I, VP]),
            "ud_stream_info": (I, [eng, C.c_int32, P(I), P(I), P(I)]),
            "ud_get_cuda_stream": (I, [eng, P(VP)]),
            "ud_pool_info": (I, [eng, P(I), P(I), P(I)]),
            "ud_synchronize": (I, [eng]),
            "ud_launch_count": (I, [eng, P(C.c_int64)]),
            "ud_debug_gemm": (I, [eng, VP, VP, I, I, I, VP, I, F, VP, F, VP, I]),
            "ud_debug_wait_probe": (I, [eng, C.c_uint64]),
            "ud_profile_enable": (I, [eng, I]),
            "ud_profile_read": (I, [eng, I, P(C.c_double), P(C.c_int64)]),
            "ud_graph_timers": (I, [eng, I]),
            "ud_graph_timers_read": (I, [eng, I, P(C.c_double), P(I)]),
            "ud_last_error": (C.c_size_t, [C.c_char_p, C.c_size_t]),
            "ud_status_string": (C.c_char_p, [I]),
            "ud_get_config": (I, [eng, P(Config)]),
            "ud_chunk_next": (I, [I, I, I, I, I, P(I), P(I), P(I), P(I), P(I)]),
            "ud_streamer_create": (I, [eng, I, I, P(VP)]),
            "ud_streamer_destroy": (I, [VP]),
            "ud_streamer_open": (I, [VP, P(F), I, P(C.c_int32)]),
            "ud_streamer_push": (I, [VP, C.c_int32, I, I]),
            "ud_streamer_step": (I, [VP, P(I), P(I)]),
            "ud_streamer_finished": (I, [VP, P(C.c_int32), I, P(I)]),
            "ud_streamer_tokens": (I, [VP, C.c_int32, P(C.c_int32), I, P(I), P(I)]),
            "ud_streamer_emissions": (I, [VP, C.c_int32, P(C.c_int32), P(C.c_int64), P(C.c_double), I, P(I)]),
            "ud_streamer_step_times": (I, [VP, C.c_int32, P(C.c_double), I, P(I)]),
            "ud_streamer_release": (I, [VP, C.c_int32]),
            "ud_streamer_set_end_padding": (I, [VP, I]),
            "ud_streamer_set_pipelined": (I, [VP, I]),
            "ud_streamer_open_audio": (I, [VP, VP, P(C.c_int32)]),
            "ud_streamer_push_audio": (I, [VP, I, P(C.c_int32), P(P(F)), P(I), P(I)]),
            "ud_mel_create": (I, [eng, P(F), I, P(F), I, P(VP)]),
            "ud_mel_destroy": (I, [VP]),
            "ud_mel_features": (I, [VP, P(F), I, P(F), I, P(I)]),
            "ud_mel_features_device": (I, [VP, I, VP, P(C.c_int64), P(I), VP, P(C.c_int64)]),
            "ud_mel_stream_open": (I, [VP, P(I)]),
            "ud_mel_stream_close": (I, [VP, I]),
            "ud_mel_push_batch": (I, [VP, I, P(I), P(P(F)), P(I), P(I), P(F), I, P(I)]),
            "ud_detok_create": (I, [C.c_char_p, C.c_size_t, P(VP)]),
            "ud_detok_create_file": (I, [C.c_char_p, P(VP)]),
            "ud_detok_destroy": (I, [VP]),
            "ud_detok_size": (I, [VP]),
            "ud_detok_decode": (I, [VP, P(C.c_int32), I, C.c_char_p, C.c_size_t, P(C.c_size_t)]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().ud_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(status: int):
    if status != UD_OK:
        raise EngineError(status, last_error())


def default_config(**kw) -> Config:
    c = Config()
    lib().ud_config_default(C.byref(c))
    for k, v in kw.items():
        if not hasattr(c, k):
            raise KeyError(k)
        setattr(c, k, int(v))
    return c


def _ptr(a: np.ndarray, ctype=C.c_float):
    return a.ctypes.data_as(C.POINTER(ctype))


def _i32(seq) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(seq, dtype=np.int32))


@dataclass(frozen=True)
class NemotronSchedule:
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
    def out_frames_per_chunk(self) -> int:
        return self.lookahead + 1

    @property
    def chunk_ms(self) -> int:
        return 80 * (self.lookahead + 1)


class Engine:
    """One libud engine: one CUDA device, one CUDA stream, shared weights, a pool of stream slots."""

    def __init__(self, config: Config | None = None, device: int = 0, **kw):
        self.cfg = config if config is not None else default_config(**kw)
        h = C.c_void_p()
        check(lib().ud_init(C.byref(self.cfg), device, C.byref(h)))
        self.h = h
        self.device = device

    def close(self):
        if getattr(self, "h", None):
            lib().ud_shutdown(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ---------------------------------------------------------------- weights
    def load_weights(self, sd: Mapping[str, object]):
        keep = []
        table = (Weight * len(sd))()
        for i, (name, t) in enumerate(sd.items()):
            a = t.detach().cpu().float().numpy() if hasattr(t, "detach") else np.asarray(t, np.float32)
            a = np.ascontiguousarray(a, dtype=np.float32)
            nm = name.encode()
            keep += [a, nm]
            table[i].name = nm
            table[i].data = _ptr(a)
            table[i].ndim = a.ndim
            for d in range(a.ndim):
                table[i].shape[d] = a.shape[d]
        check(lib().ud_load_weights(self.h, table, len(sd)))

    def load_safetensors(self, path: str | Path):
        check(lib().ud_load_safetensors(self.h, str(path).encode()))

    # ---------------------------------------------------------------- streams
    def open(self, lookahead: int) -> int:
        sid = C.c_int32()
        check(lib().ud_stream_open(self.h, lookahead, C.byref(sid)))
        return sid.value

    def close_stream(self, sid: int):
        check(lib().ud_stream_close(self.h, sid))

    def info(self, sid: int) -> tuple[int, int, int]:
        cl, hd, st = C.c_int(), C.c_int(), C.c_int()
        check(lib().ud_stream_info(self.h, sid, C.byref(cl), C.byref(hd), C.byref(st)))
        return cl.value, hd.value, st.value

    @property
    def out_width(self) -> int:
        return self.cfg.joint_dim or self.cfg.d_model

    def step(self, sid: int, mel: np.ndarray, n_rows: int, valid_rows: int, keep_all: bool):
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        out = np.zeros((self.cfg.max_chunk_frames, self.out_width), np.float32)
        fr = C.c_int()
        check(lib().ud_stream_step(self.h, sid, _ptr(mel), n_rows, valid_rows, int(keep_all), _ptr(out), C.byref(fr)))
        return out[:fr.value].copy(), fr.value

    def step_batch(self, ids: Sequence[int], mels: Sequence[np.ndarray], n_rows: Sequence[int],
                   valid_rows: Sequence[int], keep_all: Sequence[bool], decode: bool = False):
        """Host-buffer batched step. Returns (list of proj arrays, frames, list of token lists or None)."""
        n = len(ids)
        arrs = [np.ascontiguousarray(m, dtype=np.float32) for m in mels]
        ptrs = (C.POINTER(C.c_float) * n)(*[_ptr(a) for a in arrs])
        tm, W = self.cfg.max_chunk_frames, self.out_width
        out = np.empty((n, tm, W), np.float32)
        frames = np.zeros(n, np.int32)
        ids_a, nr, vr, ka = _i32(ids), _i32(n_rows), _i32(valid_rows), _i32([int(k) for k in keep_all])
        toks = np.zeros((n, tm * self.cfg.max_symbols), np.int32) if decode else None
        ntok = np.zeros(n, np.int32) if decode else None
        check(lib().ud_step_batch(self.h, n, _ptr(ids_a, C.c_int32), ptrs, _ptr(nr, C.c_int), _ptr(vr, C.c_int),
                                  _ptr(ka, C.c_int), _ptr(out), _ptr(frames, C.c_int),
                                  _ptr(toks, C.c_int32) if decode else None, _ptr(ntok, C.c_int) if decode else None))
        projs = [out[i, :frames[i]] for i in range(n)]     # views into one result block
        tok_lists = [toks[i, :ntok[i]].tolist() for i in range(n)] if decode else None
        return projs, frames.tolist(), tok_lists

    def step_batch_async(self, ids: Sequence[int], mels: Sequence[np.ndarray], n_rows: Sequence[int],
                         valid_rows: Sequence[int], keep_all: Sequence[bool], out: np.ndarray,
                         tokens: np.ndarray | None = None, n_tokens: np.ndarray | None = None) -> list[int]:
        """ud_step_batch_async: enqueues the step and returns its frames; the previous asynchronous step is
        complete on return. `out` [n, max_chunk_frames, out_width] fp32 (and `tokens` [n, max_chunk_frames *
        max_symbols] int32 with `n_tokens` [n] int32 when decoding) receive this step's results once the next
        step_batch_async or step_sync returns. Inputs and outputs should be pinned host memory (views of
        torch.empty(..., pin_memory=True)) for the copies to overlap compute; this object keeps them alive until
        the step completes."""
        n = len(ids)
        tm, W = self.cfg.max_chunk_frames, self.out_width
        if out.dtype != np.float32 or not out.flags.c_contiguous or out.size < n * tm * W:
            raise ValueError("out must be a C-contiguous float32 array of at least n * max_chunk_frames * out_width")
        if tokens is not None and (tokens.dtype != np.int32 or n_tokens is None or n_tokens.dtype != np.int32
                                   or not tokens.flags.c_contiguous or tokens.size < n * tm * self.cfg.max_symbols
                                   or n_tokens.size < n):
            raise ValueError("tokens / n_tokens: int32 arrays of n * max_chunk_frames * max_symbols and n")
        arrs = [m if (m.dtype == np.float32 and m.flags.c_contiguous) else np.ascontiguousarray(m, np.float32)
                for m in mels]
        ptrs = (C.POINTER(C.c_float) * n)(*[_ptr(a) for a in arrs])
        frames = np.zeros(n, np.int32)
        ids_a, nr, vr, ka = _i32(ids), _i32(n_rows), _i32(valid_rows), _i32([int(k) for k in keep_all])
        check(lib().ud_step_batch_async(self.h, n, _ptr(ids_a, C.c_int32), ptrs, _ptr(nr, C.c_int),
                                        _ptr(vr, C.c_int), _ptr(ka, C.c_int), _ptr(out),
                                        _ptr(frames, C.c_int),
                                        _ptr(tokens, C.c_int32) if tokens is not None else None,
                                        _ptr(n_tokens, C.c_int) if tokens is not None else None))
        refs = getattr(self, "_async_refs", [])
        self._async_refs = (refs + [(arrs, out, tokens, n_tokens)])[-2:]   # this step and the one in flight
        return frames.tolist()

    def step_sync(self):
        """ud_step_sync: every asynchronous step complete."""
        check(lib().ud_step_sync(self.h))
        self._async_refs = []

    def step_batch_device(self, ids, mel_dev_ptr: int, rows_stride: int, n_rows, valid_rows, keep_all,
                          proj_dev_ptr: int, tokens_dev_ptr: int | None = None, ntok_dev_ptr: int | None = None):
        """Device-resident batched step, asynchronous on the engine stream. Returns frames (host)."""
        n = len(ids)
        frames = np.zeros(n, np.int32)
        ids_a, nr, vr, ka = _i32(ids), _i32(n_rows), _i32(valid_rows), _i32([int(k) for k in keep_all])
        check(lib().ud_step_batch_device(self.h, n, _ptr(ids_a, C.c_int32), C.c_void_p(mel_dev_ptr), rows_stride,
                                         _ptr(nr, C.c_int), _ptr(vr, C.c_int), _ptr(ka, C.c_int),
                                         C.c_void_p(proj_dev_ptr), _ptr(frames, C.c_int),
                                         C.c_void_p(tokens_dev_ptr) if tokens_dev_ptr else None,
                                         C.c_void_p(ntok_dev_ptr) if ntok_dev_ptr else None))
        return frames.tolist()

    def rnnt_decode(self, sid: int, f: np.ndarray) -> list[int]:
        f = np.ascontiguousarray(f, dtype=np.float32)
        toks = np.zeros(max(1, f.shape[0] * self.cfg.max_symbols), np.int32)
        nt = C.c_int()
        check(lib().ud_rnnt_decode(self.h, sid, _ptr(f), f.shape[0], _ptr(toks, C.c_int32), C.byref(nt)))
        return toks[:nt.value].tolist()

    def rnnt_decode_static(self, sid: int, f: np.ndarray) -> list[int]:
        """ud_rnnt_decode_static: the same decode with its scratch in the library's static device block (no
        allocation in the call; overlapping calls on one device race)."""
        f = np.ascontiguousarray(f, dtype=np.float32)
        toks = np.zeros(max(1, f.shape[0] * self.cfg.max_symbols), np.int32)
        nt = C.c_int()
        check(lib().ud_rnnt_decode_static(self.h, sid, _ptr(f), f.shape[0], _ptr(toks, C.c_int32), C.byref(nt)))
        return toks[:nt.value].tolist()

    # ---------------------------------------------------------------- caches
    def cache_append(self, ids, k: int, kv_dev_ptr: int | None, conv_dev_ptr: int | None):
        a = _i32(ids)
        check(lib().ud_cache_append(self.h, len(a), _ptr(a, C.c_int32), k,
                                    C.c_void_p(kv_dev_ptr) if kv_dev_ptr else None,
                                    C.c_void_p(conv_dev_ptr) if conv_dev_ptr else None))

    def cache_roll(self, ids, k: int):
        a = _i32(ids)
        check(lib().ud_cache_roll(self.h, len(a), _ptr(a, C.c_int32), k))

    def cache_gather(self, ids, kv_dev_ptr: int | None, conv_dev_ptr: int | None):
        a = _i32(ids)
        check(lib().ud_cache_gather(self.h, len(a), _ptr(a, C.c_int32),
                                    C.c_void_p(kv_dev_ptr) if kv_dev_ptr else None,
                                    C.c_void_p(conv_dev_ptr) if conv_dev_ptr else None))

    def cache_evict(self, ids):
        a = _i32(ids)
        check(lib().ud_cache_evict(self.h, len(a), _ptr(a, C.c_int32)))

    def cache_read(self, sid: int, layer: int, kind: int) -> np.ndarray:
        """One stream's window of one layer: kind 0 K / 1 V -> [L, d], kind 2 conv -> [k-1, d]; raw dtype
        (float32, or bf16 returned as uint16 bit patterns)."""
        rows = self.cfg.left_context if kind < 2 else self.cfg.conv_kernel - 1
        dt = np.uint16 if self.cfg.dtype == DTYPE_BF16 else np.float32
        out = np.zeros((rows, self.cfg.d_model), dt)
        check(lib().ud_cache_read(self.h, sid, layer, kind, out.ctypes.data_as(C.c_void_p)))
        return out

    def pool_info(self) -> tuple[int, int, int]:
        f, t, e = C.c_int(), C.c_int(), C.c_int()
        check(lib().ud_pool_info(self.h, C.byref(f), C.byref(t), C.byref(e)))
        return f.value, t.value, e.value

    def cuda_stream(self) -> int:
        p = C.c_void_p()
        check(lib().ud_get_cuda_stream(self.h, C.byref(p)))
        return p.value or 0

    def synchronize(self):
        check(lib().ud_synchronize(self.h))

    def profile(self, enable: bool):
        check(lib().ud_profile_enable(self.h, int(enable)))

    def profile_read(self) -> dict[str, tuple[float, int]]:
        """{kind: (total device ms, launches)} since profiling was enabled."""
        out = {}
        for k, name in enumerate(KINDS):
            ms, n = C.c_double(), C.c_int64()
            check(lib().ud_profile_read(self.h, k, C.byref(ms), C.byref(n)))
            out[name] = (ms.value, n.value)
        return out

    def graph_timers(self, enable: bool):
        """Graph-mode kernel timers for the following steps (their graphs are captured separately)."""
        check(lib().ud_graph_timers(self.h, int(enable)))

    def graph_timers_read(self) -> dict[str, tuple[float, int]]:
        """{kind: (summed device ms of the last step's launches of that kind, each from its first CTA past the
        grid-dependency wait to its last CTA's end; launches)} for the timed kinds."""
        out = {}
        for name in ("gemm_tc2", "attention", "norm", "conv"):
            ms, n = C.c_double(), C.c_int()
            check(lib().ud_graph_timers_read(self.h, KINDS.index(name), C.byref(ms), C.byref(n)))
            out[name] = (ms.value, n.value)
        return out

    def launch_count(self) -> int:
        v = C.c_int64()
        check(lib().ud_launch_count(self.h, C.byref(v)))
        return v.value

    def debug_gemm(self, A_ptr, W_ptr, M, N, K, C_ptr, bias_ptr=None, act=0, out_scale=1.0, res_ptr=None,
                   res_scale=1.0, out_bf16=False):
        check(lib().ud_debug_gemm(self.h, C.c_void_p(A_ptr), C.c_void_p(W_ptr), M, N, K,
                                  C.c_void_p(bias_ptr) if bias_ptr else None, act, out_scale,
                                  C.c_void_p(res_ptr) if res_ptr else None, res_scale, C.c_void_p(C_ptr),
                                  int(out_bf16)))


def chunk_next(lookahead: int, idx: int, avail: int, last: bool, end_padding: bool = True):
    """ud_chunk_next: (1, start, n_rows, valid_rows, keep_all, next_idx) for a ready chunk, (0, ...) to wait,
    (-1, ...) when the stream has ended."""
    st, rows, valid, keep, nxt = C.c_int(), C.c_int(), C.c_int(), C.c_int(), C.c_int()
    r = lib().ud_chunk_next(lookahead, idx, avail, int(last), int(end_padding), C.byref(st), C.byref(rows),
                            C.byref(valid), C.byref(keep), C.byref(nxt))
    return r, st.value, rows.value, valid.value, bool(keep.value), nxt.value


class Streamer:
    """Host-side batched streamer (NemotronStreamer.swift:16-163) over one engine: streams read mel from their own
    host buffers, rows arrive with push(), and step() runs every stream with a ready chunk in one batched pass,
    appending each stream's greedy RNN-T tokens."""

    def __init__(self, engine: "Engine", lookahead: int, decode: bool = True):
        self.engine = engine
        self.h = C.c_void_p()
        check(lib().ud_streamer_create(engine.h, lookahead, int(decode), C.byref(self.h)))
        self._bufs: dict[int, np.ndarray] = {}

    def open(self, mel: np.ndarray) -> int:
        """Registers a stream over `mel` [rows, mel_bins] (kept alive here); no rows are available until pushed."""
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        sid = C.c_int32()
        check(lib().ud_streamer_open(self.h, _ptr(mel), mel.shape[0], C.byref(sid)))
        self._bufs[sid.value] = mel
        return sid.value

    def push(self, sid: int, n_rows: int, last: bool = False):
        check(lib().ud_streamer_push(self.h, sid, n_rows, int(last)))

    def set_end_padding(self, on: bool):
        check(lib().ud_streamer_set_end_padding(self.h, int(on)))

    def set_pipelined(self, on: bool):
        """ud_streamer_set_pipelined: each step's results appear one step later; the copies and the host's
        chunk gathering overlap the device's work."""
        check(lib().ud_streamer_set_pipelined(self.h, int(on)))

    def open_audio(self, frontend: "MelFrontend") -> int:
        """An audio stream whose mel comes from `frontend` (NemotronStreamer.push(samples:))."""
        sid = C.c_int32()
        check(lib().ud_streamer_open_audio(self.h, frontend.h, C.byref(sid)))
        return sid.value

    def push_audio(self, ids, chunks, last=None):
        n = len(ids)
        arrs = [np.ascontiguousarray(np.asarray(c, np.float32)) for c in chunks]
        ptrs = (C.POINTER(C.c_float) * n)(*[_ptr(a) for a in arrs])
        ids_a, ns = np.ascontiguousarray(np.asarray(ids, np.int32)), _i32([a.shape[0] for a in arrs])
        fin = _i32([int(bool(f)) for f in last]) if last is not None else None
        check(lib().ud_streamer_push_audio(self.h, n, _ptr(ids_a, C.c_int32), ptrs, _ptr(ns, C.c_int),
                                           _ptr(fin, C.c_int) if fin is not None else None))

    def step(self) -> tuple[int, int]:
        """One batched step: (streams advanced, streams finished)."""
        n, d = C.c_int(), C.c_int()
        check(lib().ud_streamer_step(self.h, C.byref(n), C.byref(d)))
        return n.value, d.value

    def finished(self) -> list[int]:
        """Ids of the streams that finished in the last step."""
        n = C.c_int()
        check(lib().ud_streamer_finished(self.h, None, 0, C.byref(n)))
        out = np.zeros(max(1, n.value), np.int32)
        check(lib().ud_streamer_finished(self.h, _ptr(out, C.c_int32), n.value, C.byref(n)))
        return out[:n.value].tolist()

    def tokens(self, sid: int) -> tuple[list[int], bool]:
        n, fin = C.c_int(), C.c_int()
        check(lib().ud_streamer_tokens(self.h, sid, None, 0, C.byref(n), C.byref(fin)))
        out = np.zeros(max(1, n.value), np.int32)
        check(lib().ud_streamer_tokens(self.h, sid, _ptr(out, C.c_int32), n.value, C.byref(n), C.byref(fin)))
        return out[:n.value].tolist(), bool(fin.value)

    def emissions(self, sid: int) -> list[tuple[int, int, float]]:
        """ud_streamer_emissions: (token, samples_seen, compute_seconds) per token (the reference's Emission)."""
        n = C.c_int()
        check(lib().ud_streamer_emissions(self.h, sid, None, None, None, 0, C.byref(n)))
        k = max(1, n.value)
        t, ss, cs = np.zeros(k, np.int32), np.zeros(k, np.int64), np.zeros(k, np.float64)
        check(lib().ud_streamer_emissions(self.h, sid, _ptr(t, C.c_int32), _ptr(ss, C.c_int64), _ptr(cs, C.c_double),
                                          n.value, C.byref(n)))
        return [(int(t[i]), int(ss[i]), float(cs[i])) for i in range(n.value)]

    def step_times(self, sid: int) -> list[float]:
        """ud_streamer_step_times: wall seconds of each step the stream took part in (wallTimes)."""
        n = C.c_int()
        check(lib().ud_streamer_step_times(self.h, sid, None, 0, C.byref(n)))
        out = np.zeros(max(1, n.value), np.float64)
        check(lib().ud_streamer_step_times(self.h, sid, _ptr(out, C.c_double), n.value, C.byref(n)))
        return out[:n.value].tolist()

    def release(self, sid: int):
        check(lib().ud_streamer_release(self.h, sid))
        self._bufs.pop(sid, None)

    def close(self):
        if self.h:
            check(lib().ud_streamer_destroy(self.h))
            self.h = C.c_void_p()
            self._bufs.clear()


class MelFrontend:
    """Log-mel frontend on an engine's device and stream (NemoMelFrontend / NemoMelStream,
    Sources/DictatorCore/Audio/NemoMel.swift:10-161): fb [n_mels, 257] and window [400] are the checkpoint's
    preprocessor.featurizer buffers."""

    HOP = 160

    def __init__(self, engine: "Engine", fb: np.ndarray, window: np.ndarray, max_streams: int = 0):
        self.engine = engine
        self.fb = np.ascontiguousarray(np.asarray(fb, np.float32).reshape(-1, 257))
        self.n_mels = self.fb.shape[0]
        w = np.ascontiguousarray(np.asarray(window, np.float32))
        if w.shape != (400,):
            raise ValueError("window must have 400 taps")
        self.h = C.c_void_p()
        check(lib().ud_mel_create(engine.h, _ptr(self.fb), self.n_mels, _ptr(w), max_streams, C.byref(self.h)))

    def features(self, audio: np.ndarray) -> np.ndarray:
        """Full utterance: [n // 160 + 1, n_mels], the last frame 0."""
        a = np.ascontiguousarray(np.asarray(audio, np.float32))
        T = a.shape[0] // self.HOP + 1
        out = np.empty((T, self.n_mels), np.float32)
        nf = C.c_int()
        check(lib().ud_mel_features(self.h, _ptr(a), a.shape[0], _ptr(out), T, C.byref(nf)))
        return out[:nf.value]

    def features_device(self, audio_dev_ptr: int, sample_off, n_samples, mel_dev_ptr: int, row_off):
        """Device-resident batch, asynchronous on the engine stream (see ud_mel_features_device)."""
        so = np.ascontiguousarray(np.asarray(sample_off, np.int64))
        ro = np.ascontiguousarray(np.asarray(row_off, np.int64))
        ns = _i32(n_samples)
        check(lib().ud_mel_features_device(self.h, len(ns), C.c_void_p(audio_dev_ptr), _ptr(so, C.c_int64),
                                           _ptr(ns, C.c_int), C.c_void_p(mel_dev_ptr), _ptr(ro, C.c_int64)))

    def open(self) -> int:
        i = C.c_int()
        check(lib().ud_mel_stream_open(self.h, C.byref(i)))
        return i.value

    def close_stream(self, sid: int):
        check(lib().ud_mel_stream_close(self.h, sid))

    def push(self, ids, chunks, finish=None, cap_frames: int | None = None) -> list[np.ndarray]:
        """Pushes one chunk of samples per stream; returns each stream's new frames [k, n_mels]."""
        n = len(ids)
        arrs = [np.ascontiguousarray(np.asarray(c, np.float32)) for c in chunks]
        if cap_frames is None:
            cap_frames = max([a.shape[0] // self.HOP + 4 for a in arrs] + [4])
        ptrs = (C.POINTER(C.c_float) * n)(*[_ptr(a) for a in arrs])
        ids_a, ns = _i32(ids), _i32([a.shape[0] for a in arrs])
        fin = _i32([int(bool(f)) for f in finish]) if finish is not None else _i32([0] * n)
        out = np.empty((n, cap_frames, self.n_mels), np.float32)
        nf = np.zeros(n, np.int32)
        check(lib().ud_mel_push_batch(self.h, n, _ptr(ids_a, C.c_int), ptrs, _ptr(ns, C.c_int), _ptr(fin, C.c_int),
                                      _ptr(out), cap_frames, _ptr(nf, C.c_int)))
        return [out[i, :nf[i]].copy() for i in range(n)]

    def close(self):
        if self.h:
            check(lib().ud_mel_destroy(self.h))
            self.h = C.c_void_p()


class SentencePieceDecoder:
    """SentencePiece detokenizer (SentencePiece.swift:5-32) over the C ABI; host only, no GPU."""

    def __init__(self, vocab_text: str | bytes | None = None, vocab_file: str | None = None):
        self.h = C.c_void_p()
        if vocab_file is not None:
            check(lib().ud_detok_create_file(str(vocab_file).encode(), C.byref(self.h)))
        else:
            b = vocab_text.encode() if isinstance(vocab_text, str) else bytes(vocab_text or b"")
            check(lib().ud_detok_create(b, len(b), C.byref(self.h)))

    @property
    def count(self) -> int:
        return lib().ud_detok_size(self.h)

    def decode(self, ids) -> str:
        a = _i32(list(ids))
        n = C.c_size_t()
        check(lib().ud_detok_decode(self.h, _ptr(a, C.c_int32), len(a), None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value + 1)
        check(lib().ud_detok_decode(self.h, _ptr(a, C.c_int32), len(a), buf, n.value + 1, C.byref(n)))
        return buf.raw[:n.value].decode("utf-8")

    def close(self):
        if self.h:
            lib().ud_detok_destroy(self.h)
            self.h = C.c_void_p()


def wait_probe(engine: "Engine", limit_ns: int):
    check(lib().ud_debug_wait_probe(engine.h, limit_ns))


class CudaNemotronEncoder:
    """NemotronEncoder conformer over libud: one object = one stream's caches (NemotronStreamer.swift:6-12)."""

    def __init__(self, engine: Engine, schedule: NemotronSchedule):
        self.engine = engine
        self.schedule = schedule
        self.sid = engine.open(schedule.lookahead)

    def step(self, mel: np.ndarray, n_rows: int, valid_rows: int, keep_all: bool):
        return self.engine.step(self.sid, mel, n_rows, valid_rows, keep_all)

    def close(self):
        if self.sid is not None:
            self.engine.close_stream(self.sid)
            self.sid = None
