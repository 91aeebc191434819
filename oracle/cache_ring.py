"""Bit-exact CPU model of the per-stream attention/conv caches (test infrastructure only).

Reference semantics (Sources/DictatorEngine/Models/FastConformer.swift):
  * StreamState (:406-435): per layer, projected K and V of the last L frames and the last K-1 depthwise-conv
    inputs, all zero-initialised; cacheLen and a step counter.
  * the roll after a step of T frames (:470-477): next K/V cache = the last L rows of [cache ; T new rows],
    next conv cache = the last K-1 rows of [conv cache ; T new rows], cacheLen = min(cacheLen + T, L).
So after any sequence of steps the K/V cache tensor is: rows [0, L - cacheLen) zero, then the last cacheLen
frames in order; the conv cache holds the last K-1 frames (zeros before the first ones exist).

This model keeps frames by absolute index (like the engine's ring, which stores frame f at a page slot
derived from f) and reproduces those tensors exactly; the engine's gather must equal `gather` bit for bit
when both are fed the same row payloads. Payload dtype is opaque (bf16 rows compare as uint16 bit patterns).
"""

from __future__ import annotations

import numpy as np


class RingModel:
    def __init__(self, n_layers: int, d: int, left_context: int = 70, conv_rows: int = 8, dtype=np.uint16):
        self.NL, self.D, self.L, self.R, self.dtype = n_layers, d, left_context, conv_rows, dtype
        self.s: dict[int, dict] = {}

    def open(self, sid: int):
        self.s[sid] = dict(head=0, cache_len=0, kv={}, conv=np.zeros((self.NL, self.R, self.D), self.dtype))

    evict = open

    def close(self, sid: int):
        del self.s[sid]

    def append(self, sid: int, kv: np.ndarray | None, conv: np.ndarray | None):
        """kv [NL, 2, k, D] and conv [NL, k, D]: the k frames after the stream's head."""
        st = self.s[sid]
        if kv is not None:
            for t in range(kv.shape[2]):
                st["kv"][st["head"] + t] = kv[:, :, t].copy()
        if conv is not None:
            k = conv.shape[1]
            for t in range(max(0, k - self.R), k):
                st["conv"][:, (st["head"] + t) % self.R] = conv[:, t]

    def roll(self, sid: int, k: int):
        st = self.s[sid]
        st["head"] += k
        st["cache_len"] = min(st["cache_len"] + k, self.L)
        lo = st["head"] - self.L
        for f in [f for f in st["kv"] if f < lo]:
            del st["kv"][f]

    def gather(self, sid: int):
        """(kv [NL, 2, L, D] with rows j < L - cacheLen zero, conv [NL, R, D] oldest first)."""
        st = self.s[sid]
        kv = np.zeros((self.NL, 2, self.L, self.D), self.dtype)
        for j in range(self.L - st["cache_len"], self.L):
            kv[:, :, j] = st["kv"][st["head"] - self.L + j]
        conv = np.stack([st["conv"][:, (st["head"] + i) % self.R] for i in range(self.R)], axis=1)
        return kv, conv

    def info(self, sid: int):
        st = self.s[sid]
        return st["cache_len"], st["head"]


def bytes_per_stream_step(n_layers: int, d: int, elem: int, k: int, left_context: int = 70, conv_rows: int = 8,
                          n_kv: int = 2) -> int:
    """Algorithmic HBM bytes of one append + roll + gather of k frames for one stream, all layers:
    read and write the k new K/V rows, read the L-row window and write it out contiguous, write the last
    min(k, R) conv rows, read and write the R conv rows. The roll moves no data."""
    row = d * elem
    kv = n_kv * (k + k + left_context + left_context)
    conv = min(k, conv_rows) + k + conv_rows + conv_rows
    return n_layers * row * (kv + conv)
