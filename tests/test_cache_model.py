"""The CPU cache model against the reference's roll semantics, and its invariants.

The reference's own sliding-cache test (Tests/DictatorEngineTests/SlidingKVTests.swift:8-29) stores each row's
absolute position as its payload and checks, after many variable-size shifts, that every query's key range
covers exactly the last `window` positions. The same pattern pins the model here."""

import numpy as np

from oracle.cache_ring import RingModel, bytes_per_stream_step


def roll_reference(cache: np.ndarray, new_rows: np.ndarray) -> np.ndarray:
    """FastConformer.swift:470-472: next cache = last L rows of [cache ; new rows]."""
    L = cache.shape[0]
    return np.concatenate([cache, new_rows], 0)[-L:]


def test_window_holds_exact_positions_after_variable_steps():
    L, D = 70, 4
    m = RingModel(n_layers=1, d=D, left_context=L, conv_rows=8, dtype=np.int64)
    m.open(0)
    ref_k = np.zeros((L, D), np.int64)
    ref_conv = np.zeros((8, D), np.int64)
    cache_len = 0
    pos = 0
    rng = np.random.default_rng(0)
    for k in rng.integers(1, 15, size=60):
        k = int(k)
        rows = np.repeat(np.arange(pos + 1, pos + k + 1, dtype=np.int64)[:, None], D, 1)   # payload = position + 1
        kv = np.stack([rows, -rows])[None]                                                    # [1, 2, k, D]
        m.append(0, kv, rows[None])
        m.roll(0, k)
        ref_k = roll_reference(ref_k, rows)
        ref_conv = roll_reference(ref_conv, rows)
        cache_len = min(cache_len + k, L)
        pos += k
        got_kv, got_conv = m.gather(0)
        assert np.array_equal(got_kv[0, 0], ref_k)
        assert np.array_equal(got_kv[0, 1], -ref_k)
        assert np.array_equal(got_conv[0], ref_conv)
        assert m.info(0) == (cache_len, pos)
        # Visible keys [L - cacheLen, L) are exactly the last cacheLen positions.
        vis = got_kv[0, 0, L - cache_len:, 0]
        assert vis.tolist() == list(range(pos - cache_len + 1, pos + 1))
    # The model keeps no frame older than the window.
    assert min(m.s[0]["kv"]) >= pos - L


def test_evict_restarts_from_zero():
    m = RingModel(n_layers=2, d=8, dtype=np.uint16)
    m.open(3)
    m.append(3, np.ones((2, 2, 5, 8), np.uint16), np.ones((2, 5, 8), np.uint16))
    m.roll(3, 5)
    m.evict(3)
    kv, conv = m.gather(3)
    assert not kv.any() and not conv.any() and m.info(3) == (0, 0)


def test_bytes_formula_worked_example():
    # 24 layers, bf16 rows of 2 KB, k = 14, K and V: 2*(14+14+70+70) + (8+14+8+8) rows = 374 rows per layer.
    b = bytes_per_stream_step(24, 1024, 2, 14)
    assert b == 24 * 2048 * (2 * (14 + 14 + 70 + 70) + (8 + 14 + 8 + 8))
