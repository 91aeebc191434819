"""The streamer's chunk walk (ud_chunk_next, host code in libud, no GPU) against the oracle's restatement of
NemotronStreamer.drainChunks (oracle/stream_step.py drain_next / live_plan, NemotronStreamer.swift:109-154):
  * over a complete buffer without end padding it is runBuffered's walk (chunk_plan, :70-91);
  * with end padding a short final tail becomes a zero-extended, masked chunk;
  * rows pushed piecemeal give the same chunks as the whole buffer at once, each full chunk as soon as its rows
    exist."""

import random

import pytest

import ud
from oracle.stream_step import chunk_plan, drain_next, live_plan


def _walk(R: int, avail: int, last: bool, idx: int = 0, end_padding: bool = True):
    out = []
    while True:
        r, start, rows, valid, keep, nxt = ud.chunk_next(R, idx, avail, last, end_padding)
        ref = drain_next(R, idx, avail, last, end_padding)
        assert (r == 1) == (ref is not None)
        if r != 1:
            return out, r, idx
        assert (start, valid, rows - valid, keep, nxt) == ref
        out.append((start, rows, valid, keep))
        idx = nxt
        if keep:
            return out, r, idx


@pytest.mark.parametrize("R", [0, 1, 6, 13])
def test_buffered_walk_without_padding_is_run_buffered(R):
    for total in list(range(0, 140)) + [1000, 3000]:
        got, _, _ = _walk(R, total, True, end_padding=False)
        assert got == list(chunk_plan(total, R)), (R, total)
        assert got == list(live_plan(total, R, end_padding=False))


@pytest.mark.parametrize("R", [0, 1, 6, 13])
def test_end_padding_extends_a_short_tail(R):
    first = 1 + 8 * R
    for total in list(range(0, 140)) + [1000, 3001]:
        got, _, _ = _walk(R, total, True)
        assert got == list(live_plan(total, R, end_padding=True)), (R, total)
        plain = list(chunk_plan(total, R))
        tail = (total - first) % (8 + 8 * R) if total > first else None
        if tail is not None and 0 < tail < 8:   # a short tail: one more chunk, padded to 8 new rows
            assert len(got) == len(plain) + 1
            start, rows, valid, keep = got[-1]
            assert keep and rows - valid == 8 - tail and valid == min(total, 9 + tail)
        else:
            assert got == plain


@pytest.mark.parametrize("R", [1, 6, 13])
@pytest.mark.parametrize("end_padding", [True, False])
def test_live_pushes_give_the_buffered_chunks(R, end_padding):
    rng = random.Random(R)
    for total in (40, 200, 777, 1500):
        idx, avail, got = 0, 0, []
        while avail < total:
            avail = min(total, avail + rng.randint(1, 90))
            part, r, idx = _walk(R, avail, avail == total, idx, end_padding)
            got += part
        assert got == list(live_plan(total, R, end_padding)), (R, total)


def test_a_full_chunk_runs_as_soon_as_its_rows_exist():
    R = 6
    first = 1 + 8 * R
    assert ud.chunk_next(R, 0, first - 1, False)[0] == 0
    assert ud.chunk_next(R, 0, first, False)[:6] == (1, 0, first, first, False, first)
    assert ud.chunk_next(R, 0, first, True)[:6] == (1, 0, first, first, True, first)
    assert ud.chunk_next(R, first, first, True)[0] == -1      # nothing left
