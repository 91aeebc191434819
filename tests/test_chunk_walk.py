"""The streamer's chunk walk (ud_chunk_next, host code in libud, no GPU) against the oracle's restatement of
NemotronStreamer.runBuffered (oracle/stream_step.py chunk_plan, NemotronStreamer.swift:70-91), and the live
rule: rows pushed piecemeal give the same chunks as the whole buffer at once."""

import random

import pytest

import ud
from oracle.stream_step import chunk_plan


def _walk(R: int, avail: int, last: bool, idx: int = 0):
    out = []
    while True:
        r, start, rows, keep, nxt = ud.chunk_next(R, idx, avail, last)
        if r != 1:
            return out, r, idx
        out.append((start, rows, rows, keep))
        idx = nxt


@pytest.mark.parametrize("R", [0, 1, 6, 13])
def test_buffered_walk_matches_oracle(R):
    for total in list(range(1, 140)) + [1000, 3000]:
        got, r, _ = _walk(R, total, True)
        assert got == list(chunk_plan(total, R)), (R, total)
        assert r == -1


@pytest.mark.parametrize("R", [1, 6, 13])
def test_live_pushes_give_the_buffered_chunks(R):
    rng = random.Random(R)
    for total in (40, 200, 777, 1500):
        idx, avail, got = 0, 0, []
        while avail < total:
            avail = min(total, avail + rng.randint(1, 90))
            part, r, idx = _walk(R, avail, avail == total, idx)
            got += part
            if avail < total:
                assert r == 0   # waits: the next chunk is not known to be final yet
        assert got == list(chunk_plan(total, R)), (R, total)


def test_a_full_chunk_waits_until_more_rows_or_the_end():
    R = 6
    first = 1 + 8 * R
    assert ud.chunk_next(R, 0, first, False)[0] == 0       # exactly one chunk: could be the final one
    assert ud.chunk_next(R, 0, first + 1, False)[0] == 1   # more rows exist: run it, not final
    r, start, rows, keep, nxt = ud.chunk_next(R, 0, first, True)
    assert (r, start, rows, keep, nxt) == (1, 0, first, True, first)
