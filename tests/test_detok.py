"""The SentencePiece detokenizer (ud_detok_*, SentencePiece.swift:5-32) through the C ABI, host only, against the
oracle restatement: word markers, byte-fallback pieces forming multi-byte UTF-8, ill-formed bytes (U+FFFD per
maximal subpart, as Swift's String(decoding:as:)), control pieces, ids outside the vocabulary, the leading
space, vocabulary lines with empty fields, and a random sweep. No GPU is used."""

import random

import pytest

import ud
from oracle.detok import decode, parse_vocab

VOCAB = "\n".join([
    "<unk>\t0", "<s>\t0", "</s>\t0", "<pad>\t0",
    "▁the\t-1.5", "▁cat\t-2", "s\t-3", "▁sat\t-2.5", "▁on\t-2", "▁a\t-1", "▁mat\t-4", ".\t-1", "▁\t-1",
    "<0xC3>\t0", "<0xA9>\t0", "<0xE2>\t0", "<0x82>\t0", "<0xAC>\t0", "<0xF0>\t0", "<0x9F>\t0", "<0x98>\t0",
    "<0x80>\t0", "<0xFF>\t0", "<0x41>\t0", "<0xed>\t0", "<0xA0>\t0", "<0x+5>\t0", "<0xZZ>\t0", "<0x4>\t0",
    "caf\t-3", "▁naïve\t-5", "a▁b\t-6", "\t\tweird\t0", "", "tail",
])


@pytest.fixture(scope="module")
def dec():
    d = ud.SentencePieceDecoder(VOCAB)
    yield d
    d.close()


def test_vocab_parse(dec):
    pieces = parse_vocab(VOCAB)
    assert dec.count == len(pieces)
    assert pieces[-2] == "weird" and pieces[-1] == "tail"


@pytest.mark.parametrize("ids", [
    [4, 5, 6, 7, 8, 9, 10, 11],            # "the cats sat on a mat."
    [29, 13, 14],                           # "café" from byte fallback
    [15, 16, 17],                           # the euro sign from three bytes
    [18, 19, 19, 20],                       # an emoji lead with a repeated continuation: ill-formed
    [13], [21], [22], [13, 23], [24, 25, 21],   # lone lead, lone continuation, invalid byte, truncated, surrogate
    [26, 27, 28],                           # "<0x+5>" (sign), "<0xZZ>", "<0x4>" (not byte pieces)
    [0, 1, 2, 3, 4], [12, 12, 5], [30, 31], [-1, 99, 4, 1000],
    [],
])
def test_matches_oracle(dec, ids):
    assert dec.decode(ids) == decode(parse_vocab(VOCAB), ids)


def test_examples(dec):
    assert dec.decode([4, 5, 6, 7, 8, 9, 10, 11]) == "the cats sat on a mat."
    assert dec.decode([29, 13, 14]) == "café"
    assert dec.decode([15, 16, 17]) == "€"
    assert dec.decode([13]) == "�"
    assert dec.decode([12, 12, 5]) == "  cat"    # three markers, only one leading space is dropped


def test_random_sweep(dec):
    pieces = parse_vocab(VOCAB)
    rng = random.Random(0)
    for _ in range(500):
        ids = [rng.randrange(-2, len(pieces) + 2) for _ in range(rng.randrange(0, 20))]
        assert dec.decode(ids) == decode(pieces, ids), ids


def test_file_and_errors(tmp_path):
    p = tmp_path / "tokenizer.vocab"
    p.write_text(VOCAB, encoding="utf-8")
    d = ud.SentencePieceDecoder(vocab_file=str(p))
    try:
        assert d.decode([4, 5]) == "the cat"
    finally:
        d.close()
    with pytest.raises(ud.EngineError):
        ud.SentencePieceDecoder(vocab_file=str(tmp_path / "missing.vocab"))
