"""CPU oracle of the SentencePiece detokenizer (test infrastructure only; the product never imports it).

Restates SentencePieceDecoder (Sources/DictatorCore/Text/SentencePiece.swift:5-32):
  pieces   one "piece\\tscore" line per id of the tokenizer.vocab text, empty lines skipped          (:8-13)
  decode   "<0xHH>" byte-fallback pieces give the byte (parsed as Swift's UInt8(_, radix: 16)); <unk>,
           <s>, </s>, <pad> give nothing; other pieces give their UTF-8 with U+2581 turned into a space;
           ids outside the vocabulary are skipped                                                       (:17-27)
  text     the bytes read as UTF-8 with ill-formed sequences replaced by U+FFFD (Swift's
           String(decoding:as:), the maximal-subpart substitution Python's "replace" handler also applies),
           one leading space dropped                                                                    (:28-30)
"""

from __future__ import annotations

_CONTROL = {"<unk>", "<s>", "</s>", "<pad>"}


def parse_vocab(text: str) -> list[str]:
    # the first non-empty tab-separated field (Swift's split omits empty fields)
    return [line.lstrip("\t").split("\t", 1)[0] for line in text.split("\n") if line]


def _swift_uint8_hex(s: str) -> int | None:
    """Swift's UInt8(s, radix: 16): optional sign, then hex digits, value in range."""
    if not s:
        return None
    sign = 1
    if s[0] in "+-":
        sign = -1 if s[0] == "-" else 1
        s = s[1:]
    if not s or any(c not in "0123456789abcdefABCDEF" for c in s):
        return None
    v = sign * int(s, 16)
    return v if 0 <= v <= 255 else None


def decode(pieces: list[str], ids) -> str:
    out = bytearray()
    for i in ids:
        if not 0 <= i < len(pieces):
            continue
        p = pieces[i]
        b = _swift_uint8_hex(p[3:-1]) if (p.startswith("<0x") and p.endswith(">") and len(p) == 6) else None
        if b is not None:
            out.append(b)
        elif p in _CONTROL:
            continue
        else:
            out += p.replace("▁", " ").encode("utf-8")
    s = out.decode("utf-8", errors="replace")
    return s[1:] if s.startswith(" ") else s
