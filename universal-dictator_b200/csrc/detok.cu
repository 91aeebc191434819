// SentencePiece detokenizer (host code): the form of SentencePieceDecoder (Sources/DictatorCore/Text/
// SentencePiece.swift:5-32) behind the C ABI.
//   pieces: one "piece\tscore" line per id of the tokenizer.vocab text, empty lines skipped, the piece being
//   the line's first non-empty tab-separated field (:8-13)
//   decode: byte-fallback pieces "<0xHH>" contribute the byte; <unk>, <s>, </s>, <pad> nothing; any other piece
//   its UTF-8 with U+2581 (the word marker) turned into a space; ids outside the vocabulary are skipped (:17-27)
//   the bytes are read as UTF-8 with each maximal ill-formed subsequence replaced by U+FFFD (Swift's
//   String(decoding:as: UTF8.self)), and one leading space is dropped (:28-30).
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "ud.h"

namespace ud {
ud_status host_fail(ud_status s, const char* msg);
}

struct ud_detok {
    std::vector<std::string> pieces;
};

namespace {

int hex_digit(char c) {
    if (c >= '0' && c <= '9') return c - '0';
    if (c >= 'a' && c <= 'f') return c - 'a' + 10;
    if (c >= 'A' && c <= 'F') return c - 'A' + 10;
    return -1;
}

// The byte of a fallback piece "<0x" a b ">", parsed as Swift's UInt8(String, radix: 16) parses "ab": two hex
// digits, or a sign and one digit ("+5" is 5, "-0" is 0); -1 if it does not parse.
int fallback_byte(const std::string& p) {
    if (p.size() != 6 || p.compare(0, 3, "<0x") != 0 || p[5] != '>') return -1;
    const int a = hex_digit(p[3]), b = hex_digit(p[4]);
    if (a >= 0 && b >= 0) return a * 16 + b;
    if (p[3] == '+' && b >= 0) return b;
    if (p[3] == '-' && b == 0) return 0;
    return -1;
}

// Appends the UTF-8 bytes `b` to `out` with every maximal ill-formed subsequence replaced by U+FFFD
// (the Unicode substitution of maximal subparts).
void utf8_repair(const std::string& b, std::string& out) {
    static const char kRepl[] = "\xEF\xBF\xBD";
    const size_t n = b.size();
    size_t i = 0;
    while (i < n) {
        const unsigned char c = static_cast<unsigned char>(b[i]);
        if (c < 0x80) {
            out.push_back(static_cast<char>(c));
            ++i;
            continue;
        }
        int len;
        unsigned char lo = 0x80, hi = 0xBF;   // allowed range of the second byte
        if (c >= 0xC2 && c <= 0xDF) len = 2;
        else if (c == 0xE0) { len = 3; lo = 0xA0; }
        else if ((c >= 0xE1 && c <= 0xEC) || c == 0xEE || c == 0xEF) len = 3;
        else if (c == 0xED) { len = 3; hi = 0x9F; }
        else if (c == 0xF0) { len = 4; lo = 0x90; }
        else if (c >= 0xF1 && c <= 0xF3) len = 4;
        else if (c == 0xF4) { len = 4; hi = 0x8F; }
        else {   // a continuation byte or an invalid lead byte: one replacement for this byte
            out.append(kRepl, 3);
            ++i;
            continue;
        }
        size_t k = 1;
        bool ok = true;
        for (; k < static_cast<size_t>(len); ++k) {
            if (i + k >= n) { ok = false; break; }
            const unsigned char d = static_cast<unsigned char>(b[i + k]);
            const unsigned char l = k == 1 ? lo : 0x80, h = k == 1 ? hi : 0xBF;
            if (d < l || d > h) { ok = false; break; }
        }
        if (ok) {
            out.append(b, i, static_cast<size_t>(len));
            i += static_cast<size_t>(len);
        } else {   // the valid prefix [i, i + k) is one maximal subpart
            out.append(kRepl, 3);
            i += k;
        }
    }
}

}  // namespace

extern "C" {

ud_status ud_detok_create(const char* vocab_text, size_t len, ud_detok** out) {
    if ((!vocab_text && len) || !out) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    ud_detok* d = new ud_detok;
    size_t i = 0;
    while (i < len) {
        size_t j = i;
        while (j < len && vocab_text[j] != '\n') ++j;
        if (j > i) {   // the first non-empty tab-separated field (Swift's split omits empty fields)
            size_t a = i;
            while (a < j && vocab_text[a] == '\t') ++a;
            size_t t = a;
            while (t < j && vocab_text[t] != '\t') ++t;
            d->pieces.emplace_back(vocab_text + a, t - a);
        }
        i = j + 1;
    }
    *out = d;
    return UD_OK;
}

ud_status ud_detok_create_file(const char* path, ud_detok** out) {
    if (!path || !out) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    FILE* f = std::fopen(path, "rb");
    if (!f) return ud::host_fail(UD_ERR_IO, "cannot open the vocabulary file");
    std::string text;
    char buf[1 << 16];
    size_t got;
    while ((got = std::fread(buf, 1, sizeof(buf), f)) > 0) text.append(buf, got);
    const bool err = std::ferror(f) != 0;
    std::fclose(f);
    if (err) return ud::host_fail(UD_ERR_IO, "cannot read the vocabulary file");
    return ud_detok_create(text.data(), text.size(), out);
}

ud_status ud_detok_destroy(ud_detok* d) {
    delete d;
    return UD_OK;
}

int ud_detok_size(const ud_detok* d) { return d ? static_cast<int>(d->pieces.size()) : 0; }

ud_status ud_detok_decode(const ud_detok* d, const int32_t* ids, int n, char* out, size_t cap, size_t* len_out) {
    if (!d || (n > 0 && !ids) || !len_out || (cap > 0 && !out))
        return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "NULL argument");
    if (n < 0) return ud::host_fail(UD_ERR_INVALID_ARGUMENT, "negative token count");
    std::string bytes;
    const int V = static_cast<int>(d->pieces.size());
    for (int i = 0; i < n; ++i) {
        const int id = ids[i];
        if (id < 0 || id >= V) continue;
        const std::string& p = d->pieces[id];
        const int fb = fallback_byte(p);
        if (fb >= 0) {
            bytes.push_back(static_cast<char>(fb));
        } else if (p == "<unk>" || p == "<s>" || p == "</s>" || p == "<pad>") {
            continue;
        } else {
            for (size_t k = 0; k < p.size();) {
                if (k + 3 <= p.size() && static_cast<unsigned char>(p[k]) == 0xE2 &&
                    static_cast<unsigned char>(p[k + 1]) == 0x96 && static_cast<unsigned char>(p[k + 2]) == 0x81) {
                    bytes.push_back(' ');
                    k += 3;
                } else {
                    bytes.push_back(p[k]);
                    ++k;
                }
            }
        }
    }
    std::string text;
    utf8_repair(bytes, text);
    if (!text.empty() && text[0] == ' ') text.erase(0, 1);
    *len_out = text.size();
    if (cap > 0) {
        const size_t m = text.size() < cap - 1 ? text.size() : cap - 1;
        std::memcpy(out, text.data(), m);
        out[m] = '\0';
    }
    return UD_OK;
}

}  // extern "C"
