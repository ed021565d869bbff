// UTF-8 decoding and encoding shared by the two host tokenizers.
//
// The two reference tokenizers read malformed UTF-8 differently, and the same
// token ids need the same reading, so there are two decoders:
//   utf8_lenient  the byte-level BPE pre-tokenizer's reading
//                 (src/tokenizer/tokenizer.cpp): the lead byte alone fixes the
//                 length (>= 0xF0: 4, >= 0xE0: 3, >= 0xC0: 2); a stray
//                 continuation byte, a truncated sequence or a bad
//                 continuation byte is one 1-byte character of its own; no
//                 overlong or surrogate checks.
//   utf8_strict   the SentencePiece normalizer's reading
//                 (src/tokenizer/bert_tokenizer.cpp:17-35): leads C2..F4 only,
//                 overlongs and surrogates refused through the first
//                 continuation byte's range; a bad sequence becomes U+FFFD and
//                 consumes the lead plus the continuation bytes that were valid.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

namespace vsb {

struct Utf8Char {
    uint32_t cp;    // code point (U+FFFD for a strict-mode error)
    uint32_t len;   // bytes consumed, >= 1
    bool ok;        // false: a malformed sequence (lenient: cp is the raw byte)
};

inline Utf8Char utf8_lenient(const char* s, size_t avail) {
    const uint32_t b0 = static_cast<unsigned char>(s[0]);
    if (b0 < 0x80) return {b0, 1, true};
    const uint32_t n = b0 >= 0xF0 ? 4 : b0 >= 0xE0 ? 3 : b0 >= 0xC0 ? 2 : 0;
    if (n == 0 || n > avail) return {b0, 1, false};
    uint32_t cp = b0 & (0xFFu >> (n + 1));
    for (uint32_t k = 1; k < n; ++k) {
        const uint32_t c = static_cast<unsigned char>(s[k]);
        if ((c >> 6) != 2) return {b0, 1, false};
        cp = (cp << 6) | (c & 0x3F);
    }
    return {cp, n, true};
}

inline Utf8Char utf8_strict(const char* s, size_t avail) {
    const uint32_t b0 = static_cast<unsigned char>(s[0]);
    if (b0 < 0x80) return {b0, 1, true};
    uint32_t more;
    if (b0 >= 0xC2 && b0 <= 0xDF) more = 1;
    else if (b0 >= 0xE0 && b0 <= 0xEF) more = 2;
    else if (b0 >= 0xF0 && b0 <= 0xF4) more = 3;
    else return {0xFFFD, 1, false};
    // allowed range of the first continuation byte
    const uint32_t lo = b0 == 0xE0 ? 0xA0 : b0 == 0xF0 ? 0x90 : 0x80;
    const uint32_t hi = b0 == 0xED ? 0x9F : b0 == 0xF4 ? 0x8F : 0xBF;
    uint32_t cp = b0 & (0x3Fu >> more);
    uint32_t used = 1;
    for (uint32_t k = 0; k < more; ++k) {
        if (used >= avail) return {0xFFFD, used, false};
        const uint32_t c = static_cast<unsigned char>(s[used]);
        const uint32_t l = k == 0 ? lo : 0x80, h = k == 0 ? hi : 0xBF;
        if (c < l || c > h) return {0xFFFD, used, false};
        cp = (cp << 6) | (c & 0x3F);
        ++used;
    }
    return {cp, used, true};
}

inline void utf8_put(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
        out.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
        out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
        out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
        out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
}

}  // namespace vsb
