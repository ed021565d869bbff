// Byte-level BPE: the reference's pre-tokenizer (GPT-2 style pieces: an
// optional leading space with a run of letters, of non-letter non-digit
// symbols, contractions, whitespace runs; every digit alone) and greedy
// lowest-rank merging, src/tokenizer/tokenizer.cpp:14-204.
#include "bpe_tokenizer.h"

#include <climits>
#include <cstdint>
#include <sstream>

namespace vsb {
namespace {

enum class Kind { Letter, Number, Blank, Symbol };

struct Range {
    uint32_t lo, hi;
};

// code points the pre-tokenizer treats as whitespace, digits and letters
// beyond ASCII (the Unicode classes it approximates)
const uint32_t kBlank[] = {0x85, 0xA0, 0x1680, 0x2028, 0x2029, 0x202F, 0x205F, 0x3000};
const Range kNumber[] = {{0xB2, 0xB3},     {0xB9, 0xB9},     {0xBC, 0xBE},     {0x660, 0x669},   {0x6F0, 0x6F9},
                         {0x966, 0x96F},   {0x2070, 0x2070}, {0x2074, 0x2079}, {0x2080, 0x2089}, {0x2150, 0x2182},
                         {0x2185, 0x2189}, {0x2460, 0x249B}, {0x24EA, 0x24FF}, {0x2776, 0x2793}, {0x3007, 0x3007},
                         {0x3021, 0x3029}, {0xFF10, 0xFF19}};
const Range kLetter[] = {{0xAA, 0xAA},     {0xB5, 0xB5},     {0xBA, 0xBA},     {0xC0, 0xD6},     {0xD8, 0xF6},
                         {0xF8, 0x2C1},    {0x370, 0x373},   {0x376, 0x377},   {0x37B, 0x37D},   {0x386, 0x386},
                         {0x388, 0x3FF},   {0x400, 0x481},   {0x48A, 0x52F},   {0x531, 0x556},   {0x561, 0x587},
                         {0x5D0, 0x5EA},   {0x620, 0x64A},   {0x1E00, 0x1FBC}, {0x3041, 0x3096}, {0x30A1, 0x30FA},
                         {0x3400, 0x4DBF}, {0x4E00, 0x9FFF}, {0xAC00, 0xD7A3}, {0xF900, 0xFAFF}, {0xFF21, 0xFF3A},
                         {0xFF41, 0xFF5A}};

template <size_t N>
bool in(const Range (&r)[N], uint32_t cp) {
    for (const Range& x : r)
        if (cp >= x.lo && cp <= x.hi) return true;
    return false;
}

// class of the character at s[i] (end e); *len = its byte length (1 for a
// malformed or truncated sequence, which is a symbol)
Kind kind_at(const std::string& s, size_t i, size_t e, size_t* len) {
    const unsigned c = static_cast<unsigned char>(s[i]);
    *len = 1;
    if (c < 0x80) {
        if ((c | 32) - 'a' < 26u) return Kind::Letter;
        if (c - '0' < 10u) return Kind::Number;
        if (c == ' ' || c - '\t' < 5u) return Kind::Blank;
        return Kind::Symbol;
    }
    const size_t n = c >= 0xF0 ? 4 : c >= 0xE0 ? 3 : c >= 0xC0 ? 2 : 0;
    if (!n || i + n > e) return Kind::Symbol;
    uint32_t cp = c & (0x7Fu >> n);
    for (size_t k = 1; k < n; ++k) {
        const unsigned d = static_cast<unsigned char>(s[i + k]);
        if ((d & 0xC0) != 0x80) return Kind::Symbol;
        cp = (cp << 6) | (d & 0x3F);
    }
    *len = n;
    for (uint32_t b : kBlank)
        if (cp == b) return Kind::Blank;
    if (cp >= 0x2000 && cp <= 0x200A) return Kind::Blank;
    if (in(kNumber, cp)) return Kind::Number;
    if (in(kLetter, cp)) return Kind::Letter;
    return Kind::Symbol;
}

size_t run_of(const std::string& s, size_t i, size_t e, Kind k) {
    size_t n;
    while (i < e && kind_at(s, i, e, &n) == k) i += n;
    return i;
}

// byte length of the piece starting at i (within a digit-free span ending at e)
size_t piece_len(const std::string& s, size_t i, size_t e) {
    if (s[i] == '\'' && i + 1 < e) {
        const char a = s[i + 1], b = i + 2 < e ? s[i + 2] : 0;
        if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
        if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
    }
    size_t n;
    const Kind k = kind_at(s, i, e, &n);
    const size_t j = i + (s[i] == ' ' ? 1 : 0);   // a single leading space joins the next run
    if (j < e) {
        const Kind kj = j == i ? k : kind_at(s, j, e, &n);
        if (kj != Kind::Blank) return run_of(s, j, e, kj) - i;
    }
    // a whitespace run: all of it at the end of the span, else all but its
    // last character (which then leads the next piece)
    const size_t end = run_of(s, i, e, Kind::Blank);
    if (end == e) return end - i;
    size_t last = i, m;
    for (size_t p = i; p < end; p += m) {
        kind_at(s, p, e, &m);
        last = p;
    }
    return last > i ? last - i : end - i;
}

std::string utf8_of(int cp) {
    std::string s;
    if (cp < 0x80) {
        s += static_cast<char>(cp);
    } else {
        s += static_cast<char>(0xC0 | (cp >> 6));
        s += static_cast<char>(0x80 | (cp & 0x3F));
    }
    return s;
}

}  // namespace

bool BpeTokenizer::load_text(const std::string& vocab, const std::string& merges) {
    vocab_.clear();
    rank_.clear();
    // the byte-to-unicode alphabet: printable Latin-1 bytes stand for
    // themselves, the other 68 bytes for code points 256.. in byte order
    {
        int extra = 0;
        for (int b = 0; b < 256; ++b) {
            const bool keep = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255);
            byte_char_[b] = utf8_of(keep ? b : 256 + extra++);
        }
    }
    std::istringstream v(vocab);
    std::string line;
    try {
        while (std::getline(v, line)) {
            const size_t tab = line.find('\t');
            if (tab == std::string::npos) continue;
            vocab_[line.substr(tab + 1)] = std::stoi(line.substr(0, tab));
        }
    } catch (...) {
        return false;
    }
    std::istringstream m(merges);
    int rank = 0;
    while (std::getline(m, line)) {
        const size_t sp = line.find(' ');
        if (sp == std::string::npos) continue;
        rank_[{line.substr(0, sp), line.substr(sp + 1)}] = rank++;
    }
    return !vocab_.empty() && !rank_.empty();
}

std::vector<int> BpeTokenizer::merge_piece(const std::string& bytes) const {
    std::vector<std::string> w;
    for (unsigned char b : bytes) w.push_back(byte_char_[b]);
    // merge the lowest-ranked adjacent pair (the leftmost on ties) until none is known
    while (w.size() > 1) {
        int best = INT_MAX;
        int at = -1;
        for (size_t i = 0; i + 1 < w.size(); ++i) {
            const auto it = rank_.find({w[i], w[i + 1]});
            if (it != rank_.end() && it->second < best) {
                best = it->second;
                at = static_cast<int>(i);
            }
        }
        if (at < 0) break;
        w[at] += w[at + 1];
        w.erase(w.begin() + at + 1);
    }
    std::vector<int> ids;
    for (const std::string& t : w) {
        const auto it = vocab_.find(t);
        if (it != vocab_.end()) ids.push_back(it->second);   // unknown symbols are dropped
    }
    return ids;
}

std::vector<int> BpeTokenizer::encode(const std::string& text) const {
    std::vector<int> ids;
    auto emit = [&](size_t i, size_t n) {
        const std::vector<int> p = merge_piece(text.substr(i, n));
        ids.insert(ids.end(), p.begin(), p.end());
    };
    const size_t N = text.size();
    for (size_t b = 0; b < N;) {
        size_t n;
        if (kind_at(text, b, N, &n) == Kind::Number) {   // every digit is a piece of its own
            emit(b, n);
            b += n;
            continue;
        }
        size_t e = b;
        while (e < N && kind_at(text, e, N, &n) != Kind::Number) e += n;
        for (size_t i = b; i < e;) {
            const size_t len = piece_len(text, i, e);
            emit(i, len);
            i += len;
        }
        b = e;
    }
    return ids;
}

}  // namespace vsb
