// Byte-level BPE with the GPT-2-style pre-tokenizer of the reference's SmolLM2
// tokenizer (src/tokenizer/tokenizer.cpp:14-204), built in three passes:
//
//   1. decode: the text becomes an array of characters (byte offset, length,
//      class), each classified once - ASCII from a 128-entry table, other code
//      points by binary search in one sorted table of class ranges;
//   2. split: a scan over that array cuts it into pieces - every digit alone;
//      inside digit-free stretches the contractions 's 't 'm 'd 're 've 'll, a
//      run of one class with at most one leading ASCII space, and whitespace
//      runs that give their last character to the next piece unless the
//      stretch ends there;
//   3. merge: each piece's bytes become symbols of the byte-to-unicode
//      alphabet in a linked list, and a min-heap of adjacent pairs keyed by
//      (merge rank, position) merges the lowest-ranked pair, the leftmost on
//      ties, until no known pair is left. Stale heap entries are recognized by
//      per-symbol versions.
//
// The class ranges, the contraction list, the split rules, the alphabet and
// the merge order are what gives the reference's ids; the code is this
// library's own.
#include "bpe_tokenizer.h"

#include "utf8.h"

#include <algorithm>
#include <cstdint>
#include <queue>
#include <string>
#include <string_view>

namespace vsb {
namespace {

enum Kind : uint8_t { kLetter, kNumber, kBlank, kSymbol };

struct ClassRange {
    uint32_t lo, hi;
    Kind kind;
};

// Code points outside ASCII that the pre-tokenizer counts as whitespace,
// digits or letters, sorted and disjoint; everything else is a symbol.
constexpr ClassRange kClasses[] = {
    {0x85, 0x85, kBlank},     {0xA0, 0xA0, kBlank},     {0xAA, 0xAA, kLetter},    {0xB2, 0xB3, kNumber},
    {0xB5, 0xB5, kLetter},    {0xB9, 0xB9, kNumber},    {0xBA, 0xBA, kLetter},    {0xBC, 0xBE, kNumber},
    {0xC0, 0xD6, kLetter},    {0xD8, 0xF6, kLetter},    {0xF8, 0x2C1, kLetter},   {0x370, 0x373, kLetter},
    {0x376, 0x377, kLetter},  {0x37B, 0x37D, kLetter},  {0x386, 0x386, kLetter},  {0x388, 0x3FF, kLetter},
    {0x400, 0x481, kLetter},  {0x48A, 0x52F, kLetter},  {0x531, 0x556, kLetter},  {0x561, 0x587, kLetter},
    {0x5D0, 0x5EA, kLetter},  {0x620, 0x64A, kLetter},  {0x660, 0x669, kNumber},  {0x6F0, 0x6F9, kNumber},
    {0x966, 0x96F, kNumber},  {0x1680, 0x1680, kBlank}, {0x1E00, 0x1FBC, kLetter}, {0x2000, 0x200A, kBlank},
    {0x2028, 0x2029, kBlank}, {0x202F, 0x202F, kBlank}, {0x205F, 0x205F, kBlank}, {0x2070, 0x2070, kNumber},
    {0x2074, 0x2079, kNumber}, {0x2080, 0x2089, kNumber}, {0x2150, 0x2182, kNumber}, {0x2185, 0x2189, kNumber},
    {0x2460, 0x249B, kNumber}, {0x24EA, 0x24FF, kNumber}, {0x2776, 0x2793, kNumber}, {0x3000, 0x3000, kBlank},
    {0x3007, 0x3007, kNumber}, {0x3021, 0x3029, kNumber}, {0x3041, 0x3096, kLetter}, {0x30A1, 0x30FA, kLetter},
    {0x3400, 0x4DBF, kLetter}, {0x4E00, 0x9FFF, kLetter}, {0xAC00, 0xD7A3, kLetter}, {0xF900, 0xFAFF, kLetter},
    {0xFF10, 0xFF19, kNumber}, {0xFF21, 0xFF3A, kLetter}, {0xFF41, 0xFF5A, kLetter},
};

constexpr bool classes_sorted() {
    for (size_t i = 1; i < sizeof(kClasses) / sizeof(kClasses[0]); ++i)
        if (kClasses[i].lo <= kClasses[i - 1].hi || kClasses[i].lo > kClasses[i].hi) return false;
    return true;
}
static_assert(classes_sorted(), "class ranges must be sorted and disjoint");

struct AsciiKinds {
    Kind k[128];
    constexpr AsciiKinds() : k{} {
        for (int c = 0; c < 128; ++c) {
            const bool letter = (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z');
            const bool digit = c >= '0' && c <= '9';
            const bool blank = c == ' ' || (c >= '\t' && c <= '\r');
            k[c] = letter ? kLetter : digit ? kNumber : blank ? kBlank : kSymbol;
        }
    }
};
constexpr AsciiKinds kAscii;

Kind kind_of(uint32_t cp) {
    if (cp < 128) return kAscii.k[cp];
    const auto* end = kClasses + sizeof(kClasses) / sizeof(kClasses[0]);
    const auto* it = std::upper_bound(kClasses, end, cp, [](uint32_t v, const ClassRange& r) { return v < r.lo; });
    if (it == kClasses) return kSymbol;
    --it;
    return cp <= it->hi ? it->kind : kSymbol;
}

struct Char {
    uint32_t off;    // byte offset in the text
    uint32_t len;    // bytes
    Kind kind;
    char ascii;      // the byte itself for a 1-byte character, else 0
};

// pass 1: characters of the text (a malformed byte is a 1-byte symbol)
std::vector<Char> decode(const std::string& text) {
    std::vector<Char> out;
    out.reserve(text.size());
    for (size_t i = 0; i < text.size();) {
        const Utf8Char u = utf8_lenient(text.data() + i, text.size() - i);
        const Kind k = u.ok ? kind_of(u.cp) : kSymbol;
        out.push_back({static_cast<uint32_t>(i), u.len, k, u.len == 1 ? text[i] : '\0'});
        i += u.len;
    }
    return out;
}

// length in characters of a contraction starting at c[i] ('s 't 'm 'd 're
// 've 'll, all ASCII), or 0; `e` ends the digit-free stretch
size_t contraction(const std::vector<Char>& c, size_t i, size_t e) {
    if (c[i].ascii != '\'' || i + 1 >= e) return 0;
    const char a = c[i + 1].ascii, b = i + 2 < e ? c[i + 2].ascii : '\0';
    if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
    if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return 3;
    return 0;
}

// end of the run of characters of kind k starting at i (bounded by e)
size_t run_end(const std::vector<Char>& c, size_t i, size_t e, Kind k) {
    while (i < e && c[i].kind == k) ++i;
    return i;
}

// pass 2: piece boundaries [first, last) in characters
std::vector<std::pair<size_t, size_t>> split(const std::vector<Char>& c) {
    std::vector<std::pair<size_t, size_t>> pieces;
    const size_t n = c.size();
    size_t i = 0;
    while (i < n) {
        if (c[i].kind == kNumber) {            // a digit is a piece of its own
            pieces.emplace_back(i, i + 1);
            ++i;
            continue;
        }
        const size_t e = [&] {                 // the digit-free stretch [i, e)
            size_t j = i;
            while (j < n && c[j].kind != kNumber) ++j;
            return j;
        }();
        while (i < e) {
            size_t len = contraction(c, i, e);
            if (!len) {
                // one leading ASCII space joins a following non-blank run
                const size_t j = c[i].ascii == ' ' ? i + 1 : i;
                if (j < e && c[j].kind != kBlank) {
                    len = run_end(c, j, e, c[j].kind) - i;
                } else {
                    // whitespace: all of it where the stretch ends, else all
                    // but its last character, which leads the next piece
                    const size_t r = run_end(c, i, e, kBlank);
                    len = (r == e || r - i == 1) ? r - i : r - i - 1;
                }
            }
            pieces.emplace_back(i, i + len);
            i += len;
        }
    }
    return pieces;
}

}  // namespace

bool BpeTokenizer::load_text(const std::string& vocab, const std::string& merges) {
    vocab_.clear();
    rank_.clear();
    // byte-to-unicode alphabet: bytes 33..126, 161..172 and 174..255 stand for
    // the code points of the same value; the other 68 bytes, in byte order,
    // for 256, 257, ...
    uint32_t next_extra = 256;
    for (int b = 0; b < 256; ++b) {
        const bool printable = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || b >= 174;
        byte_char_[b].clear();
        utf8_put(byte_char_[b], printable ? static_cast<uint32_t>(b) : next_extra++);
    }
    auto lines = [](const std::string& text, auto&& fn) {
        size_t p = 0;
        while (p < text.size()) {
            size_t q = text.find('\n', p);
            if (q == std::string::npos) q = text.size();
            fn(std::string_view(text).substr(p, q - p));
            p = q + 1;
        }
    };
    bool bad = false;
    lines(vocab, [&](std::string_view line) {
        const size_t tab = line.find('\t');
        if (tab == std::string_view::npos || bad) return;
        try {
            vocab_[std::string(line.substr(tab + 1))] = std::stoi(std::string(line.substr(0, tab)));
        } catch (...) {
            bad = true;
        }
    });
    if (bad) return false;
    // merges.txt: "left right" per line, the line's position among such lines
    // is its rank (a repeated pair takes its last rank); the whole line is the
    // key, which is how merge_piece spells a candidate pair
    int rank = 0;
    lines(merges, [&](std::string_view line) {
        if (line.find(' ') == std::string_view::npos) return;
        rank_[std::string(line)] = rank++;
    });
    return !vocab_.empty() && !rank_.empty();
}

std::vector<int> BpeTokenizer::merge_piece(const std::string& text, size_t begin, size_t end) const {
    struct Sym {
        std::string s;
        int prev, next;
        uint32_t ver;   // bumped on every change, so stale heap entries can be told apart
        bool alive;
    };
    std::vector<Sym> sym;
    sym.reserve(end - begin);
    for (size_t b = begin; b < end; ++b) {
        const int k = static_cast<int>(sym.size());
        sym.push_back({byte_char_[static_cast<unsigned char>(text[b])], k - 1, k + 1, 0, true});
    }
    if (!sym.empty()) sym.back().next = -1;

    struct Cand {
        int rank, left, right;
        uint32_t vl, vr;
    };
    auto later = [](const Cand& a, const Cand& b) { return a.rank != b.rank ? a.rank > b.rank : a.left > b.left; };
    std::priority_queue<Cand, std::vector<Cand>, decltype(later)> heap(later);
    std::string key;
    auto offer = [&](int l) {
        if (l < 0) return;
        const int r = sym[l].next;
        if (r < 0) return;
        key.assign(sym[l].s).push_back(' ');
        key += sym[r].s;
        const auto it = rank_.find(key);
        if (it != rank_.end()) heap.push({it->second, l, r, sym[l].ver, sym[r].ver});
    };
    for (int l = 0; l + 1 < static_cast<int>(sym.size()); ++l) offer(l);
    while (!heap.empty()) {
        const Cand c = heap.top();
        heap.pop();
        Sym& L = sym[c.left];
        Sym& R = sym[c.right];
        if (!L.alive || !R.alive || L.next != c.right || L.ver != c.vl || R.ver != c.vr) continue;
        L.s += R.s;
        ++L.ver;
        R.alive = false;
        L.next = R.next;
        if (R.next >= 0) sym[R.next].prev = c.left;
        offer(L.prev);
        offer(c.left);
    }
    std::vector<int> ids;
    for (int k = sym.empty() ? -1 : 0; k >= 0; k = sym[k].next) {
        const auto it = vocab_.find(sym[k].s);
        if (it != vocab_.end()) ids.push_back(it->second);   // a symbol outside the vocabulary is dropped
    }
    return ids;
}

std::vector<int> BpeTokenizer::encode(const std::string& text) const {
    const std::vector<Char> chars = decode(text);
    std::vector<int> ids;
    for (const auto& [first, last] : split(chars)) {
        const size_t b = chars[first].off;
        const size_t e = last < chars.size() ? chars[last].off : text.size();
        const std::vector<int> p = merge_piece(text, b, e);
        ids.insert(ids.end(), p.begin(), p.end());
    }
    return ids;
}

}  // namespace vsb
