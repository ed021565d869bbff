// T5 unigram tokenizer: the reference's normalization (a subset of NFKC plus
// whitespace folding into the U+2581 word marker) and its Viterbi
// segmentation over bytes, src/tokenizer/t5_tokenizer.cpp:13-129.
#include "t5_tokenizer.h"

#include <algorithm>
#include <limits>
#include <sstream>

namespace vsb {
namespace {

// UTF-8 -> code points; a malformed or truncated sequence gives U+FFFD per
// lead byte (src/tokenizer/bert_tokenizer.cpp:17-35).
std::vector<uint32_t> decode_utf8(const std::string& s) {
    std::vector<uint32_t> out;
    out.reserve(s.size());
    size_t i = 0;
    while (i < s.size()) {
        const unsigned lead = static_cast<unsigned char>(s[i++]);
        int more;
        if (lead < 0x80) more = 0;
        else if (lead >= 0xC2 && lead < 0xE0) more = 1;
        else if (lead >= 0xE0 && lead < 0xF0) more = 2;
        else if (lead >= 0xF0 && lead < 0xF5) more = 3;
        else { out.push_back(0xFFFD); continue; }
        uint32_t cp = lead & (0x7Fu >> more);
        // the first continuation byte's range excludes overlongs and surrogates
        unsigned lo = 0x80, hi = 0xBF;
        if (lead == 0xE0) lo = 0xA0;
        if (lead == 0xF0) lo = 0x90;
        if (lead == 0xED) hi = 0x9F;
        if (lead == 0xF4) hi = 0x8F;
        while (more > 0 && i < s.size()) {
            const unsigned c = static_cast<unsigned char>(s[i]);
            if (c < lo || c > hi) break;
            cp = (cp << 6) | (c & 0x3Fu);
            ++i;
            --more;
            lo = 0x80;
            hi = 0xBF;
        }
        out.push_back(more ? 0xFFFD : cp);
    }
    return out;
}

void encode_utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
        out.push_back(static_cast<char>(cp));
        return;
    }
    int n = cp < 0x800 ? 1 : cp < 0x10000 ? 2 : 3;   // continuation bytes
    static const unsigned kLead[4] = {0, 0xC0, 0xE0, 0xF0};
    out.push_back(static_cast<char>(kLead[n] | (cp >> (6 * n))));
    while (n-- > 0) out.push_back(static_cast<char>(0x80 | ((cp >> (6 * n)) & 0x3F)));
}

// Compatibility decompositions the normalizer applies (the NFKC cases of
// Latin-1 and General Punctuation that T5's normalizer rewrites):
// code point -> replacement sequence.
struct Compat {
    uint32_t cp;
    uint32_t to[4];
};
constexpr uint32_t kFrac = 0x2044, kPrime = 0x2032, kRevPrime = 0x2035;
const Compat kCompat[] = {
    {0x00A8, {' ', 0x0308}},       {0x00AA, {'a'}},
    {0x00AF, {' ', 0x0304}},       {0x00B2, {'2'}},
    {0x00B3, {'3'}},               {0x00B4, {' ', 0x0301}},
    {0x00B5, {0x03BC}},            {0x00B8, {' ', 0x0327}},
    {0x00B9, {'1'}},               {0x00BA, {'o'}},
    {0x00BC, {'1', kFrac, '4'}},   {0x00BD, {'1', kFrac, '2'}},
    {0x00BE, {'3', kFrac, '4'}},   {0x0132, {'I', 'J'}},
    {0x0133, {'i', 'j'}},          {0x013F, {'L', 0x00B7}},
    {0x0140, {'l', 0x00B7}},       {0x0149, {0x02BC, 'n'}},
    {0x017F, {'s'}},               {0x0340, {0x0300}},
    {0x0341, {0x0301}},            {0x0343, {0x0313}},
    {0x0344, {0x0308, 0x0301}},    {0x2011, {0x2010}},
    {0x2017, {' ', 0x0333}},       {0x2024, {'.'}},
    {0x2025, {'.', '.'}},          {0x2026, {'.', '.', '.'}},
    {0x2033, {kPrime, kPrime}},    {0x2034, {kPrime, kPrime, kPrime}},
    {0x2036, {kRevPrime, kRevPrime}}, {0x2037, {kRevPrime, kRevPrime, kRevPrime}},
    {0x203C, {'!', '!'}},          {0x203E, {' ', 0x0305}},
    {0x2047, {'?', '?'}},          {0x2048, {'?', '!'}},
    {0x2049, {'!', '?'}},          {0x2057, {kPrime, kPrime, kPrime, kPrime}},
};

// control characters the normalizer drops
bool dropped(uint32_t cp) {
    return (cp >= 0x01 && cp <= 0x08) || cp == 0x0B || (cp >= 0x0E && cp <= 0x1F) || cp == 0x7F || cp == 0x8F ||
           cp == 0x9F;
}

// characters that end a word (folded into one U+2581 before the next word)
bool blank(uint32_t cp) {
    switch (cp) {
        case ' ': case '\t': case '\n': case '\f': case '\r': case 0x85: case 0xA0: case 0x1680:
        case 0x2028: case 0x2029: case 0x202F: case 0x205F: case 0x2581: case 0x3000: case 0xFEFF: case 0xFFFD:
            return true;
        default:
            return cp >= 0x2000 && cp <= 0x200F;
    }
}

int utf8_bytes(unsigned char c) {
    if (c < 0x80) return 1;
    if ((c & 0xE0) == 0xC0) return 2;
    if ((c & 0xF0) == 0xE0) return 3;
    if ((c & 0xF8) == 0xF0) return 4;
    return 1;
}

constexpr int kUnk = 2, kEos = 1, kPad = 0;

}  // namespace

bool T5Tokenizer::load_text(const std::string& text) {
    piece_.clear();
    score_.clear();
    longest_ = 1;
    lowest_ = 0.0;
    std::istringstream in(text);
    std::string line;
    while (std::getline(in, line)) {
        const size_t tab = line.rfind('\t');
        if (tab == std::string::npos) continue;
        const std::string piece = line.substr(0, tab);
        double sc;
        try {
            sc = std::stod(line.substr(tab + 1));
        } catch (...) {
            return false;
        }
        const int id = static_cast<int>(score_.size());
        score_.push_back(sc);
        const bool control = piece.size() >= 2 && piece.front() == '<' && piece.back() == '>';
        if (sc == 0.0 && !control) continue;   // unused placeholder entries keep their id only
        piece_.emplace(piece, id);
        longest_ = std::max(longest_, static_cast<int>(piece.size()));
        lowest_ = std::min(lowest_, sc);
    }
    return !score_.empty();
}

void T5Tokenizer::segment(const std::string& text, std::vector<int>& ids) const {
    // normalize: compatibility rewrites, fullwidth ASCII to ASCII, dropped
    // controls, runs of blanks -> one U+2581 before the next word
    std::string s;
    bool at_word_start = true;
    auto emit = [&](uint32_t cp) {
        if (blank(cp)) {
            at_word_start = true;
            return;
        }
        if (at_word_start) {
            s += "\xE2\x96\x81";
            at_word_start = false;
        }
        encode_utf8(s, cp);
    };
    for (uint32_t cp : decode_utf8(text)) {
        if (dropped(cp)) continue;
        if (cp >= 0xFF01 && cp <= 0xFF5D) cp -= 0xFEE0;
        const Compat* hit = nullptr;
        for (const Compat& c : kCompat)
            if (c.cp == cp) hit = &c;
        if (!hit) {
            emit(cp);
            continue;
        }
        for (uint32_t r : hit->to) {
            if (!r) break;
            emit(r);
        }
    }

    // best[i]: highest total score of a segmentation of s[0, i); ties keep the
    // first candidate found (shorter pieces first, then the unknown fallback)
    const int n = static_cast<int>(s.size());
    const double kNone = -std::numeric_limits<double>::infinity();
    const double unk_score = lowest_ - 10.0;
    std::vector<double> best(n + 1, kNone);
    std::vector<int> from(n + 1, -1), tok(n + 1, kUnk);
    best[0] = 0.0;
    for (int i = 0; i < n; ++i) {
        if (best[i] == kNone) continue;
        const int lmax = std::min(longest_, n - i);
        for (int len = 1; len <= lmax; ++len) {
            const auto it = piece_.find(s.substr(i, len));
            if (it == piece_.end()) continue;
            const double cand = best[i] + score_[it->second];
            if (cand > best[i + len]) {
                best[i + len] = cand;
                from[i + len] = i;
                tok[i + len] = it->second;
            }
        }
        // one whole UTF-8 character as <unk>
        const int len = utf8_bytes(static_cast<unsigned char>(s[i]));
        if (best[i] + unk_score > best[i + len]) {
            best[i + len] = best[i] + unk_score;
            from[i + len] = i;
            tok[i + len] = kUnk;
        }
    }
    // walk back; consecutive unknowns collapse into one
    std::vector<int> back;
    for (int i = n; i > 0; i = from[i]) {
        const bool repeat_unk = tok[i] == kUnk && !back.empty() && back.back() == kUnk;
        if (!repeat_unk) back.push_back(tok[i]);
    }
    ids.insert(ids.end(), back.rbegin(), back.rend());
}

std::vector<int> T5Tokenizer::encode(const std::string& text, int max_len) const {
    if (max_len < 1) return {};
    std::vector<int> ids;
    // control pieces written literally ("<extra_id_0>") are kept whole; the
    // text between them is segmented
    size_t done = 0;
    for (size_t open = text.find('<'); open != std::string::npos; open = text.find('<', open + 1)) {
        const size_t close = text.find('>', open);
        if (close == std::string::npos) break;
        if (close - open >= static_cast<size_t>(longest_)) continue;
        const auto it = piece_.find(text.substr(open, close + 1 - open));
        if (it == piece_.end() || score_[static_cast<size_t>(it->second)] != 0.0) continue;
        segment(text.substr(done, open - done), ids);
        ids.push_back(it->second);
        done = close + 1;
    }
    segment(text.substr(done), ids);
    if (static_cast<int>(ids.size()) > max_len - 1) ids.resize(static_cast<size_t>(max_len - 1));
    ids.push_back(kEos);
    ids.resize(static_cast<size_t>(max_len), kPad);
    return ids;
}

}  // namespace vsb
