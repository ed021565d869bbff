// T5 unigram tokenizer: the reference's normalization (a subset of NFKC plus
// whitespace folding into the U+2581 word marker) and its best-score
// segmentation over bytes, src/tokenizer/t5_tokenizer.cpp:13-155. Three steps:
// normalize() rewrites the text; segment() scores every byte position from the
// pieces that end there (the best score of the text up to each position);
// encode() cuts the text at literal control pieces ("<extra_id_0>") and
// segments what lies between them.
#include "t5_tokenizer.h"

#include "utf8.h"

#include <algorithm>
#include <limits>
#include <sstream>
#include <string_view>

namespace vsb {
namespace {

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

constexpr int kUnk = 2, kEos = 1, kPad = 0;

const Compat* compat_of(uint32_t cp) {
    const Compat* end = kCompat + sizeof(kCompat) / sizeof(kCompat[0]);
    const Compat* it = std::lower_bound(kCompat, end, cp, [](const Compat& c, uint32_t v) { return c.cp < v; });
    return it != end && it->cp == cp ? it : nullptr;
}

// The normalizer: strict UTF-8 decoding (a bad sequence reads as U+FFFD),
// dropped controls, fullwidth ASCII folded to ASCII, the compatibility
// rewrites above, and every run of blanks before a word replaced by one U+2581
// (blanks after the last word vanish).
std::string normalize(const std::string& text) {
    std::string out;
    bool word_start = true;
    auto put = [&](uint32_t cp) {
        if (blank(cp)) {
            word_start = true;
            return;
        }
        if (word_start) utf8_put(out, 0x2581);
        word_start = false;
        utf8_put(out, cp);
    };
    for (size_t i = 0; i < text.size();) {
        const Utf8Char u = utf8_strict(text.data() + i, text.size() - i);
        i += u.len;
        uint32_t cp = u.cp;
        if (dropped(cp)) continue;
        if (cp >= 0xFF01 && cp <= 0xFF5D) cp -= 0xFEE0;
        if (const Compat* c = compat_of(cp)) {
            for (uint32_t r : c->to)
                if (r) put(r);
        } else {
            put(cp);
        }
    }
    return out;
}

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
    const std::string s = normalize(text);
    const int n = static_cast<int>(s.size());
    // score[j]: best total score of a segmentation of s[0, j); start[j] / id[j]
    // the last piece of that segmentation. Candidates for j are weighed in the
    // order: start position ascending, and at one start the vocabulary piece
    // before the one-character <unk>; a later candidate wins only with a
    // strictly higher score, which fixes the ties.
    const double kUnreachable = -std::numeric_limits<double>::infinity();
    const double unk_score = lowest_ - 10.0;
    std::vector<double> score(n + 1, kUnreachable);
    std::vector<int> start(n + 1, -1), id(n + 1, kUnk);
    std::vector<int> char_len(n, 1);     // UTF-8 length of the character starting at each byte
    for (int i = 0; i < n; ++i) {
        const unsigned c = static_cast<unsigned char>(s[i]);
        char_len[i] = c < 0x80 ? 1 : (c & 0xE0) == 0xC0 ? 2 : (c & 0xF0) == 0xE0 ? 3 : (c & 0xF8) == 0xF0 ? 4 : 1;
    }
    score[0] = 0.0;
    std::string_view sv(s);
    const int reach = std::max(longest_, 4);   // the farthest start a piece or a character can have
    for (int j = 1; j <= n; ++j) {
        for (int i = std::max(0, j - reach); i < j; ++i) {
            if (score[i] == kUnreachable) continue;
            if (j - i <= longest_) {
                const auto it = piece_.find(std::string(sv.substr(i, j - i)));
                if (it != piece_.end() && score[i] + score_[it->second] > score[j]) {
                    score[j] = score[i] + score_[it->second];
                    start[j] = i;
                    id[j] = it->second;
                }
            }
            if (char_len[i] == j - i && score[i] + unk_score > score[j]) {
                score[j] = score[i] + unk_score;
                start[j] = i;
                id[j] = kUnk;
            }
        }
    }
    // the winning pieces front to back; a run of <unk> pieces emits one <unk>
    std::vector<int> path;
    for (int j = n; j > 0; j = start[j]) path.push_back(id[j]);
    bool after_unk = false;
    for (auto it = path.rbegin(); it != path.rend(); ++it) {
        if (*it == kUnk && after_unk) continue;
        after_unk = *it == kUnk;
        ids.push_back(*it);
    }
}

std::vector<std::pair<size_t, size_t>> T5Tokenizer::control_pieces(const std::string& text) const {
    // every '<' opens a candidate that ends at the next '>'; the candidate is a
    // control piece when the vocabulary holds it with score 0 and it is shorter
    // than the longest piece. Scanning resumes after a match (no control piece
    // of a T5 vocabulary holds a second '<').
    std::vector<std::pair<size_t, size_t>> hits;
    size_t from = 0;
    for (;;) {
        const size_t open = text.find('<', from);
        if (open == std::string::npos) break;
        const size_t close = text.find('>', open);
        if (close == std::string::npos) break;
        from = open + 1;
        if (close - open >= static_cast<size_t>(longest_)) continue;
        const auto it = piece_.find(text.substr(open, close + 1 - open));
        if (it == piece_.end() || score_[static_cast<size_t>(it->second)] != 0.0) continue;
        hits.emplace_back(open, close + 1);
        from = close + 1;
    }
    return hits;
}

std::vector<int> T5Tokenizer::encode(const std::string& text, int max_len) const {
    if (max_len < 1) return {};
    std::vector<int> ids;
    size_t done = 0;
    for (const auto& [b, e] : control_pieces(text)) {
        segment(text.substr(done, b - done), ids);
        ids.push_back(piece_.at(text.substr(b, e - b)));
        done = e;
    }
    segment(text.substr(done), ids);
    // room for the eos, then padding to max_len
    if (static_cast<int>(ids.size()) > max_len - 1) ids.resize(static_cast<size_t>(max_len - 1));
    ids.push_back(kEos);
    ids.resize(static_cast<size_t>(max_len), kPad);
    return ids;
}

}  // namespace vsb
