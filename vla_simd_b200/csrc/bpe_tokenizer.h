// Byte-level BPE tokenizer of the SmolLM2 family, as SmolVLA's C ABI feeds
// its prompt (src/tokenizer/tokenizer.h:13-31). Host code: it turns an
// instruction into the token ids the device embedding lookup reads.
//
// vocab.txt: "id<TAB>token" per line (tokens in the byte-to-unicode alphabet);
// merges.txt: "a b" per line, the line number is the merge's rank.
#pragma once
#include <cstddef>
#include <string>
#include <unordered_map>
#include <vector>

namespace vsb {

class BpeTokenizer {
  public:
    bool load_text(const std::string& vocab, const std::string& merges);
    // ids of `text` (no special-token handling), src/tokenizer/tokenizer.cpp:151-204
    std::vector<int> encode(const std::string& text) const;

  private:
    // ids of the piece text[begin, end) after merging
    std::vector<int> merge_piece(const std::string& text, size_t begin, size_t end) const;

    std::unordered_map<std::string, int> vocab_;
    std::unordered_map<std::string, int> rank_;   // "left right" -> merge rank
    std::string byte_char_[256];                  // byte -> its symbol (UTF-8)
};

}  // namespace vsb
