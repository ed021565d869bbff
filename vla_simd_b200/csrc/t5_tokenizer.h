// SentencePiece-unigram tokenizer of the T5 family, as Octo feeds its language
// tower (src/tokenizer/t5_tokenizer.h:13-33). Host code: it turns the
// instruction string of a query into the 16 token ids the device T5 encoder
// reads, once per distinct instruction.
//
// vocab.txt: one "piece<TAB>score" per line, the line number is the id. A
// piece with score 0 is only kept when it looks like "<...>" (control
// symbols); ids 0 / 1 / 2 are pad / eos / unk.
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace vsb {

class T5Tokenizer {
  public:
    // `text` is the whole vocab.txt
    bool load_text(const std::string& text);

    // Pieces of `text` truncated to max_len - 1, then eos, then pad to max_len
    // (src/tokenizer/t5_tokenizer.cpp:131-155).
    std::vector<int> encode(const std::string& text, int max_len) const;

    int pad_id() const { return 0; }

  private:
    // ids of `text` after normalization (no control pieces inside)
    void segment(const std::string& text, std::vector<int>& ids) const;
    // [begin, end) of each literal control piece in `text`, in order
    std::vector<std::pair<size_t, size_t>> control_pieces(const std::string& text) const;

    std::unordered_map<std::string, int> piece_;
    std::vector<double> score_;
    int longest_ = 1;
    double lowest_ = 0.0;
};

}  // namespace vsb
