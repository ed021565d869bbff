// Checkpoint file access for the model loaders: a converted directory
// (<name>.meta / <name>.bin / config.txt / stats.bin files) or a vla.simd GGUF
// that carries those same files.
//
// The reference's rule for which one a model path is (src/io/files.h:13-15,
// src/io/files.cpp:84-101): a path that is a .gguf file, or a directory
// holding exactly one .gguf and no .meta file, is a GGUF; anything else is a
// plain directory. A vla.simd GGUF (general.architecture "vla-simd",
// vla_simd.format 1; written by the reference's tools/_gguf.py) stores each
// text file as the string value of "vla_simd.file.<relative path>" and each
// .bin file as a tensor named by its relative path, or as parts "<path>:0",
// "<path>:1", ... concatenated in file order (src/io/gguf_vla_simd.cpp:18-77).
// A file the GGUF does not carry is read from the directory beside it.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace vsb {

class ModelFiles {
  public:
    ModelFiles() = default;
    ~ModelFiles();
    ModelFiles(const ModelFiles&) = delete;
    ModelFiles& operator=(const ModelFiles&) = delete;

    // false (with error()) for a GGUF that does not parse or is not a vla.simd GGUF
    bool open(const std::string& path);
    const std::string& error() const { return err_; }
    bool gguf() const { return map_ != nullptr; }

    // The whole file `rel` (relative to the model path); false when absent.
    bool read(const std::string& rel, std::string& out) const;
    // A .bin of little-endian fp32 values; false when absent or not a whole number of floats.
    bool read_floats(const std::string& rel, std::vector<float>& out) const;
    // A whole file at an absolute or working-directory path, outside any model.
    static bool read_path(const std::string& path, std::string& out);

  private:
    bool parse();
    bool disk(const std::string& rel, std::string& out) const;

    std::string dir_;                      // plain directory, or the GGUF's sidecar directory
    std::string file_, err_;
    void* map_ = nullptr;
    size_t map_len_ = 0;
    // relative path -> its pieces in the mapped file (a text file: one piece of
    // its own bytes in texts_)
    std::map<std::string, std::vector<std::pair<const uint8_t*, size_t>>> bins_;
    std::map<std::string, std::string> texts_;
};

// Where a model path's GGUF is under the rule above ("" for a plain directory).
std::string find_gguf(const std::string& path);

}  // namespace vsb
