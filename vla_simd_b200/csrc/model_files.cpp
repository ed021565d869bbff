// Checkpoint file access (see model_files.h). Host code only.
//
// GGUF container (versions 2 and 3; little-endian): "GGUF", u32 version,
// u64 tensor count, u64 key/value count; key/value pairs (string key, u32 value
// type, value); tensor infos (string name, u32 n_dims, u64 dims[n_dims], u32
// element type, u64 offset into the data section); the data section at the
// next multiple of general.alignment (default 32) after the infos. Strings are
// u64 length + bytes. Every read here is bounds-checked against the mapping.
#include "model_files.h"

#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <fstream>
#include <sstream>

namespace vsb {

namespace {

bool ends_with(const std::string& s, const char* suf) {
    const size_t n = std::strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

std::string strip_slash(std::string p) {
    while (p.size() > 1 && p.back() == '/') p.pop_back();
    return p;
}

std::string parent(const std::string& p) {
    const size_t s = p.rfind('/');
    if (s == std::string::npos) return ".";
    return s == 0 ? "/" : p.substr(0, s);
}

// A relative path that stays inside the model directory.
bool relative_file(const std::string& name) {
    if (name.empty() || name.find('\0') != std::string::npos || name[0] == '/') return false;
    size_t start = 0;
    while (start <= name.size()) {
        const size_t end = name.find('/', start);
        const std::string part = name.substr(start, end == std::string::npos ? std::string::npos : end - start);
        if (part.empty() || part == "." || part == "..") return false;
        if (end == std::string::npos) break;
        start = end + 1;
    }
    return true;
}

// GGUF value types and ggml element types this reader knows the sizes of.
enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kString = 8, kArray = 9,
    kU64 = 10, kI64 = 11, kF64 = 12,
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

// bytes per element of the ggml tensor types a vla.simd GGUF uses
size_t ggml_size(uint32_t t) {
    switch (t) {
        case 0: return 4;    // F32
        case 1: return 2;    // F16
        case 24: return 1;   // I8
        case 25: return 2;   // I16
        case 26: return 4;   // I32
        case 27: return 8;   // I64
        case 28: return 8;   // F64
        case 30: return 2;   // BF16
        default: return 0;
    }
}

struct Reader {
    const uint8_t* p;
    size_t n, o = 0;
    bool ok = true;
    bool take(void* dst, size_t k) {
        if (!ok || k > n - o) { ok = false; return false; }
        std::memcpy(dst, p + o, k);
        o += k;
        return true;
    }
    uint32_t u32() { uint32_t v = 0; take(&v, 4); return v; }
    uint64_t u64() { uint64_t v = 0; take(&v, 8); return v; }
    std::string str() {
        const uint64_t len = u64();
        if (!ok || len > n - o) { ok = false; return {}; }
        std::string s(reinterpret_cast<const char*>(p + o), static_cast<size_t>(len));
        o += static_cast<size_t>(len);
        return s;
    }
    bool skip(size_t k) {
        if (!ok || k > n - o) { ok = false; return false; }
        o += k;
        return true;
    }
};

}  // namespace

std::string find_gguf(const std::string& path_in) {
    const std::string path = strip_slash(path_in);
    struct stat st;
    if (stat(path.c_str(), &st) != 0) return {};
    if (S_ISREG(st.st_mode)) return ends_with(path, ".gguf") ? path : std::string();
    if (!S_ISDIR(st.st_mode)) return {};
    DIR* d = opendir(path.c_str());
    if (!d) return {};
    std::string found;
    int n_gguf = 0, n_meta = 0;
    while (dirent* e = readdir(d)) {
        const std::string name = e->d_name;
        if (ends_with(name, ".gguf")) { n_gguf++; found = name; }
        else if (ends_with(name, ".meta")) n_meta++;
    }
    closedir(d);
    return n_gguf == 1 && n_meta == 0 ? path + "/" + found : std::string();
}

ModelFiles::~ModelFiles() {
    if (map_) munmap(map_, map_len_);
}

bool ModelFiles::open(const std::string& path_in) {
    const std::string path = strip_slash(path_in);
    file_ = find_gguf(path);
    if (file_.empty()) {
        dir_ = path;
        return true;
    }
    dir_ = file_ == path ? parent(path) : path;
    const int fd = ::open(file_.c_str(), O_RDONLY);
    if (fd < 0) { err_ = file_ + ": cannot open"; return false; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        ::close(fd);
        err_ = file_ + ": empty or unreadable";
        return false;
    }
    map_len_ = static_cast<size_t>(st.st_size);
    void* m = mmap(nullptr, map_len_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) { err_ = file_ + ": mmap failed"; map_len_ = 0; return false; }
    map_ = m;
    if (!parse()) {
        munmap(map_, map_len_);
        map_ = nullptr;
        return false;
    }
    return true;
}

bool ModelFiles::parse() {
    Reader r{static_cast<const uint8_t*>(map_), map_len_};
    char magic[4];
    if (!r.take(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) { err_ = file_ + ": not a GGUF file"; return false; }
    const uint32_t version = r.u32();
    if (version != 2 && version != 3) { err_ = file_ + ": GGUF version " + std::to_string(version) + " unsupported"; return false; }
    const uint64_t n_tensors = r.u64(), n_kv = r.u64();
    if (!r.ok || n_tensors > (1ull << 24) || n_kv > (1ull << 24)) { err_ = file_ + ": corrupt GGUF header"; return false; }
    std::string arch;
    uint64_t format = 0, alignment = 32;
    bool has_format = false;
    const std::string prefix = "vla_simd.file.";
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        const std::string key = r.str();
        const uint32_t type = r.u32();
        if (type == kString) {
            const std::string val = r.str();
            if (key == "general.architecture") arch = val;
            if (key.compare(0, prefix.size(), prefix) == 0) {
                const std::string rel = key.substr(prefix.size());
                if (!relative_file(rel)) { err_ = file_ + ": invalid embedded file " + rel; return false; }
                texts_[rel] = val;
            }
        } else if (type == kArray) {
            const uint32_t et = r.u32();
            const uint64_t count = r.u64();
            if (et == kString) {
                for (uint64_t j = 0; j < count && r.ok; ++j) r.str();
            } else {
                const size_t es = scalar_size(et);
                if (!es || count > (map_len_ / es)) { err_ = file_ + ": corrupt GGUF array"; return false; }
                r.skip(static_cast<size_t>(count) * es);
            }
        } else {
            const size_t es = scalar_size(type);
            if (!es) { err_ = file_ + ": unknown GGUF value type"; return false; }
            uint64_t v = 0;
            r.take(&v, es);
            if (key == "vla_simd.format" && (type == kU32 || type == kI32 || type == kU64 || type == kI64)) {
                format = v;
                has_format = true;
            }
            if (key == "general.alignment" && type == kU32) alignment = v;
        }
    }
    if (!r.ok) { err_ = file_ + ": truncated GGUF metadata"; return false; }
    if (arch != "vla-simd") {
        err_ = file_ + ": GGUF architecture \"" + arch + "\" is not a vla.simd checkpoint this backend loads";
        return false;
    }
    if (!has_format || format != 1) {
        err_ = file_ + ": vla.simd GGUF format " + std::to_string(format) + " is not supported (1 is)";
        return false;
    }
    if (alignment == 0 || (alignment & (alignment - 1)) || alignment > 4096) { err_ = file_ + ": invalid alignment"; return false; }
    struct Info { std::string name; uint64_t bytes, off; };
    std::vector<Info> infos;
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        Info t;
        t.name = r.str();
        const uint32_t nd = r.u32();
        if (nd == 0 || nd > 8) { err_ = file_ + ": bad tensor rank"; return false; }
        uint64_t numel = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            const uint64_t ne = r.u64();
            if (ne == 0 || numel > (map_len_ / ne)) { err_ = file_ + ": bad tensor shape " + t.name; return false; }
            numel *= ne;
        }
        const uint32_t type = r.u32();
        t.off = r.u64();
        const size_t es = ggml_size(type);
        if (!es) { err_ = file_ + ": tensor " + t.name + " has an element type vla.simd does not write"; return false; }
        t.bytes = numel * es;
        infos.push_back(t);
    }
    if (!r.ok) { err_ = file_ + ": truncated GGUF tensor table"; return false; }
    const uint64_t base = (r.o + alignment - 1) / alignment * alignment;
    std::map<std::string, size_t> parts;
    for (const Info& t : infos) {
        if (t.off % alignment || base + t.off > map_len_ || t.bytes > map_len_ - base - t.off) {
            err_ = file_ + ": tensor " + t.name + " outside the file";
            return false;
        }
        std::string rel = t.name;
        const size_t colon = rel.rfind(':');
        if (colon != std::string::npos && colon + 1 < rel.size() &&
            rel.find_first_not_of("0123456789", colon + 1) == std::string::npos) {
            const std::string suffix = rel.substr(colon + 1);
            rel.resize(colon);
            const size_t part = parts[rel]++;
            if (suffix != std::to_string(part) || (part == 0 && (bins_.count(rel) || texts_.count(rel)))) {
                err_ = file_ + ": invalid tensor part " + t.name;
                return false;
            }
        } else if (bins_.count(rel) || texts_.count(rel)) {
            err_ = file_ + ": duplicate embedded file " + rel;
            return false;
        }
        if (!relative_file(rel)) { err_ = file_ + ": invalid embedded file " + rel; return false; }
        bins_[rel].emplace_back(static_cast<const uint8_t*>(map_) + base + t.off, static_cast<size_t>(t.bytes));
    }
    if (bins_.empty() && texts_.empty()) { err_ = file_ + ": vla.simd GGUF holds no files"; return false; }
    return true;
}

bool ModelFiles::read_path(const std::string& path, std::string& out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::ostringstream ss;
    ss << f.rdbuf();
    out = ss.str();
    return true;
}

bool ModelFiles::disk(const std::string& rel, std::string& out) const { return read_path(dir_ + "/" + rel, out); }

bool ModelFiles::read(const std::string& rel, std::string& out) const {
    if (map_) {
        const auto t = texts_.find(rel);
        if (t != texts_.end()) { out = t->second; return true; }
        const auto b = bins_.find(rel);
        if (b != bins_.end()) {
            size_t n = 0;
            for (const auto& piece : b->second) n += piece.second;
            out.resize(n);
            size_t at = 0;
            for (const auto& piece : b->second) {
                std::memcpy(&out[at], piece.first, piece.second);
                at += piece.second;
            }
            return true;
        }
    }
    return disk(rel, out);   // a plain directory, or a sidecar beside the GGUF
}

bool ModelFiles::read_floats(const std::string& rel, std::vector<float>& out) const {
    if (map_) {
        const auto b = bins_.find(rel);
        if (b != bins_.end()) {
            size_t n = 0;
            for (const auto& piece : b->second) n += piece.second;
            if (n % 4) return false;
            out.resize(n / 4);
            size_t at = 0;
            for (const auto& piece : b->second) {
                std::memcpy(reinterpret_cast<char*>(out.data()) + at, piece.first, piece.second);
                at += piece.second;
            }
            return true;
        }
    }
    std::string bytes;
    if (!read(rel, bytes) || bytes.size() % 4) return false;
    out.resize(bytes.size() / 4);
    if (!bytes.empty()) std::memcpy(out.data(), bytes.data(), bytes.size());
    return true;
}

}  // namespace vsb
