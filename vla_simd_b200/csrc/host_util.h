// Host-side helpers shared by the policy loaders: environment knobs, shape
// checks, the converter's float-arena cursor and "key value" metadata.
#pragma once
#include <climits>
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <initializer_list>
#include <map>
#include <sstream>
#include <string>
#include <vector>

namespace vsb {
namespace host {

// An integer environment variable, or dflt when unset, empty or not a whole number.
inline int env_int(const char* name, int dflt) {
    const char* e = std::getenv(name);
    if (!e || !*e) return dflt;
    char* end = nullptr;
    const long v = std::strtol(e, &end, 10);
    return (end && *end == '\0') ? static_cast<int>(v) : dflt;
}

// TCPU_I8_CLIP semantics (src/hal/common/env.cpp:220-227): (0, 1], default 1.
inline float env_clip() {
    const char* e = std::getenv("TCPU_I8_CLIP");
    const float f = e ? static_cast<float>(std::atof(e)) : 1.0f;
    return f > 0.0f && f <= 1.0f ? f : 1.0f;
}

// Every dimension positive and their product at most INT_MAX (src/models/arena.h:27-35).
inline bool shape_fits(std::initializer_list<long long> dims) {
    long long c = 1;
    for (long long d : dims) {
        if (d <= 0) return false;
        c *= d;
        if (c > INT_MAX) return false;
    }
    return true;
}

inline long long round16(long long v) { return (v + 15) & ~15LL; }

// Cursor over a float arena in the converter's order (src/models/arena.h:61-72).
struct Cursor {
    const std::vector<float>& d;
    size_t off = 0;
    bool ok = true;
    const float* operator()(size_t n) {
        if (!ok || n > d.size() - off) {
            ok = false;
            return nullptr;
        }
        const float* p = d.data() + off;
        off += n;
        return p;
    }
    bool done() const { return ok && off == d.size(); }
};

// "key value" metadata where every value is a number (octo.meta, t5.meta,
// vit.meta, ...; src/models/octo/octo_transformer.cpp:18-38). false on a
// missing or non-finite value.
inline bool numeric_meta(const std::string& text, std::map<std::string, double>& kv) {
    std::istringstream in(text);
    std::string key;
    double val;
    while (in >> key) {
        if (!(in >> val) || !std::isfinite(val)) return false;
        kv[key] = val;
    }
    return true;
}

// An integer key, which must be whole and in range (src/models/arena.h:21-25);
// absent keys leave `out` unchanged.
inline bool meta_int(const std::map<std::string, double>& kv, const char* key, int& out) {
    const auto it = kv.find(key);
    if (it == kv.end()) return true;
    const double v = it->second;
    if (v < INT_MIN || v > INT_MAX || v != std::trunc(v)) return false;
    out = static_cast<int>(v);
    return true;
}

template <class T>
inline void meta_real(const std::map<std::string, double>& kv, const char* key, T& out) {
    const auto it = kv.find(key);
    if (it != kv.end()) out = static_cast<T>(it->second);
}

}  // namespace host
}  // namespace vsb
