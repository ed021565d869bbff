// Octo runtime (see octo_policy.h). Host code only: parsing, int8 packing,
// buffer planning, the T5 cache and the kernel sequence of one query batch.
#include "octo_policy.h"

#include "host_util.h"

#include "model_files.h"

#include "dp.h"
#include "f32.h"
#include "gemm_i8.h"
#include "lm_ops.h"
#include "nn.h"
#include "octo.h"
#include "polar_normal.h"
#include "quant.h"

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <sstream>

namespace vsb {

namespace {

using host::Cursor;
using host::env_clip;
using host::env_int;
using host::meta_int;
using host::numeric_meta;
using host::round16;
using host::shape_fits;

void meta_float(const std::map<std::string, double>& kv, const char* key, float& out) { host::meta_real(kv, key, out); }

// T5's bidirectional relative-position bucket of rp = key - query (the HF
// relative_position_bucket: exact buckets below num_buckets/4, log-spaced up
// to max_dist, the sign in the top half), src/nn/t5_encoder.cpp:75-88.
int t5_bucket(int rp, int num_buckets, int max_dist) {
    const int half = num_buckets / 2;
    const int base = rp > 0 ? half : 0;
    const int a = rp < 0 ? -rp : rp;
    const int exact = half / 2;
    if (a < exact) return base + a;
    const double frac = std::log(static_cast<double>(a) / exact) / std::log(static_cast<double>(max_dist) / exact);
    const int b = std::min(exact + static_cast<int>(frac * (half - exact)), half - 1);
    return base + b;
}

int grid_side(int s, int n_layers, int k, int stride, int pad) {
    for (int i = 0; i < n_layers; ++i) {
        const long long num = (long long)s + 2LL * pad - k;
        if (num < 0) return -1;
        s = static_cast<int>(num / stride + 1);
    }
    return s;
}

}  // namespace

#define VSB_TRY(x)                                     \
    do {                                               \
        const cudaError_t e_ = (x);                    \
        if (e_ != cudaSuccess) return e_;              \
    } while (0)

template <class T>
T* OctoPolicy::dalloc(size_t n) {
    void* p = nullptr;
    if (n == 0) n = 1;
    if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
        fail("cudaMalloc failed");
        return nullptr;
    }
    allocs_.push_back(p);
    return static_cast<T*>(p);
}

OctoPolicy::~OctoPolicy() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device_);
    for (auto& g : graphs_)
        if (g.second) cudaGraphExecDestroy(g.second);
    if (stream_) cudaStreamDestroy(stream_);
    for (void* p : allocs_) cudaFree(p);
    if (h_pinned_) cudaFreeHost(h_pinned_);
    if (h_noise_) cudaFreeHost(h_noise_);
    if (h_slots_) cudaFreeHost(h_slots_);
    if (h_status_pinned_) cudaFreeHost(h_status_pinned_);
    cudaSetDevice(prev);
}

// ------------------------------------------------------------------ load
// t5.meta / t5.bin (src/nn/t5_encoder.cpp:20-72): embedding [vocab][D], relative
// bias [buckets][heads], per layer ln1, q, k, v, o [D][D], ln2, wi [FF][D],
// wo [D][FF]; final norm.
bool OctoPolicy::load_t5(const ModelFiles& files) {
    std::string text;
    std::map<std::string, double> kv;
    if (!files.read("t5.meta", text) || !numeric_meta(text, kv)) { fail("cannot read t5.meta"); return false; }
    OctoConfigDev& c = cfg_;
    int d_model = c.t5_dim;
    if (!meta_int(kv, "d_model", d_model) || !meta_int(kv, "n_layers", c.t5_layers) ||
        !meta_int(kv, "n_heads", c.t5_heads) || !meta_int(kv, "d_kv", c.t5_dkv) || !meta_int(kv, "d_ff", c.t5_ff) ||
        !meta_int(kv, "vocab", c.t5_vocab) || !meta_int(kv, "n_buckets", c.t5_buckets) ||
        !meta_int(kv, "max_dist", c.t5_max_dist)) {
        fail("invalid integer in t5.meta");
        return false;
    }
    meta_float(kv, "eps", c.t5_eps);
    const int D = d_model, FF = c.t5_ff;
    if (!shape_fits({D, D}) || !shape_fits({D, FF}) || !shape_fits({c.t5_vocab, D}) || !shape_fits({c.t5_heads, c.t5_dkv}) ||
        c.t5_heads * c.t5_dkv != D || c.t5_layers < 1 || !shape_fits({c.t5_buckets, c.t5_heads}) || c.t5_buckets < 4 ||
        c.t5_buckets % 2 || c.t5_max_dist <= c.t5_buckets / 4 || !std::isfinite(c.t5_eps) || c.t5_eps <= 0) {
        fail("unsupported t5.meta");
        return false;
    }
    if (c.t5_dkv % 8) { fail("T5 head size must be a multiple of 8 on this backend"); return false; }
    c.t5_dim = D;
    std::vector<float> data;
    if (!files.read_floats("t5.bin", data)) { fail("cannot read t5.bin"); return false; }
    Cursor take{data};
    auto up = [&](size_t n) -> float* {
        const float* src = take(n);
        if (!src) return nullptr;
        float* p = dalloc<float>(n);
        if (p) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    t5_emb_ = up((size_t)c.t5_vocab * D);
    t5_rel_ = up((size_t)c.t5_buckets * c.t5_heads);
    t5_.resize(c.t5_layers);
    for (T5LayerDev& L : t5_) {
        L.ln1 = up(D);
        L.wq = up((size_t)D * D);
        L.wk = up((size_t)D * D);
        L.wv = up((size_t)D * D);
        L.wo = up((size_t)D * D);
        L.ln2 = up(D);
        L.wi = up((size_t)FF * D);
        L.wo2 = up((size_t)D * FF);
        if (!take.ok) break;
    }
    t5_final_ = up(D);
    if (!take.done()) { fail("t5.bin size does not match t5.meta"); return false; }
    return err_.empty();
}

// stem_<name>.meta / .bin (src/models/octo/small_stem.cpp:16-83): per layer conv
// w [Cout][k][k][Cin], conv b, GroupNorm scale and bias; then embed w [E][C], b.
bool OctoPolicy::load_stem(const ModelFiles& files, const std::string& name, int in_hw, bool conv_int8,
                           bool embed_int8, OctoStemDev& s) {
    std::string text;
    if (!files.read(name + ".meta", text)) { fail("cannot read " + name + ".meta"); return false; }
    constexpr int kMaxLayers = 8;
    int feat[kMaxLayers] = {32, 96, 192, 384};
    int in_ch = 6;
    std::istringstream in(text);
    std::string line;
    while (std::getline(in, line)) {
        std::istringstream ss(line);
        std::string key;
        if (!(ss >> key)) continue;
        if (key == "in_ch") ss >> in_ch;
        else if (key == "n_layers") ss >> s.n_layers;
        else if (key == "k") ss >> s.k;
        else if (key == "stride") ss >> s.stride;
        else if (key == "pad") ss >> s.pad;
        else if (key == "features") {
            for (int i = 0; i < s.n_layers && i < kMaxLayers; ++i) ss >> feat[i];
        } else if (key == "embed_dim") ss >> s.embed_dim;
        else if (key == "gn_groups") ss >> s.gn_groups;
        else if (key == "gn_eps") ss >> s.gn_eps;
        else continue;
        if (ss.fail() || !(ss >> std::ws).eof()) { fail("malformed " + name + ".meta"); return false; }
    }
    if (s.n_layers < 1 || s.n_layers > kMaxLayers || in_ch != 6 || s.k < 1 || s.embed_dim < 1 || s.stride < 1 ||
        s.pad < 0 || s.pad > (INT_MAX - 256) / 2 || s.gn_groups < 1 || !std::isfinite(s.gn_eps) || s.gn_eps <= 0) {
        fail("unsupported " + name + ".meta");
        return false;
    }
    int cin = in_ch;
    for (int i = 0; i < s.n_layers; ++i) {
        if (!shape_fits({feat[i], s.k, s.k, cin}) || feat[i] % s.gn_groups) { fail("unsupported " + name + ".meta"); return false; }
        cin = feat[i];
    }
    std::vector<float> data;
    if (!files.read_floats(name + ".bin", data)) { fail("cannot read " + name + ".bin"); return false; }
    Cursor take{data};
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    auto dev_copy = [&](const float* src, size_t n) -> float* {
        float* p = dalloc<float>(n);
        if (p && src) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    s.feat.assign(feat, feat + s.n_layers);
    s.conv.resize(s.n_layers);
    s.gn_s.resize(s.n_layers);
    s.gn_b.resize(s.n_layers);
    cin = in_ch;
    for (int i = 0; i < s.n_layers; ++i) {
        const int cout = feat[i];
        const float* w = take((size_t)cout * s.k * s.k * cin);
        const float* b = take(cout);
        const float* gs = take(cout);
        const float* gb = take(cout);
        if (!take.ok) { fail(name + ".bin too short"); return false; }
        if (!make_dev_conv(s.conv[i], w, b, cout, s.k, cin, s.stride, s.pad, conv_int8, alloc, &n_int8_)) {
            fail("conv upload failed");
            return false;
        }
        s.gn_s[i] = dev_copy(gs, cout);
        s.gn_b[i] = dev_copy(gb, cout);
        cin = cout;
    }
    const float* ew = take((size_t)s.embed_dim * cin);
    const float* eb = take(s.embed_dim);
    if (!take.done()) { fail(name + ".bin size does not match its meta"); return false; }
    if (!upload_linear(s.embed, ew, eb, s.embed_dim, cin, embed_int8, alloc, &n_int8_)) {
        fail("linear upload failed");
        return false;
    }
    s.in_hw = in_hw;
    s.side = grid_side(in_hw, s.n_layers, s.k, s.stride, s.pad);
    if (s.side < 1) { fail(name + ": the input does not survive the stem"); return false; }
    return err_.empty();
}

// octo.meta / octo.bin (src/models/octo/octo_transformer.cpp:18-100).
// OCTO_INT8 bits (src/models/octo/octo_model.cpp:53-56): 1 q/k/v/o, 2 w1,
// 4 w2, 8 token projections + stem embeds, 16 stem convs, 32 diffusion head.
bool OctoPolicy::load_transformer(const ModelFiles& files, int mask) {
    std::string text;
    std::map<std::string, double> kv;
    if (!files.read("octo.meta", text) || !numeric_meta(text, kv)) { fail("cannot read octo.meta"); return false; }
    OctoConfigDev& c = cfg_;
    int t5_dim = c.t5_dim;
    c.t5_dim = 768;
    if (!meta_int(kv, "d", c.d) || !meta_int(kv, "n_layers", c.n_layers) || !meta_int(kv, "heads", c.heads) ||
        !meta_int(kv, "head_dim", c.head_dim) || !meta_int(kv, "mlp", c.mlp) ||
        !meta_int(kv, "max_horizon", c.max_horizon) || !meta_int(kv, "n_task", c.n_task) ||
        !meta_int(kv, "tok_primary", c.tok_primary) || !meta_int(kv, "tok_wrist", c.tok_wrist) ||
        !meta_int(kv, "n_readout", c.n_readout) || !meta_int(kv, "t5_dim", c.t5_dim) ||
        !meta_int(kv, "stem_dim", c.stem_dim)) {
        fail("invalid integer in octo.meta");
        return false;
    }
    meta_float(kv, "ln_eps", c.ln_eps);
    if (kv.count("gelu_erf")) c.gelu_erf = kv["gelu_erf"] != 0;
    const int D = c.d;
    if (!shape_fits({D, D}) || !shape_fits({c.heads, c.head_dim}) || c.heads * c.head_dim != D || !shape_fits({c.mlp, D}) ||
        !shape_fits({c.n_task, D}) || !shape_fits({c.t5_dim, D}) || !shape_fits({c.stem_dim, D}) ||
        !shape_fits({c.max_horizon, c.tok_primary, D}) || !shape_fits({c.max_horizon, c.tok_wrist, D}) ||
        !shape_fits({c.max_horizon, c.n_readout, D}) || c.n_layers < 1 || !std::isfinite(c.ln_eps) || c.ln_eps <= 0) {
        fail("unsupported octo.meta");
        return false;
    }
    if (c.t5_dim != t5_dim) { fail("t5.meta d_model differs from octo.meta t5_dim"); return false; }
    if (c.head_dim != 64 || D % 4) { fail("this backend's attention needs head_dim 64"); return false; }
    std::vector<float> data;
    if (!files.read_floats("octo.bin", data)) { fail("cannot read octo.bin"); return false; }
    Cursor take{data};
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    auto up = [&](size_t n) -> float* {
        const float* src = take(n);
        if (!src) return nullptr;
        float* p = dalloc<float>(n);
        if (p) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    auto lin = [&](DevLinear& l, int N, int K, bool int8) -> bool {
        const float* w = take((size_t)N * K);
        const float* b = take(N);
        if (!take.ok) return false;
        return upload_linear(l, w, b, N, K, int8, alloc, &n_int8_);
    };
    const bool proj8 = (mask & 8) != 0;
    if (!lin(proj_task_, D, c.t5_dim, proj8) || !lin(proj_prim_, D, c.stem_dim, proj8) ||
        !lin(proj_wrist_, D, c.stem_dim, proj8)) {
        fail("octo.bin too short");
        return false;
    }
    pos_task_ = up((size_t)c.n_task * D);
    pos_prim_ = up((size_t)c.max_horizon * c.tok_primary * D);
    pos_wrist_ = up((size_t)c.max_horizon * c.tok_wrist * D);
    pos_readout_ = up((size_t)c.max_horizon * c.n_readout * D);
    layers_.resize(c.n_layers);
    std::vector<float> wqkv((size_t)3 * D * D), bqkv((size_t)3 * D);
    for (OctoLayerDev& L : layers_) {
        L.ln1s = up(D);
        L.ln1b = up(D);
        // q, k, v (each W [D][D] then b [D]) stacked into one [3D][D] layer:
        // every output keeps its own dot product, so the values are the three layers'
        for (int j = 0; j < 3; ++j) {
            const float* w = take((size_t)D * D);
            const float* b = take(D);
            if (!take.ok) { fail("octo.bin too short"); return false; }
            std::memcpy(wqkv.data() + (size_t)j * D * D, w, sizeof(float) * D * D);
            std::memcpy(bqkv.data() + (size_t)j * D, b, sizeof(float) * D);
        }
        int before = n_int8_;
        if (!upload_linear(L.wqkv, wqkv.data(), bqkv.data(), 3 * D, D, (mask & 1) != 0, alloc, &n_int8_)) {
            fail("linear upload failed");
            return false;
        }
        if (n_int8_ > before) n_int8_ += 2;   // the reference counts wq, wk, wv separately
        if (!lin(L.wo, D, D, (mask & 1) != 0)) { fail("octo.bin too short"); return false; }
        L.ln2s = up(D);
        L.ln2b = up(D);
        if (!lin(L.w1, c.mlp, D, (mask & 2) != 0) || !lin(L.w2, D, c.mlp, (mask & 4) != 0)) {
            fail("octo.bin too short");
            return false;
        }
    }
    final_s_ = up(D);
    final_b_ = up(D);
    if (!take.done()) { fail("octo.bin size does not match octo.meta"); return false; }
    return err_.empty();
}

// head.meta / head.bin (src/models/octo/diffusion_head.cpp:15-123).
bool OctoPolicy::load_head(const ModelFiles& files, bool int8) {
    std::string text;
    std::map<std::string, double> kv;
    if (!files.read("head.meta", text) || !numeric_meta(text, kv)) { fail("cannot read head.meta"); return false; }
    OctoConfigDev& c = cfg_;
    int emb = c.d;
    if (!meta_int(kv, "emb", emb) || !meta_int(kv, "action_dim", c.action_dim) ||
        !meta_int(kv, "horizon", c.horizon) || !meta_int(kv, "time_dim", c.time_dim) ||
        !meta_int(kv, "num_blocks", c.num_blocks) || !meta_int(kv, "hidden", c.hidden) ||
        !meta_int(kv, "steps", c.steps)) {
        fail("invalid integer in head.meta");
        return false;
    }
    meta_float(kv, "max_action", c.max_action);
    if (!shape_fits({c.action_dim, c.horizon}) || !shape_fits({2, c.time_dim, c.time_dim}) || c.time_dim % 2 ||
        !shape_fits({4, c.hidden, c.hidden}) || emb < 1 || c.num_blocks < 0 ||
        (long long)c.time_dim + emb + c.flat() > INT_MAX || !shape_fits({c.steps, c.time_dim}) ||
        !std::isfinite(c.max_action) || c.max_action <= 0) {
        fail("unsupported head.meta");
        return false;
    }
    if (emb != c.d) { fail("head.meta emb differs from the transformer width"); return false; }
    const int TD = c.time_dim, H = c.hidden, IN = TD + emb + c.flat();
    std::vector<float> data;
    if (!files.read_floats("head.bin", data)) { fail("cannot read head.bin"); return false; }
    Cursor take{data};
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    auto lin = [&](DevLinear& l, int N, int K, bool q) -> bool {
        const float* w = take((size_t)N * K);
        const float* b = take(N);
        if (!take.ok) return false;
        return upload_linear(l, w, b, N, K, q, alloc, &n_int8_);
    };
    auto up = [&](size_t n) -> float* {
        const float* src = take(n);
        if (!src) return nullptr;
        float* p = dalloc<float>(n);
        if (p) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    const float* fw = take(TD / 2);
    if (!fw) { fail("head.bin too short"); return false; }
    h_fourier_.assign(fw, fw + TD / 2);
    // the time conditioning MLP runs at load only; never quantized
    if (!lin(cond0_, 2 * TD, TD, false) || !lin(cond1_, TD, 2 * TD, false) || !lin(in_proj_, H, IN, int8)) {
        fail("head.bin too short");
        return false;
    }
    blocks_.resize(c.num_blocks);
    for (HeadBlock& b : blocks_) {
        b.ln_s = up(H);
        b.ln_b = up(H);
        if (!lin(b.d0, 4 * H, H, int8) || !lin(b.d1, H, 4 * H, int8)) { fail("head.bin too short"); return false; }
    }
    if (!lin(out_proj_, c.flat(), H, int8)) { fail("head.bin too short"); return false; }
    const float* betas = take(c.steps);
    const float* alphas = take(c.steps);
    const float* ahat = take(c.steps);
    if (!take.done()) { fail("head.bin size does not match head.meta"); return false; }
    for (int t = 0; t < c.steps; ++t)
        if (!(betas[t] > 0 && betas[t] < 1 && alphas[t] > 0 && alphas[t] < 1 && ahat[t] > 0 && ahat[t] < 1) ||
            (t && ahat[t] > ahat[t - 1])) {
            fail("invalid diffusion schedule in head.bin");
            return false;
        }
    // the per-step constants of DiffusionHead::denoise (diffusion_head.cpp:183-185), in float
    a1_.resize(c.steps);
    a2_.resize(c.steps);
    sb_.resize(c.steps);
    for (int t = 0; t < c.steps; ++t) {
        a1_[t] = 1.0f / std::sqrt(alphas[t]);
        a2_[t] = (1.0f - alphas[t]) / std::sqrt(1.0f - ahat[t]);
        sb_[t] = t > 0 ? std::sqrt(betas[t]) : 0.0f;
    }
    return err_.empty();
}

bool OctoPolicy::load_stats(const ModelFiles& files) {
    const size_t A = cfg_.action_dim;
    std::vector<float> mean, stdv, msk;
    auto rd = [&](const char* name, std::vector<float>& v) {
        if (!files.read_floats(name, v) || v.size() != A) return false;
        for (float f : v)
            if (!std::isfinite(f)) return false;
        return true;
    };
    if (!rd("stats_action_mean.bin", mean) || !rd("stats_action_std.bin", stdv) ||
        !rd("stats_action_mask.bin", msk)) {
        fail("cannot read the action stats");
        return false;
    }
    for (size_t i = 0; i < A; ++i)
        if (stdv[i] < 0 || (msk[i] != 0 && msk[i] != 1)) { fail("invalid action stats"); return false; }
    auto dev = [&](const std::vector<float>& v) {
        float* p = dalloc<float>(v.size());
        if (p) cudaMemcpy(p, v.data(), v.size() * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    d_act_mean_ = dev(mean);
    d_act_std_ = dev(stdv);
    d_act_mask_ = dev(msk);
    return err_.empty();
}

bool OctoPolicy::alloc_buffers() {
    const OctoConfigDev& c = cfg_;
    const int Bm = max_batch_, Wm = c.max_horizon;
    const long long F = (long long)Bm * Wm;
    if (F > kMaxConvFrames || F > 65535) { fail("max_batch x max window exceeds the frames one launch takes"); return false; }
    const int D = c.d, FL = c.flat(), T = c.total(Wm);
    const long long rows = (long long)Bm * T;
    const size_t pb = (size_t)stem_p_.in_hw * stem_p_.in_hw * 3, wb = (size_t)stem_w_.in_hw * stem_w_.in_hw * 3;

    // inputs: primary | wrist | tmask | slots | noise | z (one host-to-device copy each)
    size_t off = 0;
    auto place = [&](size_t bytes) {
        const size_t o = off;
        off = (off + bytes + 255) & ~size_t(255);
        return o;
    };
    const size_t o_p = place(F * pb), o_w = place(F * wb), o_t = place(F), o_s = place(sizeof(int) * Bm),
                 o_n = place(sizeof(float) * Bm * FL), o_z = place(sizeof(float) * (size_t)Bm * c.steps * FL);
    in_bytes_ = off;
    d_in_ = dalloc<uint8_t>(in_bytes_);
    if (!d_in_) return false;
    d_prim_u8_ = d_in_ + o_p;
    d_wrist_u8_ = d_in_ + o_w;
    d_tmask_ = d_in_ + o_t;
    d_slot_ = reinterpret_cast<int*>(d_in_ + o_s);
    d_noise_ = reinterpret_cast<float*>(d_in_ + o_n);
    d_z_ = reinterpret_cast<float*>(d_in_ + o_z);
    d_actions_ = dalloc<float>((size_t)Bm * FL);

    // stems: activations, GroupNorm affine, conv scratch, absmax slots
    size_t max_act = 0, col_i8 = 0, col_f = 0, crow = 0, max_gn = 0, qk = 0, qrows = 0;
    n_slots_ = 0;
    for (const OctoStemDev* s : {&stem_p_, &stem_w_}) {
        int h = s->in_hw;
        max_act = std::max(max_act, (size_t)F * h * h * 6);
        for (int i = 0; i < s->n_layers; ++i) {
            size_t a, b, r;
            conv_scratch_needs(s->conv[i], static_cast<int>(F), h, h, explicit_convs_, &a, &b, &r);
            col_i8 = std::max(col_i8, a);
            col_f = std::max(col_f, b);
            crow = std::max(crow, r);
            h = conv_out_size(h, s->k, s->stride, s->pad);
            max_act = std::max(max_act, (size_t)F * h * h * s->feat[i]);
            max_gn = std::max(max_gn, (size_t)F * s->feat[i]);
        }
        n_slots_ += (s->n_layers + 1) * static_cast<int>(F);
        qk = std::max(qk, (size_t)round16(s->feat.back()));
        qrows = std::max(qrows, (size_t)F * s->tokens());
    }
    d_stem_in_ = dalloc<float>(max_act);
    d_sa_ = dalloc<float>(max_act);
    d_sb_ = dalloc<float>(max_act);
    d_gnA_ = dalloc<float>(max_gn);
    d_gnB_ = dalloc<float>(max_gn);
    conv_s_.col = dalloc<int8_t>(col_i8);
    conv_s_.col_scale = dalloc<float>(crow);
    conv_s_.col_f = dalloc<float>(col_f);
    d_slots_ = dalloc<unsigned int>(n_slots_);
    d_ptok_ = dalloc<float>((size_t)F * stem_p_.tokens() * c.stem_dim);
    d_wtok_ = dalloc<float>((size_t)F * stem_w_.tokens() * c.stem_dim);
    d_pproj_ = dalloc<float>((size_t)F * stem_p_.tokens() * D);
    d_wproj_ = dalloc<float>((size_t)F * stem_w_.tokens() * D);

    // T5 scratch and cache (one instruction at a time, n_task tokens)
    const int n = c.n_task, TD5 = c.t5_dim;
    d_ids_ = dalloc<int>(n);
    d_bucket_ = dalloc<int>(2 * n - 1);
    d_t5x_ = dalloc<float>((size_t)n * TD5);
    d_t5h_ = dalloc<float>((size_t)n * TD5);
    d_t5q_ = dalloc<float>((size_t)n * TD5);
    d_t5k_ = dalloc<float>((size_t)n * TD5);
    d_t5v_ = dalloc<float>((size_t)n * TD5);
    d_t5a_ = dalloc<float>((size_t)n * TD5);
    d_t5ff_ = dalloc<float>((size_t)n * c.t5_ff);
    d_t5bias_ = dalloc<float>((size_t)c.t5_heads * n * n);
    d_t5cache_ = dalloc<float>((size_t)kT5CacheSlots * n * TD5);
    {
        std::vector<int> bk(2 * n - 1);
        for (int r = -(n - 1); r <= n - 1; ++r) bk[r + n - 1] = t5_bucket(r, c.t5_buckets, c.t5_max_dist);
        if (d_bucket_) cudaMemcpy(d_bucket_, bk.data(), sizeof(int) * bk.size(), cudaMemcpyHostToDevice);
    }

    // transformer
    d_t5in_ = dalloc<float>((size_t)Bm * n * TD5);
    d_task_ = dalloc<float>((size_t)Bm * n * D);
    d_x_ = dalloc<float>((size_t)rows * D);
    d_h_ = dalloc<float>((size_t)rows * D);
    d_qkv_ = dalloc<float>((size_t)rows * 3 * D);
    d_att_ = dalloc<float>((size_t)rows * D);
    d_ff_ = dalloc<float>((size_t)rows * c.mlp);
    d_mask_ = dalloc<float>((size_t)Bm * T * T);
    d_xr_ = dalloc<float>((size_t)Bm * D);
    d_emb_ = dalloc<float>((size_t)Bm * D);
    qk = std::max({qk, (size_t)round16(D), (size_t)round16(c.mlp), (size_t)round16(c.stem_dim),
                   (size_t)round16(TD5), (size_t)round16(c.time_dim + D + FL), (size_t)round16(4 * c.hidden)});
    qrows = std::max({qrows, (size_t)rows, (size_t)F * stem_w_.tokens(), (size_t)Bm * n});
    q_cap_ = qrows * qk;
    q_rows_ = qrows;
    d_q_ = dalloc<int8_t>(q_cap_);
    d_qs_ = dalloc<float>(qrows);
    d_att_cnt_ = dalloc<unsigned int>(kAttCounters);
    if (d_att_cnt_ && cudaMemset(d_att_cnt_, 0, sizeof(unsigned int) * kAttCounters) != cudaSuccess)
        fail("cudaMemset failed");

    // head
    d_cond_table_ = dalloc<float>((size_t)c.steps * c.time_dim);
    d_hin_ = dalloc<float>((size_t)Bm * (c.time_dim + D + FL));
    d_hh_ = dalloc<float>((size_t)Bm * c.hidden);
    d_hn_ = dalloc<float>((size_t)Bm * c.hidden);
    d_wide_ = dalloc<float>((size_t)Bm * 4 * c.hidden);
    d_eps_ = dalloc<float>((size_t)Bm * FL);
    d_sample_ = dalloc<float>((size_t)Bm * FL);
    return err_.empty();
}

// The time conditioning of every integer diffusion time (DiffusionHead::time_cond,
// diffusion_head.cpp:126-145): Fourier features with the host C library's
// cosf / sinf (the reference's own calls), then Dense -> swish -> Dense on the device.
bool OctoPolicy::time_cond() {
    const OctoConfigDev& c = cfg_;
    const int TD = c.time_dim, S = c.steps;
    std::vector<float> tff((size_t)S * TD);
    const float two_pi = 6.283185307179586f;
    for (int t = 0; t < S; ++t)
        for (int i = 0; i < TD / 2; ++i) {
            const float f = two_pi * static_cast<float>(t) * h_fourier_[i];
            tff[(size_t)t * TD + i] = std::cos(f);
            tff[(size_t)t * TD + TD / 2 + i] = std::sin(f);
        }
    float* d_tff = dalloc<float>(tff.size());
    float* d_c1 = dalloc<float>((size_t)S * 2 * TD);
    if (!d_tff || !d_c1) return false;
    cudaMemcpy(d_tff, tff.data(), sizeof(float) * tff.size(), cudaMemcpyHostToDevice);
    cudaError_t e = linear_f32(d_tff, TD, cond0_.W, cond0_.bias, d_c1, 2 * TD, S, 2 * TD, TD, nullptr, nullptr, stream_);
    if (e == cudaSuccess) e = silu_exact(d_c1, (long long)S * 2 * TD, stream_);
    if (e == cudaSuccess)
        e = linear_f32(d_c1, 2 * TD, cond1_.W, cond1_.bias, d_cond_table_, TD, S, TD, 2 * TD, nullptr, nullptr, stream_);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) { fail("time conditioning failed"); return false; }
    return true;
}

bool OctoPolicy::load(const std::string& dir, const std::string& tok_dir, int max_batch) {
    const int want_dev = env_int("VLA_CUDA_DEVICE", -1);
    if (want_dev >= 0 && cudaSetDevice(want_dev) != cudaSuccess) { fail("VLA_CUDA_DEVICE not usable"); return false; }
    cudaGetDevice(&device_);
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_);
    if (major != 10) { fail("needs an sm_100 (B200) device"); return false; }
    if (max_batch < 1) { fail("max_batch must be >= 1"); return false; }
    max_batch_ = max_batch;
    use_graph_ = env_int("VLA_CUDA_GRAPH", 1) != 0;
    explicit_convs_ = env_int("VLA_CONV_IM2COL", 0) != 0;
    i8_clip_ = env_clip();
    const int mask = env_int("OCTO_INT8", 0);

    // a converted directory or a vla.simd GGUF (src/models/octo/octo_model.cpp:60-62
    // mounts it before the tokenizer: a GGUF carries tok/)
    ModelFiles files;
    if (!files.open(dir)) { fail(files.error()); return false; }
    {
        std::string vocab;
        std::string rel;
        const std::string prefix = dir + "/";
        if (tok_dir.compare(0, prefix.size(), prefix) == 0) rel = tok_dir.substr(prefix.size()) + "/vocab.txt";
        const bool ok = rel.empty() ? ModelFiles::read_path(tok_dir + "/vocab.txt", vocab) : files.read(rel, vocab);
        if (!ok || !tok_.load_text(vocab)) { fail("cannot read the tokenizer's vocab.txt"); return false; }
    }
    if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess) { fail("stream"); return false; }
    if (!load_t5(files)) return false;
    if (!load_stem(files, "stem_primary", 256, (mask & 16) != 0, (mask & 8) != 0, stem_p_)) return false;
    if (!load_stem(files, "stem_wrist", 128, (mask & 16) != 0, (mask & 8) != 0, stem_w_)) return false;
    if (!load_transformer(files, mask)) return false;
    if (!load_head(files, (mask & 32) != 0)) return false;
    // the reference's shape agreement checks (octo_model.cpp:74-79)
    if (stem_p_.embed_dim != cfg_.stem_dim || stem_w_.embed_dim != cfg_.stem_dim ||
        stem_p_.tokens() != cfg_.tok_primary || stem_w_.tokens() != cfg_.tok_wrist) {
        fail("stems disagree with octo.meta");
        return false;
    }
    if (!load_stats(files)) return false;
    if (!alloc_buffers()) return false;
    if (mask) std::fprintf(stderr, "[octo] int8 GEMMs on device: %d (OCTO_INT8=%d)\n", n_int8_, mask);
    const int FL = cfg_.flat();
    if (cudaMallocHost(&h_pinned_, sizeof(float) * (size_t)max_batch_ * FL) != cudaSuccess ||
        cudaMallocHost(&h_noise_, sizeof(float) * (size_t)max_batch_ * (1 + cfg_.steps) * FL) != cudaSuccess ||
        cudaMallocHost(&h_slots_, sizeof(int) * (size_t)max_batch_) != cudaSuccess ||
        cudaMallocHost(&h_status_pinned_, sizeof(int)) != cudaSuccess) {
        fail("pinned host buffers");
        return false;
    }
    d_status_ = static_cast<int*>(device_status_address());
    if (!d_status_) { fail("device status word"); return false; }
    cudaMemset(d_in_, 0, in_bytes_);
    cudaDeviceSynchronize();
    if (!time_cond()) return false;
    // one eager batch validates every launch before capture (instruction "")
    cudaError_t e = set_instruction(0, "");
    if (e == cudaSuccess) {
        const uint8_t one = 1;
        e = cudaMemcpy(d_tmask_, &one, 1, cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = forward(1, 1, true, stream_, true);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) { fail(std::string("warm-up query failed: ") + cudaGetErrorString(e)); return false; }
    if (device_status_take() != 0) { fail("device status error in warm-up"); return false; }
    return true;
}

// ------------------------------------------------------------------ T5
// T5Encoder::encode (src/nn/t5_encoder.cpp:90-136): pre-RMSNorm blocks, fp32
// dense_linear projections (the exact-order fp32 linear), per-head-bias
// attention without scaling, ReLU FFN, final RMSNorm.
cudaError_t OctoPolicy::run_t5(const std::vector<int>& ids, float* out, cudaStream_t st) {
    const OctoConfigDev& c = cfg_;
    const int n = c.n_task, D = c.t5_dim, FF = c.t5_ff;
    VSB_TRY(cudaMemcpyAsync(d_ids_, ids.data(), sizeof(int) * n, cudaMemcpyHostToDevice, st));
    VSB_TRY(t5_embed(d_ids_, n, t5_emb_, c.t5_vocab, D, tok_.pad_id(), t5_rel_, d_bucket_, c.t5_heads, d_t5x_,
                     d_t5bias_, st));
    for (const T5LayerDev& L : t5_) {
        VSB_TRY(rmsnorm(d_t5x_, L.ln1, d_t5h_, n, D, c.t5_eps, st));
        VSB_TRY(linear_f32(d_t5h_, D, L.wq, nullptr, d_t5q_, D, n, D, D, nullptr, nullptr, st));
        VSB_TRY(linear_f32(d_t5h_, D, L.wk, nullptr, d_t5k_, D, n, D, D, nullptr, nullptr, st));
        VSB_TRY(linear_f32(d_t5h_, D, L.wv, nullptr, d_t5v_, D, n, D, D, nullptr, nullptr, st));
        VSB_TRY(t5_attention(d_t5q_, d_t5k_, d_t5v_, d_t5bias_, n, c.t5_heads, c.t5_dkv, 1.0f, d_t5a_, st));
        VSB_TRY(linear_f32(d_t5a_, D, L.wo, nullptr, d_t5h_, D, n, D, D, nullptr, nullptr, st));
        VSB_TRY(add_f32(d_t5x_, d_t5h_, d_t5x_, (long long)n * D, st));
        VSB_TRY(rmsnorm(d_t5x_, L.ln2, d_t5h_, n, D, c.t5_eps, st));
        VSB_TRY(linear_f32(d_t5h_, D, L.wi, nullptr, d_t5ff_, FF, n, FF, D, nullptr, nullptr, st));
        VSB_TRY(activation(kActRelu, d_t5ff_, d_t5ff_, nullptr, (long long)n * FF, st));
        VSB_TRY(linear_f32(d_t5ff_, FF, L.wo2, nullptr, d_t5h_, D, n, D, FF, nullptr, nullptr, st));
        VSB_TRY(add_f32(d_t5x_, d_t5h_, d_t5x_, (long long)n * D, st));
    }
    return rmsnorm(d_t5x_, t5_final_, out, n, D, c.t5_eps, st);
}

// The cache slot of an instruction's T5 encoding, encoding it first when it
// is new; the cache is emptied when full (octo_model.cpp:149-164).
int OctoPolicy::t5_slot(const std::string& instruction, cudaStream_t st, cudaError_t* err) {
    *err = cudaSuccess;
    const auto it = t5_slots_.find(instruction);
    if (it != t5_slots_.end()) return it->second;
    if (static_cast<int>(t5_slots_.size()) >= kT5CacheSlots) t5_slots_.clear();
    const int slot = static_cast<int>(t5_slots_.size());
    const std::vector<int> ids = tok_.encode(instruction, cfg_.n_task);
    *err = run_t5(ids, d_t5cache_ + (size_t)slot * cfg_.n_task * cfg_.t5_dim, st);
    if (*err == cudaSuccess) *err = cudaStreamSynchronize(st);   // ids staging is reused
    if (*err != cudaSuccess) return -1;
    ++t5_runs_;
    t5_slots_.emplace(instruction, slot);
    return slot;
}

cudaError_t OctoPolicy::set_instruction(int b, const char* instruction) {
    if (b < 0 || b >= max_batch_ || !instruction) return cudaErrorInvalidValue;
    cudaError_t e;
    const int slot = t5_slot(instruction, stream_, &e);
    if (e != cudaSuccess) return e;
    VSB_TRY(cudaMemcpyAsync(d_slot_ + b, &slot, sizeof(int), cudaMemcpyHostToDevice, stream_));
    return cudaStreamSynchronize(stream_);
}

// ------------------------------------------------------------- layers
// int8 layers: quantize_act_i8 of each row of x, then the W8A8 GEMM
// (nn::Linear::forward, src/nn/linear.cpp:121-133); fp32 layers: the fp32 GEMM.
// The int8 row copy (d_q_ / d_qs_) of an attention output of `rows` rows of K
// columns, written by the attention launch itself (nn.h AttQuant); sequences
// of seq_rows rows each. Null q when the scratch cannot hold it.
AttQuant OctoPolicy::att_quant(int rows, int K, int seq_rows) const {
    AttQuant a;
    const long long ldq = round16(K);
    if ((size_t)rows > q_rows_ || (size_t)rows * ldq > q_cap_) return a;
    a.q = d_q_;
    a.ldq = ldq;
    a.scale = d_qs_;
    a.counters = d_att_cnt_;
    a.n_counters = kAttCounters;
    a.zq = (long long)seq_rows * ldq;
    a.zs = seq_rows;
    return a;
}

cudaError_t OctoPolicy::linear(const DevLinear& l, const float* x, long long ldx, int M, float* out, long long ldo,
                               int mode, const float* res, long long ldr, cudaStream_t st) {
    if (l.int8) {
        if ((size_t)M * round16(l.K) > q_cap_) return cudaErrorInvalidValue;
        VSB_TRY(quantize_rows(x, ldx, nullptr, 0, M, l.K, d_q_, round16(l.K), d_qs_, nullptr, 0, nullptr, st));
    }
    return linear_q(l, d_q_, d_qs_, x, ldx, M, out, ldo, mode, res, ldr, st);
}

cudaError_t OctoPolicy::linear_q(const DevLinear& l, const int8_t* q, const float* qs, const float* x, long long ldx,
                                 int M, float* out, long long ldo, int mode, const float* res, long long ldr,
                                 cudaStream_t st) {
    if (l.int8) {
        GemmI8Args a;
        a.A = q;
        a.lda = round16(l.K);
        a.B = l.Wq;
        a.ldb = l.ldw;
        a.M = M;
        a.N = l.N;
        a.K = l.K;
        a.out = out;
        a.ldo = ldo;
        a.ascale = qs;
        a.wscale = l.wscale;
        a.bias = l.bias;
        a.res = res;
        a.ldr = ldr;
        a.mode = mode;
        a.static_weights = true;   // uploaded once at load
        return gemm_i8(a, st);
    }
    return gemm_f32(x, ldx, l.W, l.K, l.bias, out, ldo, res, ldr, M, l.N, l.K, mode, nullptr, 1, st);
}

// SmallStem::encode over F frames (src/models/octo/small_stem.cpp:86-141): the
// 6-channel input, n x (conv -> GroupNorm + ReLU), then the 1x1 embedding.
cudaError_t OctoPolicy::run_stem(const OctoStemDev& s, const uint8_t* img, int F, float* tokens, cudaStream_t st) {
    unsigned int* slot = d_slots_ + (&s == &stem_w_ ? (stem_p_.n_layers + 1) * (long long)max_batch_ * cfg_.max_horizon : 0);
    VSB_TRY(octo_stem_input(img, F, (long long)s.in_hw * s.in_hw, d_stem_in_, slot, st));
    const float* in = d_stem_in_;
    float* bufs[2] = {d_sa_, d_sb_};
    int h = s.in_hw;
    for (int i = 0; i < s.n_layers; ++i) {
        float* out = bufs[i & 1];
        unsigned int* next = slot + (long long)F * (i + 1);
        VSB_TRY(conv2d_dev(s.conv[i], in, F, h, h, out, 0, nullptr, slot + (long long)F * i, nullptr, i8_clip_,
                           explicit_convs_, conv_s_, st));
        h = conv_out_size(h, s.k, s.stride, s.pad);
        const int C = s.feat[i];
        VSB_TRY(gn_affine(out, F, h * h, C, C, s.gn_groups, s.gn_eps, s.gn_s[i], s.gn_b[i], d_gnA_, d_gnB_,
                          st));
        VSB_TRY(gn_apply(out, d_gnA_, d_gnB_, out, F, h * h, C, C, kGnRelu, nullptr, next, st));
        in = out;
    }
    const int C = s.feat.back();
    return linear(s.embed, in, C, F * h * h, tokens, s.embed_dim, 0, nullptr, 0, st);
}

// ------------------------------------------------------------ forward
cudaError_t OctoPolicy::forward(int B, int wnd, bool wrist, cudaStream_t st, bool unnormalize) {
    const OctoConfigDev& c = cfg_;
    const int D = c.d, T = c.total(wnd), F = B * wnd;
    const int ro = c.n_task + wnd * c.per_step() - 1;   // the last step's readout row (octo_transformer.h:61)
    const long long rows = (long long)B * T;
    VSB_TRY(cudaMemsetAsync(d_slots_, 0, sizeof(unsigned int) * n_slots_, st));

    // observation tokens (SmallStem + projection; the frame cache of the
    // reference changes no values, every frame is encoded)
    VSB_TRY(run_stem(stem_p_, d_prim_u8_, F, d_ptok_, st));
    VSB_TRY(linear(proj_prim_, d_ptok_, c.stem_dim, F * c.tok_primary, d_pproj_, D, 0, nullptr, 0, st));
    if (wrist) {
        VSB_TRY(run_stem(stem_w_, d_wrist_u8_, F, d_wtok_, st));
        VSB_TRY(linear(proj_wrist_, d_wtok_, c.stem_dim, F * c.tok_wrist, d_wproj_, D, 0, nullptr, 0, st));
    }
    // task tokens: cached T5 encodings of each query's instruction, projected
    VSB_TRY(gather_rows(d_t5cache_, d_slot_, B, (long long)c.n_task * c.t5_dim, d_t5in_, st));
    VSB_TRY(linear(proj_task_, d_t5in_, c.t5_dim, B * c.n_task, d_task_, D, 0, nullptr, 0, st));
    const OctoSeq seq{B, wnd, c.n_task, c.tok_primary, c.tok_wrist, c.n_readout, D};
    VSB_TRY(octo_assemble(seq, d_task_, pos_task_, d_pproj_, pos_prim_, wrist ? d_wproj_ : nullptr, pos_wrist_,
                          pos_readout_, d_x_, st));
    VSB_TRY(octo_mask(seq, d_tmask_, wrist, d_mask_, st));

    // encoder blocks (pre-LN, masked MHA, gelu MLP; octo_transformer.cpp:205-211,
    // src/nn/encoder.cpp:25-78)
    const float scale = 1.0f / std::sqrt(static_cast<float>(c.head_dim));
    const int act = c.gelu_erf ? kActGeluErf : kActGeluTanh;
    const long long ldq = round16(D);
    for (int li = 0; li < c.n_layers; ++li) {
        const OctoLayerDev& L = layers_[li];
        const bool last = li + 1 == c.n_layers;
        VSB_TRY(layernorm(d_x_, d_h_, L.ln1s, L.ln1b, static_cast<int>(rows), D, c.ln_eps, nullptr,
                          L.wqkv.int8 ? d_q_ : nullptr, L.wqkv.int8 ? d_qs_ : nullptr, nullptr, nullptr, ldq, st));
        VSB_TRY(linear_q(L.wqkv, d_q_, d_qs_, d_h_, D, static_cast<int>(rows), d_qkv_, 3 * D, 0, nullptr, 0, st));
        AttBatch bs;
        bs.n = B;
        bs.q = bs.k = bs.v = (long long)T * 3 * D;
        bs.mask = (long long)T * T;
        if (!last) {
            bs.o = (long long)T * D;
            // the o-projection's int8 input comes out of the attention launch
            const AttQuant aq = att_quant(static_cast<int>(rows), D, T);
            if (L.wo.int8 && !aq.q) return cudaErrorInvalidValue;
            VSB_TRY(attention_batched(d_qkv_, 3 * D, d_qkv_ + D, 3 * D, d_qkv_ + 2 * D, 3 * D, d_att_, D, T, T, c.heads,
                                      c.heads, c.head_dim, scale, d_mask_, bs, st, L.wo.int8 ? &aq : nullptr));
            VSB_TRY(linear_q(L.wo, d_q_, d_qs_, d_att_, D, static_cast<int>(rows), d_x_, D, kEpiAdd, d_x_, D, st));
            VSB_TRY(layernorm(d_x_, d_h_, L.ln2s, L.ln2b, static_cast<int>(rows), D, c.ln_eps, nullptr,
                              L.w1.int8 ? d_q_ : nullptr, L.w1.int8 ? d_qs_ : nullptr, nullptr, nullptr, ldq, st));
            VSB_TRY(linear_q(L.w1, d_q_, d_qs_, d_h_, D, static_cast<int>(rows), d_ff_, c.mlp, 0, nullptr, 0, st));
            VSB_TRY(mlp_out(L, act, static_cast<int>(rows), d_x_, st));
        } else {
            // readout-only final layer (EncoderLayer::forward_last_row,
            // src/nn/encoder.cpp:80-111): K/V of every token, the rest for row ro
            bs.o = D;
            const AttQuant aq = att_quant(B, D, 1);
            if (L.wo.int8 && !aq.q) return cudaErrorInvalidValue;
            VSB_TRY(attention_batched(d_qkv_ + (long long)ro * 3 * D, 3 * D, d_qkv_ + D, 3 * D, d_qkv_ + 2 * D, 3 * D,
                                      d_att_, D, 1, T, c.heads, c.heads, c.head_dim, scale,
                                      d_mask_ + (long long)ro * T, bs, st, L.wo.int8 ? &aq : nullptr));
            VSB_TRY(linear_q(L.wo, d_q_, d_qs_, d_att_, D, B, d_xr_, D, kEpiAdd, d_x_ + (long long)ro * D,
                             (long long)T * D, st));
            VSB_TRY(layernorm(d_xr_, d_h_, L.ln2s, L.ln2b, B, D, c.ln_eps, nullptr, L.w1.int8 ? d_q_ : nullptr,
                              L.w1.int8 ? d_qs_ : nullptr, nullptr, nullptr, ldq, st));
            VSB_TRY(linear_q(L.w1, d_q_, d_qs_, d_h_, D, B, d_ff_, c.mlp, 0, nullptr, 0, st));
            VSB_TRY(mlp_out(L, act, B, d_xr_, st));
        }
    }
    VSB_TRY(layernorm(d_xr_, d_emb_, final_s_, final_b_, B, D, c.ln_eps, nullptr, nullptr, nullptr, nullptr, nullptr,
                      0, st));

    // DDPM over the score network (DiffusionHead::denoise, diffusion_head.cpp:172-191;
    // nn::DiffusionMlp::forward, src/nn/diffusion.cpp:15-36)
    return run_head(B, st, unnormalize);
}

// The MLP's second half of M rows: gelu(ff) -> w2 -> x += . (src/nn/encoder.cpp:62-77).
// An int8 w2 takes gelu and its row quantization in one pass.
cudaError_t OctoPolicy::mlp_out(const OctoLayerDev& L, int act, int M, float* x, cudaStream_t st) {
    const OctoConfigDev& c = cfg_;
    if (L.w2.int8) {
        VSB_TRY(act_rows_q(act, d_ff_, M, c.mlp, false, d_q_, round16(c.mlp), d_qs_, st));
        return linear_q(L.w2, d_q_, d_qs_, nullptr, 0, M, x, c.d, kEpiAdd, x, c.d, st);
    }
    VSB_TRY(activation(act, d_ff_, d_ff_, nullptr, (long long)M * c.mlp, st));
    return linear(L.w2, d_ff_, c.mlp, M, x, c.d, kEpiAdd, x, c.d, st);
}

// The diffusion head of B queries: per step in_proj -> blocks (LN -> d0 ->
// silu -> d1, residual) -> the fused tail (silu, out_proj, DDPM update, next
// input row and its quantization).
cudaError_t OctoPolicy::run_head(int B, cudaStream_t st, bool unnormalize) {
    const OctoConfigDev& c = cfg_;
    const int D = c.d, FL = c.flat(), TD = c.time_dim, H = c.hidden, IN = TD + D + FL;
    const bool fused_tail = !out_proj_.int8;   // the fp32 out_proj of a flat size that is not a multiple of 16
    auto dense = [&](const DevLinear& l, const float* x, int K, float* out, int mode, const float* res) -> cudaError_t {
        if (l.int8) return linear(l, x, K, B, out, l.N, mode, res, l.N, st);
        // fp32 score-net layers are the reference's plain dense_linear (Role::Generic)
        VSB_TRY(linear_f32(x, K, l.W, l.bias, mode == kEpiAdd ? d_hn_ : out, l.N, B, l.N, K, nullptr, nullptr, st));
        if (mode == kEpiAdd) return add_f32(res, d_hn_, out, (long long)B * l.N, st);
        return cudaSuccess;
    };
    auto input_row = [&](const float* h, const float* z, int t, int t_next) -> cudaError_t {
        OctoHeadTail a;
        a.B = B;
        a.H = H;
        a.FL = FL;
        a.TD = TD;
        a.E = D;
        a.h = h;
        a.x0 = h ? nullptr : d_noise_;
        a.W = out_proj_.W;
        a.bias = out_proj_.bias;
        a.sample = d_sample_;
        a.z = z;
        a.z_stride = (long long)c.steps * FL;
        if (t >= 0) {
            a.a1 = a1_[t];
            a.a2 = a2_[t];
            a.sb = sb_[t];
        }
        a.max_action = c.max_action;
        a.cond_next = t_next >= 0 ? d_cond_table_ + (size_t)t_next * TD : nullptr;
        a.emb = d_emb_;
        if (in_proj_.int8) {
            a.q = d_q_;
            a.ldq = round16(IN);
            a.qscale = d_qs_;
        } else {
            a.in_f32 = d_hin_;
        }
        return octo_head_tail(a, st);
    };
    if (fused_tail) {
        VSB_TRY(input_row(nullptr, nullptr, -1, c.steps - 1));
    } else {
        VSB_TRY(cudaMemcpyAsync(d_sample_, d_noise_, sizeof(float) * (size_t)B * FL, cudaMemcpyDeviceToDevice, st));
    }
    for (int s = 0; s < c.steps; ++s) {
        const int t = c.steps - 1 - s;
        if (fused_tail) {
            if (in_proj_.int8) VSB_TRY(linear_q(in_proj_, d_q_, d_qs_, nullptr, 0, B, d_hh_, H, 0, nullptr, 0, st));
            else VSB_TRY(dense(in_proj_, d_hin_, IN, d_hh_, 0, nullptr));
        } else {
            VSB_TRY(octo_head_input(d_cond_table_ + (size_t)t * TD, TD, d_emb_, D, d_sample_, FL, B, d_hin_, st));
            VSB_TRY(dense(in_proj_, d_hin_, IN, d_hh_, 0, nullptr));
        }
        for (const HeadBlock& hb : blocks_) {
            VSB_TRY(layernorm(d_hh_, d_hn_, hb.ln_s, hb.ln_b, B, H, 1e-6f, nullptr, hb.d0.int8 ? d_q_ : nullptr,
                              hb.d0.int8 ? d_qs_ : nullptr, nullptr, nullptr, round16(H), st));
            if (hb.d0.int8) VSB_TRY(linear_q(hb.d0, d_q_, d_qs_, nullptr, 0, B, d_wide_, 4 * H, 0, nullptr, 0, st));
            else VSB_TRY(dense(hb.d0, d_hn_, H, d_wide_, 0, nullptr));
            if (hb.d1.int8) {
                VSB_TRY(act_rows_q(kActSiluLibm, d_wide_, B, 4 * H, false, d_q_, round16(4 * H), d_qs_, st));
                VSB_TRY(linear_q(hb.d1, d_q_, d_qs_, nullptr, 0, B, d_hh_, H, kEpiAdd, d_hh_, H, st));
            } else {
                VSB_TRY(silu_exact(d_wide_, (long long)B * 4 * H, st));
                VSB_TRY(dense(hb.d1, d_wide_, 4 * H, d_hh_, kEpiAdd, d_hh_));
            }
        }
        if (fused_tail) {
            VSB_TRY(input_row(d_hh_, d_z_ + (size_t)s * FL, t, t > 0 ? t - 1 : -1));
        } else {
            VSB_TRY(silu_exact(d_hh_, (long long)B * H, st));
            VSB_TRY(dense(out_proj_, d_hh_, H, d_eps_, 0, nullptr));
            VSB_TRY(octo_ddpm_step(d_sample_, d_eps_, d_z_ + (size_t)s * FL, (long long)c.steps * FL, B, FL, a1_[t],
                                   a2_[t], sb_[t], c.max_action, st));
        }
    }
    return octo_actions(d_sample_, B, FL, c.action_dim, d_act_mean_, d_act_std_, d_act_mask_, unnormalize,
                        d_actions_, st);
}

cudaError_t OctoPolicy::enqueue(int B, int wnd, bool wrist, cudaStream_t st, bool unnormalize) {
    if (B < 1 || B > max_batch_ || wnd < 1 || wnd > cfg_.max_horizon) return cudaErrorInvalidValue;
    last_batch_ = B;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device_) cudaSetDevice(device_);
    cudaError_t e = cudaSuccess;
    if (!use_graph_) {
        e = forward(B, wnd, wrist, st, unnormalize);
    } else {
        const long long key = (((long long)B * 64 + wnd) * 2 + (wrist ? 1 : 0)) * 2 + (unnormalize ? 1 : 0);
        cudaGraphExec_t& g = graphs_[key];
        if (!g) {
            cudaGraph_t gr = nullptr;
            e = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal);
            if (e == cudaSuccess) {
                const cudaError_t fe = forward(B, wnd, wrist, stream_, unnormalize);
                const cudaError_t ce = cudaStreamEndCapture(stream_, &gr);
                e = fe != cudaSuccess ? fe : ce;
            }
            if (e == cudaSuccess) {
                size_t n_nodes = 0;
                cudaGraphGetNodes(gr, nullptr, &n_nodes);
                std::vector<cudaGraphNode_t> nodes(n_nodes);
                cudaGraphGetNodes(gr, nodes.data(), &n_nodes);
                int nk = 0;
                for (cudaGraphNode_t nd : nodes) {
                    cudaGraphNodeType t;
                    if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) nk++;
                }
                kernels_per_step_ = nk;
                e = cudaGraphInstantiate(&g, gr, 0);
            }
            if (gr) cudaGraphDestroy(gr);
            if (e != cudaSuccess) g = nullptr;
        }
        if (e == cudaSuccess) e = cudaGraphLaunch(g, st);
    }
    if (prev != device_) cudaSetDevice(prev);
    return e;
}

cudaError_t OctoPolicy::predict(int B, const uint8_t* primary, const uint8_t* wrist, int wnd, const uint8_t* tmask,
                                const char* const* instructions, const float* noise, const float* z,
                                const uint64_t* seeds, bool unnormalize, float* actions) {
    if (B < 1 || B > max_batch_ || wnd < 1 || wnd > cfg_.max_horizon || !primary || !tmask || !instructions ||
        !actions || (noise == nullptr) != (z == nullptr) || (!noise && !seeds))
        return cudaErrorInvalidValue;
    for (int b = 0; b < B; ++b)
        if (!instructions[b]) return cudaErrorInvalidValue;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device_) cudaSetDevice(device_);
    const cudaError_t e0 = [&]() -> cudaError_t {
        const OctoConfigDev& c = cfg_;
        const int FL = c.flat();
        for (int b = 0; b < B; ++b) {
            cudaError_t e;
            h_slots_[b] = t5_slot(instructions[b], stream_, &e);
            if (e != cudaSuccess) return e;
        }
        const size_t pb = (size_t)stem_p_.in_hw * stem_p_.in_hw * 3, wb = (size_t)stem_w_.in_hw * stem_w_.in_hw * 3;
        VSB_TRY(cudaMemcpyAsync(d_prim_u8_, primary, (size_t)B * wnd * pb, cudaMemcpyHostToDevice, stream_));
        if (wrist) VSB_TRY(cudaMemcpyAsync(d_wrist_u8_, wrist, (size_t)B * wnd * wb, cudaMemcpyHostToDevice, stream_));
        VSB_TRY(cudaMemcpyAsync(d_tmask_, tmask, (size_t)B * wnd, cudaMemcpyHostToDevice, stream_));
        VSB_TRY(cudaMemcpyAsync(d_slot_, h_slots_, sizeof(int) * B, cudaMemcpyHostToDevice, stream_));
        if (noise) {
            VSB_TRY(cudaMemcpyAsync(d_noise_, noise, sizeof(float) * (size_t)B * FL, cudaMemcpyHostToDevice, stream_));
            VSB_TRY(cudaMemcpyAsync(d_z_, z, sizeof(float) * (size_t)B * c.steps * FL, cudaMemcpyHostToDevice, stream_));
        } else {
            // the reference's draw (octo_model.cpp:198-210): initial x, then every step's z
            float* hn = h_noise_;
            float* hz = h_noise_ + (size_t)B * FL;
            for (int b = 0; b < B; ++b) {
                PolarNormal N(seeds[b]);
                for (int i = 0; i < FL; ++i) hn[(size_t)b * FL + i] = N();
                for (int i = 0; i < c.steps * FL; ++i) hz[(size_t)b * c.steps * FL + i] = N();
            }
            VSB_TRY(cudaMemcpyAsync(d_noise_, hn, sizeof(float) * (size_t)B * FL, cudaMemcpyHostToDevice, stream_));
            VSB_TRY(cudaMemcpyAsync(d_z_, hz, sizeof(float) * (size_t)B * c.steps * FL, cudaMemcpyHostToDevice,
                                    stream_));
        }
        VSB_TRY(enqueue(B, wnd, wrist != nullptr, stream_, unnormalize));
        VSB_TRY(cudaMemcpyAsync(h_pinned_, d_actions_, sizeof(float) * (size_t)B * FL, cudaMemcpyDeviceToHost, stream_));
        VSB_TRY(cudaMemcpyAsync(h_status_pinned_, d_status_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        VSB_TRY(cudaStreamSynchronize(stream_));
        if (*h_status_pinned_ != 0) {
            device_status_take();
            return cudaErrorLaunchFailure;
        }
        std::memcpy(actions, h_pinned_, sizeof(float) * (size_t)B * FL);
        return cudaSuccess;
    }();
    if (prev != device_) cudaSetDevice(prev);
    return e0;
}

long long OctoPolicy::readout(float* out, long long cap) {
    const long long n = (long long)last_batch_ * cfg_.d;
    if (!out || n <= 0 || n > cap) return -1;
    cudaSetDevice(device_);
    if (cudaMemcpy(out, d_emb_, sizeof(float) * n, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return n;
}

}  // namespace vsb
