// ACT policy runtime (see act_policy.h). Host code only: parsing, int8 packing,
// buffer planning, and the kernel sequence of one step.
#include "act_policy.h"

#include "host_util.h"

#include "model_files.h"

#include "f32.h"
#include "gemm_i8.h"
#include "host_quant.h"
#include "nn.h"
#include "quant.h"

#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>

namespace vsb {

namespace {

using host::Cursor;
using host::env_clip;
using host::env_int;
using host::round16;
using host::shape_fits;

int conv_out(int in, int k, int stride, int pad) {
    const long long num = (long long)in + 2LL * pad - k;
    if (in <= 0 || stride <= 0 || num < 0) return 0;
    return static_cast<int>(num / stride + 1);
}


#define VSB_TRY(expr)                                  \
    do {                                               \
        const cudaError_t e_ = (expr);                 \
        if (e_ != cudaSuccess) return e_;              \
    } while (0)

}  // namespace

template <class T>
T* ActPolicy::dalloc(size_t n) {
    void* p = nullptr;
    if (n == 0) n = 1;
    if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
        fail("cudaMalloc failed");
        return nullptr;
    }
    allocs_.push_back(p);
    return static_cast<T*>(p);
}

ActPolicy::~ActPolicy() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device_);
    for (auto& g : graph_)
        if (g) cudaGraphExecDestroy(g);
    if (stream_) cudaStreamDestroy(stream_);
    if (side_) cudaStreamDestroy(side_);
    if (ev_fork_) cudaEventDestroy(ev_fork_);
    if (ev_join_) cudaEventDestroy(ev_join_);
    for (void* p : allocs_) cudaFree(p);
    if (h_state_pinned_) cudaFreeHost(h_state_pinned_);
    if (h_actions_pinned_) cudaFreeHost(h_actions_pinned_);
    if (h_status_pinned_) cudaFreeHost(h_status_pinned_);
    cudaSetDevice(prev);
}

bool ActPolicy::upload_linear(DevLinear& l, const float* W, const float* b, int N, int K, bool int8) {
    return vsb::upload_linear(l, W, b, N, K, int8, [this](size_t n) -> void* { return dalloc<char>(n); }, &n_int8_);
}

bool ActPolicy::load_config(const ModelFiles& files) {
    std::string text;
    if (!files.read("config.txt", text)) { fail("cannot open config.txt"); return false; }
    std::istringstream f(text);
    std::string line;
    while (std::getline(f, line)) {
        std::istringstream ss(line);
        std::string key;
        if (!(ss >> key)) continue;
        if (key == "img_h") ss >> img_h_;
        else if (key == "img_w") ss >> img_w_;
        else if (key == "n_cams") ss >> n_cams_;
        else if (key == "norm_eps") ss >> norm_eps_;
        else if (key.rfind("cam", 0) == 0) { std::string name; ss >> name; }
        else continue;
        if (ss.fail() || !(ss >> std::ws).eof()) { fail("malformed config.txt"); return false; }
    }
    if (!shape_fits({img_h_, img_w_, n_cams_, 3}) || !std::isfinite(norm_eps_) || norm_eps_ <= 0) {
        fail("bad config.txt values");
        return false;
    }
    if (n_cams_ > 8) {   // the conv kernels batch the cameras as up to 8 frames
        fail("more than 8 cameras");
        return false;
    }
    return true;
}

bool ActPolicy::load_backbone(const ModelFiles& files, bool int8) {
    std::string meta_text;
    if (!files.read("backbone.meta", meta_text)) { fail("cannot open backbone.meta"); return false; }
    std::istringstream meta(meta_text);
    struct BM { int cin, cout, stride, has_down; };
    std::vector<BM> bm;
    int in_ch = 3, gn = 0;
    std::string line;
    while (std::getline(meta, line)) {
        std::istringstream ss(line);
        std::string key;
        if (!(ss >> key)) continue;
        if (key == "in_ch") ss >> in_ch;
        else if (key == "stem_out") ss >> stem_out_;
        else if (key == "stem_k") ss >> stem_k_;
        else if (key == "stem_stride") ss >> stem_stride_;
        else if (key == "stem_pad") ss >> stem_pad_;
        else if (key == "pool_k") ss >> pool_k_;
        else if (key == "pool_stride") ss >> pool_stride_;
        else if (key == "pool_pad") ss >> pool_pad_;
        else if (key == "gn_group_size") ss >> gn;
        else if (key == "block") { BM b{}; ss >> b.cin >> b.cout >> b.stride >> b.has_down; bm.push_back(b); }
        else if (key == "film_after") { int i; ss >> i; fail("FiLM backbones are not supported"); return false; }
        else continue;
        if (ss.fail() || !(ss >> std::ws).eof()) { fail("malformed backbone.meta"); return false; }
    }
    if (in_ch != 3 || gn != 0 || !shape_fits({stem_out_, stem_k_, stem_k_, in_ch}) || stem_stride_ < 1 ||
        stem_pad_ < 0 || pool_k_ < 1 || pool_stride_ < 1 || pool_pad_ < 0) {
        fail("unsupported backbone.meta");
        return false;
    }
    std::vector<float> data;
    if (!files.read_floats("backbone.bin", data)) { fail("cannot read backbone.bin"); return false; }
    Cursor take{data};
    // ACT_I8_CONV_FROM / ACT_I8_CONV_TO (src/models/act/act_model.cpp:57-65,
    // src/models/act/resnet_backbone.cpp:171-188): stage 0 = stem, i+1 = block i.
    const int from = env_int("ACT_I8_CONV_FROM", 0);
    int to = env_int("ACT_I8_CONV_TO", -1);
    if (to < 0) to = static_cast<int>(bm.size()) + 1;
    auto want = [&](int stage) { return int8 && stage >= from && stage < to; };

    auto make_conv = [&](DevConv& c, int cout, int k, int cin, int stride, int pad, bool q) -> bool {
        const float* w = take((size_t)cout * k * k * cin);
        const float* b = take(cout);
        if (!take.ok) { fail("backbone.bin too short"); return false; }
        return make_dev_conv(c, w, b, cout, k, cin, stride, pad, q,
                             [this](size_t n) -> void* { return dalloc<char>(n); }, &n_int8_);
    };
    if (!make_conv(stem_, stem_out_, stem_k_, in_ch, stem_stride_, stem_pad_, want(0))) return false;
    blocks_.resize(bm.size());
    int prev = stem_out_;
    for (size_t i = 0; i < bm.size(); ++i) {
        DevBlock& blk = blocks_[i];
        if (bm[i].cin != prev || bm[i].cout < 1 || bm[i].stride < 1 || (bm[i].has_down != 0 && bm[i].has_down != 1)) {
            fail("inconsistent backbone block table");
            return false;
        }
        if (!bm[i].has_down && (bm[i].stride != 1 || bm[i].cin != bm[i].cout)) {
            fail("block without downsample changes shape");
            return false;
        }
        blk.has_down = bm[i].has_down != 0;
        const bool q = want(static_cast<int>(i) + 1);
        if (!make_conv(blk.conv1, bm[i].cout, 3, bm[i].cin, bm[i].stride, 1, q)) return false;
        if (!make_conv(blk.conv2, bm[i].cout, 3, bm[i].cout, 1, 1, q)) return false;
        if (blk.has_down && !make_conv(blk.down, bm[i].cout, 1, bm[i].cin, bm[i].stride, 0, q)) return false;
        prev = bm[i].cout;
    }
    if (!take.done()) { fail("backbone.bin size does not match backbone.meta"); return false; }
    return true;
}

bool ActPolicy::load_transformer(const ModelFiles& files, int mask) {
    std::string meta_text;
    if (!files.read("act.meta", meta_text)) { fail("cannot open act.meta"); return false; }
    std::istringstream meta(meta_text);
    std::string line;
    ActConfigDev& c = cfg_;
    while (std::getline(meta, line)) {
        std::istringstream ss(line);
        std::string key;
        if (!(ss >> key)) continue;
        if (key == "dim") ss >> c.dim;
        else if (key == "heads") ss >> c.heads;
        else if (key == "head_dim") ss >> c.head_dim;
        else if (key == "ff") ss >> c.ff;
        else if (key == "n_enc") ss >> c.n_enc;
        else if (key == "n_dec") ss >> c.n_dec;
        else if (key == "chunk") ss >> c.chunk;
        else if (key == "state_dim") ss >> c.state_dim;
        else if (key == "action_dim") ss >> c.action_dim;
        else if (key == "n_1d") ss >> c.n_1d;
        else if (key == "n_text") ss >> c.n_text;
        else if (key == "ln_eps") ss >> c.ln_eps;
        else continue;
        if (ss.fail() || !(ss >> std::ws).eof()) { fail("malformed act.meta"); return false; }
    }
    const int img_ch = blocks_.empty() ? stem_out_ : blocks_.back().conv1.cout;
    if (!shape_fits({c.dim, c.dim}) || c.dim % 4 || c.heads * c.head_dim != c.dim || c.head_dim != 64 ||
        !shape_fits({c.ff, c.dim}) || !shape_fits({c.chunk, c.dim}) || !shape_fits({c.state_dim, c.dim}) ||
        !shape_fits({c.action_dim, c.dim}) || !shape_fits({img_ch, c.dim}) || c.n_enc < 1 || c.n_dec < 1 ||
        c.n_1d != 2 || c.n_text != 0 || !std::isfinite(c.ln_eps) || c.ln_eps <= 0) {
        fail("unsupported act.meta (head_dim 64, no text tokens)");
        return false;
    }
    std::vector<float> data;
    if (!files.read_floats("act.bin", data)) { fail("cannot read act.bin"); return false; }
    Cursor take{data};
    const int d = c.dim;
    // bits of ACT_INT8 (src/models/act/act_transformer.cpp:23-27)
    const bool q_attn = mask & 1, q_w1 = mask & 2, q_w2 = mask & 4, q_img = mask & 8, q_dec = mask & 16;
    struct Raw { const float* w; const float* b; };
    auto raw = [&](int N, int K) -> Raw {
        const float* w = take((size_t)N * K);
        const float* b = take(N);
        return {w, b};
    };
    auto dev_copy = [&](const float* src, size_t n) -> float* {
        float* p = dalloc<float>(n);
        if (p && src) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    // stacked [wq; wk] -> one [2d, d] layer
    auto stack_qk = [&](DevLinear& l, Raw q, Raw k, bool int8) -> bool {
        if (!take.ok) return false;
        std::vector<float> w((size_t)2 * d * d), b((size_t)2 * d);
        std::memcpy(w.data(), q.w, sizeof(float) * d * d);
        std::memcpy(w.data() + (size_t)d * d, k.w, sizeof(float) * d * d);
        std::memcpy(b.data(), q.b, sizeof(float) * d);
        std::memcpy(b.data() + d, k.b, sizeof(float) * d);
        return upload_linear(l, w.data(), b.data(), 2 * d, d, int8);
    };
    auto lin = [&](DevLinear& l, Raw r, int N, int K, bool int8) -> bool {
        if (!take.ok) return false;
        return upload_linear(l, r.w, r.b, N, K, int8);
    };

    Raw r_img = raw(d, img_ch);
    if (!lin(img_proj_, r_img, d, img_ch, q_img)) { fail("act.bin too short"); return false; }
    Raw r_state = raw(d, c.state_dim);
    if (!lin(state_proj_, r_state, d, c.state_dim, false)) { fail("act.bin too short"); return false; }
    const float* latent = take(d);
    const float* pos1d = take((size_t)c.n_1d * d);
    if (!take.ok) { fail("act.bin too short"); return false; }
    d_latent_ = dev_copy(latent, d);
    std::vector<float> pos1d_h(pos1d, pos1d + (size_t)c.n_1d * d);

    enc_.resize(c.n_enc);
    for (EncLayerDev& l : enc_) {
        Raw wq = raw(d, d), wk = raw(d, d), wv = raw(d, d), wo = raw(d, d);
        if (!stack_qk(l.wqk, wq, wk, q_attn) || !lin(l.wv, wv, d, d, q_attn) || !lin(l.wo, wo, d, d, q_attn)) {
            fail("act.bin too short");
            return false;
        }
        const float* n1s = take(d); const float* n1b = take(d);
        Raw w1 = raw(c.ff, d), w2 = raw(d, c.ff);
        const float* n2s = take(d); const float* n2b = take(d);
        if (!take.ok || !lin(l.w1, w1, c.ff, d, q_w1) || !lin(l.w2, w2, d, c.ff, q_w2)) {
            fail("act.bin too short");
            return false;
        }
        l.n1s = dev_copy(n1s, d); l.n1b = dev_copy(n1b, d); l.n2s = dev_copy(n2s, d); l.n2b = dev_copy(n2b, d);
    }
    dec_.resize(c.n_dec);
    for (DecLayerDev& l : dec_) {
        Raw sq = raw(d, d), sk = raw(d, d), sv = raw(d, d), so = raw(d, d);
        if (!stack_qk(l.s_wqk, sq, sk, q_dec) || !lin(l.s_wv, sv, d, d, q_dec) || !lin(l.s_wo, so, d, d, q_dec)) {
            fail("act.bin too short");
            return false;
        }
        const float* n1s = take(d); const float* n1b = take(d);
        Raw cq = raw(d, d), ck = raw(d, d), cv = raw(d, d), co = raw(d, d);
        if (!lin(l.c_wq, cq, d, d, q_dec) || !lin(l.c_wk, ck, d, d, q_dec) || !lin(l.c_wv, cv, d, d, q_dec) ||
            !lin(l.c_wo, co, d, d, q_dec)) {
            fail("act.bin too short");
            return false;
        }
        const float* n2s = take(d); const float* n2b = take(d);
        Raw w1 = raw(c.ff, d), w2 = raw(d, c.ff);
        const float* n3s = take(d); const float* n3b = take(d);
        if (!take.ok || !lin(l.w1, w1, c.ff, d, q_dec) || !lin(l.w2, w2, d, c.ff, q_dec)) {
            fail("act.bin too short");
            return false;
        }
        l.n1s = dev_copy(n1s, d); l.n1b = dev_copy(n1b, d); l.n2s = dev_copy(n2s, d);
        l.n2b = dev_copy(n2b, d); l.n3s = dev_copy(n3s, d); l.n3b = dev_copy(n3b, d);
    }
    const float* dec_pos = take((size_t)c.chunk * d);
    const float* dec_ns = take(d);
    const float* dec_nb = take(d);
    Raw hd = raw(c.action_dim, d);
    if (!take.ok || !lin(head_, hd, c.action_dim, d, false)) { fail("act.bin too short"); return false; }
    if (!take.done()) { fail("act.bin size does not match act.meta"); return false; }
    d_dec_pos_ = dev_copy(dec_pos, (size_t)c.chunk * d);
    d_dec_ns_ = dev_copy(dec_ns, d);
    d_dec_nb_ = dev_copy(dec_nb, d);

    // Token positions [latent | state | cam0 | cam1 ...]: the 1D table, then
    // the 2D sinusoid per camera (ActTransformer::build_tokens).
    const int n_img = fh_ * fw_;
    const int T = c.n_1d + n_cams_ * n_img;
    std::vector<float> pos((size_t)T * d), cam((size_t)n_img * d);
    sinusoid_pos_2d_host(fh_, fw_, d, cam.data());
    std::memcpy(pos.data(), pos1d_h.data(), sizeof(float) * pos1d_h.size());
    for (int cc = 0; cc < n_cams_; ++cc)
        std::memcpy(pos.data() + ((size_t)c.n_1d + (size_t)cc * n_img) * d, cam.data(), sizeof(float) * cam.size());
    d_pos_ = dev_copy(pos.data(), pos.size());
    return true;
}

bool ActPolicy::load_stats(const ModelFiles& files) {
    std::vector<float> raw;
    const int sd = cfg_.state_dim, ad = cfg_.action_dim;
    if (!files.read_floats("stats.bin", raw) || raw.size() != (size_t)2 * sd + 2 * ad + (size_t)n_cams_ * 6) {
        fail("stats.bin missing or wrong size");
        return false;
    }
    for (float v : raw)
        if (!std::isfinite(v)) { fail("non-finite stats"); return false; }
    const float* p = raw.data();
    std::vector<float> im((size_t)n_cams_ * 3), is((size_t)n_cams_ * 3);
    const float* sm = p; p += sd;
    const float* ss = p; p += sd;
    const float* am = p; p += ad;
    const float* as = p; p += ad;
    for (int cc = 0; cc < n_cams_; ++cc) {
        for (int i = 0; i < 3; ++i) im[(size_t)cc * 3 + i] = *p++;
        for (int i = 0; i < 3; ++i) is[(size_t)cc * 3 + i] = *p++;
    }
    for (int i = 0; i < sd; ++i) if (ss[i] < 0) { fail("negative std"); return false; }
    for (int i = 0; i < ad; ++i) if (as[i] < 0) { fail("negative std"); return false; }
    for (float v : is) if (v < 0) { fail("negative std"); return false; }
    auto up = [&](const float* s, size_t n) {
        float* d = dalloc<float>(n);
        if (d) cudaMemcpy(d, s, n * sizeof(float), cudaMemcpyHostToDevice);
        return d;
    };
    d_state_mean_ = up(sm, sd); d_state_std_ = up(ss, sd);
    d_act_mean_ = up(am, ad); d_act_std_ = up(as, ad);
    d_img_mean_ = up(im.data(), im.size()); d_img_std_ = up(is.data(), is.size());
    return err_.empty();
}

bool ActPolicy::alloc_buffers() {
    const int F = n_cams_;
    // backbone activations: the largest map is the stem output
    const int sh = conv_out(img_h_, stem_k_, stem_stride_, stem_pad_), sw = conv_out(img_w_, stem_k_, stem_stride_, stem_pad_);
    size_t max_act = (size_t)F * sh * sw * stem_out_;
    size_t max_col_i8 = 0, max_col_f = 0, max_rows = 0;
    size_t max_col_side = 0, max_rows_side = 0;   // downsample convs, run beside conv1
    auto visit_side = [&](const DevConv& c, int H, int W) {
        if (!c.lin.int8) return;
        const int Ho = conv_out(H, c.k, c.stride, c.pad), Wo = conv_out(W, c.k, c.stride, c.pad);
        const size_t rows = (size_t)F * Ho * Wo;
        max_rows_side = std::max(max_rows_side, std::max(rows, (size_t)F));
        max_col_side = std::max(max_col_side, std::max(rows * (size_t)c.lin.ldw, (size_t)F * H * W * c.cin));
    };
    auto visit = [&](const DevConv& c, int H, int W) {
        const int Ho = conv_out(H, c.k, c.stride, c.pad), Wo = conv_out(W, c.k, c.stride, c.pad);
        const size_t rows = (size_t)F * Ho * Wo;
        max_rows = std::max(max_rows, rows);
        max_act = std::max(max_act, rows * c.cout);
        if (c.lin.int8) max_col_i8 = std::max(max_col_i8, rows * (size_t)c.lin.ldw);
        if (c.Wq_s2d) max_col_i8 = std::max(max_col_i8, (size_t)F * (Ho + (c.k + 1) / 2 - 1) * Wo * 64);
        else max_col_f = std::max(max_col_f, rows * (size_t)c.lin.K);
    };
    visit(stem_, img_h_, img_w_);
    int h = conv_out(sh, pool_k_, pool_stride_, pool_pad_), w = conv_out(sw, pool_k_, pool_stride_, pool_pad_);
    for (const DevBlock& b : blocks_) {
        visit(b.conv1, h, w);
        const int oh = conv_out(h, 3, b.conv1.stride, 1), ow = conv_out(w, 3, b.conv1.stride, 1);
        visit(b.conv2, oh, ow);
        if (b.has_down) {
            visit(b.down, h, w);
            visit_side(b.down, h, w);
        }
        h = oh;
        w = ow;
    }
    fh_ = h;
    fw_ = w;
    if (fh_ <= 0 || fw_ <= 0) { fail("image too small for the backbone"); return false; }

    const size_t npx = (size_t)img_h_ * img_w_;
    // frames and state share one device buffer (one host-to-device copy per call)
    state_off_ = ((size_t)F * npx * 3 + 255) & ~size_t(255);
    d_img_u8_ = dalloc<uint8_t>(state_off_ + sizeof(float) * cfg_.state_dim);
    d_img_f_ = dalloc<float>((size_t)F * npx * 3);
    d_ba_ = dalloc<float>(max_act);
    d_bb_ = dalloc<float>(max_act);
    d_bc_ = dalloc<float>(max_act);
    d_bres_ = dalloc<float>(max_act);
    if (max_col_i8) d_col_ = dalloc<int8_t>(max_col_i8);
    if (max_col_f) d_col_f_ = dalloc<float>(max_col_f);
    d_col_scale_ = dalloc<float>(max_rows);
    if (max_col_side) {
        d_col2_ = dalloc<int8_t>(max_col_side);
        d_col_scale2_ = dalloc<float>(max_rows_side);
    }
    n_amax_ = (2 + 2 * static_cast<int>(blocks_.size())) * F;
    d_amax_ = dalloc<unsigned int>(n_amax_);
    return err_.empty();
}

bool ActPolicy::load(const std::string& dir) {
    const int want_dev = env_int("VLA_CUDA_DEVICE", -1);
    if (want_dev >= 0) {
        if (cudaSetDevice(want_dev) != cudaSuccess) { fail("VLA_CUDA_DEVICE not usable"); return false; }
    }
    cudaGetDevice(&device_);
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device_);
    if (major != 10) { fail("needs an sm_100 (B200) device"); return false; }
    use_graph_ = env_int("VLA_CUDA_GRAPH", 1) != 0;
    explicit_convs_ = env_int("VLA_CONV_IM2COL", 0) != 0;
    i8_clip_ = env_clip();
    const int mask = env_int("ACT_INT8", 0);

    // a converted directory or a vla.simd GGUF (src/models/act/act_model.cpp:22-24 mounts it the same way)
    ModelFiles files;
    if (!files.open(dir)) { fail(files.error()); return false; }
    if (!load_config(files)) return false;
    if (!load_backbone(files, (mask & 32) != 0)) return false;
    if (!alloc_buffers()) return false;   // also fixes the feature map size
    if (!load_transformer(files, mask)) return false;
    if (!load_stats(files)) return false;
    if (env_int("ACT_PROFILE", 0) >= 2)
        std::fprintf(stderr, "[act] int8 GEMMs on device: %d\n", n_int8_);

    // transformer activations
    const int T = n_tokens(), d = cfg_.dim, C = cfg_.chunk;
    const int R = std::max(T, C);
    ldq_ = round16(d);
    ldqff_ = round16(cfg_.ff);
    const int img_rows = n_cams_ * fh_ * fw_;
    const int img_ch = blocks_.empty() ? stem_out_ : blocks_.back().conv1.cout;
    const long long ldqi = round16(img_ch);
    d_state_ = d_img_u8_ ? reinterpret_cast<float*>(d_img_u8_ + state_off_) : nullptr;
    d_state_n_ = dalloc<float>(cfg_.state_dim);
    d_actions_ = dalloc<float>((size_t)cfg_.chunk * cfg_.action_dim);
    d_x_ = dalloc<float>((size_t)T * d);
    d_qk_ = dalloc<float>((size_t)R * 2 * d);
    d_v_ = dalloc<float>((size_t)R * d);
    d_att_ = dalloc<float>((size_t)R * d);
    d_ff_ = dalloc<float>((size_t)R * cfg_.ff);
    d_dx_ = dalloc<float>((size_t)C * d);
    d_ck_ = dalloc<float>((size_t)T * d);
    d_cv_ = dalloc<float>((size_t)T * d);
    d_qa_ = dalloc<int8_t>((size_t)std::max(R, img_rows) * std::max(ldq_, ldqi));
    d_qb_ = dalloc<int8_t>((size_t)R * ldq_);
    d_qatt_ = dalloc<int8_t>((size_t)R * ldq_);
    d_qff_ = dalloc<int8_t>((size_t)R * ldqff_);
    d_sa_ = dalloc<float>(std::max(R, img_rows));
    d_sb_ = dalloc<float>(R);
    d_satt_ = dalloc<float>(R);
    d_sff_ = dalloc<float>(R);
    d_qamax_ = dalloc<unsigned int>(R);
    d_qsync_ = dalloc<unsigned int>(2 * ((R + 127) / 128));
    if (d_qamax_ && d_qsync_ &&
        (cudaMemset(d_qamax_, 0, sizeof(unsigned int) * R) != cudaSuccess ||
         cudaMemset(d_qsync_, 0, sizeof(unsigned int) * 2 * ((R + 127) / 128)) != cudaSuccess))
        fail("cudaMemset failed");
    d_att_cnt_ = dalloc<unsigned int>(kAttCounters);
    if (d_att_cnt_ && cudaMemset(d_att_cnt_, 0, sizeof(unsigned int) * kAttCounters) != cudaSuccess)
        fail("cudaMemset failed");
    d_xp_ = dalloc<float>((size_t)R * d);
    d_qea_ = dalloc<int8_t>((size_t)T * ldq_);
    d_qeb_ = dalloc<int8_t>((size_t)T * ldq_);
    d_sea_ = dalloc<float>(T);
    d_seb_ = dalloc<float>(T);
    d_dec_x0_ = dalloc<float>((size_t)C * d);
    d_dec_q0_ = dalloc<float>((size_t)C * d);
    if (!err_.empty()) return false;

    if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&side_, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_join_, cudaEventDisableTiming) != cudaSuccess) {
        fail("streams / events");
        return false;
    }
    if (cudaMallocHost(&h_state_pinned_, sizeof(float) * cfg_.state_dim) != cudaSuccess ||
        cudaMallocHost(&h_actions_pinned_, sizeof(float) * cfg_.chunk * cfg_.action_dim) != cudaSuccess ||
        cudaMallocHost(&h_status_pinned_, sizeof(int)) != cudaSuccess) {
        fail("pinned host buffers");
        return false;
    }
    d_status_ = static_cast<int*>(device_status_address());
    if (!d_status_) { fail("device status word"); return false; }
    // zero inputs so the warm-up step reads defined memory
    cudaMemset(d_img_u8_, 0, (size_t)n_cams_ * img_h_ * img_w_ * 3);
    cudaMemset(d_state_, 0, sizeof(float) * cfg_.state_dim);
    cudaDeviceSynchronize();
    if (dec0_consts(stream_) != cudaSuccess) {
        fail("decoder layer-0 constants failed");
        return false;
    }
    // one eager step validates every launch before capture
    if (forward(stream_, true) != cudaSuccess || cudaStreamSynchronize(stream_) != cudaSuccess) {
        fail("warm-up step failed");
        return false;
    }
    if (device_status_take() != 0) { fail("device status error in warm-up"); return false; }
    return true;
}

cudaError_t ActPolicy::run_linear(const DevLinear& l, const float* x_f32, const int8_t* xq, const float* xs,
                                  const CUtensorMap* tmap_a, int M, float* out, long long ldo, int mode,
                                  const float* res, long long ldr, cudaStream_t st, unsigned int* amax,
                                  int amax_rows) {
    if (l.int8) {
        GemmI8Args a;
        a.A = xq;
        a.lda = round16(l.K);
        a.B = l.Wq;
        a.ldb = l.ldw;
        a.M = M;
        a.N = l.N;
        a.K = l.K;
        a.out = out;
        a.ldo = ldo;
        a.ascale = xs;
        a.wscale = l.wscale;
        a.bias = l.bias;
        a.res = res;
        a.ldr = ldr;
        a.mode = mode;
        a.amax = amax;
        a.amax_rows = amax_rows;
        a.static_weights = true;   // uploaded once at load
        (void)tmap_a;
        return gemm_i8(a, st);
    }
    return gemm_f32(x_f32, l.K, l.W, l.K, l.bias, out, ldo, res, ldr, M, l.N, l.K, mode, amax, amax_rows, st);
}

cudaError_t ActPolicy::run_conv(const DevConv& c, const float* in, int F, int H, int W, float* out, int mode,
                                const float* res, const unsigned int* amax_in, unsigned int* amax_out,
                                cudaStream_t st, bool side) {
    // a conv running beside another (a downsample next to conv1) has its own scratch
    ConvScratch s;
    s.col = side ? d_col2_ : d_col_;
    s.col_scale = side ? d_col_scale2_ : d_col_scale_;
    s.col_f = d_col_f_;
    return conv2d_dev(c, in, F, H, W, out, mode, res, amax_in, amax_out, i8_clip_, explicit_convs_, s, st);
}

cudaStream_t ActPolicy::fork(cudaStream_t st) {
    if (cudaEventRecord(ev_fork_, st) != cudaSuccess || cudaStreamWaitEvent(side_, ev_fork_, 0) != cudaSuccess)
        return nullptr;
    return side_;
}

cudaError_t ActPolicy::join(cudaStream_t st) {
    VSB_TRY(cudaEventRecord(ev_join_, side_));
    return cudaStreamWaitEvent(st, ev_join_, 0);
}

// FFN up-projection + ReLU straight to the down-projection's int8 input
// (d_qff_ / d_sff_: the row quantization quantize_rows would make of the fp32
// hidden, which is then never written), where the GEMM can do it (w1 and w2
// both int8, one wave of slab CTAs); else the fp32 hidden and quantize_rows.
cudaError_t ActPolicy::ffn_up(const DevLinear& w1, const DevLinear& w2, const int8_t* xq, const float* xs,
                              const float* x_f32, int M, cudaStream_t st) {
    if (w1.int8 && w2.int8 && d_qamax_ && gemm_i8_rowq_supported(M, w1.N, w1.K) && ldqff_ == w1.N) {
        GemmI8Args a;
        a.A = xq;
        a.lda = round16(w1.K);
        a.B = w1.Wq;
        a.ldb = w1.ldw;
        a.M = M;
        a.N = w1.N;
        a.K = w1.K;
        a.ascale = xs;
        a.wscale = w1.wscale;
        a.bias = w1.bias;
        a.mode = kEpiRelu;
        a.static_weights = true;
        a.qout = d_qff_;
        a.ldq = ldqff_;
        a.qscale = d_sff_;
        a.qamax = d_qamax_;
        a.qsync = d_qsync_;
        return gemm_i8(a, st);
    }
    VSB_TRY(run_linear(w1, x_f32, xq, xs, nullptr, M, d_ff_, cfg_.ff, kEpiRelu, nullptr, 0, st));
    if (w2.int8)
        VSB_TRY(quantize_rows(d_ff_, cfg_.ff, nullptr, 0, M, cfg_.ff, d_qff_, ldqff_, d_sff_, nullptr, 0, nullptr, st));
    return cudaSuccess;
}

// The attention output's int8 row copy (d_qatt_ / d_satt_), written by the
// attention launch (nn.h AttQuant).
AttQuant ActPolicy::att_quant() const {
    AttQuant a;
    a.q = d_qatt_;
    a.ldq = ldq_;
    a.scale = d_satt_;
    a.counters = d_att_cnt_;
    a.n_counters = kAttCounters;
    return a;
}

cudaError_t ActPolicy::run_backbone(cudaStream_t st) {
    const int F = n_cams_;
    unsigned int* slot = d_amax_;
    VSB_TRY(normalize_frames(d_img_u8_, d_img_f_, F, (long long)img_h_ * img_w_, d_img_mean_, d_img_std_, norm_eps_,
                             slot, st));
    int h = conv_out(img_h_, stem_k_, stem_stride_, stem_pad_), w = conv_out(img_w_, stem_k_, stem_stride_, stem_pad_);
    VSB_TRY(run_conv(stem_, d_img_f_, F, img_h_, img_w_, d_ba_, 0, nullptr, slot, nullptr, st));
    const int ph = conv_out(h, pool_k_, pool_stride_, pool_pad_), pw = conv_out(w, pool_k_, pool_stride_, pool_pad_);
    unsigned int* pool_slot = slot + F;
    VSB_TRY(maxpool_relu(d_ba_, d_bb_, F, h, w, stem_out_, pool_k_, pool_stride_, pool_pad_, ph, pw, pool_slot, st));
    h = ph;
    w = pw;
    float *b = d_bb_, *a = d_ba_, *c = d_bc_;
    unsigned int* in_slot = pool_slot;
    for (size_t i = 0; i < blocks_.size(); ++i) {
        const DevBlock& blk = blocks_[i];
        unsigned int* mid_slot = d_amax_ + (2 + 2 * i) * F;
        unsigned int* out_slot = mid_slot + F;
        const int oh = conv_out(h, 3, blk.conv1.stride, 1), ow = conv_out(w, 3, blk.conv1.stride, 1);
        const float* idn = b;
        // the downsample conv runs beside conv1 (both read the block input; it
        // has its own scratch); conv2 waits for both
        const bool side = blk.has_down && blk.down.lin.int8 && d_col2_;
        if (blk.has_down) {
            cudaStream_t ds = side ? fork(st) : st;
            if (!ds) return cudaErrorUnknown;
            VSB_TRY(run_conv(blk.down, b, F, h, w, d_bres_, 0, nullptr, in_slot, nullptr, ds, side));
            idn = d_bres_;
        }
        VSB_TRY(run_conv(blk.conv1, b, F, h, w, a, kEpiRelu, nullptr, in_slot, mid_slot, st));
        if (side) VSB_TRY(join(st));
        VSB_TRY(run_conv(blk.conv2, a, F, oh, ow, c, kEpiAddRelu, idn, mid_slot, out_slot, st));
        std::swap(b, c);
        h = oh;
        w = ow;
        in_slot = out_slot;
    }
    d_feat_ = b;
    return cudaSuccess;
}

cudaError_t ActPolicy::run_encoder(cudaStream_t st) {
    const int T = n_tokens(), d = cfg_.dim;
    const float scale = 1.0f / std::sqrt(static_cast<float>(cfg_.head_dim));
    // layer 0 inputs: q(x + pos) and q(x); later layers get them from LN2
    VSB_TRY(quantize_rows(d_x_, d, d_pos_, d, T, d, d_qa_, ldq_, d_sa_, d_qb_, ldq_, d_sb_, st));
    for (size_t li = 0; li < enc_.size(); ++li) {
        const EncLayerDev& l = enc_[li];
        const bool last = li + 1 == enc_.size();
        if (!l.wqk.int8) VSB_TRY(add_f32(d_x_, d_pos_, d_xp_, (long long)T * d, st));   // fp32 q/k read x + pos
        {   // V beside Q/K (separate inputs and outputs); attention waits for both
            cudaStream_t sv = fork(st);
            if (!sv) return cudaErrorUnknown;
            VSB_TRY(run_linear(l.wv, d_x_, d_qb_, d_sb_, nullptr, T, d_v_, d, 0, nullptr, 0, sv));
            VSB_TRY(run_linear(l.wqk, d_xp_, d_qa_, d_sa_, nullptr, T, d_qk_, 2 * d, 0, nullptr, 0, st));
            VSB_TRY(join(st));
        }
        // the o-projection's int8 input comes out of the attention launch itself
        const AttQuant aq = att_quant();
        VSB_TRY(attention(d_qk_, 2 * d, d_qk_ + d, 2 * d, d_v_, d, d_att_, d, T, T, cfg_.heads, cfg_.heads,
                          cfg_.head_dim, scale, nullptr, st, l.wo.int8 ? &aq : nullptr));
        VSB_TRY(run_linear(l.wo, d_att_, d_qatt_, d_satt_, nullptr, T, d_x_, d, kEpiAdd, d_x_, d, st));
        VSB_TRY(layernorm(d_x_, d_x_, l.n1s, l.n1b, T, d, cfg_.ln_eps, nullptr, d_qa_, d_sa_, nullptr, nullptr, ldq_, st));
        VSB_TRY(ffn_up(l.w1, l.w2, d_qa_, d_sa_, d_x_, T, st));
        VSB_TRY(run_linear(l.w2, d_ff_, d_qff_, d_sff_, nullptr, T, d_x_, d, kEpiAdd, d_x_, d, st));
        // LN2, then q(x + pos) and q(x) for the next layer (or for the decoder's
        // cross-attention keys / values after the last layer)
        VSB_TRY(layernorm(d_x_, d_x_, l.n2s, l.n2b, T, d, cfg_.ln_eps, d_pos_, last ? d_qea_ : d_qa_,
                          last ? d_sea_ : d_sa_, last ? d_qeb_ : d_qb_, last ? d_seb_ : d_sb_, ldq_, st));
    }
    return cudaSuccess;
}

cudaError_t ActPolicy::run_decoder(cudaStream_t st, bool unnormalize) {
    const int T = n_tokens(), d = cfg_.dim, C = cfg_.chunk;
    const float scale = 1.0f / std::sqrt(static_cast<float>(cfg_.head_dim));
    // cross-attention keys / values: q(enc + pos) is in qa, q(enc) in qb
    // (last encoder LN2). With one decoder layer they are used once; with
    // more, each layer projects them with its own weights.
    // Queries start at zero every step, so decoder layer 0's self-attention
    // block (and its LayerNorm) and its cross-attention query projection depend
    // on the weights alone: they ran once at load (dec0_consts) - the step
    // prologue seeded d_dx_ with that LayerNorm output and layer 0 reads its
    // cross queries from d_dec_q0_. Later layers run in full.
    for (size_t li = 0; li < dec_.size(); ++li) {
        const DecLayerDev& l = dec_[li];
        if (!l.c_wk.int8) VSB_TRY(add_f32(d_x_, d_pos_, d_xp_, (long long)T * d, st));   // fp32 keys read enc + pos
        {   // cross V beside cross K
            cudaStream_t sv = fork(st);
            if (!sv) return cudaErrorUnknown;
            VSB_TRY(run_linear(l.c_wv, d_x_, d_qeb_, d_seb_, nullptr, T, d_cv_, d, 0, nullptr, 0, sv));
            VSB_TRY(run_linear(l.c_wk, d_xp_, d_qea_, d_sea_, nullptr, T, d_ck_, d, 0, nullptr, 0, st));
            VSB_TRY(join(st));
        }
        const float* cq = d_qk_;
        if (li == 0 && dec0_ready_) {
            cq = d_dec_q0_;
        } else {
            VSB_TRY(decoder_self_block(l, st));
            VSB_TRY(decoder_cross_queries(l, d_qk_, st));
        }
        const AttQuant aq = att_quant();
        VSB_TRY(attention(cq, d, d_ck_, d, d_cv_, d, d_att_, d, C, T, cfg_.heads, cfg_.heads, cfg_.head_dim,
                          scale, nullptr, st, &aq));
        VSB_TRY(run_linear(l.c_wo, d_att_, d_qatt_, d_satt_, nullptr, C, d_dx_, d, kEpiAdd, d_dx_, d, st));
        VSB_TRY(layernorm(d_dx_, d_dx_, l.n2s, l.n2b, C, d, cfg_.ln_eps, nullptr, d_qatt_, d_satt_, nullptr, nullptr,
                          ldq_, st));
        VSB_TRY(ffn_up(l.w1, l.w2, d_qatt_, d_satt_, d_dx_, C, st));
        VSB_TRY(run_linear(l.w2, d_ff_, d_qff_, d_sff_, nullptr, C, d_dx_, d, kEpiAdd, d_dx_, d, st));
        VSB_TRY(layernorm(d_dx_, d_dx_, l.n3s, l.n3b, C, d, cfg_.ln_eps, nullptr, nullptr, nullptr, nullptr, nullptr,
                          0, st));
    }
    VSB_TRY(layernorm(d_dx_, d_dx_, d_dec_ns_, d_dec_nb_, C, d, cfg_.ln_eps, nullptr, nullptr, nullptr, nullptr,
                      nullptr, 0, st));
    VSB_TRY(linear_f32(d_dx_, d, head_.W, head_.bias, d_actions_, cfg_.action_dim, C, cfg_.action_dim, d,
                       unnormalize ? d_act_std_ : nullptr, unnormalize ? d_act_mean_ : nullptr, st));
    return cudaSuccess;
}

// Self-attention block of a decoder layer over the queries in d_dx_, ending
// with LayerNorm n1 (whose fused int8 output q(x + pos) feeds the cross
// queries): src/models/act/act_transformer.cpp:301-312.
cudaError_t ActPolicy::decoder_self_block(const DecLayerDev& l, cudaStream_t st) {
    const int d = cfg_.dim, C = cfg_.chunk;
    const float scale = 1.0f / std::sqrt(static_cast<float>(cfg_.head_dim));
    VSB_TRY(quantize_rows(d_dx_, d, d_dec_pos_, d, C, d, d_qatt_, ldq_, d_satt_, d_qb_, ldq_, d_sb_, st));
    if (!l.s_wqk.int8) VSB_TRY(add_f32(d_dx_, d_dec_pos_, d_xp_, (long long)C * d, st));
    VSB_TRY(run_linear(l.s_wqk, d_xp_, d_qatt_, d_satt_, nullptr, C, d_qk_, 2 * d, 0, nullptr, 0, st));
    VSB_TRY(run_linear(l.s_wv, d_dx_, d_qb_, d_sb_, nullptr, C, d_v_, d, 0, nullptr, 0, st));
    const AttQuant aq = att_quant();
    VSB_TRY(attention(d_qk_, 2 * d, d_qk_ + d, 2 * d, d_v_, d, d_att_, d, C, C, cfg_.heads, cfg_.heads,
                      cfg_.head_dim, scale, nullptr, st, &aq));
    VSB_TRY(run_linear(l.s_wo, d_att_, d_qatt_, d_satt_, nullptr, C, d_dx_, d, kEpiAdd, d_dx_, d, st));
    return layernorm(d_dx_, d_dx_, l.n1s, l.n1b, C, d, cfg_.ln_eps, d_dec_pos_, d_qatt_, d_satt_, nullptr, nullptr,
                     ldq_, st);
}

// Cross-attention queries from x + pos (act_transformer.cpp:314-319) into q [C][d].
cudaError_t ActPolicy::decoder_cross_queries(const DecLayerDev& l, float* q, cudaStream_t st) {
    const int d = cfg_.dim, C = cfg_.chunk;
    if (!l.c_wq.int8) VSB_TRY(add_f32(d_dx_, d_dec_pos_, d_xp_, (long long)C * d, st));
    return run_linear(l.c_wq, d_xp_, d_qatt_, d_satt_, nullptr, C, q, d, 0, nullptr, 0, st);
}

// Decoder layer 0 on zero queries, once per load: its LayerNorm-n1 output goes
// to d_dec_x0_ (the step prologue copies it into d_dx_), its cross queries to
// d_dec_q0_. The same kernels on the same inputs as a per-step run, so the
// results are bit-identical to computing them every step.
cudaError_t ActPolicy::dec0_consts(cudaStream_t st) {
    if (dec_.empty()) return cudaSuccess;
    const size_t n = (size_t)cfg_.chunk * cfg_.dim;
    VSB_TRY(cudaMemsetAsync(d_dx_, 0, sizeof(float) * n, st));
    VSB_TRY(decoder_self_block(dec_[0], st));
    VSB_TRY(decoder_cross_queries(dec_[0], d_dec_q0_, st));
    VSB_TRY(cudaMemcpyAsync(d_dec_x0_, d_dx_, sizeof(float) * n, cudaMemcpyDeviceToDevice, st));
    VSB_TRY(cudaStreamSynchronize(st));
    dec0_ready_ = true;
    return cudaSuccess;
}

cudaError_t ActPolicy::forward(cudaStream_t st, bool unnormalize) {
    const int d = cfg_.dim;
    // absmax slots zeroed, decoder state set (layer 0's constant LayerNorm-n1
    // output, or zero queries), latent token placed, state normalized
    VSB_TRY(act_prologue(d_amax_, n_amax_, d_dx_, (long long)cfg_.chunk * d, dec0_ready_ ? d_dec_x0_ : nullptr, d_x_,
                         d_latent_, d, d_state_, d_state_mean_, d_state_std_, norm_eps_, d_state_n_, cfg_.state_dim,
                         st));
    VSB_TRY(run_backbone(st));
    // tokens: [latent | state_proj(state_norm) | img_proj(features per camera)]
    VSB_TRY(linear_f32(d_state_n_, cfg_.state_dim, state_proj_.W, state_proj_.bias, d_x_ + d, d, 1, d,
                       cfg_.state_dim, nullptr, nullptr, st));
    const int img_rows = n_cams_ * fh_ * fw_;
    const int img_ch = blocks_.empty() ? stem_out_ : blocks_.back().conv1.cout;
    if (img_proj_.int8) {
        VSB_TRY(quantize_rows(d_feat_, img_ch, nullptr, 0, img_rows, img_ch, d_qa_, round16(img_ch), d_sa_, nullptr,
                              0, nullptr, st));
    }
    VSB_TRY(run_linear(img_proj_, d_feat_, d_qa_, d_sa_, nullptr, img_rows, d_x_ + (size_t)cfg_.n_1d * d, d, 0,
                       nullptr, 0, st));
    VSB_TRY(run_encoder(st));
    return run_decoder(st, unnormalize);
}

cudaError_t ActPolicy::enqueue_step(cudaStream_t st, bool unnormalize) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device_) cudaSetDevice(device_);
    const cudaError_t e = enqueue_on_device(st, unnormalize);
    if (prev != device_) cudaSetDevice(prev);
    return e;
}

cudaError_t ActPolicy::enqueue_on_device(cudaStream_t st, bool unnormalize) {
    const int gi = unnormalize ? 1 : 0;
    if (!use_graph_) return forward(st, unnormalize);
    if (!graph_[gi]) {
        // capture on the policy's own stream, instantiate once
        cudaGraph_t g = nullptr;
        VSB_TRY(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
        const cudaError_t fe = forward(stream_, unnormalize);
        const cudaError_t ce = cudaStreamEndCapture(stream_, &g);
        if (fe != cudaSuccess) { if (g) cudaGraphDestroy(g); return fe; }
        VSB_TRY(ce);
        size_t n_nodes = 0;
        cudaGraphGetNodes(g, nullptr, &n_nodes);
        std::vector<cudaGraphNode_t> nodes(n_nodes);
        cudaGraphGetNodes(g, nodes.data(), &n_nodes);
        int nk = 0;
        for (cudaGraphNode_t nd : nodes) {
            cudaGraphNodeType t;
            if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) nk++;
        }
        kernels_per_step_ = nk;
        const cudaError_t ie = cudaGraphInstantiate(&graph_[gi], g, 0);
        cudaGraphDestroy(g);
        VSB_TRY(ie);
    }
    return cudaGraphLaunch(graph_[gi], st);
}

cudaError_t ActPolicy::predict(const uint8_t* images, const float* state, bool unnormalize, float* actions) {
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device_) cudaSetDevice(device_);
    const size_t img_bytes = (size_t)n_cams_ * img_h_ * img_w_ * 3;
    // The frames go straight from the caller's (pageable) buffer: the driver
    // overlaps its staging copy with the DMA, which measured faster than a
    // memcpy into our pinned buffer followed by the DMA (~109 vs ~145 us for
    // 1.8 MB). The small state goes through pinned staging.
    std::memcpy(h_state_pinned_, state, sizeof(float) * cfg_.state_dim);
    cudaError_t e = cudaMemcpyAsync(d_img_u8_, images, img_bytes, cudaMemcpyHostToDevice, stream_);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_state_, h_state_pinned_, sizeof(float) * cfg_.state_dim, cudaMemcpyHostToDevice,
                            stream_);
    if (e == cudaSuccess) e = enqueue_on_device(stream_, unnormalize);
    const size_t ab = sizeof(float) * cfg_.chunk * cfg_.action_dim;
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_actions_pinned_, d_actions_, ab, cudaMemcpyDeviceToHost, stream_);
    // the kernels' status word comes back in the same stream (no extra sync)
    if (e == cudaSuccess) e = cudaMemcpyAsync(h_status_pinned_, d_status_, sizeof(int), cudaMemcpyDeviceToHost, stream_);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
    if (e == cudaSuccess && *h_status_pinned_ != 0) {
        device_status_take();   // clear it for the next call
        e = cudaErrorLaunchFailure;
    }
    if (e == cudaSuccess) std::memcpy(actions, h_actions_pinned_, ab);
    if (prev != device_) cudaSetDevice(prev);
    return e;
}

}  // namespace vsb
