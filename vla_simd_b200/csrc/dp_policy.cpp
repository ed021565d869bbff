// Diffusion Policy runtime (see dp_policy.h). Host code only: parsing, int8
// packing, the noise schedule, buffer planning and the kernel sequence of one
// query batch.
#include "dp_policy.h"

#include "host_util.h"

#include "model_files.h"

#include "f32.h"
#include "gemm_i8.h"
#include "lm_ops.h"
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

constexpr float kNormEps = 1e-8f;   // src/models/diffusion/diffusion_model.cpp:17

using host::Cursor;
using host::env_clip;
using host::env_int;
using host::round16;
using host::shape_fits;

// numpy's linspace as the reference builds the keypoint grid
// (src/models/diffusion/rgb_encoder.cpp:22-28): start + step*i in double (its
// build fuses that into one fma), cast once, endpoint pinned.
void linspace_np(std::vector<float>& v, double start, double stop, int n) {
    v.resize(n);
    if (n == 1) { v[0] = static_cast<float>(start); return; }
    const double step = (stop - start) / static_cast<double>(n - 1);
    for (int i = 0; i < n; ++i) v[i] = static_cast<float>(std::fma(step, static_cast<double>(i), start));
    v[n - 1] = static_cast<float>(stop);
}

double alpha_bar_cosine(double t) {
    const double c = std::cos((t + 0.008) / 1.008 * M_PI / 2.0);
    return c * c;
}

#define VSB_TRY(expr)                                  \
    do {                                               \
        const cudaError_t e_ = (expr);                 \
        if (e_ != cudaSuccess) return e_;              \
    } while (0)

}  // namespace

template <class T>
T* DpPolicy::dalloc(size_t n) {
    void* p = nullptr;
    if (n == 0) n = 1;
    if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
        fail("cudaMalloc failed");
        return nullptr;
    }
    allocs_.push_back(p);
    return static_cast<T*>(p);
}

DpPolicy::~DpPolicy() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device_);
    for (auto& g : graphs_)
        if (g) cudaGraphExecDestroy(g);
    if (stream_) cudaStreamDestroy(stream_);
    if (side_) cudaStreamDestroy(side_);
    if (ev_fork_) cudaEventDestroy(ev_fork_);
    if (ev_join_) cudaEventDestroy(ev_join_);
    for (void* p : allocs_) cudaFree(p);
    if (h_pinned_) cudaFreeHost(h_pinned_);
    if (h_status_pinned_) cudaFreeHost(h_status_pinned_);
    cudaSetDevice(prev);
}

// diffusion.meta as DiffusionModel::load reads it (src/models/diffusion/diffusion_model.cpp:25-103).
bool DpPolicy::load_meta(const ModelFiles& files) {
    std::string meta_text;
    if (!files.read("diffusion.meta", meta_text)) { fail("cannot open diffusion.meta"); return false; }
    std::istringstream meta(meta_text);
    DpConfigDev& c = cfg_;
    std::string line, sched = "DDPM";
    std::vector<int> dd;
    while (std::getline(meta, line)) {
        std::istringstream ss(line);
        std::string key;
        if (!(ss >> key)) continue;
        if (key == "n_obs_steps") ss >> c.n_obs;
        else if (key == "n_cams") ss >> c.n_cams;
        else if (key == "img_h") ss >> c.img_h;
        else if (key == "img_w") ss >> c.img_w;
        else if (key == "crop_h") ss >> c.crop_h;
        else if (key == "crop_w") ss >> c.crop_w;
        else if (key == "resize_h") ss >> c.resize_h;
        else if (key == "resize_w") ss >> c.resize_w;
        else if (key == "state_dim") ss >> c.state_dim;
        else if (key == "action_dim") ss >> c.action_dim;
        else if (key == "horizon") ss >> c.horizon;
        else if (key == "n_action_steps") ss >> c.n_action_steps;
        else if (key == "num_keypoints") ss >> c.num_keypoints;
        else if (key == "kernel_size") ss >> c.kernel_size;
        else if (key == "n_groups") ss >> c.n_groups;
        else if (key == "step_embed_dim") ss >> c.step_embed_dim;
        else if (key == "num_train_timesteps") ss >> c.num_train_timesteps;
        else if (key == "num_inference_steps") ss >> c.num_inference_steps;
        else if (key == "beta_start") ss >> c.beta_start;
        else if (key == "beta_end") ss >> c.beta_end;
        else if (key == "beta_schedule") ss >> c.beta_schedule;
        else if (key == "prediction_type") ss >> c.prediction_type;
        else if (key == "clip_sample_range") ss >> c.clip_sample_range;
        else if (key == "gn_eps") ss >> c.gn_eps;
        else if (key == "scheduler") ss >> sched;
        else if (key == "film_scale") { int v = 0; ss >> v; c.film_scale = v != 0; }
        else if (key == "clip_sample") { int v = 0; ss >> v; c.clip_sample = v != 0; }
        else if (key == "separate_encoders") { int v = 0; ss >> v; c.separate = v != 0; }
        else if (key == "down_dims") {
            int v;
            while (ss >> v) dd.push_back(v);
            if (!ss.eof() || dd.empty()) { fail("malformed down_dims"); return false; }
            continue;
        } else if (key == "cam") { std::string n; ss >> n; }
        else continue;
        if (ss.fail() || !(ss >> std::ws).eof()) { fail("malformed diffusion.meta line: " + line); return false; }
    }
    if (!dd.empty()) c.down_dims = dd;
    if (sched != "DDPM" && sched != "DDIM") { fail("unknown scheduler"); return false; }
    c.ddim = sched == "DDIM";
    // the deployment knobs, read once at load (diffusion_model.cpp:79-87)
    const int steps = env_int("DP_STEPS", 0);
    if (steps > 0) c.num_inference_steps = steps;
    if (const char* e = std::getenv("DP_SCHEDULER")) {
        const std::string s(e);
        if (s != "DDIM" && s != "DDPM") { fail("DP_SCHEDULER must be DDIM or DDPM"); return false; }
        c.ddim = s == "DDIM";
    }
    if (!shape_fits({c.n_cams, c.n_obs, c.img_h, c.img_w, 3}) || !shape_fits({c.state_dim, c.n_obs}) ||
        !shape_fits({c.horizon, c.action_dim}) || !shape_fits({2, c.num_keypoints, c.n_cams, c.n_obs}) ||
        (long long)c.step_embed_dim + (long long)c.state_dim * c.n_obs +
                (long long)2 * c.num_keypoints * c.n_cams * c.n_obs > INT_MAX ||
        c.crop_h < 0 || c.crop_w < 0 || (c.crop_h == 0) != (c.crop_w == 0) || c.resize_h < 0 || c.resize_w < 0 ||
        c.n_action_steps <= 0 || (long long)c.n_obs - 1 + c.n_action_steps > c.horizon || c.crop_h > c.img_h ||
        c.crop_w > c.img_w || (c.resize_h > 0 && c.resize_h != c.img_h) || (c.resize_w > 0 && c.resize_w != c.img_w) ||
        c.num_inference_steps > c.num_train_timesteps) {
        fail("diffusion.meta values out of range");
        return false;
    }
    return true;
}

// DPNoiseScheduler::init (src/models/diffusion/scheduler.cpp:19-69): betas
// and alphas_cumprod in double, the "leading" inference ladder. No product
// here is followed by an add, so the reference build's contraction does not
// change any of these values.
bool DpPolicy::init_schedule() {
    const DpConfigDev& c = cfg_;
    const int N = c.num_train_timesteps;
    if (N <= 0 || c.num_inference_steps <= 0 || c.num_inference_steps > N || c.horizon <= 0 || c.action_dim <= 0) {
        fail("bad scheduler sizes");
        return false;
    }
    if (c.clip_sample && (!std::isfinite(c.clip_sample_range) || c.clip_sample_range <= 0)) {
        fail("bad clip_sample_range");
        return false;
    }
    if (c.prediction_type != "epsilon") { fail("prediction_type must be epsilon"); return false; }
    std::vector<double> betas((size_t)N);
    if (c.beta_schedule == "squaredcos_cap_v2") {
        for (int i = 0; i < N; ++i) {
            const double t1 = (double)i / (double)N, t2 = (double)(i + 1) / (double)N;
            betas[i] = std::min(1.0 - alpha_bar_cosine(t2) / alpha_bar_cosine(t1), 0.999);
        }
    } else if (c.beta_schedule == "linear" || c.beta_schedule == "scaled_linear") {
        if (!(c.beta_start > 0 && c.beta_start < 1 && c.beta_end > 0 && c.beta_end < 1)) {
            fail("bad beta range");
            return false;
        }
        const bool scaled = c.beta_schedule == "scaled_linear";
        const double a = scaled ? std::sqrt((double)c.beta_start) : (double)c.beta_start;
        const double b = scaled ? std::sqrt((double)c.beta_end) : (double)c.beta_end;
        for (int i = 0; i < N; ++i) {
            const double v = a + (b - a) * (double)i / (double)std::max(N - 1, 1);
            betas[i] = scaled ? v * v : v;
        }
    } else {
        fail("unknown beta_schedule");
        return false;
    }
    alphas_cumprod_.resize((size_t)N);
    double run = 1.0;
    for (int i = 0; i < N; ++i) {
        run *= (1.0 - betas[i]);
        alphas_cumprod_[i] = run;
    }
    const int ratio = N / c.num_inference_steps;
    timesteps_.clear();
    for (int i = c.num_inference_steps - 1; i >= 0; --i) timesteps_.push_back(i * ratio);
    return true;
}

// One observation encoder: "{name}_backbone.meta/.bin" (ResNet with
// GroupNorm, src/models/act/resnet_backbone.cpp:50-151) and "{name}.bin"
// (keypoint conv + output projection, src/models/diffusion/rgb_encoder.cpp:30-68).
bool DpPolicy::load_encoder(const ModelFiles& files, int idx, bool int8) {
    DpEncoderDev& e = enc_[idx];
    const std::string name = "rgb_encoder" + std::to_string(idx);
    std::string meta_text;
    if (!files.read(name + "_backbone.meta", meta_text)) { fail("cannot open " + name + "_backbone.meta"); return false; }
    std::istringstream meta(meta_text);
    struct BM { int cin, cout, stride, has_down; };
    std::vector<BM> bm;
    int in_ch = 3, gs = 0, block_k = 3;
    std::string line;
    while (std::getline(meta, line)) {
        std::istringstream ss(line);
        std::string key;
        if (!(ss >> key)) continue;
        if (key == "in_ch") ss >> in_ch;
        else if (key == "stem_out") ss >> e.stem_out;
        else if (key == "stem_k") ss >> e.stem_k;
        else if (key == "stem_stride") ss >> e.stem_stride;
        else if (key == "stem_pad") ss >> e.stem_pad;
        else if (key == "pool_k") ss >> e.pool_k;
        else if (key == "pool_stride") ss >> e.pool_stride;
        else if (key == "pool_pad") ss >> e.pool_pad;
        else if (key == "block_k") ss >> block_k;
        else if (key == "gn_group_size") ss >> gs;
        else if (key == "block") { BM b{}; ss >> b.cin >> b.cout >> b.stride >> b.has_down; bm.push_back(b); }
        else if (key == "film_after") { fail("FiLM backbones are not part of Diffusion Policy"); return false; }
        else continue;
        if (ss.fail() || !(ss >> std::ws).eof()) { fail("malformed " + name + "_backbone.meta"); return false; }
    }
    if (in_ch != 3 || gs < 0 || block_k != 3 || !shape_fits({e.stem_out, e.stem_k, e.stem_k, in_ch}) ||
        e.stem_stride < 1 || e.stem_pad < 0 || e.pool_k < 1 || e.pool_stride < 1 || e.pool_pad < 0) {
        fail("unsupported " + name + "_backbone.meta");
        return false;
    }
    e.gs = gs;
    std::vector<float> data;
    if (!files.read_floats(name + "_backbone.bin", data)) { fail("cannot read " + name + "_backbone.bin"); return false; }
    Cursor take{data};
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    auto dev_copy = [&](const float* src, size_t n) -> float* {
        float* p = dalloc<float>(n);
        if (p && src) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    // weights, then either GroupNorm scale/shift (no conv bias) or a bias
    auto make = [&](DpGnConv& c, int cout, int k, int cin, int stride, int pad) -> bool {
        const float* w = take((size_t)cout * k * k * cin);
        const float* b = nullptr;
        if (gs) {
            if (cout % gs) { fail("GroupNorm group size does not divide the channels"); return false; }
            const float* s = take(cout);
            const float* sb = take(cout);
            if (!take.ok) { fail(name + "_backbone.bin too short"); return false; }
            c.gn_s = dev_copy(s, cout);
            c.gn_b = dev_copy(sb, cout);
            c.groups = cout / gs;
        } else {
            b = take(cout);
        }
        if (!take.ok) { fail(name + "_backbone.bin too short"); return false; }
        return make_dev_conv(c.conv, w, b, cout, k, cin, stride, pad, int8, alloc, &n_int8_);
    };
    if (!make(e.stem, e.stem_out, e.stem_k, in_ch, e.stem_stride, e.stem_pad)) return false;
    e.blocks.resize(bm.size());
    int prev = e.stem_out;
    for (size_t i = 0; i < bm.size(); ++i) {
        DpBasicBlock& blk = e.blocks[i];
        if (bm[i].cin != prev || bm[i].cout < 1 || bm[i].stride < 1 || (bm[i].has_down != 0 && bm[i].has_down != 1) ||
            (!bm[i].has_down && (bm[i].stride != 1 || bm[i].cin != bm[i].cout))) {
            fail("inconsistent backbone block table");
            return false;
        }
        blk.has_down = bm[i].has_down != 0;
        if (!make(blk.c1, bm[i].cout, 3, bm[i].cin, bm[i].stride, 1)) return false;
        if (!make(blk.c2, bm[i].cout, 3, bm[i].cout, 1, 1)) return false;
        if (blk.has_down && !make(blk.down, bm[i].cout, 1, bm[i].cin, bm[i].stride, 0)) return false;
        prev = bm[i].cout;
    }
    if (!take.done()) { fail(name + "_backbone.bin size does not match its meta"); return false; }
    e.C = prev;

    // feature map size for the (cropped) input the encoder sees
    const int in_h = cfg_.crop_h > 0 ? cfg_.crop_h : cfg_.img_h, in_w = cfg_.crop_w > 0 ? cfg_.crop_w : cfg_.img_w;
    int h = conv_out_size(in_h, e.stem_k, e.stem_stride, e.stem_pad), w = conv_out_size(in_w, e.stem_k, e.stem_stride, e.stem_pad);
    h = conv_out_size(h, e.pool_k, e.pool_stride, e.pool_pad);
    w = conv_out_size(w, e.pool_k, e.pool_stride, e.pool_pad);
    for (const DpBasicBlock& b : e.blocks) {
        h = conv_out_size(h, 3, b.c1.conv.stride, 1);
        w = conv_out_size(w, 3, b.c1.conv.stride, 1);
    }
    if (h <= 0 || w <= 0) { fail("image too small for the backbone"); return false; }
    e.fh = h;
    e.fw = w;

    std::vector<float> head;
    if (!files.read_floats(name + ".bin", head)) { fail("cannot read " + name + ".bin"); return false; }
    Cursor t2{head};
    const int K = cfg_.num_keypoints, F2 = 2 * K, C = e.C;
    const float* kw = t2((size_t)K * C);
    const float* kb = t2(K);
    const float* ow = t2((size_t)F2 * F2);
    const float* ob = t2(F2);
    if (!t2.done()) { fail(name + ".bin size does not match"); return false; }
    if (!upload_linear(e.kp, kw, kb, K, C, false, alloc) || !upload_linear(e.out, ow, ob, F2, F2, false, alloc))
        return false;
    std::vector<float> px, py, grid((size_t)h * w * 2);
    linspace_np(px, -1.0, 1.0, w);
    linspace_np(py, -1.0, 1.0, h);
    for (int y = 0; y < h; ++y)
        for (int x = 0; x < w; ++x) {
            grid[((size_t)y * w + x) * 2 + 0] = px[x];
            grid[((size_t)y * w + x) * 2 + 1] = py[y];
        }
    e.grid = dev_copy(grid.data(), grid.size());
    return err_.empty();
}

// unet.bin in DPUNet1d::load order (src/models/diffusion/unet1d.cpp:18-160).
bool DpPolicy::load_unet(const ModelFiles& files, bool int8) {
    const DpConfigDev& c = cfg_;
    const int ndown = static_cast<int>(c.down_dims.size());
    if (c.down_dims.empty() || ndown > 30 || c.n_groups <= 0 || c.step_embed_dim < 4 || c.step_embed_dim % 2 ||
        !shape_fits({4, c.step_embed_dim, c.step_embed_dim}) || c.kernel_size < 1 || c.kernel_size % 2 == 0 ||
        c.horizon <= 0 || c.horizon % (1 << (ndown - 1)) || !std::isfinite(c.gn_eps) || c.gn_eps <= 0) {
        fail("unsupported U-Net configuration");
        return false;
    }
    for (int width : c.down_dims)
        if (!shape_fits({2, width, c.kernel_size, width}) || width % c.n_groups || !shape_fits({c.horizon, width}) ||
            !shape_fits({2, width, c.cond_dim()})) {
            fail("unsupported U-Net width");
            return false;
        }
    if (c.down_dims[0] % 8) {   // the final block's GroupNorm uses 8 groups (unet1d.cpp:297)
        fail("down_dims[0] must be a multiple of 8");
        return false;
    }
    std::vector<float> data;
    if (!files.read_floats("unet.bin", data)) { fail("cannot read unet.bin"); return false; }
    Cursor take{data};
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    const int A = c.action_dim, D = c.step_embed_dim, CD = c.cond_dim(), k = c.kernel_size;
    std::vector<float> cond_w, cond_b;   // every block's cond linear, stacked
    auto lin = [&](DevLinear& L, int N, int K, bool q) -> bool {
        const float* w = take((size_t)N * K);
        const float* b = take(N);
        if (!take.ok) { fail("unet.bin too short"); return false; }
        return upload_linear(L, w, b, N, K, q, alloc, &n_int8_);
    };
    auto dev_copy = [&](const float* src, size_t n) -> float* {
        float* p = dalloc<float>(n);
        if (p && src) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    auto conv_block = [&](DpConvBlockDev& cb, int cin, int cout, int kk) -> bool {
        cb.cin = cin; cb.cout = cout; cb.k = kk;
        if (!lin(cb.conv, cout, kk * cin, int8)) return false;
        const float* s = take(cout);
        const float* b = take(cout);
        if (!take.ok) { fail("unet.bin too short"); return false; }
        cb.gn_s = dev_copy(s, cout);
        cb.gn_b = dev_copy(b, cout);
        return err_.empty();
    };
    auto res_block = [&](DpResBlockDev& rb, int cin, int cout) -> bool {
        rb.cin = cin; rb.cout = cout;
        if (!conv_block(rb.c1, cin, cout, k)) return false;
        const int nc = c.film_scale ? 2 * cout : cout;
        const float* w = take((size_t)nc * CD);
        const float* b = take(nc);
        if (!take.ok) { fail("unet.bin too short"); return false; }
        rb.film_off = (long long)cond_b.size();
        cond_w.insert(cond_w.end(), w, w + (size_t)nc * CD);
        cond_b.insert(cond_b.end(), b, b + nc);
        if (!conv_block(rb.c2, cout, cout, k)) return false;
        rb.has_res = cin != cout;
        if (rb.has_res && !lin(rb.res, cout, cin, int8)) return false;
        return true;
    };
    if (!lin(step1_, 4 * D, D, false) || !lin(step2_, D, 4 * D, false)) return false;
    std::vector<std::pair<int, int>> in_out;
    in_out.emplace_back(A, c.down_dims[0]);
    for (size_t i = 0; i + 1 < c.down_dims.size(); ++i) in_out.emplace_back(c.down_dims[i], c.down_dims[i + 1]);
    down_.clear();
    down_.resize(in_out.size());
    for (size_t i = 0; i < in_out.size(); ++i) {
        DpDownDev& d = down_[i];
        if (!res_block(d.r1, in_out[i].first, in_out[i].second) || !res_block(d.r2, in_out[i].second, in_out[i].second))
            return false;
        d.has = i + 1 < in_out.size();
        if (d.has && !lin(d.ds, in_out[i].second, 3 * in_out[i].second, int8)) return false;
    }
    const int mid = c.down_dims.back();
    if (!res_block(mid1_, mid, mid) || !res_block(mid2_, mid, mid)) return false;
    up_.clear();
    up_.resize(in_out.size() - 1);
    for (size_t ind = 0; ind + 1 < in_out.size(); ++ind) {
        const std::pair<int, int>& p = in_out[in_out.size() - 1 - ind];
        const int dim_out = p.first, dim_in = p.second;
        DpUpDev& u = up_[ind];
        if (!res_block(u.r1, dim_in * 2, dim_out) || !res_block(u.r2, dim_out, dim_out)) return false;
        u.has = ind < in_out.size() - 1;
        if (u.has) {
            u.uc = dim_out;
            const float* w = take((size_t)dim_out * 4 * dim_out);
            const float* b = take(dim_out);
            if (!take.ok) { fail("unet.bin too short"); return false; }
            u.uw = dev_copy(w, (size_t)dim_out * 4 * dim_out);
            // [Cout][k][Cin] copy for the several-sample kernel
            std::vector<float> wt((size_t)dim_out * 4 * dim_out);
            for (int ci = 0; ci < dim_out; ++ci)
                for (int kt = 0; kt < 4; ++kt)
                    for (int co = 0; co < dim_out; ++co)
                        wt[((size_t)co * 4 + kt) * dim_out + ci] = w[((size_t)ci * 4 + kt) * dim_out + co];
            u.uwt = dev_copy(wt.data(), wt.size());
            u.ub = dev_copy(b, dim_out);
        }
    }
    if (!conv_block(final_block_, c.down_dims[0], c.down_dims[0], k)) return false;
    if (!lin(final_conv_, A, c.down_dims[0], false)) return false;
    if (!take.done()) { fail("unet.bin size does not match diffusion.meta"); return false; }
    film_cols_ = (long long)cond_b.size();
    if (!upload_linear(cond_all_, cond_w.data(), cond_b.data(), (int)film_cols_, CD, false, alloc)) return false;
    return err_.empty();
}

// stats.bin: state min/max, action min/max, per camera image mean/std
// (src/models/diffusion/diffusion_model.cpp:123-162), with the same refusals.
bool DpPolicy::load_stats(const ModelFiles& files) {
    const int sd = cfg_.state_dim, ad = cfg_.action_dim, N = cfg_.n_cams;
    std::vector<float> raw;
    if (!files.read_floats("stats.bin", raw) || raw.size() != (size_t)2 * sd + 2 * ad + (size_t)6 * N) {
        fail("stats.bin missing or wrong size");
        return false;
    }
    for (float v : raw)
        if (!std::isfinite(v)) { fail("non-finite stats"); return false; }
    const float* smin = raw.data();
    const float* smax = smin + sd;
    const float* amin = smax + sd;
    const float* amax = amin + ad;
    const float* img = amax + ad;
    std::vector<float> im((size_t)N * 3), is((size_t)N * 3);
    for (int c = 0; c < N; ++c)
        for (int i = 0; i < 3; ++i) {
            im[(size_t)c * 3 + i] = img[(size_t)c * 6 + i];
            is[(size_t)c * 3 + i] = img[(size_t)c * 6 + 3 + i];
        }
    for (int i = 0; i < sd; ++i) if (smax[i] < smin[i]) { fail("state max < min"); return false; }
    for (int i = 0; i < ad; ++i) if (amax[i] < amin[i]) { fail("action max < min"); return false; }
    for (float v : is) if (v < 0) { fail("negative image std"); return false; }
    bool degenerate = true;
    for (int i = 0; i < ad; ++i) if (amax[i] - amin[i] > 1e-6f) degenerate = false;
    if (degenerate) { fail("degenerate action statistics"); return false; }
    auto up = [&](const float* s, size_t n) {
        float* d = dalloc<float>(n);
        if (d) cudaMemcpy(d, s, n * sizeof(float), cudaMemcpyHostToDevice);
        return d;
    };
    d_smin_ = up(smin, sd); d_smax_ = up(smax, sd);
    d_amin_ = up(amin, ad); d_amax_ = up(amax, ad);
    d_img_mean_ = up(im.data(), im.size()); d_img_std_ = up(is.data(), is.size());
    return err_.empty();
}

bool DpPolicy::alloc_buffers() {
    const DpConfigDev& c = cfg_;
    const int Bm = max_batch_;
    const int S = c.n_obs, N = c.n_cams;
    const int oh = c.crop_h > 0 ? c.crop_h : c.img_h, ow = c.crop_w > 0 ? c.crop_w : c.img_w;
    const long long nframes = (long long)Bm * S * N;
    if (nframes > 65535) { fail("batch too large"); return false; }
    // frames per encoder run: one camera's B*S frames, or all of them with a shared encoder
    const int Fe = c.separate ? Bm * S : Bm * S * N;

    // inputs: frames | state | noise in one buffer (one host-to-device copy)
    const size_t fb = (size_t)Bm * frame_bytes();
    state_off_ = (fb + 255) & ~size_t(255);
    noise_off_ = (state_off_ + sizeof(float) * (size_t)Bm * S * c.state_dim + 255) & ~size_t(255);
    in_bytes_ = noise_off_ + sizeof(float) * (size_t)Bm * noise_floats();
    d_in_ = dalloc<uint8_t>(in_bytes_);
    if (!d_in_) return false;
    d_frames_ = d_in_;
    d_state_ = reinterpret_cast<float*>(d_in_ + state_off_);
    d_noise_ = reinterpret_cast<float*>(d_in_ + noise_off_);
    d_img_f_ = dalloc<float>((size_t)nframes * oh * ow * 3);

    // backbone activations / scratch: the largest map over all encoders
    size_t max_act = 0, col_i8 = 0, col_f = 0, rows = 0, max_gn = 0;
    int nslots = 0;
    for (const DpEncoderDev& e : enc_) {
        auto visit = [&](const DevConv& cv, int H, int W) {
            size_t a, b, r;
            conv_scratch_needs(cv, Fe, H, W, explicit_convs_, &a, &b, &r);
            col_i8 = std::max(col_i8, a);
            col_f = std::max(col_f, b);
            rows = std::max(rows, r);
            const int Ho = conv_out_size(H, cv.k, cv.stride, cv.pad), Wo = conv_out_size(W, cv.k, cv.stride, cv.pad);
            max_act = std::max(max_act, (size_t)Fe * Ho * Wo * cv.cout);
            max_gn = std::max(max_gn, (size_t)Fe * cv.cout);
        };
        visit(e.stem.conv, oh, ow);
        int h = conv_out_size(oh, e.stem_k, e.stem_stride, e.stem_pad), w = conv_out_size(ow, e.stem_k, e.stem_stride, e.stem_pad);
        h = conv_out_size(h, e.pool_k, e.pool_stride, e.pool_pad);
        w = conv_out_size(w, e.pool_k, e.pool_stride, e.pool_pad);
        for (const DpBasicBlock& b : e.blocks) {
            visit(b.c1.conv, h, w);
            const int h2 = conv_out_size(h, 3, b.c1.conv.stride, 1), w2 = conv_out_size(w, 3, b.c1.conv.stride, 1);
            visit(b.c2.conv, h2, w2);
            if (b.has_down) visit(b.down.conv, h, w);
            h = h2;
            w = w2;
        }
        nslots = std::max(nslots, 2 + 2 * static_cast<int>(e.blocks.size()));
    }
    const int n_runs = c.separate ? N : 1;
    n_slots_ = nslots * Fe * n_runs;
    d_ba_ = dalloc<float>(max_act);
    if (debug_stage_ >= 0) {
        d_debug_ = dalloc<float>(max_act);
        debug_cap_ = max_act;
    }
    d_bb_ = dalloc<float>(max_act);
    d_bc_ = dalloc<float>(max_act);
    d_bres_ = dalloc<float>(max_act);
    d_gnA_ = dalloc<float>(std::max(max_gn, (size_t)1));
    d_gnB_ = dalloc<float>(std::max(max_gn, (size_t)1));
    if (col_i8) conv_s_.col = dalloc<int8_t>(col_i8);
    if (col_f) conv_s_.col_f = dalloc<float>(col_f);
    conv_s_.col_scale = dalloc<float>(std::max(rows, (size_t)Fe));
    // per-row absmax arena of the U-Net (after the encoders' slots, zeroed with them):
    // per step at most 2 per res block + 3 (downsample, concat, upsample) per level
    const long long per_step_uses = 2LL * (2 * (long long)down_.size() + 2 + 2 * (long long)up_.size()) +
                                    3LL * (long long)down_.size() + 2;
    rm_cap_ = per_step_uses * num_steps() * (long long)Bm * c.horizon;
    if (n_slots_ + rm_cap_ > INT_MAX) { fail("batch too large"); return false; }
    d_slots_ = dalloc<unsigned int>(n_slots_ + rm_cap_);
    d_rowmax_ = d_slots_ ? d_slots_ + n_slots_ : nullptr;
    size_t kp = 0;
    for (const DpEncoderDev& e : enc_) kp = std::max(kp, (size_t)Fe * e.fh * e.fw * c.num_keypoints);
    d_kp_ = dalloc<float>(kp);
    d_feat_ = dalloc<float>((size_t)nframes * c.cam_feature_dim());

    const int steps = num_steps(), CD = c.cond_dim(), D = c.step_embed_dim;
    d_stepfeat_ = dalloc<float>((size_t)steps * D);
    d_gcond_ = dalloc<float>((size_t)Bm * c.global_cond_dim());
    d_gm_ = dalloc<float>((size_t)steps * Bm * CD);
    d_film_ = dalloc<float>((size_t)steps * Bm * film_cols_);

    // U-Net: the widest [B*T][C] map over all levels (the concat doubles it)
    size_t act = (size_t)c.horizon * c.action_dim, qcols = 16, colf = 1;
    int T = c.horizon;
    auto need = [&](int t, int ch, int k) {
        act = std::max(act, (size_t)t * ch);
        qcols = std::max(qcols, (size_t)round16((long long)k * ch));
        colf = std::max(colf, (size_t)t * k * ch);
    };
    d_skip_.clear();
    for (size_t i = 0; i < down_.size(); ++i) {
        const DpDownDev& d = down_[i];
        need(T, d.r1.cin, c.kernel_size);
        need(T, d.r1.cout, c.kernel_size);
        d_skip_.push_back(dalloc<float>((size_t)Bm * T * d.r2.cout));
        if (d.has) {
            need(T, d.r2.cout, 3);
            T = (T + 2 - 3) / 2 + 1;
        }
    }
    need(T, mid1_.cout, c.kernel_size);
    for (const DpUpDev& u : up_) {
        need(T, u.r1.cin, c.kernel_size);
        need(T, u.r1.cout, c.kernel_size);
        if (u.has) T = (T - 1) * 2 - 2 + 4;
    }
    need(T, final_block_.cin, c.kernel_size);
    if (T != c.horizon) { fail("U-Net does not return to the horizon"); return false; }
    if ((size_t)c.kernel_size * std::max(act, (size_t)1) == 0) return false;
    const size_t A = (size_t)Bm * act;
    d_x_ = dalloc<float>(A);
    d_a_ = dalloc<float>(A);
    d_b_ = dalloc<float>(A);
    d_cat_ = dalloc<float>(A);
    d_h_ = dalloc<float>(A);
    d_o_ = dalloc<float>(A);
    d_r_ = dalloc<float>(A);
    const size_t qrows = (size_t)Bm * c.horizon;
    d_q_ = dalloc<int8_t>(qrows * qcols);
    d_q2_ = dalloc<int8_t>(qrows * qcols);
    d_qs_ = dalloc<float>(qrows);
    d_qs2_ = dalloc<float>(qrows);
    {
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_);
        for (DpSplitWs* w : {&ws_main_, &ws_side_}) {
            w->elems = (long long)sms * 128 * 128;   // one CTA per SM, 128 rows x 128 columns each
            w->n_counters = 4096;
            w->ws = dalloc<int32_t>((size_t)w->elems);
            w->counters = dalloc<unsigned int>(w->n_counters);
            if (w->counters) cudaMemset(w->counters, 0, sizeof(unsigned int) * w->n_counters);
        }
    }
    d_colf_ = dalloc<float>((size_t)Bm * colf);
    d_sample_ = dalloc<float>((size_t)Bm * c.horizon * c.action_dim);
    d_eps_ = dalloc<float>((size_t)Bm * c.horizon * c.action_dim);
    d_actions_ = dalloc<float>((size_t)Bm * c.n_action_steps * c.action_dim);
    if (qcols * sizeof(float) > 200 * 1024) { fail("U-Net conv rows too wide (k*C > 51200)"); return false; }
    return err_.empty();
}

// The timestep part of the U-Net's global feature for every step of the
// ladder, once at load: sinusoidal embedding (host libm, as DPUNet1d::step_embedding,
// src/models/diffusion/unet1d.cpp:217-228) -> Linear -> Mish -> Linear.
bool DpPolicy::step_features() {
    const int D = cfg_.step_embed_dim, half = D / 2, steps = num_steps();
    std::vector<float> emb((size_t)steps * D);
    const float sc = std::log(10000.0f) / static_cast<float>(half - 1);
    for (int s = 0; s < steps; ++s) {
        const int t = timesteps_[s];
        for (int i = 0; i < half; ++i) {
            const float f = static_cast<float>(t) * std::exp(-static_cast<float>(i) * sc);
            emb[(size_t)s * D + i] = std::sin(f);
            emb[(size_t)s * D + half + i] = std::cos(f);
        }
    }
    float* d_emb = dalloc<float>(emb.size());
    float* d_wide = dalloc<float>((size_t)steps * 4 * D);
    if (!d_emb || !d_wide) return false;
    cudaMemcpy(d_emb, emb.data(), sizeof(float) * emb.size(), cudaMemcpyHostToDevice);
    cudaError_t e = linear_f32(d_emb, D, step1_.W, step1_.bias, d_wide, 4 * D, steps, 4 * D, D, nullptr, nullptr, stream_);
    if (e == cudaSuccess) e = activation(kActMish, d_wide, d_wide, nullptr, (long long)steps * 4 * D, stream_);
    if (e == cudaSuccess)
        e = linear_f32(d_wide, 4 * D, step2_.W, step2_.bias, d_stepfeat_, D, steps, D, 4 * D, nullptr, nullptr, stream_);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream_);
    if (e != cudaSuccess) { fail("timestep features failed"); return false; }
    return true;
}

bool DpPolicy::load(const std::string& dir, int max_batch) {
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
    debug_stage_ = env_int("VLA_DP_DEBUG_STAGE", -1);
    i8_clip_ = env_clip();
    // DIFFUSION_INT8: bit 1 the U-Net's GEMM layers, bit 2 the backbone convs
    // (src/models/diffusion/diffusion_model.cpp:110-121)
    const int i8 = env_int("DIFFUSION_INT8", 0);

    // a converted directory or a vla.simd GGUF (src/models/diffusion/diffusion_model.cpp:25-27 mounts it the same way)
    ModelFiles files;
    if (!files.open(dir)) { fail(files.error()); return false; }
    if (!load_meta(files) || !init_schedule()) return false;
    enc_.resize(cfg_.separate ? cfg_.n_cams : 1);
    for (size_t i = 0; i < enc_.size(); ++i)
        if (!load_encoder(files, static_cast<int>(i), (i8 & 2) != 0)) return false;
    for (const DpEncoderDev& e : enc_)
        if (e.C != enc_[0].C || e.fh != enc_[0].fh || e.fw != enc_[0].fw) { fail("encoders differ in shape"); return false; }
    if (!load_unet(files, (i8 & 1) != 0)) return false;
    if (!load_stats(files)) return false;
    if (!alloc_buffers()) return false;
    if (env_int("DP_PROFILE", 0) >= 1)
        std::fprintf(stderr, "[diffusion] int8 GEMMs on device: %d (DIFFUSION_INT8=%d)\n", n_int8_, i8);

    if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&side_, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_join_, cudaEventDisableTiming) != cudaSuccess) {
        fail("streams / events");
        return false;
    }
    if (cudaMallocHost(&h_pinned_, sizeof(float) * (size_t)max_batch_ * cfg_.n_action_steps * cfg_.action_dim) !=
            cudaSuccess ||
        cudaMallocHost(&h_status_pinned_, sizeof(int)) != cudaSuccess) {
        fail("pinned host buffers");
        return false;
    }
    d_status_ = static_cast<int*>(device_status_address());
    if (!d_status_) { fail("device status word"); return false; }
    tail_n_ = cfg_.cond_dim() % 8;
    if (tail_n_) {
        d_tail_ = dalloc<float>((size_t)max_batch_ * tail_n_);
        if (!d_tail_) return false;
    }
    graphs_.assign((size_t)max_batch_ * 2, nullptr);
    cudaMemset(d_in_, 0, in_bytes_);
    cudaDeviceSynchronize();
    if (!step_features()) return false;
    // one eager batch validates every launch before capture
    if (forward(1, stream_, true) != cudaSuccess || cudaStreamSynchronize(stream_) != cudaSuccess) {
        fail("warm-up step failed");
        return false;
    }
    if (device_status_take() != 0) { fail("device status error in warm-up"); return false; }
    return true;
}

cudaStream_t DpPolicy::fork(cudaStream_t st) {
    if (cudaEventRecord(ev_fork_, st) != cudaSuccess || cudaStreamWaitEvent(side_, ev_fork_, 0) != cudaSuccess)
        return nullptr;
    return side_;
}

cudaError_t DpPolicy::join(cudaStream_t st) {
    VSB_TRY(cudaEventRecord(ev_join_, side_));
    return cudaStreamWaitEvent(st, ev_join_, 0);
}

// conv (no bias) -> GroupNorm (per frame, eps 1e-5 as ResNetBackbone::forward,
// src/models/act/resnet_backbone.cpp:217-220) with the epilogue `epi`, or, for
// a backbone without GroupNorm, the conv's own epilogue. amax_out receives the
// per-frame absmax of the output (the next int8 conv's scale).
cudaError_t DpPolicy::run_gn_conv(const DpGnConv& c, const float* in, int F, int H, int W, float* out, int epi,
                                  const float* res, const unsigned int* amax_in, unsigned int* amax_out,
                                  cudaStream_t st) {
    if (!c.gn_s) {
        const int mode = (epi & kGnAdd) ? kEpiAddRelu : (epi & kGnRelu) ? kEpiRelu : 0;
        return conv2d_dev(c.conv, in, F, H, W, out, mode, res, amax_in, amax_out, i8_clip_, explicit_convs_, conv_s_,
                          st);
    }
    VSB_TRY(conv2d_dev(c.conv, in, F, H, W, out, 0, nullptr, amax_in, nullptr, i8_clip_, explicit_convs_, conv_s_, st));
    const int Ho = conv_out_size(H, c.conv.k, c.conv.stride, c.conv.pad);
    const int Wo = conv_out_size(W, c.conv.k, c.conv.stride, c.conv.pad);
    const int C = c.conv.cout;
    VSB_TRY(gn_affine(out, F, Ho * Wo, C, C, c.groups, 1e-5f, c.gn_s, c.gn_b, d_gnA_, d_gnB_, st));
    return gn_apply(out, d_gnA_, d_gnB_, out, F, Ho * Wo, C, C, epi, res, amax_out, st);
}

// DPRgbEncoder::forward (src/models/diffusion/rgb_encoder.cpp:70-93) over F
// frames: ResNet (resnet_backbone.cpp:211-315) -> 1x1 keypoint conv -> spatial
// soft-argmax -> feat [F][2K]. `slots`: [pool | mid0 | out0 | mid1 | out1 ...],
// F per-frame absmax slots each; img_slot: the frames' own absmax.
cudaError_t DpPolicy::tap_stage(int stage, const float* map, size_t n, cudaStream_t st) {
    if (stage != debug_stage_ || !d_debug_ || n > debug_cap_) return cudaSuccess;
    debug_n_ = n;
    return cudaMemcpyAsync(d_debug_, map, n * sizeof(float), cudaMemcpyDeviceToDevice, st);
}

cudaError_t DpPolicy::run_encoder(const DpEncoderDev& e, const float* img, int F, unsigned int* slots, float* feat,
                                  bool tap, cudaStream_t st) {
    const int in_h = cfg_.crop_h > 0 ? cfg_.crop_h : cfg_.img_h, in_w = cfg_.crop_w > 0 ? cfg_.crop_w : cfg_.img_w;
    const unsigned int* img_slot = slots - F;   // the frames' absmax sits just before this run's slots
    int h = conv_out_size(in_h, e.stem_k, e.stem_stride, e.stem_pad), w = conv_out_size(in_w, e.stem_k, e.stem_stride, e.stem_pad);
    VSB_TRY(run_gn_conv(e.stem, img, F, in_h, in_w, d_ba_, 0, nullptr, img_slot, nullptr, st));
    if (tap) VSB_TRY(tap_stage(0, d_ba_, (size_t)F * h * w * e.stem_out, st));
    const int ph = conv_out_size(h, e.pool_k, e.pool_stride, e.pool_pad), pw = conv_out_size(w, e.pool_k, e.pool_stride, e.pool_pad);
    unsigned int* in_slot = slots;
    VSB_TRY(maxpool_relu(d_ba_, d_bb_, F, h, w, e.stem_out, e.pool_k, e.pool_stride, e.pool_pad, ph, pw, in_slot, st));
    h = ph;
    w = pw;
    if (tap) VSB_TRY(tap_stage(1, d_bb_, (size_t)F * h * w * e.stem_out, st));
    float *b = d_bb_, *a = d_ba_, *c = d_bc_;
    for (size_t i = 0; i < e.blocks.size(); ++i) {
        const DpBasicBlock& blk = e.blocks[i];
        unsigned int* mid_slot = slots + (1 + 2 * i) * F;
        unsigned int* out_slot = mid_slot + F;
        const int oh = conv_out_size(h, 3, blk.c1.conv.stride, 1), ow = conv_out_size(w, 3, blk.c1.conv.stride, 1);
        const float* idn = b;
        if (blk.has_down) {
            VSB_TRY(run_gn_conv(blk.down, b, F, h, w, d_bres_, 0, nullptr, in_slot, nullptr, st));
            idn = d_bres_;
        }
        VSB_TRY(run_gn_conv(blk.c1, b, F, h, w, a, kGnRelu, nullptr, in_slot, mid_slot, st));
        VSB_TRY(run_gn_conv(blk.c2, a, F, oh, ow, c, kGnAdd | kGnRelu, idn, mid_slot, out_slot, st));
        std::swap(b, c);
        h = oh;
        w = ow;
        in_slot = out_slot;
        if (tap) VSB_TRY(tap_stage(2 + static_cast<int>(i), b, (size_t)F * h * w * blk.c1.conv.cout, st));
    }
    const int npx = e.fh * e.fw, K = cfg_.num_keypoints;
    VSB_TRY(linear_f32(b, e.C, e.kp.W, e.kp.bias, d_kp_, K, F * npx, K, e.C, nullptr, nullptr, st));
    return spatial_softmax_f(d_kp_, e.grid, feat, F, npx, K, st);
}

cudaError_t DpPolicy::gemm_rows(const DevLinear& l, const int8_t* q, const float* qs, const float* xf, int M,
                                float* out, const DpSplitWs& ws, cudaStream_t st) {
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
        a.ldo = l.N;
        a.ascale = qs;
        a.wscale = l.wscale;
        a.bias = l.bias;
        a.static_weights = true;   // uploaded once at load
        a.splitk_ws = ws.ws;
        a.splitk_ws_elems = ws.elems;
        a.splitk_counters = ws.counters;
        a.splitk_counters_n = ws.n_counters;
        return gemm_i8(a, st);
    }
    return gemm_f32(xf, l.K, l.W, l.K, l.bias, out, l.N, nullptr, 0, M, l.N, l.K, 0, nullptr, 1, st);
}

// Per-row absmax slots of one query batch: handed out in a fixed order by
// forward(), so a captured graph keeps its addresses; the step prologue zeroes
// the whole arena (it follows the encoders' slots in d_slots_).
unsigned int* DpPolicy::rm_take(long long n) {
    if (rm_used_ + n > rm_cap_) {
        rm_overflow_ = true;
        return nullptr;
    }
    unsigned int* p = d_rowmax_ + rm_used_;
    rm_used_ += n;
    return p;
}

// A Conv1d as the reference's nn::Linear over the im2col'd taps
// (DPConvBlock::forward, src/models/diffusion/unet1d.cpp:185-191): int8 layers
// quantize each im2col row (dense_linear_i8) with the row scales that rm_x
// (the per-time-step absmax of x) determines; fp32 layers take the fp32 rows.
// rm_out (optional): per-row absmax of the output, for the next conv.
cudaError_t DpPolicy::im2col_gemm(const DevLinear& l, const float* x, const unsigned int* rm_x, int B, int T, int C,
                                  int k, int stride, int pad, int Tout, float* out, unsigned int* rm_out,
                                  cudaStream_t st, bool side) {
    // side: the residual 1x1 conv on the forked stream, with its own A buffer
    // and split-K workspace
    int8_t* q = side ? d_q2_ : d_q_;
    float* qs = side ? d_qs2_ : d_qs_;
    const DpSplitWs& ws = side ? ws_side_ : ws_main_;
    if (l.int8) {
        const long long ldq = round16((long long)k * C);
        GemmI8Args a;
        a.A = q;
        a.lda = ldq;
        a.B = l.Wq;
        a.ldb = l.ldw;
        a.M = B * Tout;
        a.N = l.N;
        a.K = l.K;
        a.out = out;
        a.ldo = l.N;
        a.ascale = qs;
        a.wscale = l.wscale;
        a.bias = l.bias;
        a.amax = rm_out;
        a.amax_rows = 1;
        a.static_weights = true;   // uploaded once at load
        a.splitk_ws = ws.ws;
        a.splitk_ws_elems = ws.elems;
        a.splitk_counters = ws.counters;
        a.splitk_counters_n = ws.n_counters;
        // the GEMM quantizes the im2col rows itself where it can (one launch
        // less), except where a few short rows take the GEMV; else
        // im2col1d_q8w writes them first
        const bool gemv = gemm_i8_takes_gemv(a);
        a.im_x = x;
        a.im_rowmax = rm_x;
        a.im_T = T;
        a.im_C = C;
        a.im_k = k;
        a.im_stride = stride;
        a.im_pad = pad;
        a.im_Tout = Tout;
        if (!gemv && gemm_i8_im2col_supported(a)) return gemm_i8(a, st);
        a.im_x = nullptr;
        VSB_TRY(im2col1d_q8w(x, B, T, C, k, stride, pad, Tout, rm_x, q, ldq, qs, st));
        return gemm_i8(a, st);
    }
    if (side) return gemm_rows(l, nullptr, nullptr, x, B * T, out, ws, st);
    VSB_TRY(im2col1d_f32x(x, B, T, C, C, k, stride, pad, Tout, d_colf_, st));
    return gemm_f32(d_colf_, l.K, l.W, l.K, l.bias, out, l.N, nullptr, 0, B * Tout, l.N, l.K, 0, rm_out, 1, st);
}

// DPResBlock::forward (src/models/diffusion/unet1d.cpp:193-215) for B samples:
// conv1 -> GroupNorm -> Mish -> FiLM (this step's cond vector), conv2 ->
// GroupNorm -> Mish -> + residual (1x1 conv when the width changes, on the side
// stream, else identity). Returns the output's per-row absmax slots.
unsigned int* DpPolicy::res_block(const DpResBlockDev& rb, const float* x, const unsigned int* rm_x, int B, int T,
                                  int step, float* out, cudaStream_t st, cudaError_t* err) {
    const int k = cfg_.kernel_size, G = cfg_.n_groups;
    const float* film = d_film_ + (size_t)step * B * film_cols_ + rb.film_off;
    unsigned int* rm_h = rm_take((long long)B * T);
    unsigned int* rm_o = rm_take((long long)B * T);
    cudaError_t e = rm_h && rm_o ? cudaSuccess : cudaErrorInvalidValue;
    const float* resp = x;
    if (e == cudaSuccess && rb.has_res) {
        cudaStream_t sd = fork(st);
        if (!sd) e = cudaErrorUnknown;
        // a 1x1 conv: the one-tap im2col, whose row scales come from x's
        // absmax slots (the same per-row quantization as the reference's
        // Linear over x, res.forward in src/models/diffusion/unet1d.cpp:188-191)
        if (e == cudaSuccess) e = im2col_gemm(rb.res, x, rm_x, B, T, rb.cin, 1, 1, 0, T, d_r_, nullptr, sd, true);
        resp = d_r_;
    }
    // conv1 into d_o_ and its GroupNorm out of place into d_h_ (lets unet_gn
    // spread each group over several CTAs)
    if (e == cudaSuccess)
        e = im2col_gemm(rb.c1.conv, x, rm_x, B, T, rb.cin, k, 1, k / 2, T, d_o_, nullptr, st);
    if (e == cudaSuccess)
        e = unet_gn(d_o_, B, T, rb.cout, G, cfg_.gn_eps, rb.c1.gn_s, rb.c1.gn_b,
                    cfg_.film_scale ? kUgFilmScale : kUgFilmBias, film, film_cols_, nullptr, d_h_, rm_h, st);
    if (e == cudaSuccess)
        e = im2col_gemm(rb.c2.conv, d_h_, rm_h, B, T, rb.cout, k, 1, k / 2, T, d_o_, nullptr, st);
    if (e == cudaSuccess && rb.has_res) e = join(st);
    if (e == cudaSuccess)
        e = unet_gn(d_o_, B, T, rb.cout, G, cfg_.gn_eps, rb.c2.gn_s, rb.c2.gn_b, kUgRes, nullptr, 0, resp, out, rm_o,
                    st);
    *err = e;
    return rm_o;
}

// DPUNet1d::forward (src/models/diffusion/unet1d.cpp:230-303) on d_sample_ -> d_eps_.
cudaError_t DpPolicy::unet(int B, int step, cudaStream_t st) {
    int T = cfg_.horizon;
    const float* x = d_sample_;
    const unsigned int* rm = nullptr;   // the sample's rows are action_dim wide: scanned directly
    cudaError_t e = cudaSuccess;
    std::vector<int> skipC;
    std::vector<unsigned int*> skip_rm;
    for (size_t i = 0; i < down_.size(); ++i) {
        const DpDownDev& d = down_[i];
        const unsigned int* rm_a = res_block(d.r1, x, rm, B, T, step, d_a_, st, &e);
        VSB_TRY(e);
        unsigned int* rm_s = res_block(d.r2, d_a_, rm_a, B, T, step, d_skip_[i], st, &e);
        VSB_TRY(e);
        skipC.push_back(d.r2.cout);
        skip_rm.push_back(rm_s);
        if (d.has) {
            const int Tout = (T + 2 - 3) / 2 + 1;
            unsigned int* rm_ds = rm_take((long long)B * Tout);
            if (!rm_ds) return cudaErrorInvalidValue;
            VSB_TRY(im2col_gemm(d.ds, d_skip_[i], rm_s, B, T, d.r2.cout, 3, 2, 1, Tout, d_x_, rm_ds, st));
            T = Tout;
            x = d_x_;
            rm = rm_ds;
        } else {
            x = d_skip_[i];
            rm = rm_s;
        }
    }
    const unsigned int* rm_m = res_block(mid1_, x, rm, B, T, step, d_a_, st, &e);
    VSB_TRY(e);
    rm = res_block(mid2_, d_a_, rm_m, B, T, step, d_b_, st, &e);
    VSB_TRY(e);
    x = d_b_;
    int C = mid2_.cout;
    for (size_t ind = 0; ind < up_.size(); ++ind) {
        const DpUpDev& u = up_[ind];
        const size_t si = down_.size() - 1 - ind;
        unsigned int* rm_cat = rm_take((long long)B * T);
        if (!rm_cat) return cudaErrorInvalidValue;
        VSB_TRY(concat_channels(x, C, d_skip_[si], skipC[si], d_cat_, B, T, rm_cat, st));
        const unsigned int* rm_a = res_block(u.r1, d_cat_, rm_cat, B, T, step, d_a_, st, &e);
        VSB_TRY(e);
        rm = res_block(u.r2, d_a_, rm_a, B, T, step, d_b_, st, &e);
        VSB_TRY(e);
        C = u.r2.cout;
        if (u.has) {
            const int Tout = (T - 1) * 2 - 2 + 4;
            unsigned int* rm_u = rm_take((long long)B * Tout);
            if (!rm_u) return cudaErrorInvalidValue;
            VSB_TRY(conv_transpose1d_f(d_b_, u.uw, u.uwt, u.ub, d_x_, B, T, C, u.uc, 4, 2, 1, rm_u, st));
            T = Tout;
            C = u.uc;
            x = d_x_;
            rm = rm_u;
        } else {
            x = d_b_;
        }
    }
    // final block: Conv1d -> GroupNorm (8 groups, unet1d.cpp:297) -> Mish, then the 1x1 fp32 conv
    const DpConvBlockDev& fb = final_block_;
    VSB_TRY(im2col_gemm(fb.conv, x, rm, B, T, fb.cin, fb.k, 1, fb.k / 2, T, d_o_, nullptr, st));
    VSB_TRY(unet_gn(d_o_, B, T, fb.cout, 8, cfg_.gn_eps, fb.gn_s, fb.gn_b, kUgMish, nullptr, 0, nullptr, d_h_,
                    nullptr, st));
    return linear_f32(d_h_, fb.cout, final_conv_.W, final_conv_.bias, d_eps_, cfg_.action_dim, B * T,
                      cfg_.action_dim, fb.cout, nullptr, nullptr, st);
}

cudaError_t DpPolicy::forward(int B, cudaStream_t st, bool unnormalize) {
    const DpConfigDev& c = cfg_;
    if (B < 1 || B > max_batch_) return cudaErrorInvalidValue;
    const int S = c.n_obs, N = c.n_cams, BS = B * S, F2 = c.cam_feature_dim();
    const int oh = c.crop_h > 0 ? c.crop_h : c.img_h, ow = c.crop_w > 0 ? c.crop_w : c.img_w;
    const int HA = c.horizon * c.action_dim;
    rm_used_ = 0;
    rm_overflow_ = false;
    VSB_TRY(dp_prologue(d_slots_, n_slots_ + static_cast<int>(rm_cap_), d_state_, B, S, c.state_dim, d_smin_, d_smax_,
                        kNormEps, d_gcond_, c.per_step(), d_noise_, (long long)noise_floats(), HA, d_sample_, st));
    // center crop offsets as torchvision's CenterCrop (diffusion_model.cpp:176-178)
    const int dh = c.img_h - oh, dw = c.img_w - ow;
    const int top = dh / 2 + ((dh & 3) == 3), left = dw / 2 + ((dw & 3) == 3);
    // absmax slots, per encoder run of Fr frames: [frames | pool | mid0 | out0 | ...]
    const int runs = c.separate ? N : 1;
    const int Fr = c.separate ? BS : BS * N;
    const int per_run = 1 + 2 * static_cast<int>(enc_[0].blocks.size());
    const long long run_stride = (long long)(1 + per_run) * Fr;
    if (run_stride * runs > n_slots_) return cudaErrorInvalidValue;
    VSB_TRY(dp_preprocess(d_frames_, B, S, N, c.img_h, c.img_w, top, left, oh, ow, d_img_mean_, d_img_std_, kNormEps,
                          d_img_f_, d_slots_, Fr, run_stride, st));
    for (int r = 0; r < runs; ++r) {
        unsigned int* base = d_slots_ + r * run_stride;
        const float* img = d_img_f_ + (size_t)r * Fr * oh * ow * 3;
        VSB_TRY(run_encoder(enc_[r], img, Fr, base + Fr, d_feat_ + (size_t)r * Fr * F2, r == 0, st));
    }
    // output projection + ReLU per camera, into the global conditioning rows (b, s)
    for (int cam = 0; cam < N; ++cam) {
        const DpEncoderDev& e = enc_[c.separate ? cam : 0];
        float* dst = d_gcond_ + c.state_dim + (size_t)cam * F2;
        VSB_TRY(linear_f32(d_feat_ + (size_t)cam * BS * F2, F2, e.out.W, e.out.bias, dst, c.per_step(), BS, F2, F2,
                           nullptr, nullptr, st));
        VSB_TRY(relu_rows(dst, BS, F2, c.per_step(), st));
    }
    const int steps = num_steps(), CD = c.cond_dim(), D = c.step_embed_dim;
    if (tail_n_) {
        // the cond input's scalar Mish tail, with the host library's functions restated on the device
        VSB_TRY(dp_mish_tail(d_gcond_, c.global_cond_dim(), tail_n_, B, d_tail_, st));
    }
    VSB_TRY(dp_cond_input(d_stepfeat_, steps, D, d_gcond_, d_tail_, B, CD, d_gm_, st));
    VSB_TRY(linear_f32(d_gm_, CD, cond_all_.W, cond_all_.bias, d_film_, film_cols_, steps * B, (int)film_cols_, CD,
                       nullptr, nullptr, st));
    const int Ntrain = c.num_train_timesteps;
    for (int i = 0; i < steps; ++i) {
        VSB_TRY(unet(B, i, st));
        // DPNoiseScheduler::step constants (src/models/diffusion/scheduler.cpp:76-101)
        const int t = timesteps_[i];
        int prev_t;
        if (!c.ddim) prev_t = (i + 1 < steps) ? timesteps_[i + 1] : -1;
        else prev_t = t - Ntrain / c.num_inference_steps;
        const double ap = alphas_cumprod_[t];
        const double app = prev_t >= 0 ? alphas_cumprod_[prev_t] : 1.0;
        const double bp = 1.0 - ap;
        DdStepConsts k{};
        k.sqrt_ap = std::sqrt(ap);
        k.sqrt_bp = std::sqrt(bp);
        k.clip = c.clip_sample ? 1 : 0;
        k.lo = -(double)c.clip_sample_range;
        k.hi = (double)c.clip_sample_range;
        const float* nz = nullptr;
        if (!c.ddim) {
            const double bpp = 1.0 - app, cur_a = ap / app, cur_b = 1.0 - cur_a;
            k.ddpm = 1;
            k.a = (std::sqrt(app) * cur_b) / bp;
            k.b = std::sqrt(cur_a) * bpp / bp;
            k.var = t > 0 ? std::sqrt(std::max((1.0 - app) / (1.0 - ap) * cur_b, 1e-20)) : 0.0;
            if (t > 0) nz = d_noise_ + (size_t)(i + 1) * HA;
        } else {
            k.ddpm = 0;
            k.a = std::sqrt(app);
            k.b = std::sqrt(std::max(0.0, 1.0 - app));
        }
        VSB_TRY(dp_sched_step(d_sample_, d_eps_, nz, (long long)noise_floats(), B, HA, k, st));
    }
    if (rm_overflow_) return cudaErrorInvalidValue;
    return dp_actions(d_sample_, B, c.horizon, c.action_dim, c.n_obs - 1, c.n_action_steps,
                      unnormalize ? d_amin_ : nullptr, d_amax_, kNormEps, d_actions_, st);
}

cudaError_t DpPolicy::enqueue(int B, cudaStream_t st, bool unnormalize) {
    if (B < 1 || B > max_batch_) return cudaErrorInvalidValue;
    last_batch_ = B;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device_) cudaSetDevice(device_);
    cudaError_t e = cudaSuccess;
    if (!use_graph_) {
        e = forward(B, st, unnormalize);
    } else {
        cudaGraphExec_t& g = graphs_[(size_t)(B - 1) * 2 + (unnormalize ? 1 : 0)];
        if (!g) {
            cudaGraph_t gr = nullptr;
            e = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal);
            if (e == cudaSuccess) {
                const cudaError_t fe = forward(B, stream_, unnormalize);
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
        }
        if (e == cudaSuccess) e = cudaGraphLaunch(g, st);
    }
    if (prev != device_) cudaSetDevice(prev);
    return e;
}

cudaError_t DpPolicy::predict(int B, const uint8_t* frames, const float* state, const float* noise, bool unnormalize,
                              float* actions) {
    if (B < 1 || B > max_batch_ || !frames || !state || !actions) return cudaErrorInvalidValue;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != device_) cudaSetDevice(device_);
    const cudaError_t e0 = [&]() -> cudaError_t {
        VSB_TRY(cudaMemcpyAsync(d_frames_, frames, (size_t)B * frame_bytes(), cudaMemcpyHostToDevice, stream_));
        VSB_TRY(cudaMemcpyAsync(d_state_, state, sizeof(float) * (size_t)B * cfg_.n_obs * cfg_.state_dim,
                                cudaMemcpyHostToDevice, stream_));
        // no noise: the sampler starts from zeros (vla_diffusion_predict's contract)
        const size_t nb = sizeof(float) * (size_t)B * noise_floats();
        if (noise) VSB_TRY(cudaMemcpyAsync(d_noise_, noise, nb, cudaMemcpyHostToDevice, stream_));
        else VSB_TRY(cudaMemsetAsync(d_noise_, 0, nb, stream_));
        VSB_TRY(enqueue(B, stream_, unnormalize));
        const size_t ab = sizeof(float) * (size_t)B * cfg_.n_action_steps * cfg_.action_dim;
        VSB_TRY(cudaMemcpyAsync(h_pinned_, d_actions_, ab, cudaMemcpyDeviceToHost, stream_));
        VSB_TRY(cudaMemcpyAsync(h_status_pinned_, d_status_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
        VSB_TRY(cudaStreamSynchronize(stream_));
        if (*h_status_pinned_ != 0) {
            device_status_take();
            return cudaErrorLaunchFailure;
        }
        std::memcpy(actions, h_pinned_, ab);
        return cudaSuccess;
    }();
    if (prev != device_) cudaSetDevice(prev);
    return e0;
}

long long DpPolicy::global_cond(float* out, long long cap) {
    const long long n = (long long)last_batch_ * cfg_.global_cond_dim();
    if (!out || n <= 0 || n > cap) return -1;
    cudaSetDevice(device_);
    if (cudaMemcpy(out, d_gcond_, sizeof(float) * n, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return n;
}

long long DpPolicy::debug_map(float* out, long long cap) {
    const long long n = (long long)debug_n_;
    if (!out || !d_debug_ || n <= 0 || n > cap) return -1;
    cudaSetDevice(device_);
    if (cudaMemcpy(out, d_debug_, sizeof(float) * n, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return n;
}

}  // namespace vsb
