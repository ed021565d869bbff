// SmolVLA runtime (see smolvla_policy.h). Host code only: parsing, bf16
// widening, int8 packing, the RoPE / time-embedding tables, buffer planning
// and the kernel sequence of one query batch.
#include "smolvla_policy.h"

#include "host_util.h"

#include "model_files.h"

#include "f32.h"
#include "gemm_i8.h"
#include "lm_ops.h"
#include "nn.h"
#include "octo.h"
#include "polar_normal.h"
#include "quant.h"
#include "smolvla.h"

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <sstream>

namespace vsb {

namespace {

using host::env_int;
using host::meta_int;
using host::meta_real;
using host::numeric_meta;
using host::round16;
using host::shape_fits;

// fp32 values of bf16 words (exact: the bf16 bits are the top half)
std::vector<float> widen(const uint16_t* p, size_t n) {
    std::vector<float> out(n);
    for (size_t i = 0; i < n; ++i) {
        const uint32_t u = static_cast<uint32_t>(p[i]) << 16;
        std::memcpy(&out[i], &u, 4);
    }
    return out;
}

// rope_neox's per-position table (src/hal/common/norms.cpp:31-49): theta starts
// at the position and is multiplied by base^(-2/hd) per pair; cos / sin from
// the host C library, in double.
std::vector<double> rope_cos_sin(int max_pos, int hd, double base) {
    const int half = hd / 2;
    const double scale = std::pow(base, -2.0 / hd);
    std::vector<double> t((size_t)(max_pos + 1) * half * 2);
    for (int p = 0; p <= max_pos; ++p) {
        double theta = static_cast<double>(p);
        for (int i = 0; i < half; ++i) {
            t[((size_t)p * half + i) * 2] = std::cos(theta);
            t[((size_t)p * half + i) * 2 + 1] = std::sin(theta);
            theta *= scale;
        }
    }
    return t;
}

}  // namespace

#define VSB_TRY(x)                                     \
    do {                                               \
        const cudaError_t e_ = (x);                    \
        if (e_ != cudaSuccess) return e_;              \
    } while (0)

template <class T>
T* SmolvlaPolicy::dalloc(size_t n) {
    void* p = nullptr;
    if (n == 0) n = 1;
    if (cudaMalloc(&p, n * sizeof(T)) != cudaSuccess) {
        fail("cudaMalloc failed");
        return nullptr;
    }
    allocs_.push_back(p);
    return static_cast<T*>(p);
}

SmolvlaPolicy::~SmolvlaPolicy() {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device_);
    for (auto& g : graphs_)
        if (g.second) cudaGraphExecDestroy(g.second);
    if (stream_) cudaStreamDestroy(stream_);
    for (void* p : allocs_) cudaFree(p);
    if (h_pinned_) cudaFreeHost(h_pinned_);
    if (h_noise_) cudaFreeHost(h_noise_);
    if (h_status_pinned_) cudaFreeHost(h_status_pinned_);
    cudaSetDevice(prev);
}

// ------------------------------------------------------------------ load
// vit.meta / vit.bin (src/models/smolvla/siglip_vision.cpp:16-144): the fp32
// region (patch bias, position embedding, per layer norms and biases, post
// norm), then the bf16 region (patch weights, per layer q k v o fc1 fc2, the
// connector). SMOLVLA_INT8 bits (smolvla_model.cpp:62-63): 1 q/k/v/o, 2 fc1,
// 4 fc2, 8 patch embedding + connector.
bool SmolvlaPolicy::load_vit(const ModelFiles& files, int mask) {
    std::string text;
    std::map<std::string, double> kv;
    if (!files.read("vit.meta", text) || !numeric_meta(text, kv)) { fail("cannot read vit.meta"); return false; }
    SmolvlaConfigDev& c = cfg_;
    if (!meta_int(kv, "hidden", c.v_hidden) || !meta_int(kv, "n_heads", c.v_heads) ||
        !meta_int(kv, "head_dim", c.v_hd) || !meta_int(kv, "inter", c.v_inter) ||
        !meta_int(kv, "n_layers", c.v_layers) || !meta_int(kv, "patch", c.patch) || !meta_int(kv, "img", c.img) ||
        !meta_int(kv, "n_patches", c.n_patches) || !meta_int(kv, "scale_factor", c.sf) ||
        !meta_int(kv, "mm_out", c.mm_out) || !meta_int(kv, "n_img_tok", c.n_img_tok)) {
        fail("invalid integer in vit.meta");
        return false;
    }
    meta_real(kv, "ln_eps", c.v_eps);
    const int H = c.v_hidden, I = c.v_inter, PD = 3 * c.patch * c.patch, NP = c.n_patches, SD = H * c.sf * c.sf;
    if (c.n_patches < 1 || !shape_fits({c.img, c.img, 3}) || !shape_fits({c.v_heads, c.v_hd}) || !shape_fits({H, c.sf, c.sf}) ||
        !shape_fits({c.v_layers, H, H}) || !shape_fits({c.v_layers, I, H}) || !shape_fits({c.mm_out, SD}) ||
        !std::isfinite(c.v_eps) || c.v_eps <= 0) {
        fail("unsupported vit.meta");
        return false;
    }
    const int side = static_cast<int>(std::lround(std::sqrt(static_cast<double>(NP))));
    if (c.v_heads * c.v_hd != H || side * side != NP || c.img % c.patch || (c.img / c.patch) * (c.img / c.patch) != NP ||
        side % c.sf || (side / c.sf) * (side / c.sf) != c.n_img_tok) {
        fail("vit.meta shapes do not close");
        return false;
    }
    if (c.v_hd != 64) { fail("this backend's attention needs head_dim 64"); return false; }
    const size_t fcount = (size_t)H + (size_t)NP * H + (size_t)c.v_layers * (8 * H + I + H) + 2 * (size_t)H;
    const size_t wcount = (size_t)H * PD + (size_t)c.v_layers * (4 * (size_t)H * H + 2 * (size_t)I * H) +
                          (size_t)c.mm_out * SD;
    std::string bin;
    if (!files.read("vit.bin", bin) || bin.size() != fcount * 4 + wcount * 2) {
        fail("vit.bin size does not match vit.meta");
        return false;
    }
    const float* f = reinterpret_cast<const float*>(bin.data());
    const uint16_t* w = reinterpret_cast<const uint16_t*>(bin.data() + fcount * 4);
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    auto up = [&](const float* src, size_t n) {
        float* p = dalloc<float>(n);
        if (p) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    size_t fo = 0, wo = 0;
    auto tf = [&](size_t n) { const float* p = f + fo; fo += n; return p; };
    auto tw = [&](size_t n) { std::vector<float> v = widen(w + wo, n); wo += n; return v; };
    const float* patch_b = tf(H);
    pos_emb_ = up(tf((size_t)NP * H), (size_t)NP * H);
    struct LF { const float *l1w, *l1b, *bq, *bk, *bv, *bo, *l2w, *l2b, *b1, *b2; };
    std::vector<LF> lf(c.v_layers);
    for (LF& l : lf) {
        l.l1w = tf(H); l.l1b = tf(H); l.bq = tf(H); l.bk = tf(H); l.bv = tf(H); l.bo = tf(H);
        l.l2w = tf(H); l.l2b = tf(H); l.b1 = tf(I); l.b2 = tf(H);
    }
    post_s_ = up(tf(H), H);
    post_b_ = up(tf(H), H);
    {
        std::vector<float> pw = tw((size_t)H * PD);
        if (!upload_linear(patch_, pw.data(), patch_b, H, PD, (mask & 8) != 0, alloc, &n_int8_)) return false;
    }
    vit_.resize(c.v_layers);
    std::vector<float> bqkv(3 * (size_t)H);
    for (int L = 0; L < c.v_layers; ++L) {
        SmolVitLayerDev& d = vit_[L];
        d.ln1s = up(lf[L].l1w, H);
        d.ln1b = up(lf[L].l1b, H);
        d.ln2s = up(lf[L].l2w, H);
        d.ln2b = up(lf[L].l2b, H);
        std::vector<float> qkv = tw(3 * (size_t)H * H);   // Wq, Wk, Wv are consecutive: the stacked [3H][H]
        std::memcpy(bqkv.data(), lf[L].bq, 4 * (size_t)H);
        std::memcpy(bqkv.data() + H, lf[L].bk, 4 * (size_t)H);
        std::memcpy(bqkv.data() + 2 * H, lf[L].bv, 4 * (size_t)H);
        const int before = n_int8_;
        if (!upload_linear(d.wqkv, qkv.data(), bqkv.data(), 3 * H, H, (mask & 1) != 0, alloc, &n_int8_)) return false;
        if (n_int8_ > before) n_int8_ += 2;   // the reference counts q, k, v separately
        std::vector<float> wo_ = tw((size_t)H * H), w1 = tw((size_t)I * H), w2 = tw((size_t)H * I);
        if (!upload_linear(d.wo, wo_.data(), lf[L].bo, H, H, (mask & 1) != 0, alloc, &n_int8_) ||
            !upload_linear(d.w1, w1.data(), lf[L].b1, I, H, (mask & 2) != 0, alloc, &n_int8_) ||
            !upload_linear(d.w2, w2.data(), lf[L].b2, H, I, (mask & 4) != 0, alloc, &n_int8_))
            return false;
    }
    std::vector<float> mm = tw((size_t)c.mm_out * SD);
    if (!upload_linear(mm_proj_, mm.data(), nullptr, c.mm_out, SD, (mask & 8) != 0, alloc, &n_int8_)) return false;
    return err_.empty();
}

// vlm.meta / vlm.bin (src/models/smolvla/smollm2_lm.cpp:13-78): per layer
// norms, the output norm, then bf16 q k v o gate up down per layer.
bool SmolvlaPolicy::load_vlm(const ModelFiles& files, bool int8) {
    std::string text;
    std::map<std::string, double> kv;
    if (!files.read("vlm.meta", text) || !numeric_meta(text, kv)) { fail("cannot read vlm.meta"); return false; }
    SmolvlaConfigDev& c = cfg_;
    if (!meta_int(kv, "hidden", c.hidden) || !meta_int(kv, "n_q", c.n_q) || !meta_int(kv, "n_kv", c.n_kv) ||
        !meta_int(kv, "head_dim", c.hd) || !meta_int(kv, "ffn", c.ffn) || !meta_int(kv, "n_layers", c.vlm_layers)) {
        fail("invalid integer in vlm.meta");
        return false;
    }
    meta_real(kv, "eps", c.rms_eps);
    meta_real(kv, "rope_base", c.rope_base);
    if (!shape_fits({c.n_q, c.hd}) || !shape_fits({c.n_kv, c.hd}) || c.n_q % c.n_kv || c.hd % 2 || c.qf() != c.hidden ||
        !shape_fits({c.vlm_layers, c.hidden, c.hidden}) || !shape_fits({c.vlm_layers, c.ffn, c.hidden}) ||
        !std::isfinite(c.rms_eps) || c.rms_eps <= 0 || !std::isfinite(c.rope_base) || c.rope_base <= 0) {
        fail("unsupported vlm.meta");
        return false;
    }
    if (c.hd != 64) { fail("this backend's attention needs head_dim 64"); return false; }
    const int H = c.hidden, QF = c.qf(), KV = c.kvf(), F = c.ffn, NL = c.vlm_layers;
    const size_t fcount = 2 * (size_t)H * NL + H;
    const size_t per = (size_t)QF * H + 2 * (size_t)KV * H + (size_t)H * QF + 3 * (size_t)F * H;
    std::string bin;
    if (!files.read("vlm.bin", bin) || bin.size() != fcount * 4 + per * NL * 2) {
        fail("vlm.bin size does not match vlm.meta");
        return false;
    }
    const float* f = reinterpret_cast<const float*>(bin.data());
    const uint16_t* w = reinterpret_cast<const uint16_t*>(bin.data() + fcount * 4);
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    auto up = [&](const float* src, size_t n) {
        float* p = dalloc<float>(n);
        if (p) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    vlm_.resize(NL);
    for (int L = 0; L < NL; ++L) {
        vlm_[L].ln_in = up(f + 2 * (size_t)H * L, H);
        vlm_[L].ln_post = up(f + 2 * (size_t)H * L + H, H);
    }
    size_t wo = 0;
    auto tw = [&](size_t n) { std::vector<float> v = widen(w + wo, n); wo += n; return v; };
    for (int L = 0; L < NL; ++L) {
        SmolVlmLayerDev& d = vlm_[L];
        std::vector<float> qkv = tw((size_t)(QF + 2 * KV) * H);   // q, k, v consecutive
        int before = n_int8_;
        if (!upload_linear(d.wqkv, qkv.data(), nullptr, QF + 2 * KV, H, int8, alloc, &n_int8_)) return false;
        if (n_int8_ > before) n_int8_ += 2;
        std::vector<float> o = tw((size_t)H * QF), gu = tw(2 * (size_t)F * H), dn = tw((size_t)H * F);
        if (!upload_linear(d.wo, o.data(), nullptr, H, QF, int8, alloc, &n_int8_)) return false;
        before = n_int8_;
        if (!upload_linear(d.wgu, gu.data(), nullptr, 2 * F, H, int8, alloc, &n_int8_)) return false;
        if (n_int8_ > before) n_int8_ += 1;   // gate and up
        if (!upload_linear(d.wdown, dn.data(), nullptr, H, F, int8, alloc, &n_int8_)) return false;
    }
    return err_.empty();
}

// aex.meta / aex.bin (src/models/smolvla/action_expert.cpp:49-164): fp32; per
// layer ln_in, q, k, v, o, ln_post, gate, up, down (k / v over the expert
// stream on self-attention layers, over the cached VLM K / V on the others),
// then the output norm and the flow projections.
bool SmolvlaPolicy::load_expert(const ModelFiles& files, bool int8) {
    std::string text;
    std::map<std::string, double> kv;
    if (!files.read("aex.meta", text) || !numeric_meta(text, kv)) { fail("cannot read aex.meta"); return false; }
    SmolvlaConfigDev& c = cfg_;
    if (!meta_int(kv, "expert_h", c.eh) || !meta_int(kv, "expert_ffn", c.ef) || !meta_int(kv, "n_q", c.e_nq) ||
        !meta_int(kv, "n_kv", c.e_nkv) || !meta_int(kv, "head_dim", c.e_hd) || !meta_int(kv, "n_layers", c.e_layers) ||
        !meta_int(kv, "self_attn_every_n", c.san) || !meta_int(kv, "chunk", c.chunk) ||
        !meta_int(kv, "num_steps", c.num_steps) || !meta_int(kv, "max_action_dim", c.mad)) {
        fail("invalid integer in aex.meta");
        return false;
    }
    meta_real(kv, "eps", c.e_eps);
    meta_real(kv, "rope_base", c.e_rope_base);
    meta_real(kv, "min_period", c.min_period);
    meta_real(kv, "max_period", c.max_period);
    const int steps = env_int("SMOLVLA_NUM_STEPS", 0);   // the reference's override (action_expert.cpp:71-76)
    if (steps > 0) c.num_steps = steps;
    const int QF = c.e_nq * c.e_hd, KV = c.e_nkv * c.e_hd, EH = c.eh, EF = c.ef, MAD = c.mad, NL = c.e_layers;
    if (!shape_fits({c.e_nq, c.e_hd}) || !shape_fits({c.e_nkv, c.e_hd}) || c.e_nq % c.e_nkv || c.e_hd % 2 || EH % 2 ||
        !shape_fits({NL, EH, QF}) || !shape_fits({NL, KV, KV}) || !shape_fits({NL, EF, EH}) || !shape_fits({2, EH, EH}) ||
        !shape_fits({c.chunk, MAD}) || !shape_fits({EH, MAD}) || c.num_steps < 1 || c.san < 0 || !std::isfinite(c.e_eps) ||
        c.e_eps <= 0 || !std::isfinite(c.e_rope_base) || c.e_rope_base <= 0 || !std::isfinite(c.min_period) ||
        !std::isfinite(c.max_period) || c.min_period <= 0 || c.max_period <= c.min_period) {
        fail("unsupported aex.meta");
        return false;
    }
    if (c.e_hd != 64) { fail("this backend's attention needs head_dim 64"); return false; }
    if (c.chunk > 1023) { fail("chunk larger than this backend takes"); return false; }
    std::vector<float> data;
    if (!files.read_floats("aex.bin", data)) { fail("cannot read aex.bin"); return false; }
    size_t total = 0;
    for (int L = 0; L < NL; ++L) {
        const bool self = c.san > 0 && L % c.san == 0;
        const size_t kk = self ? EH : KV;
        total += (size_t)QF * EH + 2 * (size_t)KV * kk + (size_t)EH * QF + 3 * (size_t)EF * EH + 2 * (size_t)EH;
    }
    total += (size_t)EH + (size_t)EH * MAD + EH + (size_t)EH * 2 * EH + EH + (size_t)EH * EH + EH + (size_t)MAD * EH + MAD;
    if (data.size() != total) { fail("aex.bin size does not match aex.meta"); return false; }
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    size_t off = 0;
    auto take = [&](size_t n) { const float* p = data.data() + off; off += n; return p; };
    auto up = [&](const float* src, size_t n) {
        float* p = dalloc<float>(n);
        if (p) cudaMemcpy(p, src, n * sizeof(float), cudaMemcpyHostToDevice);
        return p;
    };
    aex_.resize(NL);
    for (int L = 0; L < NL; ++L) {
        SmolExpertLayerDev& d = aex_[L];
        d.self_attn = c.san > 0 && L % c.san == 0;
        const int kk = d.self_attn ? EH : KV;
        d.ln_in = up(take(EH), EH);
        const float* wq = take((size_t)QF * EH);
        const float* wk = take((size_t)KV * kk);
        const float* wv = take((size_t)KV * kk);
        const float* wo = take((size_t)EH * QF);
        d.ln_post = up(take(EH), EH);
        const float* wg = take(2 * (size_t)EF * EH);   // gate, up consecutive
        const float* wd = take((size_t)EH * EF);
        if (!upload_linear(d.wq, wq, nullptr, QF, EH, int8, alloc, &n_int8_)) return false;
        if (d.self_attn) {   // k and v read the same normalized stream: one stacked GEMM
            const int before = n_int8_;
            if (!upload_linear(d.wkv, wk, nullptr, 2 * KV, kk, int8, alloc, &n_int8_)) return false;
            if (n_int8_ > before) n_int8_ += 1;
        } else if (!upload_linear(d.wk, wk, nullptr, KV, kk, int8, alloc, &n_int8_) ||
                   !upload_linear(d.wv, wv, nullptr, KV, kk, int8, alloc, &n_int8_)) {
            return false;
        }
        if (!upload_linear(d.wo, wo, nullptr, EH, QF, int8, alloc, &n_int8_)) return false;
        const int before = n_int8_;
        if (!upload_linear(d.wgu, wg, nullptr, 2 * EF, EH, int8, alloc, &n_int8_)) return false;
        if (n_int8_ > before) n_int8_ += 1;
        if (!upload_linear(d.wdown, wd, nullptr, EH, EF, int8, alloc, &n_int8_)) return false;
        (void)wv;
    }
    out_norm_ = up(take(EH), EH);
    auto flow = [&](DevLinear& l, int N, int K) {
        const float* W = take((size_t)N * K);
        const float* b = take(N);
        return upload_linear(l, W, b, N, K, false, alloc, nullptr);
    };
    if (!flow(ain_, EH, MAD) || !flow(at1_, EH, 2 * EH) || !flow(at2_, EH, EH) || !flow(aout_, MAD, EH)) return false;
    return err_.empty();
}

// heads.meta, emb.bin, heads.bin, the stats and config.txt (smolvla_model.cpp:52-117,
// smolvla_capi.cpp:35-60).
bool SmolvlaPolicy::load_heads(const ModelFiles& files) {
    std::string text;
    std::map<std::string, double> kv;
    if (!files.read("heads.meta", text) || !numeric_meta(text, kv)) { fail("cannot read heads.meta"); return false; }
    SmolvlaConfigDev& c = cfg_;
    int hidden = 0;
    if (!meta_int(kv, "vocab", c.vocab) || !meta_int(kv, "hidden", hidden) || !meta_int(kv, "max_state_dim", c.msd) ||
        !meta_int(kv, "real_state_dim", c.sd) || !meta_int(kv, "real_action_dim", c.ad) ||
        !meta_int(kv, "n_views", c.n_views)) {
        fail("invalid integer in heads.meta");
        return false;
    }
    meta_real(kv, "norm_eps", c.norm_eps);
    if (!shape_fits({c.vocab, hidden}) || !shape_fits({c.msd, hidden}) || c.n_views <= 0 || !std::isfinite(c.norm_eps) ||
        c.norm_eps <= 0 || c.sd <= 0 || c.sd > c.msd || c.ad <= 0 || c.ad > c.mad || hidden != c.hidden ||
        hidden != c.mm_out || c.e_nkv * c.e_hd != c.kvf() || c.e_layers > c.vlm_layers) {
        fail("heads.meta is missing or malformed");
        return false;
    }
    std::string emb;
    if (!files.read("emb.bin", emb) || emb.size() != (size_t)c.vocab * hidden * 2) { fail("emb.bin size"); return false; }
    emb_ = dalloc<uint16_t>((size_t)c.vocab * hidden);
    if (!emb_) return false;
    cudaMemcpy(emb_, emb.data(), emb.size(), cudaMemcpyHostToDevice);
    std::vector<float> heads;
    if (!files.read_floats("heads.bin", heads) || heads.size() != (size_t)hidden * c.msd + hidden) {
        fail("heads.bin size");
        return false;
    }
    const DevAlloc alloc = [this](size_t n) -> void* { return dalloc<char>(n); };
    if (!upload_linear(state_proj_, heads.data(), heads.data() + (size_t)hidden * c.msd, hidden, c.msd, false, alloc,
                       nullptr))
        return false;
    auto stat = [&](const char* name, int n, float** dst, bool nonneg) {
        std::vector<float> v;
        if (!files.read_floats(name, v) || (int)v.size() != n) return false;
        for (float x : v)
            if (!std::isfinite(x) || (nonneg && x < 0)) return false;
        *dst = dalloc<float>(n);
        if (!*dst) return false;
        cudaMemcpy(*dst, v.data(), n * sizeof(float), cudaMemcpyHostToDevice);
        return true;
    };
    if (!stat("stats_state_mean.bin", c.sd, &s_mean_, false) || !stat("stats_state_std.bin", c.sd, &s_std_, true) ||
        !stat("stats_action_mean.bin", c.ad, &a_mean_, false) || !stat("stats_action_std.bin", c.ad, &a_std_, true)) {
        fail("cannot read the state / action stats");
        return false;
    }
    // config.txt: tokenizer_max_length / pad_token_id, one "key value" per line
    // split at the first space (smolvla_capi.cpp:35-60)
    std::string cfg;
    if (files.read("config.txt", cfg)) {
        std::istringstream in(cfg);
        std::string line;
        while (std::getline(in, line)) {
            if (!line.empty() && line.back() == '\r') line.pop_back();
            const size_t sp = line.find(' ');
            if (sp == std::string::npos) continue;
            const std::string k = line.substr(0, sp), v = line.substr(sp + 1);
            try {
                if (k == "tokenizer_max_length") c.tok_maxlen = std::stoi(v);
                else if (k == "pad_token_id") c.pad_id = std::stoi(v);
            } catch (...) {
            }
        }
        if (c.tok_maxlen < 1) c.tok_maxlen = 48;
    }
    return err_.empty();
}

bool SmolvlaPolicy::alloc_buffers() {
    const SmolvlaConfigDev& c = cfg_;
    const int Bm = max_batch_, F = Bm * c.n_views, NP = c.n_patches, H = c.v_hidden, I = c.v_inter;
    const int np = c.n_prefix(), C = c.chunk, SK = np + C, D = c.hidden, QF = c.qf(), KV = c.kvf();
    const int EH = c.eh, EF = c.ef, MAD = c.mad, TOK = c.n_img_tok, SD = H * c.sf * c.sf;
    const int eQF = c.e_nq * c.e_hd;
    d_tokens_ = dalloc<int>((size_t)Bm * c.tok_maxlen);
    d_lmask_ = dalloc<int>((size_t)Bm * c.tok_maxlen);
    d_state_raw_ = dalloc<float>((size_t)Bm * c.sd);
    d_noise_ = dalloc<float>((size_t)Bm * C * MAD);
    d_prev_ = dalloc<float>((size_t)Bm * C * c.ad);
    d_weights_ = dalloc<float>((size_t)Bm * C + c.num_steps);   // + the per-step guidance weights
    d_actions_ = dalloc<float>((size_t)Bm * C * c.ad);
    d_pix_ = dalloc<float>((size_t)F * 3 * c.img * c.img);
    d_patches_ = dalloc<float>((size_t)F * NP * 3 * c.patch * c.patch);
    d_vh_ = dalloc<float>((size_t)F * NP * H);
    d_vn_ = dalloc<float>((size_t)F * NP * H);
    d_vqkv_ = dalloc<float>((size_t)F * NP * 3 * H);
    d_vatt_ = dalloc<float>((size_t)F * NP * H);
    d_vff_ = dalloc<float>((size_t)F * NP * I);
    d_shuf_ = dalloc<float>((size_t)F * TOK * SD);
    d_img_ = dalloc<float>((size_t)F * TOK * D);
    d_state_n_ = dalloc<float>((size_t)Bm * c.msd);
    d_state_row_ = dalloc<float>((size_t)Bm * D);
    d_x_ = dalloc<float>((size_t)Bm * np * D);
    d_xn_ = dalloc<float>((size_t)Bm * np * D);
    d_att_ = dalloc<float>((size_t)Bm * np * QF);
    d_gu_ = dalloc<float>((size_t)Bm * np * 2 * c.ffn);
    d_pmask_ = dalloc<float>((size_t)Bm * np * np);
    d_dmask_ = dalloc<float>((size_t)Bm * C * SK);
    d_cmask_ = dalloc<float>((size_t)Bm * C * np);
    d_pos_ = dalloc<int>((size_t)Bm * np);
    d_pos_full_ = dalloc<int>((size_t)Bm * C);
    d_pos_reb_ = dalloc<int>((size_t)Bm * C);
    d_cache_.resize(c.vlm_layers);
    for (float*& p : d_cache_) p = dalloc<float>((size_t)Bm * np * (QF + 2 * KV));
    d_kvf_.assign(c.e_layers, nullptr);
    d_ckv_.assign(c.e_layers, nullptr);
    for (int L = 0; L < c.e_layers; ++L) {
        if (aex_[L].self_attn) d_kvf_[L] = dalloc<float>((size_t)Bm * SK * 2 * KV);
        else d_ckv_[L] = dalloc<float>((size_t)Bm * np * 2 * KV);
    }
    d_eh_ = dalloc<float>((size_t)Bm * C * EH);
    d_ehn_ = dalloc<float>((size_t)Bm * C * EH);
    d_eq_ = dalloc<float>((size_t)Bm * C * eQF);
    d_ekv_ = dalloc<float>((size_t)Bm * C * 2 * KV);
    d_eatt_ = dalloc<float>((size_t)Bm * C * eQF);
    d_egu_ = dalloc<float>((size_t)Bm * C * 2 * EF);
    d_act_ = dalloc<float>(std::max((size_t)Bm * np * c.ffn, (size_t)Bm * C * EF));
    d_aemb_ = dalloc<float>((size_t)Bm * C * EH);
    d_at_ = dalloc<float>((size_t)Bm * C * 2 * EH);
    d_mlp1_ = dalloc<float>((size_t)Bm * C * EH);
    d_x_t_ = dalloc<float>((size_t)Bm * C * MAD);
    d_v_t_ = dalloc<float>((size_t)Bm * C * MAD);
    d_guide_ = dalloc<float>((size_t)Bm * C * MAD);
    // int8 row quantization scratch: the largest rows x padded K of any int8 layer
    const size_t rows_max = std::max({(size_t)F * NP, (size_t)F * TOK, (size_t)Bm * np, (size_t)Bm * C});
    const size_t k_max = std::max({(size_t)round16(3 * c.patch * c.patch), (size_t)round16(H), (size_t)round16(I),
                                   (size_t)round16(SD), (size_t)round16(D), (size_t)round16(QF),
                                   (size_t)round16(c.ffn), (size_t)round16(EH), (size_t)round16(EF),
                                   (size_t)round16(KV), (size_t)round16(eQF)});
    q_rows_ = rows_max;
    q_cap_ = rows_max * k_max;
    d_q_ = dalloc<int8_t>(q_cap_);
    d_qs_ = dalloc<float>(rows_max);
    d_att_cnt_ = dalloc<unsigned int>(kAttCounters);
    if (d_att_cnt_ && cudaMemset(d_att_cnt_, 0, sizeof(unsigned int) * kAttCounters) != cudaSuccess)
        fail("cudaMemset failed");
    // RoPE tables: positions up to the prefix plus the chunk
    max_pos_ = np + C;
    {
        const std::vector<double> tv = rope_cos_sin(max_pos_, c.hd, c.rope_base);
        rope_vlm_ = dalloc<double>(tv.size());
        if (rope_vlm_) cudaMemcpy(rope_vlm_, tv.data(), tv.size() * sizeof(double), cudaMemcpyHostToDevice);
        const std::vector<double> ta = rope_cos_sin(max_pos_, c.e_hd, c.e_rope_base);
        rope_aex_ = dalloc<double>(ta.size());
        if (rope_aex_) cudaMemcpy(rope_aex_, ta.data(), ta.size() * sizeof(double), cudaMemcpyHostToDevice);
    }
    // per-step time, its sinusoidal embedding (double, action_expert.cpp:188-195) and
    // the RTC weight before the max_guidance clamp (action_expert.cpp:372-378)
    {
        const int half = EH / 2, S = c.num_steps;
        std::vector<float> te((size_t)S * EH);
        time_.resize(S);
        gw_base_.resize(S);
        for (int k = 0; k < S; ++k) {
            const double td = std::fma(static_cast<double>(k), -1.0 / S, 1.0);
            const float time = static_cast<float>(td);
            time_[k] = time;
            for (int i = 0; i < half; ++i) {
                const double frac = half == 1 ? 0.0 : static_cast<double>(i) / static_cast<double>(half - 1);
                const double period = c.min_period * std::pow(c.max_period / c.min_period, frac);
                const double s = (2.0 * M_PI / period) * static_cast<double>(time);
                te[(size_t)k * EH + i] = static_cast<float>(std::sin(s));
                te[(size_t)k * EH + half + i] = static_cast<float>(std::cos(s));
            }
            const float tau = static_cast<float>(1.0 - td), s1 = (1.0f - tau) * (1.0f - tau);
            gw_base_[k] = (1.0f - tau) / tau * (std::fma(tau, tau, s1) / s1);
        }
        te_ = dalloc<float>(te.size());
        if (te_) cudaMemcpy(te_, te.data(), te.size() * sizeof(float), cudaMemcpyHostToDevice);
        dt_ = -1.0f / static_cast<float>(S);
        gw_.assign(S, 0.0f);
    }
    return err_.empty();
}

bool SmolvlaPolicy::ensure_frames(int h, int w) {
    const size_t need = (size_t)max_batch_ * cfg_.n_views * h * w * 3;
    if (need <= frames_cap_) return true;
    // a larger frame size: new input buffer, and the captured graphs read the old one
    for (auto& g : graphs_)
        if (g.second) cudaGraphExecDestroy(g.second);
    graphs_.clear();
    d_frames_ = dalloc<uint8_t>(need);
    if (!d_frames_) return false;
    frames_cap_ = need;
    return true;
}

bool SmolvlaPolicy::load(const std::string& dir, const std::string& tok_dir, int max_batch) {
    const int want_dev = env_int("VLA_CUDA_DEVICE", -1);
    if (want_dev >= 0 && cudaSetDevice(want_dev) != cudaSuccess) { fail("VLA_CUDA_DEVICE not usable"); return false; }
    cudaGetDevice(&device_);
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_);
    if (major != 10) { fail("needs an sm_100 (B200) device"); return false; }
    if (max_batch < 1 || max_batch > 256) { fail("max_batch must be in [1, 256]"); return false; }
    max_batch_ = max_batch;
    use_graph_ = env_int("VLA_CUDA_GRAPH", 1) != 0;
    const int mask = env_int("SMOLVLA_INT8", 0);
    ModelFiles files;
    if (!files.open(dir)) { fail(files.error()); return false; }
    {
        std::string vocab, merges;
        const std::string prefix = dir + "/";
        const bool inside = tok_dir.compare(0, prefix.size(), prefix) == 0;
        const std::string rel = inside ? tok_dir.substr(prefix.size()) + "/" : "";
        const bool ok = inside ? (files.read(rel + "vocab.txt", vocab) && files.read(rel + "merges.txt", merges))
                               : (ModelFiles::read_path(tok_dir + "/vocab.txt", vocab) &&
                                  ModelFiles::read_path(tok_dir + "/merges.txt", merges));
        if (!ok || !tok_.load_text(vocab, merges)) { fail("cannot load the tokenizer (vocab.txt, merges.txt)"); return false; }
    }
    if (cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess) { fail("stream"); return false; }
    if (!load_vit(files, mask) || !load_vlm(files, (mask & 16) != 0) || !load_expert(files, (mask & 32) != 0) ||
        !load_heads(files))
        return false;
    if (!alloc_buffers()) return false;
    if (mask) std::fprintf(stderr, "[smolvla] int8 GEMMs on device: %d (SMOLVLA_INT8=%d)\n", n_int8_, mask);
    const int FLo = cfg_.chunk * cfg_.ad;
    if (cudaMallocHost(&h_pinned_, sizeof(float) * (size_t)max_batch_ * FLo) != cudaSuccess ||
        cudaMallocHost(&h_noise_, sizeof(float) * (size_t)max_batch_ * cfg_.chunk * cfg_.mad) != cudaSuccess ||
        cudaMallocHost(&h_status_pinned_, sizeof(int)) != cudaSuccess) {
        fail("pinned host buffers");
        return false;
    }
    d_status_ = static_cast<int*>(device_status_address());
    if (!d_status_) { fail("device status word"); return false; }
    return err_.empty();
}

int SmolvlaPolicy::tokenize(const char* text, int32_t* ids, int32_t* mask) const {
    // lerobot's pipeline appends one newline (smolvla_capi.cpp:94-114)
    std::string s(text);
    if (s.size() > 65536) s.erase(0, s.size() - 65536);
    while (!s.empty() && s.back() == '\n') s.pop_back();
    s.push_back('\n');
    std::vector<int> enc = tok_.encode(s);
    const int n = cfg_.tok_maxlen;
    if (static_cast<int>(enc.size()) > n) enc.erase(enc.begin(), enc.end() - n);   // keeps the last n
    for (int i = 0; i < n; ++i) {
        ids[i] = i < static_cast<int>(enc.size()) ? enc[i] : cfg_.pad_id;
        mask[i] = i < static_cast<int>(enc.size()) ? 1 : 0;
    }
    return static_cast<int>(enc.size());
}

// ------------------------------------------------------------- layers
cudaError_t SmolvlaPolicy::linear(const DevLinear& l, const float* x, long long ldx, int M, float* out, long long ldo,
                                  int mode, const float* res, long long ldr, cudaStream_t st) {
    if (l.int8) {
        if ((size_t)M > q_rows_ || (size_t)M * round16(l.K) > q_cap_) return cudaErrorInvalidValue;
        VSB_TRY(quantize_rows(x, ldx, nullptr, 0, M, l.K, d_q_, round16(l.K), d_qs_, nullptr, 0, nullptr, st));
    }
    return linear_q(l, d_q_, d_qs_, x, ldx, M, out, ldo, mode, res, ldr, st);
}

// The int8 row copy (d_q_ / d_qs_) of an attention output of `rows` rows of K
// columns, written by the attention launch itself (nn.h AttQuant); sequences
// of seq_rows rows each. Null q when the scratch cannot hold it.
AttQuant SmolvlaPolicy::att_quant(int rows, int K, int seq_rows) const {
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

cudaError_t SmolvlaPolicy::rmsnorm_for(const float* x, const float* w, float* xn, int rows, int K, float eps, bool int8,
                                       cudaStream_t st) {
    if (int8 && ((size_t)rows > q_rows_ || (size_t)rows * round16(K) > q_cap_)) return cudaErrorInvalidValue;
    return rmsnorm(x, w, xn, rows, K, eps, st, int8 ? d_q_ : nullptr, round16(K), d_qs_);
}

cudaError_t SmolvlaPolicy::linear_q(const DevLinear& l, const int8_t* q, const float* qs, const float* x,
                                    long long ldx, int M, float* out, long long ldo, int mode, const float* res,
                                    long long ldr, cudaStream_t st) {
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
        a.static_weights = true;
        return gemm_i8(a, st);
    }
    return gemm_f32(x, ldx, l.W, l.K, l.bias, out, ldo, res, ldr, M, l.N, l.K, mode, nullptr, 1, st);
}

// SiglipVision::encode over F = B x n_views images (siglip_vision.cpp:163-210):
// patches -> embedding + position -> n pre-LN layers (dense attention) -> post
// LayerNorm -> pixel shuffle -> connector.
cudaError_t SmolvlaPolicy::run_vision(int F, int h, int w, cudaStream_t st) {
    const SmolvlaConfigDev& c = cfg_;
    const int H = c.v_hidden, I = c.v_inter, NP = c.n_patches, PD = 3 * c.patch * c.patch;
    const long long rows = (long long)F * NP;
    SmolvlaResize g;
    {   // resize_with_pad geometry (src/preprocess/image.cpp:19-25), in double
        const int S = c.img;
        const double ratio = std::max(static_cast<double>(w) / S, static_cast<double>(h) / S);
        int rw = static_cast<int>(w / ratio), rh = static_cast<int>(h / ratio);
        if (rw < 1) rw = 1;
        if (rh < 1) rh = 1;
        g.S = S;
        g.pad_w = S - rw;
        g.pad_h = S - rh;
        g.sx = static_cast<double>(w) / rw;
        g.sy = static_cast<double>(h) / rh;
    }
    VSB_TRY(smolvla_resize(d_frames_, F, h, w, g, d_pix_, st));
    VSB_TRY(smolvla_patches(d_pix_, F, c.img, c.patch, d_patches_, st));
    VSB_TRY(linear(patch_, d_patches_, PD, static_cast<int>(rows), d_vh_, H, 0, nullptr, 0, st));
    VSB_TRY(add_rows_mod(d_vh_, rows, H, pos_emb_, NP, st));
    const float scale = 1.0f / std::sqrt(static_cast<float>(c.v_hd));
    const long long ldq = round16(H);
    for (const SmolVitLayerDev& L : vit_) {
        VSB_TRY(layernorm(d_vh_, d_vn_, L.ln1s, L.ln1b, static_cast<int>(rows), H, c.v_eps, nullptr,
                          L.wqkv.int8 ? d_q_ : nullptr, L.wqkv.int8 ? d_qs_ : nullptr, nullptr, nullptr, ldq, st));
        VSB_TRY(linear_q(L.wqkv, d_q_, d_qs_, d_vn_, H, static_cast<int>(rows), d_vqkv_, 3 * H, 0, nullptr, 0, st));
        AttBatch bs;
        bs.n = F;
        bs.q = bs.k = bs.v = (long long)NP * 3 * H;
        bs.o = (long long)NP * H;
        {   // the o-projection's int8 input comes out of the attention launch
            const AttQuant aq = att_quant(static_cast<int>(rows), H, NP);
            if (L.wo.int8 && !aq.q) return cudaErrorInvalidValue;
            VSB_TRY(attention_batched(d_vqkv_, 3 * H, d_vqkv_ + H, 3 * H, d_vqkv_ + 2 * H, 3 * H, d_vatt_, H, NP, NP,
                                      c.v_heads, c.v_heads, c.v_hd, scale, nullptr, bs, st, L.wo.int8 ? &aq : nullptr));
            VSB_TRY(linear_q(L.wo, d_q_, d_qs_, d_vatt_, H, static_cast<int>(rows), d_vh_, H, kEpiAdd, d_vh_, H, st));
        }
        VSB_TRY(layernorm(d_vh_, d_vn_, L.ln2s, L.ln2b, static_cast<int>(rows), H, c.v_eps, nullptr,
                          L.w1.int8 ? d_q_ : nullptr, L.w1.int8 ? d_qs_ : nullptr, nullptr, nullptr, ldq, st));
        VSB_TRY(linear_q(L.w1, d_q_, d_qs_, d_vn_, H, static_cast<int>(rows), d_vff_, I, 0, nullptr, 0, st));
        if (L.w2.int8) {
            VSB_TRY(act_rows_q(kActGeluTanh, d_vff_, static_cast<int>(rows), I, false, d_q_, round16(I), d_qs_, st));
            VSB_TRY(linear_q(L.w2, d_q_, d_qs_, nullptr, 0, static_cast<int>(rows), d_vh_, H, kEpiAdd, d_vh_, H, st));
        } else {
            VSB_TRY(activation(kActGeluTanh, d_vff_, d_vff_, nullptr, rows * I, st));
            VSB_TRY(linear(L.w2, d_vff_, I, static_cast<int>(rows), d_vh_, H, kEpiAdd, d_vh_, H, st));
        }
    }
    VSB_TRY(layernorm(d_vh_, d_vh_, post_s_, post_b_, static_cast<int>(rows), H, c.v_eps, nullptr, nullptr, nullptr,
                      nullptr, nullptr, 0, st));
    const int side = static_cast<int>(std::lround(std::sqrt(static_cast<double>(NP))));
    VSB_TRY(pixel_shuffle(d_vh_, F, side, c.sf, H, d_shuf_, st));
    return linear(mm_proj_, d_shuf_, (long long)H * c.sf * c.sf, F * c.n_img_tok, d_img_, c.hidden, 0, nullptr, 0,
                  st);
}

// The SmolLM2 prefix pass (smollm2_lm.cpp:80-132): every layer's q | rotated k | v
// stay in d_cache_ as the expert's K/V cache; the last layer stops after K / V.
cudaError_t SmolvlaPolicy::run_vlm(int B, cudaStream_t st) {
    const SmolvlaConfigDev& c = cfg_;
    const int np = c.n_prefix(), D = c.hidden, QF = c.qf(), KV = c.kvf(), F = c.ffn, LD = QF + 2 * KV;
    const int rows = B * np;
    const float scale = 1.0f / std::sqrt(static_cast<float>(c.hd));
    for (int L = 0; L < c.vlm_layers; ++L) {
        const SmolVlmLayerDev& w = vlm_[L];
        float* qkv = d_cache_[L];
        VSB_TRY(rmsnorm_for(d_x_, w.ln_in, d_xn_, rows, D, c.rms_eps, w.wqkv.int8, st));
        VSB_TRY(linear_q(w.wqkv, d_q_, d_qs_, d_xn_, D, rows, qkv, LD, 0, nullptr, 0, st));
        VSB_TRY(rope_table(qkv + QF, LD, rows, c.n_kv, c.hd, d_pos_, rope_vlm_, max_pos_, d_status_, st));
        if (L + 1 == c.vlm_layers) break;
        VSB_TRY(rope_table(qkv, LD, rows, c.n_q, c.hd, d_pos_, rope_vlm_, max_pos_, d_status_, st));
        AttBatch bs;
        bs.n = B;
        bs.q = bs.k = bs.v = (long long)np * LD;
        bs.o = (long long)np * QF;
        bs.mask = (long long)np * np;
        {
            const AttQuant aq = att_quant(rows, QF, np);
            if (w.wo.int8 && !aq.q) return cudaErrorInvalidValue;
            VSB_TRY(attention_batched(qkv, LD, qkv + QF, LD, qkv + QF + KV, LD, d_att_, QF, np, np, c.n_q, c.n_kv,
                                      c.hd, scale, d_pmask_, bs, st, w.wo.int8 ? &aq : nullptr));
            VSB_TRY(linear_q(w.wo, d_q_, d_qs_, d_att_, QF, rows, d_x_, D, kEpiAdd, d_x_, D, st));
        }
        VSB_TRY(rmsnorm_for(d_x_, w.ln_post, d_xn_, rows, D, c.rms_eps, w.wgu.int8, st));
        VSB_TRY(linear_q(w.wgu, d_q_, d_qs_, d_xn_, D, rows, d_gu_, 2 * F, 0, nullptr, 0, st));
        if (w.wdown.int8) {
            VSB_TRY(silu_gate_rows(d_gu_, rows, F, nullptr, d_q_, round16(F), d_qs_, st));
            VSB_TRY(linear_q(w.wdown, d_q_, d_qs_, nullptr, 0, rows, d_x_, D, kEpiAdd, d_x_, D, st));
        } else {
            VSB_TRY(silu_gate_rows(d_gu_, rows, F, d_act_, nullptr, 0, nullptr, st));
            VSB_TRY(linear(w.wdown, d_act_, F, rows, d_x_, D, kEpiAdd, d_x_, D, st));
        }
    }
    return cudaSuccess;
}

// ActionExpert::denoise (action_expert.cpp:343-392) for B queries.
cudaError_t SmolvlaPolicy::run_expert(int B, bool guided, cudaStream_t st) {
    const SmolvlaConfigDev& c = cfg_;
    const int np = c.n_prefix(), C = c.chunk, SK = np + C, QF = c.qf(), KV = c.kvf(), LD = QF + 2 * KV;
    const int EH = c.eh, EF = c.ef, MAD = c.mad, eQF = c.e_nq * c.e_hd;
    const int rows = B * C;
    const float scale = 1.0f / std::sqrt(static_cast<float>(c.e_hd));
    // the step-invariant halves: the prefix K / V of the self-attention layers,
    // the cross-attention layers' reprojected K / V
    for (int L = 0; L < c.e_layers; ++L) {
        const SmolExpertLayerDev& w = aex_[L];
        const float* cache = d_cache_[L];
        if (w.self_attn) {
            VSB_TRY(copy_rows(cache + QF, (long long)np * LD, LD, d_kvf_[L], (long long)SK * 2 * KV, 2 * KV, B, np,
                              2 * KV, st));
        } else {
            VSB_TRY(linear(w.wk, cache + QF, LD, B * np, d_ckv_[L], 2 * KV, 0, nullptr, 0, st));
            VSB_TRY(linear(w.wv, cache + QF + KV, LD, B * np, d_ckv_[L] + KV, 2 * KV, 0, nullptr, 0, st));
        }
    }
    VSB_TRY(cudaMemcpyAsync(d_x_t_, d_noise_, sizeof(float) * (size_t)rows * MAD, cudaMemcpyDeviceToDevice, st));
    for (int k = 0; k < c.num_steps; ++k) {
        // embed_suffix (action_expert.cpp:180-211): the reference's plain dense_linear
        VSB_TRY(linear_f32(d_x_t_, MAD, ain_.W, ain_.bias, d_aemb_, EH, rows, EH, MAD, nullptr, nullptr, st));
        VSB_TRY(concat_time(d_aemb_, te_ + (size_t)k * EH, rows, EH, d_at_, st));
        VSB_TRY(linear_f32(d_at_, 2 * EH, at1_.W, at1_.bias, d_mlp1_, EH, rows, EH, 2 * EH, nullptr, nullptr, st));
        VSB_TRY(silu_exact(d_mlp1_, (long long)rows * EH, st));
        VSB_TRY(linear_f32(d_mlp1_, EH, at2_.W, at2_.bias, d_eh_, EH, rows, EH, EH, nullptr, nullptr, st));
        for (int L = 0; L < c.e_layers; ++L) {
            const SmolExpertLayerDev& w = aex_[L];
            // one int8 copy of the normalized rows serves q and (self-attention) k / v
            VSB_TRY(rmsnorm_for(d_eh_, w.ln_in, d_ehn_, rows, EH, c.e_eps, w.wq.int8 || (w.self_attn && w.wkv.int8),
                                st));
            VSB_TRY(linear_q(w.wq, d_q_, d_qs_, d_ehn_, EH, rows, d_eq_, eQF, 0, nullptr, 0, st));
            AttBatch bs;
            bs.n = B;
            bs.q = (long long)C * eQF;
            bs.o = (long long)C * eQF;
            const AttQuant eq = att_quant(rows, eQF, C);   // the o-projection's int8 input, from the attention
            if (w.wo.int8 && !eq.q) return cudaErrorInvalidValue;
            if (w.self_attn) {
                VSB_TRY(linear_q(w.wkv, d_q_, d_qs_, d_ehn_, EH, rows, d_ekv_, 2 * KV, 0, nullptr, 0, st));
                VSB_TRY(rope_table(d_eq_, eQF, rows, c.e_nq, c.e_hd, d_pos_full_, rope_aex_, max_pos_, d_status_, st));
                VSB_TRY(kv_scatter_rope(d_ekv_, B, C, KV, c.e_hd, d_pos_full_, rope_aex_, max_pos_, d_kvf_[L], np,
                                        d_status_, st));
                bs.k = bs.v = (long long)SK * 2 * KV;
                bs.mask = (long long)C * SK;
                VSB_TRY(attention_batched(d_eq_, eQF, d_kvf_[L], 2 * KV, d_kvf_[L] + KV, 2 * KV, d_eatt_, eQF, C, SK,
                                          c.e_nq, c.e_nkv, c.e_hd, scale, d_dmask_, bs, st, w.wo.int8 ? &eq : nullptr));
            } else {
                VSB_TRY(rope_table(d_eq_, eQF, rows, c.e_nq, c.e_hd, d_pos_reb_, rope_aex_, max_pos_, d_status_, st));
                bs.k = bs.v = (long long)np * 2 * KV;
                bs.mask = (long long)C * np;
                VSB_TRY(attention_batched(d_eq_, eQF, d_ckv_[L], 2 * KV, d_ckv_[L] + KV, 2 * KV, d_eatt_, eQF, C, np,
                                          c.e_nq, c.e_nkv, c.e_hd, scale, d_cmask_, bs, st, w.wo.int8 ? &eq : nullptr));
            }
            VSB_TRY(linear_q(w.wo, d_q_, d_qs_, d_eatt_, eQF, rows, d_eh_, EH, kEpiAdd, d_eh_, EH, st));
            VSB_TRY(rmsnorm_for(d_eh_, w.ln_post, d_ehn_, rows, EH, c.e_eps, w.wgu.int8, st));
            VSB_TRY(linear_q(w.wgu, d_q_, d_qs_, d_ehn_, EH, rows, d_egu_, 2 * EF, 0, nullptr, 0, st));
            if (w.wdown.int8) {
                VSB_TRY(silu_gate_rows(d_egu_, rows, EF, nullptr, d_q_, round16(EF), d_qs_, st));
                VSB_TRY(linear_q(w.wdown, d_q_, d_qs_, nullptr, 0, rows, d_eh_, EH, kEpiAdd, d_eh_, EH, st));
            } else {
                VSB_TRY(silu_gate_rows(d_egu_, rows, EF, d_act_, nullptr, 0, nullptr, st));
                VSB_TRY(linear(w.wdown, d_act_, EF, rows, d_eh_, EH, kEpiAdd, d_eh_, EH, st));
            }
        }
        VSB_TRY(rmsnorm(d_eh_, out_norm_, d_ehn_, rows, EH, c.e_eps, st));
        VSB_TRY(linear_f32(d_ehn_, EH, aout_.W, aout_.bias, d_v_t_, MAD, rows, MAD, EH, nullptr, nullptr, st));
        VSB_TRY(flow_update(d_x_t_, d_v_t_, B, C, MAD, guided ? d_guide_ : nullptr, guided ? d_weights_ : nullptr,
                            time_[k], guided ? d_weights_ + (size_t)max_batch_ * C + k : nullptr, dt_, st));
    }
    return cudaSuccess;
}

cudaError_t SmolvlaPolicy::forward(int B, int h, int w, bool guided, cudaStream_t st, bool unnormalize) {
    const SmolvlaConfigDev& c = cfg_;
    const int np = c.n_prefix(), C = c.chunk;
    VSB_TRY(run_vision(B * c.n_views, h, w, st));
    VSB_TRY(smolvla_state(d_state_raw_, B, c.sd, c.msd, s_mean_, s_std_, c.norm_eps, d_state_n_, st));
    VSB_TRY(linear_f32(d_state_n_, c.msd, state_proj_.W, state_proj_.bias, d_state_row_, c.hidden, B, c.hidden, c.msd,
                       nullptr, nullptr, st));
    SmolvlaPrefix p;
    p.B = B;
    p.n_img = c.n_views * c.n_img_tok;
    p.n_lang = c.tok_maxlen;
    p.D = c.hidden;
    p.sq = std::sqrt(static_cast<float>(c.hidden));
    p.img = d_img_;
    p.emb = emb_;
    p.tokens = d_tokens_;
    p.state_row = d_state_row_;
    VSB_TRY(smolvla_prefix(p, d_x_, st));
    SmolvlaMaskArgs m;
    m.B = B;
    m.n_img = p.n_img;
    m.n_lang = p.n_lang;
    m.C = C;
    m.pmask = d_pmask_;
    m.dmask = d_dmask_;
    m.cmask = d_cmask_;
    m.pos = d_pos_;
    m.pos_full = d_pos_full_;
    m.pos_rebased = d_pos_reb_;
    VSB_TRY(smolvla_masks(d_lmask_, m, st));
    VSB_TRY(run_vlm(B, st));
    if (guided)
        VSB_TRY(smolvla_guide(d_prev_, B, C, c.mad, c.ad, prev_rows_, a_mean_, a_std_, c.norm_eps, d_guide_, st));
    VSB_TRY(run_expert(B, guided, st));
    (void)np;
    return smolvla_actions(d_x_t_, B, C, c.mad, c.ad, a_mean_, a_std_, c.norm_eps, unnormalize, d_actions_, st);
}

cudaError_t SmolvlaPolicy::predict(int B, const uint8_t* frames, int h, int w, const int32_t* tokens,
                                   const int32_t* mask, int n_lang, const float* state, const float* noise,
                                   const uint64_t* seeds, const float* prev, int n_prev, const float* weights,
                                   float max_guidance, bool unnormalize, float* actions) {
    const SmolvlaConfigDev& c = cfg_;
    if (B < 1 || B > max_batch_ || !frames || h <= 0 || w <= 0 || !tokens || !mask || !state || !actions ||
        (!noise && !seeds) || n_lang != c.tok_maxlen || n_prev < 0 || n_prev > c.chunk || (n_prev > 0 && !weights))
        return cudaErrorInvalidValue;
    for (int i = 0; i < B * n_lang; ++i)
        if (tokens[i] < 0 || tokens[i] >= c.vocab) return cudaErrorInvalidValue;   // smolvla_model.cpp:157-167
    int prevdev = 0;
    cudaGetDevice(&prevdev);
    if (prevdev != device_) cudaSetDevice(device_);
    const cudaError_t e0 = [&]() -> cudaError_t {
        if (!ensure_frames(h, w)) return cudaErrorMemoryAllocation;
        const int C = c.chunk, MAD = c.mad;
        VSB_TRY(cudaMemcpyAsync(d_frames_, frames, (size_t)B * c.n_views * h * w * 3, cudaMemcpyHostToDevice, stream_));
        VSB_TRY(cudaMemcpyAsync(d_tokens_, tokens, sizeof(int) * (size_t)B * n_lang, cudaMemcpyHostToDevice, stream_));
        VSB_TRY(cudaMemcpyAsync(d_lmask_, mask, sizeof(int) * (size_t)B * n_lang, cudaMemcpyHostToDevice, stream_));
        VSB_TRY(cudaMemcpyAsync(d_state_raw_, state, sizeof(float) * (size_t)B * c.sd, cudaMemcpyHostToDevice, stream_));
        if (noise) {
            VSB_TRY(cudaMemcpyAsync(d_noise_, noise, sizeof(float) * (size_t)B * C * MAD, cudaMemcpyHostToDevice,
                                    stream_));
        } else {
            for (int b = 0; b < B; ++b) {   // the reference's draw (smolvla_capi.cpp:143-149)
                PolarNormal N(seeds[b]);
                for (int i = 0; i < C * MAD; ++i) h_noise_[(size_t)b * C * MAD + i] = N();
            }
            VSB_TRY(cudaMemcpyAsync(d_noise_, h_noise_, sizeof(float) * (size_t)B * C * MAD, cudaMemcpyHostToDevice,
                                    stream_));
        }
        const bool guided = n_prev > 0;
        if (guided) {
            for (int b = 0; b < B; ++b)
                VSB_TRY(cudaMemcpyAsync(d_prev_ + (size_t)b * n_prev * c.ad, prev + (size_t)b * n_prev * c.ad,
                                        sizeof(float) * (size_t)n_prev * c.ad, cudaMemcpyHostToDevice, stream_));
            VSB_TRY(cudaMemcpyAsync(d_weights_, weights, sizeof(float) * (size_t)B * C, cudaMemcpyHostToDevice,
                                    stream_));
            for (int k = 0; k < c.num_steps; ++k) gw_[k] = std::min(gw_base_[k], max_guidance);
            VSB_TRY(cudaMemcpyAsync(d_weights_ + (size_t)max_batch_ * C, gw_.data(), sizeof(float) * c.num_steps,
                                    cudaMemcpyHostToDevice, stream_));
            VSB_TRY(cudaStreamSynchronize(stream_));   // gw_ is host memory the copy reads
        }
        prev_rows_ = n_prev;
        const long long key = (((((long long)B * 8192 + h) * 8192 + w) * 2 + (guided ? 1 : 0)) * 1024 + n_prev) * 2 +
                              (unnormalize ? 1 : 0);
        if (!use_graph_) {
            VSB_TRY(forward(B, h, w, guided, stream_, unnormalize));
        } else {
            cudaGraphExec_t& g = graphs_[key];
            if (!g) {
                cudaGraph_t gr = nullptr;
                cudaError_t e = cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal);
                if (e == cudaSuccess) {
                    const cudaError_t fe = forward(B, h, w, guided, stream_, unnormalize);
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
                if (e != cudaSuccess) {
                    g = nullptr;
                    return e;
                }
            }
            VSB_TRY(cudaGraphLaunch(g, stream_));
        }
        const size_t ab = sizeof(float) * (size_t)B * C * c.ad;
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
    if (prevdev != device_) cudaSetDevice(prevdev);
    return e0;
}

}  // namespace vsb
