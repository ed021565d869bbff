// extern "C" boundary of libvla_simd_b200.so: include/vla_simd.h (model level)
// and include/vla_simd_cuda.h (op level). Exceptions are fenced here, CUDA
// errors map to VLA_ERR_DEVICE, argument checks to VLA_ERR_ARG.
#include "../../include/vla_simd.h"
#include "../../include/vla_simd_cuda.h"

#include "act_policy.h"
#include "dp_policy.h"
#include "dp.h"
#include "octo_policy.h"
#include "smolvla_policy.h"
#include "bpe_tokenizer.h"
#include "t5_tokenizer.h"
#include "gemm_i8.h"
#include "lm_ops.h"
#include "nn.h"
#include "quant.h"

#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <new>
#include <vector>

using vsb::ActPolicy;
using vsb::DpPolicy;
using vsb::OctoPolicy;
using vsb::SmolvlaPolicy;

namespace {

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int32_t status_of(cudaError_t e) {
    if (e == cudaSuccess) return VLA_OK;
    if (e == cudaErrorInvalidValue) return VLA_ERR_ARG;
    return VLA_ERR_DEVICE;
}

int64_t ld16(int64_t k) { return (k + 15) & ~int64_t(15); }

bool k_ok(int32_t K) { return K > 0 && K <= INT_MAX / (255 * 127); }

// Grow-only device workspace for the host-pointer shims (one per thread).
struct Workspace {
    void* p = nullptr;
    size_t n = 0;
    int dev = -1;
    ~Workspace() {
        if (p) cudaFree(p);
    }
    void* get(size_t bytes) {
        int d = 0;
        cudaGetDevice(&d);
        if (p && (bytes > n || d != dev)) {
            cudaFree(p);
            p = nullptr;
            n = 0;
        }
        if (!p) {
            if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
            n = bytes;
            dev = d;
        }
        return p;
    }
};
thread_local Workspace g_ws;

// carve 256-byte aligned pieces out of one allocation
struct Carver {
    char* base;
    size_t off = 0;
    template <class T>
    T* take(size_t count) {
        off = (off + 255) & ~size_t(255);
        T* r = reinterpret_cast<T*>(base + off);
        off += count * sizeof(T);
        return r;
    }
};
size_t carve_size(std::initializer_list<size_t> bytes) {
    size_t s = 0;
    for (size_t b : bytes) s += ((b + 255) & ~size_t(255)) + 256;
    return s;
}

}  // namespace

extern "C" {

// ------------------------------------------------------------ model level

int32_t vla_abi_version(void) { return VLA_ABI_VERSION; }

const char* vla_backend_name(void) { return "cuda-sm100a"; }

int32_t vla_int8_available(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) return 0;
    int dev = 0;
    cudaGetDevice(&dev);
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    return major == 10 ? 1 : 0;
}

void* vla_act_load(const char* model_dir) try {
    if (!model_dir) return nullptr;
    auto m = std::make_unique<ActPolicy>();
    if (!m->load(model_dir)) {
        std::fprintf(stderr, "vla_act_load: %s\n", m->error().c_str());
        return nullptr;
    }
    return m.release();
} catch (...) {
    return nullptr;
}

void vla_act_free(void* h) { delete static_cast<ActPolicy*>(h); }

int32_t vla_act_chunk(void* h) { return h ? static_cast<ActPolicy*>(h)->chunk() : 0; }
int32_t vla_act_action_dim(void* h) { return h ? static_cast<ActPolicy*>(h)->action_dim() : 0; }
int32_t vla_act_state_dim(void* h) { return h ? static_cast<ActPolicy*>(h)->state_dim() : 0; }
int32_t vla_act_n_cams(void* h) { return h ? static_cast<ActPolicy*>(h)->n_cams() : 0; }
int32_t vla_act_img_h(void* h) { return h ? static_cast<ActPolicy*>(h)->img_h() : 0; }
int32_t vla_act_img_w(void* h) { return h ? static_cast<ActPolicy*>(h)->img_w() : 0; }

int32_t vla_act_predict(void* h, const uint8_t* images, const float* state, int32_t unnormalize,
                        float* actions) try {
    if (!h || !images || !state || !actions) return VLA_ERR_ARG;
    return static_cast<ActPolicy*>(h)->predict(images, state, unnormalize != 0, actions) == cudaSuccess
               ? VLA_OK
               : VLA_ERR_DEVICE;
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_act_device_buffers(void* h, uint8_t** images, float** state, const float** actions) {
    if (!h) return VLA_ERR_ARG;
    auto* m = static_cast<ActPolicy*>(h);
    if (images) *images = m->device_images();
    if (state) *state = m->device_state();
    if (actions) *actions = m->device_actions();
    return VLA_OK;
}

int32_t vla_act_enqueue(void* h, void* stream, int32_t unnormalize) try {
    if (!h) return VLA_ERR_ARG;
    return status_of(static_cast<ActPolicy*>(h)->enqueue_step(as_stream(stream), unnormalize != 0));
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_act_kernels_per_step(void* h) { return h ? static_cast<ActPolicy*>(h)->kernels_per_step() : 0; }
int32_t vla_act_int8_layers(void* h) { return h ? static_cast<ActPolicy*>(h)->int8_layers() : 0; }

// ---------------------------------------------------- Diffusion Policy

void* vla_diffusion_load_batch(const char* model_dir, int32_t max_batch) try {
    if (!model_dir || max_batch < 1) return nullptr;
    auto m = std::make_unique<DpPolicy>();
    if (!m->load(model_dir, max_batch)) {
        std::fprintf(stderr, "vla_diffusion_load: %s\n", m->error().c_str());
        return nullptr;
    }
    return m.release();
} catch (...) {
    return nullptr;
}

void* vla_diffusion_load(const char* model_dir) { return vla_diffusion_load_batch(model_dir, 1); }

void vla_diffusion_free(void* h) { delete static_cast<DpPolicy*>(h); }

#define VSB_DP_GET(name, expr)                          \
    int32_t vla_diffusion_##name(void* h) {             \
        if (!h) return VLA_ERR_ARG;                     \
        const DpPolicy* m = static_cast<DpPolicy*>(h);  \
        return static_cast<int32_t>(expr);              \
    }
VSB_DP_GET(chunk, m->config().n_action_steps)
VSB_DP_GET(horizon, m->config().horizon)
VSB_DP_GET(action_dim, m->config().action_dim)
VSB_DP_GET(state_dim, m->config().state_dim)
VSB_DP_GET(n_cams, m->config().n_cams)
VSB_DP_GET(n_obs_steps, m->config().n_obs)
VSB_DP_GET(img_h, m->config().img_h)
VSB_DP_GET(img_w, m->config().img_w)
VSB_DP_GET(num_steps, m->num_steps())
VSB_DP_GET(is_ddim, m->config().ddim ? 1 : 0)
VSB_DP_GET(kernels_per_step, m->kernels_per_step())
VSB_DP_GET(int8_layers, m->int8_layers())
#undef VSB_DP_GET

int32_t vla_diffusion_predict_batch(void* h, int32_t batch, const uint8_t* frames, const float* state,
                                    int32_t unnormalize, float* actions, const float* noise) try {
    if (!h || !frames || !state || !actions) return VLA_ERR_ARG;
    auto* m = static_cast<DpPolicy*>(h);
    if (batch < 1 || batch > m->max_batch()) return VLA_ERR_SHAPE;
    return status_of(m->predict(batch, frames, state, noise, unnormalize != 0, actions));
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_diffusion_predict(void* h, const uint8_t* frames, const float* state, int32_t unnormalize,
                              float* actions, const float* noise) {
    return vla_diffusion_predict_batch(h, 1, frames, state, unnormalize, actions, noise);
}

int64_t vla_diffusion_global_cond(void* h, float* out, int64_t cap) try {
    return h ? static_cast<DpPolicy*>(h)->global_cond(out, cap) : -1;
} catch (...) {
    return -1;
}

int64_t vla_diffusion_debug_map(void* h, float* out, int64_t cap) try {
    return h ? static_cast<DpPolicy*>(h)->debug_map(out, cap) : -1;
} catch (...) {
    return -1;
}

int32_t vla_diffusion_device_buffers(void* h, uint8_t** frames, float** state, float** noise,
                                     const float** actions) {
    if (!h) return VLA_ERR_ARG;
    auto* m = static_cast<DpPolicy*>(h);
    if (frames) *frames = m->device_frames();
    if (state) *state = m->device_state();
    if (noise) *noise = m->device_noise();
    if (actions) *actions = m->device_actions();
    return VLA_OK;
}

int32_t vla_diffusion_enqueue(void* h, int32_t batch, void* stream, int32_t unnormalize) try {
    if (!h) return VLA_ERR_ARG;
    auto* m = static_cast<DpPolicy*>(h);
    if (batch < 1 || batch > m->max_batch()) return VLA_ERR_SHAPE;
    return status_of(m->enqueue(batch, as_stream(stream), unnormalize != 0));
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

// ---------------------------------------------------------------- Octo

void* vla_octo_load_batch(const char* model_dir, const char* tok_dir, int32_t max_batch) try {
    if (!model_dir || !tok_dir || max_batch < 1) return nullptr;
    auto m = std::make_unique<OctoPolicy>();
    if (!m->load(model_dir, tok_dir, max_batch)) {
        std::fprintf(stderr, "vla_octo_load: %s\n", m->error().c_str());
        return nullptr;
    }
    return m.release();
} catch (...) {
    return nullptr;
}

void* vla_octo_load(const char* model_dir, const char* tok_dir) { return vla_octo_load_batch(model_dir, tok_dir, 1); }

void vla_octo_free(void* h) { delete static_cast<OctoPolicy*>(h); }

int32_t vla_octo_horizon(void* h) { return h ? static_cast<OctoPolicy*>(h)->config().horizon : 0; }
int32_t vla_octo_action_dim(void* h) { return h ? static_cast<OctoPolicy*>(h)->config().action_dim : 0; }
int32_t vla_octo_max_window(void* h) { return h ? static_cast<OctoPolicy*>(h)->config().max_horizon : 0; }
int32_t vla_octo_num_steps(void* h) { return h ? static_cast<OctoPolicy*>(h)->config().steps : 0; }
int32_t vla_octo_embed_dim(void* h) { return h ? static_cast<OctoPolicy*>(h)->config().d : 0; }
int32_t vla_octo_int8_layers(void* h) { return h ? static_cast<OctoPolicy*>(h)->int8_layers() : 0; }
int32_t vla_octo_kernels_per_step(void* h) { return h ? static_cast<OctoPolicy*>(h)->kernels_per_step() : 0; }
int32_t vla_octo_t5_runs(void* h) { return h ? static_cast<OctoPolicy*>(h)->t5_runs() : 0; }

int32_t vla_octo_predict_batch(void* h, int32_t batch, const uint8_t* primary, const uint8_t* wrist, int32_t wnd,
                               const uint8_t* timestep_mask, const char* const* instructions, const float* noise,
                               const float* z, const uint64_t* seeds, int32_t unnormalize, float* actions) try {
    if (!h || !primary || !timestep_mask || !instructions || !actions) return VLA_ERR_ARG;
    auto* m = static_cast<OctoPolicy*>(h);
    if (batch < 1 || batch > m->max_batch()) return VLA_ERR_SHAPE;
    // the position tables hold max_window steps (octo_capi.cpp:46-48)
    if (wnd < 1 || wnd > m->config().max_horizon) return VLA_ERR_SHAPE;
    if ((noise == nullptr) != (z == nullptr) || (!noise && !seeds)) return VLA_ERR_ARG;
    for (int32_t b = 0; b < batch; ++b)
        if (!instructions[b]) return VLA_ERR_ARG;
    return status_of(m->predict(batch, primary, wrist, wnd, timestep_mask, instructions, noise, z, seeds,
                                unnormalize != 0, actions));
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_octo_predict_ex(void* h, const uint8_t* primary, const uint8_t* wrist, int32_t wnd,
                            const uint8_t* timestep_mask, const char* instruction, const float* noise, const float* z,
                            uint64_t seed, int32_t unnormalize, float* actions) {
    if (!instruction) return VLA_ERR_ARG;
    return vla_octo_predict_batch(h, 1, primary, wrist, wnd, timestep_mask, &instruction, noise, z, &seed,
                                  unnormalize, actions);
}

int32_t vla_octo_predict(void* h, const uint8_t* primary, const uint8_t* wrist, int32_t wnd,
                         const uint8_t* timestep_mask, const char* instruction, uint64_t seed, int32_t unnormalize,
                         float* actions) {
    return vla_octo_predict_ex(h, primary, wrist, wnd, timestep_mask, instruction, nullptr, nullptr, seed,
                               unnormalize, actions);
}

int32_t vla_t5_tokenize(const char* vocab_text, const char* text, int32_t max_len, int32_t* ids) try {
    if (!vocab_text || !text || !ids || max_len < 1) return VLA_ERR_ARG;
    vsb::T5Tokenizer tok;
    if (!tok.load_text(vocab_text)) return VLA_ERR_ARG;
    const std::vector<int> v = tok.encode(text, max_len);
    for (int32_t i = 0; i < max_len; ++i) ids[i] = v[static_cast<size_t>(i)];
    return VLA_OK;
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int64_t vla_octo_readout(void* h, float* out, int64_t cap) try {
    return h ? static_cast<OctoPolicy*>(h)->readout(out, cap) : -1;
} catch (...) {
    return -1;
}

int32_t vla_octo_device_buffers(void* h, uint8_t** primary, uint8_t** wrist, uint8_t** timestep_mask, float** noise,
                                float** z, const float** actions) {
    if (!h) return VLA_ERR_ARG;
    auto* m = static_cast<OctoPolicy*>(h);
    if (primary) *primary = m->device_primary();
    if (wrist) *wrist = m->device_wrist();
    if (timestep_mask) *timestep_mask = m->device_tmask();
    if (noise) *noise = m->device_noise();
    if (z) *z = m->device_z();
    if (actions) *actions = m->device_actions();
    return VLA_OK;
}

int32_t vla_octo_set_instruction(void* h, int32_t b, const char* instruction) try {
    if (!h || !instruction) return VLA_ERR_ARG;
    auto* m = static_cast<OctoPolicy*>(h);
    if (b < 0 || b >= m->max_batch()) return VLA_ERR_SHAPE;
    return status_of(m->set_instruction(b, instruction));
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_octo_enqueue(void* h, int32_t batch, int32_t wnd, int32_t wrist, void* stream, int32_t unnormalize) try {
    if (!h) return VLA_ERR_ARG;
    auto* m = static_cast<OctoPolicy*>(h);
    if (batch < 1 || batch > m->max_batch() || wnd < 1 || wnd > m->config().max_horizon) return VLA_ERR_SHAPE;
    return status_of(m->enqueue(batch, wnd, wrist != 0, as_stream(stream), unnormalize != 0));
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

// ------------------------------------------------------------- SmolVLA

void* vla_smolvla_load_batch(const char* model_dir, const char* tok_dir, int32_t max_batch) try {
    if (!model_dir || !tok_dir || max_batch < 1) return nullptr;
    auto m = std::make_unique<SmolvlaPolicy>();
    if (!m->load(model_dir, tok_dir, max_batch)) {
        std::fprintf(stderr, "vla_smolvla_load: %s\n", m->error().c_str());
        return nullptr;
    }
    return m.release();
} catch (...) {
    return nullptr;
}

void* vla_smolvla_load(const char* model_dir, const char* tok_dir) {
    return vla_smolvla_load_batch(model_dir, tok_dir, 1);
}

void vla_smolvla_free(void* h) { delete static_cast<SmolvlaPolicy*>(h); }

int32_t vla_smolvla_chunk(void* h) { return h ? static_cast<SmolvlaPolicy*>(h)->config().chunk : 0; }
int32_t vla_smolvla_action_dim(void* h) { return h ? static_cast<SmolvlaPolicy*>(h)->config().ad : 0; }
int32_t vla_smolvla_state_dim(void* h) { return h ? static_cast<SmolvlaPolicy*>(h)->config().sd : 0; }
int32_t vla_smolvla_n_views(void* h) { return h ? static_cast<SmolvlaPolicy*>(h)->config().n_views : 0; }
int32_t vla_smolvla_img_size(void* h) { return h ? static_cast<SmolvlaPolicy*>(h)->config().img : 0; }
int32_t vla_smolvla_tok_maxlen(void* h) { return h ? static_cast<SmolvlaPolicy*>(h)->config().tok_maxlen : 0; }
int32_t vla_smolvla_int8_layers(void* h) { return h ? static_cast<SmolvlaPolicy*>(h)->int8_layers() : 0; }
int32_t vla_smolvla_kernels_per_step(void* h) { return h ? static_cast<SmolvlaPolicy*>(h)->kernels_per_step() : 0; }

int32_t vla_smolvla_tokenize(void* h, const char* text, int32_t* ids, int32_t* mask) try {
    if (!h || !text || !ids || !mask) return VLA_ERR_ARG;
    return static_cast<SmolvlaPolicy*>(h)->tokenize(text, ids, mask);
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_smolvla_predict_batch(void* h, int32_t batch, const uint8_t* frames, int32_t n_views, int32_t height,
                                  int32_t width, const int32_t* lang_tokens, const int32_t* lang_mask, int32_t n_lang,
                                  const float* state, const float* noise, const uint64_t* seeds, float* actions,
                                  const float* prev, int32_t n_prev, const float* weights, float max_guidance) try {
    if (!h || !frames || !lang_tokens || !lang_mask || !state || !actions) return VLA_ERR_ARG;
    if (height <= 0 || width <= 0 || n_lang < 0 || n_prev < 0) return VLA_ERR_ARG;
    if (!noise && !seeds) return VLA_ERR_ARG;
    if (!prev) n_prev = 0;
    if (n_prev > 0 && (!weights || !(std::isfinite(max_guidance) && max_guidance > 0))) return VLA_ERR_ARG;
    auto* m = static_cast<SmolvlaPolicy*>(h);
    const vsb::SmolvlaConfigDev& c = m->config();
    if (batch < 1 || batch > m->max_batch() || n_views != c.n_views || n_prev > c.chunk) return VLA_ERR_SHAPE;
    if (n_lang != c.tok_maxlen) return VLA_ERR_SHAPE;
    for (int64_t i = 0; n_prev > 0 && i < (int64_t)batch * c.chunk; i++)
        if (!std::isfinite(weights[i])) return VLA_ERR_ARG;
    for (int64_t i = 0; i < (int64_t)batch * n_prev * c.ad; i++)
        if (!std::isfinite(prev[i])) return VLA_ERR_ARG;
    for (int64_t i = 0; i < (int64_t)batch * n_lang; i++)   // a token past the vocab (smolvla_model.cpp:157-167)
        if (lang_tokens[i] < 0 || lang_tokens[i] >= c.vocab) return VLA_ERR_SHAPE;
    return status_of(m->predict(batch, frames, height, width, lang_tokens, lang_mask, n_lang, state, noise, seeds,
                                prev, n_prev, weights, max_guidance, true, actions));
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_smolvla_predict_rtc(void* h, const uint8_t* frames, int32_t n_views, int32_t height, int32_t width,
                                const int32_t* lang_tokens, const int32_t* lang_mask, int32_t n_lang,
                                const float* state, const float* noise, uint64_t seed, float* actions,
                                const float* prev, int32_t n_prev, const float* weights, float max_guidance) {
    return vla_smolvla_predict_batch(h, 1, frames, n_views, height, width, lang_tokens, lang_mask, n_lang, state,
                                     noise, &seed, actions, prev, n_prev, weights, max_guidance);
}

int32_t vla_smolvla_predict(void* h, const uint8_t* frames, int32_t n_views, int32_t height, int32_t width,
                            const int32_t* lang_tokens, const int32_t* lang_mask, int32_t n_lang, const float* state,
                            const float* noise, uint64_t seed, float* actions) {
    return vla_smolvla_predict_rtc(h, frames, n_views, height, width, lang_tokens, lang_mask, n_lang, state, noise,
                                   seed, actions, nullptr, 0, nullptr, 0.0f);
}

int32_t vla_bpe_tokenize(const char* vocab_text, const char* merges_text, const char* text, int32_t* ids,
                         int32_t cap) try {
    if (!vocab_text || !merges_text || !text || cap < 0 || (!ids && cap > 0)) return VLA_ERR_ARG;
    vsb::BpeTokenizer tok;
    if (!tok.load_text(vocab_text, merges_text)) return VLA_ERR_ARG;
    const std::vector<int> v = tok.encode(text);
    for (int32_t i = 0; i < cap && i < (int32_t)v.size(); ++i) ids[i] = v[static_cast<size_t>(i)];
    return static_cast<int32_t>(v.size());
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

// --------------------------------------------------------------- op level

int64_t vla_cuda_i8_ld(int32_t K) { return K > 0 ? ld16(K) : 0; }

int32_t vla_cuda_device_status(void) { return vsb::device_status_take(); }

int32_t vla_cuda_quantize_act_i8(const float* x, int8_t* xq, float* ascale, int32_t seq, int32_t K, int64_t ldq,
                                 void* stream) {
    if (!x || !xq || !ascale || seq <= 0 || K <= 0 || ldq < K) return VLA_ERR_ARG;
    return status_of(vsb::quantize_rows(x, K, nullptr, 0, seq, K, xq, ldq, ascale, nullptr, 0, nullptr,
                                        as_stream(stream)));
}

int32_t vla_cuda_quantize_span_i8(const float* x, int8_t* q, int64_t n, float inv, void* stream) {
    if (n < 0 || (n > 0 && (!x || !q))) return VLA_ERR_ARG;
    return status_of(vsb::quantize_span_i8(x, q, n, inv, as_stream(stream)));
}

int32_t vla_cuda_pack_weights_i8(const float* W, int8_t* Wq, float* wscale, int32_t N, int32_t K, int64_t ldw,
                                 void* stream) {
    if (!W || !Wq || !wscale || N <= 0 || K <= 0 || ldw < K) return VLA_ERR_ARG;
    return status_of(vsb::quantize_rows(W, K, nullptr, 0, N, K, Wq, ldw, wscale, nullptr, 0, nullptr,
                                        as_stream(stream)));
}

int32_t vla_cuda_gemm_i8(void* out, int64_t ldo, const int8_t* xq, int64_t ldx, const float* ascale,
                         int32_t ascale_per_row, const int8_t* Wq, int64_t ldw, const float* wscale,
                         const float* bias, const float* res, int64_t ldr, int32_t M, int32_t N, int32_t K,
                         int32_t mode, uint32_t* amax, int32_t amax_rows, int32_t force_simt, void* stream) {
    if (!out || !xq || !Wq || M <= 0 || N <= 0 || !k_ok(K) || ldx < K || ldw < K || ldo < N) return VLA_ERR_ARG;
    if (!(mode & VLA_EPI_ACC) && (!ascale || !wscale)) return VLA_ERR_ARG;
    if ((mode & (VLA_EPI_ADD | VLA_EPI_ADD_RELU)) && (!res || ldr < N)) return VLA_ERR_ARG;
    if (mode & ~(VLA_EPI_RELU | VLA_EPI_ADD | VLA_EPI_ADD_RELU | VLA_EPI_ACC)) return VLA_ERR_ARG;
    vsb::GemmI8Args a;
    a.A = xq;
    a.lda = ldx;
    a.B = Wq;
    a.ldb = ldw;
    a.M = M;
    a.N = N;
    a.K = K;
    a.out = out;
    a.ldo = ldo;
    a.ascale = ascale;
    a.ascale_per_row = ascale_per_row != 0;
    a.wscale = wscale;
    a.bias = bias;
    a.res = res;
    a.ldr = ldr;
    a.mode = mode;
    a.amax = amax;
    a.amax_rows = amax_rows > 0 ? amax_rows : 1;
    a.force_simt = force_simt != 0;
    return status_of(vsb::gemm_i8(a, as_stream(stream)));
}

int32_t vla_cuda_gemm_i8_rowq_supported(int32_t M, int32_t N, int32_t K) {
    return (M > 0 && N > 0 && k_ok(K) && vsb::gemm_i8_rowq_supported(M, N, K)) ? 1 : 0;
}

int32_t vla_cuda_gemm_i8_rowq(int8_t* q, int64_t ldq, float* qscale, const int8_t* xq, int64_t ldx,
                              const float* ascale, const int8_t* Wq, int64_t ldw, const float* wscale,
                              const float* bias, int32_t M, int32_t N, int32_t K, int32_t relu, uint32_t* qamax,
                              uint32_t* qsync, void* stream) {
    if (!q || !qscale || !xq || !ascale || !Wq || !wscale || !qamax || !qsync || M <= 0 || N <= 0 || !k_ok(K) ||
        ldx < K || ldw < K || ldq != N)
        return VLA_ERR_ARG;
    if (!vsb::gemm_i8_rowq_supported(M, N, K)) return VLA_ERR_SHAPE;
    vsb::GemmI8Args a;
    a.A = xq;
    a.lda = ldx;
    a.B = Wq;
    a.ldb = ldw;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ascale = ascale;
    a.wscale = wscale;
    a.bias = bias;
    a.mode = relu ? VLA_EPI_RELU : 0;
    a.qout = q;
    a.ldq = ldq;
    a.qscale = qscale;
    a.qamax = qamax;
    a.qsync = qsync;
    return status_of(vsb::gemm_i8(a, as_stream(stream)));
}

int32_t vla_cuda_gemm_i8_splitk(void* out, int64_t ldo, const int8_t* xq, int64_t ldx, const float* ascale,
                                const int8_t* Wq, int64_t ldw, const float* wscale, const float* bias,
                                const float* res, int64_t ldr, int32_t M, int32_t N, int32_t K, int32_t mode,
                                int32_t* ws, int64_t ws_elems, uint32_t* counters, int32_t n_counters,
                                void* stream) {
    if (!out || !xq || !Wq || M <= 0 || M > 128 || N <= 0 || !k_ok(K) || ldx < K || ldw < K || ldo < N ||
        !ws || ws_elems <= 0 || !counters || n_counters <= 0)
        return VLA_ERR_ARG;
    if (!(mode & VLA_EPI_ACC) && (!ascale || !wscale)) return VLA_ERR_ARG;
    if ((mode & (VLA_EPI_ADD | VLA_EPI_ADD_RELU)) && (!res || ldr < N)) return VLA_ERR_ARG;
    if (mode & ~(VLA_EPI_RELU | VLA_EPI_ADD | VLA_EPI_ADD_RELU | VLA_EPI_ACC)) return VLA_ERR_ARG;
    vsb::GemmI8Args a;
    a.A = xq;
    a.lda = ldx;
    a.B = Wq;
    a.ldb = ldw;
    a.M = M;
    a.N = N;
    a.K = K;
    a.out = out;
    a.ldo = ldo;
    a.ascale = ascale;
    a.wscale = wscale;
    a.bias = bias;
    a.res = res;
    a.ldr = ldr;
    a.mode = mode;
    a.splitk_ws = ws;
    a.splitk_ws_elems = ws_elems;
    a.splitk_counters = counters;
    a.splitk_counters_n = n_counters;
    return status_of(vsb::gemm_i8(a, as_stream(stream)));
}

int32_t vla_cuda_dense_linear_i8_pre(float* out, const int8_t* xq, const float* ascale, const int8_t* Wq,
                                     const float* wscale, const float* bias, int32_t seq, int32_t N, int32_t K,
                                     int64_t ldx, int64_t ldw, void* stream) {
    if (!ascale || !wscale) return VLA_ERR_ARG;
    return vla_cuda_gemm_i8(out, N, xq, ldx, ascale, 1, Wq, ldw, wscale, bias, nullptr, 0, seq, N, K, 0, nullptr,
                            1, 0, stream);
}

int32_t vla_cuda_dense_linear_i8(float* out, const float* x, const int8_t* Wq, const float* wscale,
                                 const float* bias, int32_t seq, int32_t N, int32_t K, int64_t ldw,
                                 int8_t* xq_scratch, float* ascale_scratch, void* stream) {
    if (!out || !x || !xq_scratch || !ascale_scratch || seq <= 0 || !k_ok(K)) return VLA_ERR_ARG;
    const int32_t r = vla_cuda_quantize_act_i8(x, xq_scratch, ascale_scratch, seq, K, ld16(K), stream);
    if (r != VLA_OK) return r;
    return vla_cuda_dense_linear_i8_pre(out, xq_scratch, ascale_scratch, Wq, wscale, bias, seq, N, K, ld16(K), ldw,
                                        stream);
}

int32_t vla_cuda_conv2d_i8(float* out, const float* x, int32_t F, int32_t H, int32_t W, int32_t Cin,
                           const int8_t* Wq, int64_t ldw, const float* wscale, const float* bias, int32_t Cout,
                           int32_t k, int32_t stride, int32_t pad, float clip, int32_t mode, const float* res,
                           int8_t* col_scratch, float* rscale_scratch, uint32_t* amax_scratch, void* stream) {
    if (!out || !x || !Wq || !wscale || !col_scratch || !rscale_scratch || !amax_scratch) return VLA_ERR_ARG;
    if (F <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0 || k <= 0 || stride <= 0 || pad < 0) return VLA_ERR_ARG;
    if (!(clip > 0.0f && clip <= 1.0f)) return VLA_ERR_ARG;
    const int32_t K = k * k * Cin;
    if (!k_ok(K) || ldw < K || (ldw & 15)) return VLA_ERR_ARG;
    const int Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
    if (H + 2 * pad < k || W + 2 * pad < k || Ho <= 0 || Wo <= 0) return VLA_ERR_ARG;
    cudaStream_t st = as_stream(stream);
    cudaError_t e = cudaMemsetAsync(amax_scratch, 0, sizeof(uint32_t) * F, st);
    if (e == cudaSuccess) e = vsb::absmax_slots(x, (long long)F * H * W * Cin, (long long)H * W * Cin, amax_scratch, st);
    if (e == cudaSuccess && vsb::conv_i8_implicit_supported(Cin, k, stride) && !std::getenv("VLA_CONV_IM2COL")) {
        // stride 1, >= 64 channels: quantized NHWC input (fits col_scratch: F*H*W*Cin <= the
        // im2col matrix), taps gathered by the GEMM itself; VLA_CONV_IM2COL=1 keeps im2col
        e = vsb::quantize_frames_i8(x, F, (long long)H * W * Cin, amax_scratch, clip, col_scratch, rscale_scratch, st);
        if (e != cudaSuccess) return status_of(e);
        vsb::ConvI8Args a;
        a.x = col_scratch;
        a.F = F;
        a.H = H;
        a.W = W;
        a.C = Cin;
        a.k = k;
        a.pad = pad;
        a.Wq = Wq;
        a.ldw = ldw;
        a.N = Cout;
        a.fscale = rscale_scratch;
        a.wscale = wscale;
        a.bias = bias;
        a.out = out;
        a.res = res;
        a.mode = mode;
        return status_of(vsb::conv_i8_implicit(a, st));
    }
    if (e == cudaSuccess)
        e = vsb::im2col_i8(x, F, H, W, Cin, k, stride, pad, Ho, Wo, ldw, amax_scratch, clip, col_scratch,
                           rscale_scratch, st);
    if (e != cudaSuccess) return status_of(e);
    return vla_cuda_gemm_i8(out, Cout, col_scratch, ldw, rscale_scratch, 1, Wq, ldw, wscale, bias, res, Cout,
                            F * Ho * Wo, Cout, K, mode, nullptr, 1, 0, stream);
}

int32_t vla_cuda_layernorm(float* out, const float* x, const float* w, const float* b, int32_t seq, int32_t hidden,
                           float eps, void* stream) {
    if (!out || !x || !w || seq <= 0 || hidden <= 0 || hidden > 2048) return VLA_ERR_ARG;
    return status_of(vsb::layernorm(x, out, w, b, seq, hidden, eps, nullptr, nullptr, nullptr, nullptr, nullptr, 0,
                                    as_stream(stream)));
}

int32_t vla_cuda_gqa_attention(float* out, const float* Q, const float* K, const float* V, int32_t seq_q,
                               int32_t seq_k, int32_t n_q, int32_t n_kv, int32_t head_dim, float scale,
                               const float* mask, void* stream) {
    if (!out || !Q || !K || !V || seq_q <= 0 || seq_k <= 0 || n_q <= 0 || n_kv <= 0 || n_q % n_kv || head_dim != 64)
        return VLA_ERR_ARG;
    return status_of(vsb::attention(Q, (long long)n_q * head_dim, K, (long long)n_kv * head_dim, V,
                                    (long long)n_kv * head_dim, out, (long long)n_q * head_dim, seq_q, seq_k, n_q,
                                    n_kv, head_dim, scale, mask, as_stream(stream)));
}

int32_t vla_cuda_gqa_attention_tc(float* out, const float* Q, const float* K, const float* V, int32_t seq_q,
                                  int32_t seq_k, int32_t n_q, int32_t n_kv, int32_t head_dim, float scale,
                                  const float* mask, void* stream) {
    if (!out || !Q || !K || !V || seq_q <= 0 || seq_k <= 0 || n_q <= 0 || n_kv <= 0 || n_q % n_kv || head_dim != 64)
        return VLA_ERR_ARG;
    const uintptr_t a = reinterpret_cast<uintptr_t>(Q) | reinterpret_cast<uintptr_t>(K) |
                        reinterpret_cast<uintptr_t>(V) | reinterpret_cast<uintptr_t>(out);
    if (a & 15) return VLA_ERR_ARG;
    return status_of(vsb::attention_tc(Q, (long long)n_q * head_dim, K, (long long)n_kv * head_dim, V,
                                       (long long)n_kv * head_dim, out, (long long)n_q * head_dim, seq_q, seq_k, n_q,
                                       n_kv, scale, mask, vsb::AttBatch{}, as_stream(stream)));
}

int32_t vla_cuda_dense_linear_f32(float* out, const float* x, const float* W, const float* bias, int32_t seq,
                                  int32_t N, int32_t K, void* stream) {
    if (!out || !x || !W || seq <= 0 || N <= 0 || K <= 0) return VLA_ERR_ARG;
    return status_of(vsb::linear_f32(x, K, W, bias, out, N, seq, N, K, nullptr, nullptr, as_stream(stream)));
}

int32_t vla_cuda_maxpool2d_relu(float* out, const float* x, int32_t F, int32_t H, int32_t W, int32_t C, int32_t k,
                                int32_t stride, int32_t pad, void* stream) {
    if (!out || !x || F <= 0 || H <= 0 || W <= 0 || C <= 0 || k <= 0 || stride <= 0 || pad < 0) return VLA_ERR_ARG;
    const int Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
    if (Ho <= 0 || Wo <= 0) return VLA_ERR_ARG;
    return status_of(vsb::maxpool_relu(x, out, F, H, W, C, k, stride, pad, Ho, Wo, nullptr, as_stream(stream)));
}

// ------------------------------------------- lm / conv ops (other policies)

int32_t vla_cuda_rmsnorm(float* out, const float* x, const float* w, int32_t seq, int32_t hidden, float eps,
                         void* stream) {
    if (!out || !x || !w || seq <= 0 || hidden <= 0 || hidden > 6144) return VLA_ERR_ARG;
    return status_of(vsb::rmsnorm(x, w, out, seq, hidden, eps, as_stream(stream)));
}

int32_t vla_cuda_rope_neox(float* x, const int32_t* pos, int32_t seq, int32_t n_heads, int32_t head_dim, float base,
                           void* stream) {
    if (!x || !pos || seq <= 0 || n_heads <= 0 || head_dim <= 0 || head_dim % 2) return VLA_ERR_ARG;
    return status_of(vsb::rope_neox(x, pos, seq, n_heads, head_dim, base, as_stream(stream)));
}

static int32_t act_call(int kind, float* out, const float* x, const float* u, int64_t n, void* stream) {
    if (!out || !x || n <= 0) return VLA_ERR_ARG;
    return status_of(vsb::activation(kind, out, x, u, n, as_stream(stream)));
}
int32_t vla_cuda_silu_gate(float* out, const float* g, const float* u, int64_t n, void* stream) {
    if (!u) return VLA_ERR_ARG;
    return act_call(vsb::kActSiluGate, out, g, u, n, stream);
}
int32_t vla_cuda_silu(float* out, const float* x, int64_t n, void* stream) {
    return act_call(vsb::kActSilu, out, x, nullptr, n, stream);
}
int32_t vla_cuda_gelu_tanh(float* out, const float* x, int64_t n, void* stream) {
    return act_call(vsb::kActGeluTanh, out, x, nullptr, n, stream);
}
int32_t vla_cuda_gelu_erf(float* out, const float* x, int64_t n, void* stream) {
    return act_call(vsb::kActGeluErf, out, x, nullptr, n, stream);
}
int32_t vla_cuda_relu(float* out, const float* x, int64_t n, void* stream) {
    return act_call(vsb::kActRelu, out, x, nullptr, n, stream);
}
int32_t vla_cuda_mish(float* out, const float* x, int64_t n, void* stream) {
    return act_call(vsb::kActMish, out, x, nullptr, n, stream);
}

uint64_t vla_cuda_groupnorm_scratch_bytes(int32_t C) { return C > 0 ? vsb::groupnorm_scratch_bytes(C) : 0; }

int32_t vla_cuda_groupnorm(float* out, const float* x, const float* scale, const float* bias, int32_t n_pixels,
                           int32_t C, int32_t groups, float eps, int32_t fuse_relu, void* scratch, void* stream) {
    if (!out || !x || !scale || !bias || !scratch || n_pixels <= 0 || C <= 0 || groups <= 0 || C % groups)
        return VLA_ERR_ARG;
    return status_of(vsb::groupnorm(x, scale, bias, out, n_pixels, C, groups, eps, fuse_relu != 0, scratch,
                                    as_stream(stream)));
}

int32_t vla_cuda_spatial_softmax(float* out, const float* x, const float* grid, int32_t n_pixels, int32_t C,
                                 void* stream) {
    if (!out || !x || !grid || n_pixels <= 0 || C <= 0) return VLA_ERR_ARG;
    return status_of(vsb::spatial_softmax(x, grid, out, n_pixels, C, as_stream(stream)));
}

int32_t vla_cuda_im2col1d(float* col, const float* x, int32_t T, int32_t Cin, int32_t k, int32_t stride, int32_t pad,
                          int32_t Tout, void* stream) {
    if (!col || !x || T <= 0 || Cin <= 0 || k <= 0 || stride <= 0 || pad < 0 || Tout <= 0) return VLA_ERR_ARG;
    return status_of(vsb::im2col1d(x, col, T, Cin, k, stride, pad, Tout, as_stream(stream)));
}

int32_t vla_cuda_conv_transpose1d(float* out, const float* x, const float* W, const float* bias, int32_t T,
                                  int32_t Cin, int32_t Cout, int32_t k, int32_t stride, int32_t pad, void* stream) {
    if (!out || !x || !W || T <= 0 || Cin <= 0 || Cout <= 0 || k <= 0 || stride <= 0 || pad < 0 ||
        (T - 1) * stride - 2 * pad + k <= 0)
        return VLA_ERR_ARG;
    // the U-Net's one-sample kernels where they take the shape, else the general one
    cudaError_t e = vsb::conv_transpose1d_f(x, W, nullptr, bias, out, 1, T, Cin, Cout, k, stride, pad, nullptr,
                                            as_stream(stream));
    if (e == cudaErrorInvalidValue) {
        cudaGetLastError();
        e = vsb::conv_transpose1d(x, W, bias, out, T, Cin, Cout, k, stride, pad, as_stream(stream));
    }
    return status_of(e);
}

// ------------------------------------------------------ host-pointer shims

int32_t vla_tcpu_int8_gemm_available(void) { return vla_int8_available(); }

int32_t vla_tcpu_i8_kpad(int32_t K) { return (K + 3) & ~3; }

uint64_t vla_tcpu_packed_i8_words(int32_t N, int32_t K) {
    const uint64_t panel = (uint64_t)N * (uint64_t)vla_tcpu_i8_kpad(K);
    return (panel + (uint64_t)N * 4) / 4;
}

int32_t vla_tcpu_pack_weights_i8(const float* W, int8_t* Wq, float* wscale, int32_t N, int32_t K) try {
    if (!W || !Wq || !wscale || N <= 0 || N % 16 || K <= 0) return VLA_ERR_ARG;
    // quantize and pack on the device, then copy the reference's layout back
    const int64_t ld = ld16(K);
    const size_t packed = (size_t)N * vla_tcpu_i8_kpad(K) + sizeof(int32_t) * (size_t)N;
    void* base = g_ws.get(carve_size({sizeof(float) * (size_t)N * K, (size_t)N * ld, sizeof(float) * N, packed}));
    if (!base) return VLA_ERR_DEVICE;
    Carver c{static_cast<char*>(base)};
    float* dW = c.take<float>((size_t)N * K);
    int8_t* dq = c.take<int8_t>((size_t)N * ld);
    float* ds = c.take<float>(N);
    int8_t* dp = c.take<int8_t>(packed);
    cudaError_t e = cudaMemcpy(dW, W, sizeof(float) * (size_t)N * K, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = vsb::quantize_rows(dW, K, nullptr, 0, N, K, dq, ld, ds, nullptr, 0, nullptr, 0);
    if (e == cudaSuccess) e = vsb::pack_panels_i8(dq, ld, N, K, dp, 0);
    if (e == cudaSuccess) e = cudaMemcpy(Wq, dp, packed, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(wscale, ds, sizeof(float) * N, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && vsb::device_status_take() != 0) e = cudaErrorLaunchFailure;
    return status_of(e);
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

const int32_t* vla_tcpu_i8_rowsums(const int8_t* Wq, int32_t N, int32_t K) {
    if (!Wq || N <= 0 || K <= 0) return nullptr;
    return reinterpret_cast<const int32_t*>(Wq + (size_t)N * vla_tcpu_i8_kpad(K));
}

int32_t vla_tcpu_quantize_span_i8(const float* x, int8_t* q, uint64_t n, float inv) try {
    if (n == 0) return VLA_OK;
    if (!x || !q) return VLA_ERR_ARG;
    void* base = g_ws.get(carve_size({sizeof(float) * (size_t)n, (size_t)n}));
    if (!base) return VLA_ERR_DEVICE;
    Carver c{static_cast<char*>(base)};
    float* dx = c.take<float>(n);
    int8_t* dq = c.take<int8_t>(n);
    cudaError_t e = cudaMemcpy(dx, x, sizeof(float) * n, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = vsb::quantize_span_i8(dx, dq, (long long)n, inv, 0);
    if (e == cudaSuccess) e = cudaMemcpy(q, dq, n, cudaMemcpyDeviceToHost);
    return status_of(e);
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_tcpu_quantize_act_i8(const float* x, int8_t* xq, float* ascale, int32_t seq, int32_t K) try {
    if (!x || !xq || !ascale || seq <= 0 || K <= 0) return VLA_ERR_ARG;
    const int64_t ld = ld16(K);
    const int Kp = vla_tcpu_i8_kpad(K);
    void* base = g_ws.get(carve_size({sizeof(float) * (size_t)seq * K, (size_t)seq * ld, sizeof(float) * seq}));
    if (!base) return VLA_ERR_DEVICE;
    Carver c{static_cast<char*>(base)};
    float* dx = c.take<float>((size_t)seq * K);
    int8_t* dq = c.take<int8_t>((size_t)seq * ld);
    float* ds = c.take<float>(seq);
    cudaError_t e = cudaMemcpy(dx, x, sizeof(float) * (size_t)seq * K, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = vsb::quantize_rows(dx, K, nullptr, 0, seq, K, dq, ld, ds, nullptr, 0, nullptr, 0);
    if (e == cudaSuccess) e = cudaMemcpy2D(xq, Kp, dq, ld, Kp, seq, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(ascale, ds, sizeof(float) * seq, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && vsb::device_status_take() != 0) e = cudaErrorLaunchFailure;
    return status_of(e);
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

static int32_t tcpu_linear_pre(float* out, const int8_t* xq, const float* ascale, const int8_t* Wq,
                               const float* wscale, const float* bias, int32_t seq, int32_t N, int32_t K,
                               int32_t force_simt) try {
    if (!out || !xq || !ascale || !Wq || !wscale || seq <= 0 || N <= 0 || N % 16 || !k_ok(K)) return VLA_ERR_ARG;
    const int64_t ld = ld16(K);
    const int Kp = vla_tcpu_i8_kpad(K);
    const size_t panel_bytes = (size_t)N * Kp;
    void* base = g_ws.get(carve_size({(size_t)seq * ld, sizeof(float) * seq, panel_bytes, (size_t)N * ld,
                                      sizeof(float) * N, sizeof(float) * N, sizeof(float) * (size_t)seq * N}));
    if (!base) return VLA_ERR_DEVICE;
    Carver c{static_cast<char*>(base)};
    int8_t* dq = c.take<int8_t>((size_t)seq * ld);
    float* ds = c.take<float>(seq);
    int8_t* dp = c.take<int8_t>(panel_bytes);
    int8_t* dw = c.take<int8_t>((size_t)N * ld);
    float* dws = c.take<float>(N);
    float* db = c.take<float>(N);
    float* dout = c.take<float>((size_t)seq * N);
    cudaError_t e = cudaMemcpy2D(dq, ld, xq, Kp, Kp, seq, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(ds, ascale, sizeof(float) * seq, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dp, Wq, panel_bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(dws, wscale, sizeof(float) * N, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && bias) e = cudaMemcpy(db, bias, sizeof(float) * N, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = vsb::unpack_panels_i8(dp, N, K, dw, ld, 0);
    if (e != cudaSuccess) return status_of(e);
    const int32_t r = vla_cuda_gemm_i8(dout, N, dq, ld, ds, 1, dw, ld, dws, bias ? db : nullptr, nullptr, 0, seq, N,
                                       K, 0, nullptr, 1, force_simt, nullptr);
    if (r != VLA_OK) return r;
    e = cudaMemcpy(out, dout, sizeof(float) * (size_t)seq * N, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && vsb::device_status_take() != 0) e = cudaErrorLaunchFailure;
    return status_of(e);
} catch (...) {
    return VLA_ERR_EXCEPTION;
}

int32_t vla_tcpu_dense_linear_i8_pre(float* out, const int8_t* xq, const float* ascale, const int8_t* Wq,
                                     const float* wscale, const float* bias, int32_t seq, int32_t N, int32_t K) {
    return tcpu_linear_pre(out, xq, ascale, Wq, wscale, bias, seq, N, K, 0);
}

int32_t vla_tcpu_dense_linear_i8_ref(float* out, const int8_t* xq, const float* ascale, const int8_t* Wq,
                                     const float* wscale, const float* bias, int32_t seq, int32_t N, int32_t K) {
    return tcpu_linear_pre(out, xq, ascale, Wq, wscale, bias, seq, N, K, 1);
}

int32_t vla_tcpu_dense_linear_i8(float* out, const float* x, const int8_t* Wq, const float* wscale, const float* bias,
                                 int32_t seq, int32_t N, int32_t K, int8_t* xq_scratch, float* ascale_scratch) {
    if (!xq_scratch || !ascale_scratch) return VLA_ERR_ARG;
    const int32_t r = vla_tcpu_quantize_act_i8(x, xq_scratch, ascale_scratch, seq, K);
    if (r != VLA_OK) return r;
    return vla_tcpu_dense_linear_i8_pre(out, xq_scratch, ascale_scratch, Wq, wscale, bias, seq, N, K);
}

}  // extern "C"
