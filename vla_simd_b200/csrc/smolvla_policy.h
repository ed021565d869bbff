// SmolVLA on one B200: the reference's SmolvlaModel (src/models/smolvla/smolvla_model.h:18-58)
// and its C ABI handle (smolvla_capi.cpp:28-33) re-built around device-resident
// weights, batched queries and one CUDA graph per (batch, frame size, guidance,
// unnormalize).
//
// Load reads the converter's checkpoint (vit / vlm / aex / heads .meta + .bin,
// emb.bin, stats, config.txt, and the tokenizer's vocab.txt + merges.txt),
// widens the bf16 towers to fp32 once, packs the layers SMOLVLA_INT8 selects
// exactly as the reference's apply_int8 does, and uploads everything. A query
// (one graph): resize-with-pad of every view, the SigLIP tower and connector,
// the prefix [image tokens | prompt | state], the SmolLM2 prefix pass that
// fills the K/V cache, the expert's cross-attention K/V reprojections, then
// `num_steps` flow-matching steps of the action expert (optionally with
// real-time-chunking guidance) and the unnormalized chunk.
#pragma once
#include <cuda_runtime.h>

#include "bpe_tokenizer.h"
#include "conv_exec.h"
#include "nn.h"

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace vsb {

class ModelFiles;

struct SmolvlaConfigDev {
    // vision (vit.meta)
    int v_hidden = 768, v_heads = 12, v_hd = 64, v_inter = 3072, v_layers = 12, patch = 16, img = 512,
        n_patches = 1024, sf = 4, mm_out = 960, n_img_tok = 64;
    float v_eps = 1e-6f;
    // text tower (vlm.meta)
    int hidden = 960, n_q = 15, n_kv = 5, hd = 64, ffn = 2560, vlm_layers = 32;
    float rms_eps = 1e-5f, rope_base = 10000.0f;
    // action expert (aex.meta)
    int eh = 480, ef = 1280, e_nq = 15, e_nkv = 5, e_hd = 64, e_layers = 32, san = 2, chunk = 50, num_steps = 10,
        mad = 32;
    float e_eps = 1e-5f, e_rope_base = 10000.0f;
    double min_period = 4e-3, max_period = 4.0;
    // heads.meta / config.txt
    int vocab = 0, msd = 32, sd = 0, ad = 0, n_views = 2, tok_maxlen = 48, pad_id = 2;
    float norm_eps = 1e-8f;
    int qf() const { return n_q * hd; }
    int kvf() const { return n_kv * hd; }
    int n_prefix() const { return n_views * n_img_tok + tok_maxlen + 1; }
};

struct SmolVitLayerDev {
    float *ln1s = nullptr, *ln1b = nullptr, *ln2s = nullptr, *ln2b = nullptr;
    DevLinear wqkv, wo, w1, w2;
};

struct SmolVlmLayerDev {
    float *ln_in = nullptr, *ln_post = nullptr;
    DevLinear wqkv, wo, wgu, wdown;   // q;k;v stacked, gate;up stacked
};

struct SmolExpertLayerDev {
    bool self_attn = true;
    float *ln_in = nullptr, *ln_post = nullptr;
    DevLinear wq, wkv, wk, wv, wo, wgu, wdown;   // wkv (k;v) for self layers, wk / wv for cross layers
};

class SmolvlaPolicy {
  public:
    ~SmolvlaPolicy();
    bool load(const std::string& dir, const std::string& tok_dir, int max_batch = 1);
    const std::string& error() const { return err_; }

    // vla_smolvla_tokenize (smolvla_capi.cpp:94-114): ids / mask [tok_maxlen]; returns the token count.
    int tokenize(const char* text, int32_t* ids, int32_t* mask) const;

    // Host buffers, `batch` queries of one frame size: frames [batch][n_views][h][w][3]
    // uint8, lang tokens / mask [batch][n_lang] (n_lang == tok_maxlen), raw
    // state [batch][state_dim], noise [batch][chunk][max_action_dim] or null
    // (drawn per query from seeds[b] as the reference draws it); optional RTC
    // guidance prev [batch][n_prev][action_dim] with weights [batch][chunk] and
    // max_guidance. actions [batch][chunk][action_dim]. Synchronous.
    cudaError_t predict(int batch, const uint8_t* frames, int h, int w, const int32_t* tokens, const int32_t* mask,
                        int n_lang, const float* state, const float* noise, const uint64_t* seeds, const float* prev,
                        int n_prev, const float* weights, float max_guidance, bool unnormalize, float* actions);

    const SmolvlaConfigDev& config() const { return cfg_; }
    int max_batch() const { return max_batch_; }
    int int8_layers() const { return n_int8_; }
    int kernels_per_step() const { return kernels_per_step_; }

    cudaError_t forward(int B, int h, int w, bool guided, cudaStream_t st, bool unnormalize);

  private:
    bool load_vit(const ModelFiles& files, int mask);
    bool load_vlm(const ModelFiles& files, bool int8);
    bool load_expert(const ModelFiles& files, bool int8);
    bool load_heads(const ModelFiles& files);
    bool alloc_buffers();
    bool ensure_frames(int h, int w);
    cudaError_t linear(const DevLinear& l, const float* x, long long ldx, int M, float* out, long long ldo, int mode,
                       const float* res, long long ldr, cudaStream_t st);
    // RMSNorm of x into xn; with int8, also the per-row int8 copy into the
    // shared quantization buffer (d_q_ / d_qs_) for the linears that read xn.
    cudaError_t rmsnorm_for(const float* x, const float* w, float* xn, int rows, int K, float eps, bool int8,
                            cudaStream_t st);
    cudaError_t linear_q(const DevLinear& l, const int8_t* q, const float* qs, const float* x, long long ldx, int M,
                         float* out, long long ldo, int mode, const float* res, long long ldr, cudaStream_t st);
    cudaError_t run_vision(int F, int h, int w, cudaStream_t st);
    cudaError_t run_vlm(int B, cudaStream_t st);
    cudaError_t run_expert(int B, bool guided, cudaStream_t st);
    template <class T> T* dalloc(size_t n);
    void fail(const std::string& m) { if (err_.empty()) err_ = m; }

    std::string err_;
    SmolvlaConfigDev cfg_;
    int device_ = 0;
    int max_batch_ = 1;
    int n_int8_ = 0;
    int kernels_per_step_ = 0;
    BpeTokenizer tok_;

    // vision
    DevLinear patch_, mm_proj_;
    float *pos_emb_ = nullptr, *post_s_ = nullptr, *post_b_ = nullptr;
    std::vector<SmolVitLayerDev> vit_;
    // text tower, expert
    std::vector<SmolVlmLayerDev> vlm_;
    std::vector<SmolExpertLayerDev> aex_;
    float* out_norm_ = nullptr;
    DevLinear ain_, at1_, at2_, aout_;   // fp32 (the reference's plain dense_linear)
    // heads
    uint16_t* emb_ = nullptr;
    DevLinear state_proj_;
    float *s_mean_ = nullptr, *s_std_ = nullptr, *a_mean_ = nullptr, *a_std_ = nullptr;
    // RoPE tables [max_pos + 1][hd/2][2] (double) for the text tower and the expert
    double *rope_vlm_ = nullptr, *rope_aex_ = nullptr;
    int max_pos_ = 0;
    // per-step flow constants
    float* te_ = nullptr;   // [num_steps][eh] time embeddings
    std::vector<float> time_, gw_base_;
    float dt_ = 0.0f;

    // inputs
    uint8_t* d_frames_ = nullptr;
    size_t frames_cap_ = 0;
    int *d_tokens_ = nullptr, *d_lmask_ = nullptr;
    float *d_state_raw_ = nullptr, *d_noise_ = nullptr, *d_prev_ = nullptr, *d_weights_ = nullptr;
    float* d_actions_ = nullptr;
    int prev_rows_ = 0;
    float max_guidance_ = 0.0f;
    std::vector<float> gw_;   // per step, min(base, max_guidance) of the current call

    // vision scratch
    float *d_pix_ = nullptr, *d_patches_ = nullptr, *d_vh_ = nullptr, *d_vn_ = nullptr, *d_vqkv_ = nullptr,
          *d_vatt_ = nullptr, *d_vff_ = nullptr, *d_shuf_ = nullptr, *d_img_ = nullptr;
    // prefix + text tower
    float *d_state_n_ = nullptr, *d_state_row_ = nullptr, *d_x_ = nullptr, *d_xn_ = nullptr, *d_att_ = nullptr,
          *d_gu_ = nullptr;
    float *d_pmask_ = nullptr, *d_dmask_ = nullptr, *d_cmask_ = nullptr;
    int *d_pos_ = nullptr, *d_pos_full_ = nullptr, *d_pos_reb_ = nullptr;
    std::vector<float*> d_cache_;   // per text layer: [B*np][qf + 2kvf] (q | rotated k | v)
    // expert
    std::vector<float*> d_kvf_;     // self layers: [B][np + C][2kvf]
    std::vector<float*> d_ckv_;     // cross layers: [B*np][2kvf]
    float *d_eh_ = nullptr, *d_ehn_ = nullptr, *d_eq_ = nullptr, *d_ekv_ = nullptr, *d_eatt_ = nullptr,
          *d_egu_ = nullptr, *d_aemb_ = nullptr, *d_at_ = nullptr, *d_mlp1_ = nullptr, *d_x_t_ = nullptr,
          *d_v_t_ = nullptr, *d_guide_ = nullptr;
    float* d_act_ = nullptr;   // SwiGLU output of fp32 down projections
    int8_t* d_q_ = nullptr;
    float* d_qs_ = nullptr;
    size_t q_cap_ = 0, q_rows_ = 0;
    static constexpr int kAttCounters = 1 << 17;   // attention query-tile arrival counters (fused quantization)
    unsigned int* d_att_cnt_ = nullptr;
    AttQuant att_quant(int rows, int K, int seq_rows) const;

    std::vector<void*> allocs_;
    float* h_pinned_ = nullptr;
    float* h_noise_ = nullptr;
    int* h_status_pinned_ = nullptr;
    int* d_status_ = nullptr;
    cudaStream_t stream_ = nullptr;
    std::map<long long, cudaGraphExec_t> graphs_;
    bool use_graph_ = true;
};

}  // namespace vsb
