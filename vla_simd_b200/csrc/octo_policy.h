// Octo on one B200: the reference's OctoModel (src/models/octo/octo_model.h:21-52)
// re-built around device-resident weights, batched queries and one CUDA graph
// per (batch, window, wrist, unnormalize).
//
// Load reads the converter's checkpoint (t5.meta/.bin, stem_primary / stem_wrist
// .meta/.bin, octo.meta/.bin, head.meta/.bin, stats_action_{mean,std,mask}.bin,
// and the tokenizer's vocab.txt) from a directory or a vla.simd GGUF, packs the
// layers OCTO_INT8 selects exactly as the reference's apply_int8 does, and
// uploads everything once. A query: the instruction's T5 encoding (device,
// cached per instruction string like the reference's lang_cache), then one
// graph: both SmallStems over every frame of the window, the token sequence,
// the block-causal ViT (the last layer only for the readout row), and the
// 20-step DDPM diffusion head.
#pragma once
#include <cuda_runtime.h>

#include "conv_exec.h"
#include "nn.h"
#include "t5_tokenizer.h"

#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace vsb {

class ModelFiles;

struct OctoStemDev {
    int n_layers = 4, k = 3, stride = 2, pad = 1, embed_dim = 512, gn_groups = 32;
    float gn_eps = 1e-6f;
    std::vector<int> feat;
    std::vector<DevConv> conv;
    std::vector<float*> gn_s, gn_b;
    DevLinear embed;
    int in_hw = 256;   // square input side (256 primary, 128 wrist)
    int side = 16;     // output grid side
    int tokens() const { return side * side; }
};

struct OctoLayerDev {
    float *ln1s = nullptr, *ln1b = nullptr, *ln2s = nullptr, *ln2b = nullptr;
    DevLinear wqkv, wo, w1, w2;   // wq / wk / wv stacked: one GEMM, N = 3d
};

struct T5LayerDev {
    float *ln1 = nullptr, *ln2 = nullptr;
    float *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr, *wi = nullptr, *wo2 = nullptr;
};

struct OctoConfigDev {
    // transformer (octo.meta)
    int d = 384, n_layers = 12, heads = 6, head_dim = 64, mlp = 1536;
    int max_horizon = 10, n_task = 16, tok_primary = 256, tok_wrist = 64, n_readout = 1;
    int t5_dim = 768, stem_dim = 512;
    float ln_eps = 1e-6f;
    bool gelu_erf = false;
    // T5 (t5.meta)
    int t5_layers = 12, t5_heads = 12, t5_dkv = 64, t5_ff = 3072, t5_vocab = 32128, t5_buckets = 32, t5_max_dist = 128;
    float t5_eps = 1e-6f;
    // diffusion head (head.meta)
    int action_dim = 7, horizon = 4, time_dim = 32, num_blocks = 3, hidden = 256, steps = 20;
    float max_action = 5.0f;
    int flat() const { return action_dim * horizon; }
    int per_step() const { return tok_primary + tok_wrist + n_task + n_readout; }
    int total(int wnd) const { return n_task + wnd * per_step(); }
};

class OctoPolicy {
  public:
    ~OctoPolicy();
    // tok_dir holds vocab.txt (read through the model's GGUF when it lies
    // inside the model path). max_batch: the most queries one predict carries.
    bool load(const std::string& dir, const std::string& tok_dir, int max_batch = 1);
    const std::string& error() const { return err_; }

    // Host buffers, `batch` queries: primary [batch][wnd][256][256][3], wrist
    // [batch][wnd][128][128][3] or null, timestep masks [batch][wnd],
    // instructions[batch]; noise [batch][flat] and z [batch][steps][flat], or
    // both null to draw them per query from seeds[b] the way the reference
    // does (std::mt19937_64 + std::normal_distribution<float>). actions
    // [batch][horizon][action_dim]. Synchronous.
    cudaError_t predict(int batch, const uint8_t* primary, const uint8_t* wrist, int wnd, const uint8_t* tmask,
                        const char* const* instructions, const float* noise, const float* z, const uint64_t* seeds,
                        bool unnormalize, float* actions);

    // Device-side batch for benchmarks: frames, masks, noise and the cache
    // slots already in the device buffers (set_instruction fills slot b).
    cudaError_t enqueue(int batch, int wnd, bool wrist, cudaStream_t st, bool unnormalize);
    cudaError_t set_instruction(int b, const char* instruction);
    uint8_t* device_primary() { return d_prim_u8_; }
    uint8_t* device_wrist() { return d_wrist_u8_; }
    uint8_t* device_tmask() { return d_tmask_; }
    float* device_noise() { return d_noise_; }
    float* device_z() { return d_z_; }
    const float* device_actions() const { return d_actions_; }

    const OctoConfigDev& config() const { return cfg_; }
    int max_batch() const { return max_batch_; }
    int int8_layers() const { return n_int8_; }
    int kernels_per_step() const { return kernels_per_step_; }
    int device() const { return device_; }
    int t5_runs() const { return t5_runs_; }

    // Eager (uncaptured) forward of `batch` queries.
    cudaError_t forward(int batch, int wnd, bool wrist, cudaStream_t st, bool unnormalize);

    // Parity tap (host copy, after a predict): the readout embeddings
    // [batch][d] of the last query batch. Returns the element count, or -1.
    long long readout(float* out, long long cap);

  private:
    bool load_t5(const ModelFiles& files);
    bool load_stem(const ModelFiles& files, const std::string& name, int in_hw, bool conv_int8, bool embed_int8,
                   OctoStemDev& s);
    bool load_transformer(const ModelFiles& files, int mask);
    bool load_head(const ModelFiles& files, bool int8);
    bool load_stats(const ModelFiles& files);
    bool alloc_buffers();
    bool time_cond();
    int t5_slot(const std::string& instruction, cudaStream_t st, cudaError_t* err);
    cudaError_t run_t5(const std::vector<int>& ids, float* out, cudaStream_t st);
    cudaError_t run_stem(const OctoStemDev& s, const uint8_t* img, int F, float* tokens, cudaStream_t st);
    cudaError_t mlp_out(const OctoLayerDev& L, int act, int M, float* x, cudaStream_t st);
    cudaError_t run_head(int B, cudaStream_t st, bool unnormalize);
    cudaError_t linear(const DevLinear& l, const float* x, long long ldx, int M, float* out, long long ldo, int mode,
                       const float* res, long long ldr, cudaStream_t st);
    cudaError_t linear_q(const DevLinear& l, const int8_t* q, const float* qs, const float* x, long long ldx, int M,
                         float* out, long long ldo, int mode, const float* res, long long ldr, cudaStream_t st);
    template <class T> T* dalloc(size_t n);
    void fail(const std::string& m) { if (err_.empty()) err_ = m; }

    std::string err_;
    OctoConfigDev cfg_;
    int device_ = 0;
    int max_batch_ = 1;
    int n_int8_ = 0;
    int kernels_per_step_ = 0;
    float i8_clip_ = 1.0f;
    bool explicit_convs_ = false;
    int t5_runs_ = 0;

    T5Tokenizer tok_;

    // T5 (fp32, the reference never quantizes it)
    float *t5_emb_ = nullptr, *t5_rel_ = nullptr, *t5_final_ = nullptr;
    std::vector<T5LayerDev> t5_;
    int* d_bucket_ = nullptr;   // relative-position buckets of j - i + n_task - 1
    int* d_ids_ = nullptr;
    float *d_t5x_ = nullptr, *d_t5h_ = nullptr, *d_t5q_ = nullptr, *d_t5k_ = nullptr, *d_t5v_ = nullptr,
          *d_t5a_ = nullptr, *d_t5ff_ = nullptr, *d_t5bias_ = nullptr;
    static constexpr int kT5CacheSlots = 64;   // the reference's lang_cache bound
    float* d_t5cache_ = nullptr;               // [64][n_task][t5_dim]
    std::unordered_map<std::string, int> t5_slots_;

    OctoStemDev stem_p_, stem_w_;
    DevLinear proj_task_, proj_prim_, proj_wrist_;
    float *pos_task_ = nullptr, *pos_prim_ = nullptr, *pos_wrist_ = nullptr, *pos_readout_ = nullptr;
    std::vector<OctoLayerDev> layers_;
    float *final_s_ = nullptr, *final_b_ = nullptr;

    // diffusion head
    float* fourier_ = nullptr;
    std::vector<float> h_fourier_;
    DevLinear cond0_, cond1_, in_proj_, out_proj_;
    struct HeadBlock {
        float *ln_s = nullptr, *ln_b = nullptr;
        DevLinear d0, d1;
    };
    std::vector<HeadBlock> blocks_;
    std::vector<float> a1_, a2_, sb_;   // per diffusion time t
    float* d_cond_table_ = nullptr;     // [steps][time_dim]
    float *d_act_mean_ = nullptr, *d_act_std_ = nullptr, *d_act_mask_ = nullptr;

    // inputs: primary | wrist | tmask | slots | noise | z in one device buffer
    uint8_t* d_in_ = nullptr;
    size_t in_bytes_ = 0;
    uint8_t *d_prim_u8_ = nullptr, *d_wrist_u8_ = nullptr, *d_tmask_ = nullptr;
    int* d_slot_ = nullptr;
    float *d_noise_ = nullptr, *d_z_ = nullptr;
    float* d_actions_ = nullptr;

    // stems
    float *d_stem_in_ = nullptr, *d_sa_ = nullptr, *d_sb_ = nullptr, *d_gnA_ = nullptr, *d_gnB_ = nullptr;
    ConvScratch conv_s_;
    unsigned int* d_slots_ = nullptr;   // per-frame absmax slots, zeroed per query
    int n_slots_ = 0;
    float *d_ptok_ = nullptr, *d_wtok_ = nullptr;      // stem tokens [F*P][stem_dim]
    float *d_pproj_ = nullptr, *d_wproj_ = nullptr;    // projected [F*P][d]

    // transformer
    float *d_t5in_ = nullptr, *d_task_ = nullptr;
    float *d_x_ = nullptr, *d_h_ = nullptr, *d_qkv_ = nullptr, *d_att_ = nullptr, *d_ff_ = nullptr, *d_mask_ = nullptr;
    float *d_xr_ = nullptr, *d_emb_ = nullptr;
    int8_t* d_q_ = nullptr;
    float* d_qs_ = nullptr;
    size_t q_cap_ = 0, q_rows_ = 0;
    static constexpr int kAttCounters = 1 << 16;   // attention query-tile arrival counters (fused quantization)
    unsigned int* d_att_cnt_ = nullptr;
    AttQuant att_quant(int rows, int K, int seq_rows) const;

    // head
    float *d_hin_ = nullptr, *d_hh_ = nullptr, *d_hn_ = nullptr, *d_wide_ = nullptr, *d_eps_ = nullptr,
          *d_sample_ = nullptr;

    int last_batch_ = 0;
    std::vector<void*> allocs_;
    float* h_pinned_ = nullptr;   // actions staging
    float* h_noise_ = nullptr;    // noise | z staging for seeded queries
    int* h_slots_ = nullptr;
    int* h_status_pinned_ = nullptr;
    int* d_status_ = nullptr;
    cudaStream_t stream_ = nullptr;
    std::map<long long, cudaGraphExec_t> graphs_;
    bool use_graph_ = true;
};

}  // namespace vsb
