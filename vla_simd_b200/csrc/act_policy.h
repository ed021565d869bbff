// ACT policy on one B200: the reference's ActModel (src/models/act/act_model.cpp)
// re-built around device-resident weights and one CUDA graph per step.
//
// Load reads the reference converter's checkpoint directory unchanged
// (config.txt, backbone.meta/.bin, act.meta/.bin, stats.bin), quantizes the
// layers ACT_INT8 selects exactly as pack_weights_i8 does, and uploads
// everything once. predict() copies the camera frames + state in, replays the
// captured graph (normalize -> ResNet-18 -> token assembly -> 4 post-LN encoder
// layers -> 1 decoder layer -> head -> unnormalize) and copies the actions out.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "conv_exec.h"
#include "nn.h"

#include <cstdint>
#include <string>
#include <vector>

namespace vsb {

class ModelFiles;

struct DevBlock {
    DevConv conv1, conv2, down;
    bool has_down = false;
};

struct ActConfigDev {
    int dim = 512, heads = 8, head_dim = 64, ff = 3200;
    int n_enc = 4, n_dec = 1, chunk = 100, state_dim = 6, action_dim = 6, n_1d = 2, n_text = 0;
    float ln_eps = 1e-5f;
};

struct EncLayerDev {
    DevLinear wqk, wv, wo, w1, w2;   // wq and wk stacked: one GEMM, N = 2*dim
    float *n1s, *n1b, *n2s, *n2b;
};

struct DecLayerDev {
    DevLinear s_wqk, s_wv, s_wo, c_wq, c_wk, c_wv, c_wo, w1, w2;
    float *n1s, *n1b, *n2s, *n2b, *n3s, *n3b;
};

class ActPolicy {
  public:
    ~ActPolicy();
    // Returns false (with a message in error()) on any load failure. `dir`: a
    // converted directory or a vla.simd GGUF (model_files.h).
    bool load(const std::string& dir);
    const std::string& error() const { return err_; }

    // Host buffers: images n_cams*img_h*img_w*3 uint8, state [state_dim] raw,
    // actions [chunk*action_dim]. Synchronous (returns when actions are written).
    cudaError_t predict(const uint8_t* images, const float* state, bool unnormalize, float* actions);

    // Device-side step for benchmarks: inputs already in d_images/d_state,
    // enqueue the graph on `st` (no host copies, no sync).
    cudaError_t enqueue_step(cudaStream_t st, bool unnormalize);
    uint8_t* device_images() { return d_img_u8_; }
    float* device_state() { return d_state_; }
    const float* device_actions() const { return d_actions_; }

    int chunk() const { return cfg_.chunk; }
    int action_dim() const { return cfg_.action_dim; }
    int state_dim() const { return cfg_.state_dim; }
    int n_cams() const { return n_cams_; }
    int img_h() const { return img_h_; }
    int img_w() const { return img_w_; }
    int n_tokens() const { return cfg_.n_1d + n_cams_ * fh_ * fw_; }
    int int8_layers() const { return n_int8_; }
    int kernels_per_step() const { return kernels_per_step_; }
    int device() const { return device_; }

    // Eager (uncaptured) forward, for debugging and for graph capture.
    cudaError_t forward(cudaStream_t st, bool unnormalize);

  private:
    bool load_config(const ModelFiles& files);
    bool load_backbone(const ModelFiles& files, bool int8);
    bool load_transformer(const ModelFiles& files, int mask);
    bool load_stats(const ModelFiles& files);
    bool alloc_buffers();
    bool upload_linear(DevLinear& l, const float* W, const float* b, int N, int K, bool int8);
    cudaError_t run_linear(const DevLinear& l, const float* x_f32, const int8_t* xq, const float* xs,
                           const CUtensorMap* tmap_a, int M, float* out, long long ldo, int mode,
                           const float* res, long long ldr, cudaStream_t st, unsigned int* amax = nullptr,
                           int amax_rows = 1);
    // Independent kernel pairs of the step run on `st` and a side stream:
    // fork() returns the side stream, ordered after everything issued on st so
    // far; join() orders st after everything issued on the side stream. In a
    // captured step they become parallel branches of the graph.
    cudaStream_t fork(cudaStream_t st);
    cudaError_t join(cudaStream_t st);
    cudaError_t run_conv(const DevConv& c, const float* in, int F, int H, int W, float* out, int mode,
                         const float* res, const unsigned int* amax_in, unsigned int* amax_out,
                         cudaStream_t st, bool side = false);
    cudaError_t enqueue_on_device(cudaStream_t st, bool unnormalize);
    cudaError_t run_backbone(cudaStream_t st);
    cudaError_t run_encoder(cudaStream_t st);
    cudaError_t run_decoder(cudaStream_t st, bool unnormalize);
    cudaError_t decoder_self_block(const DecLayerDev& l, cudaStream_t st);
    cudaError_t decoder_cross_queries(const DecLayerDev& l, float* q, cudaStream_t st);
    cudaError_t dec0_consts(cudaStream_t st);
    template <class T> T* dalloc(size_t n);
    void fail(const std::string& m) { if (err_.empty()) err_ = m; }

    std::string err_;
    int device_ = 0;
    int img_h_ = 0, img_w_ = 0, n_cams_ = 0;
    float norm_eps_ = 1e-5f;
    float i8_clip_ = 1.0f;
    int fh_ = 0, fw_ = 0;
    int n_int8_ = 0;
    int kernels_per_step_ = 0;

    // backbone
    int stem_out_ = 64, stem_k_ = 7, stem_stride_ = 2, stem_pad_ = 3;
    int pool_k_ = 3, pool_stride_ = 2, pool_pad_ = 1;
    DevConv stem_;
    std::vector<DevBlock> blocks_;

    // transformer
    ActConfigDev cfg_;
    DevLinear img_proj_, state_proj_, head_;
    std::vector<EncLayerDev> enc_;
    std::vector<DecLayerDev> dec_;
    float *d_latent_ = nullptr, *d_pos_ = nullptr, *d_dec_pos_ = nullptr, *d_dec_ns_ = nullptr, *d_dec_nb_ = nullptr;

    // stats
    float *d_state_mean_ = nullptr, *d_state_std_ = nullptr, *d_act_mean_ = nullptr, *d_act_std_ = nullptr;
    float *d_img_mean_ = nullptr, *d_img_std_ = nullptr;

    // activations / scratch
    uint8_t* d_img_u8_ = nullptr;
    float* d_state_ = nullptr;
    float* d_state_n_ = nullptr;
    float* d_actions_ = nullptr;
    float *d_img_f_ = nullptr, *d_ba_ = nullptr, *d_bb_ = nullptr, *d_bc_ = nullptr, *d_bres_ = nullptr;
    int8_t* d_col_ = nullptr;
    int8_t* d_col2_ = nullptr;              // scratch of the conv on the side stream
    float* d_col_scale2_ = nullptr;
    float* d_col_f_ = nullptr;
    float* d_col_scale_ = nullptr;
    unsigned int* d_amax_ = nullptr;
    static constexpr int kAttCounters = 4096;   // attention query-tile arrival counters (fused quantization)
    unsigned int* d_att_cnt_ = nullptr;
    AttQuant att_quant() const;
    // row-quantized FFN hidden (GemmI8Args::qout): per-row absmax slots, tile counters
    unsigned int* d_qamax_ = nullptr;
    unsigned int* d_qsync_ = nullptr;
    cudaError_t ffn_up(const DevLinear& w1, const DevLinear& w2, const int8_t* xq, const float* xs,
                       const float* x_f32, int M, cudaStream_t st);
    int n_amax_ = 0;
    float *d_x_ = nullptr, *d_qk_ = nullptr, *d_v_ = nullptr, *d_att_ = nullptr, *d_ff_ = nullptr;
    float *d_dx_ = nullptr, *d_ck_ = nullptr, *d_cv_ = nullptr, *d_feat_ = nullptr;
    float* d_xp_ = nullptr;    // fp32 x + pos, only for fp32 q/k projections
    int8_t *d_qa_ = nullptr, *d_qb_ = nullptr, *d_qatt_ = nullptr, *d_qff_ = nullptr;
    int8_t *d_qea_ = nullptr, *d_qeb_ = nullptr;   // q(enc + pos), q(enc) for cross-attention
    float *d_sea_ = nullptr, *d_seb_ = nullptr;
    float *d_sa_ = nullptr, *d_sb_ = nullptr, *d_satt_ = nullptr, *d_sff_ = nullptr;
    // decoder layer 0 on its (always zero) queries, evaluated once at load
    float *d_dec_x0_ = nullptr, *d_dec_q0_ = nullptr;
    bool dec0_ready_ = false;
    long long ldq_ = 0, ldqff_ = 0;

    std::vector<void*> allocs_;
    size_t state_off_ = 0;                  // d_state_ = d_img_u8_ + state_off_ (one input buffer)
    float* h_state_pinned_ = nullptr;
    float* h_actions_pinned_ = nullptr;
    int* h_status_pinned_ = nullptr;        // device status word, read back with the actions
    int* d_status_ = nullptr;               // its device address
    cudaStream_t stream_ = nullptr;
    cudaStream_t side_ = nullptr;
    cudaEvent_t ev_fork_ = nullptr, ev_join_ = nullptr;
    cudaGraphExec_t graph_[2] = {nullptr, nullptr};
    bool use_graph_ = true;
    bool explicit_convs_ = false;   // VLA_CONV_IM2COL: im2col + GEMM for every int8 conv
};

}  // namespace vsb
