// Diffusion Policy on one B200: the reference's DiffusionModel
// (src/models/diffusion/diffusion_model.cpp) re-built around device-resident
// weights and one CUDA graph per query batch.
//
// Load reads the reference converter's checkpoint directory unchanged
// (diffusion.meta, rgb_encoder{i}_backbone.meta/.bin, rgb_encoder{i}.bin,
// unet.bin, stats.bin), quantizes the layers DIFFUSION_INT8 selects (bit 1 the
// U-Net's conv GEMMs, bit 2 the backbone convs) exactly as pack_weights_i8
// does, and uploads everything once. A query batch of up to max_batch
// independent observations runs as one graph: preprocess -> per-camera
// ResNet-18 (GroupNorm) -> keypoints -> conditioning -> num_inference_steps x
// (conditional U-Net -> DDIM / DDPM step) -> actions. Requests of a batch are
// independent: each keeps its own GroupNorm statistics and quantization
// scales, so a batched result equals the single-query result.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "conv_exec.h"
#include "dp.h"

namespace vsb {

class ModelFiles;

struct DpGnConv {           // conv (no bias) followed by GroupNorm, or a conv with bias
    DevConv conv;
    float* gn_s = nullptr;      // null: no GroupNorm (BatchNorm folded into the conv)
    float* gn_b = nullptr;
    int groups = 0;
};

struct DpBasicBlock {
    DpGnConv c1, c2, down;
    bool has_down = false;
};

struct DpEncoderDev {
    DpGnConv stem;
    std::vector<DpBasicBlock> blocks;
    int stem_out = 64, stem_k = 7, stem_stride = 2, stem_pad = 3;
    int pool_k = 3, pool_stride = 2, pool_pad = 1;
    int gs = 16;                    // GroupNorm group size (channels per group)
    DevLinear kp, out;              // fp32: 1x1 keypoint conv, output projection
    float* grid = nullptr;          // [fh*fw][2]
    int fh = 0, fw = 0, C = 0;
};

struct DpConvBlockDev {             // Conv1d -> GroupNorm -> Mish
    DevLinear conv;                 // N = cout, K = k*cin (taps major)
    float* gn_s = nullptr;
    float* gn_b = nullptr;
    int cin = 0, cout = 0, k = 0;
};

struct DpResBlockDev {
    DpConvBlockDev c1, c2;
    DevLinear res;                  // 1x1 residual conv when cin != cout
    bool has_res = false;
    int cin = 0, cout = 0;
    long long film_off = 0;         // column of this block's FiLM vector in the stacked cond output
};

struct DpDownDev { DpResBlockDev r1, r2; DevLinear ds; bool has = false; };
struct DpUpDev {
    DpResBlockDev r1, r2;
    float* uw = nullptr;    // [Cin][4][Cout]
    float* uwt = nullptr;   // the same as [Cout][4][Cin]
    float* ub = nullptr;
    bool has = false;
    int uc = 0;
};

// Workspace of the split-K GEMM path (GemmI8Args::splitk_ws / splitk_counters).
struct DpSplitWs {
    int32_t* ws = nullptr;
    long long elems = 0;
    unsigned int* counters = nullptr;
    int n_counters = 0;
};

struct DpConfigDev {
    int n_obs = 2, n_cams = 2, img_h = 480, img_w = 640, crop_h = 0, crop_w = 0, resize_h = 0, resize_w = 0;
    int state_dim = 6, action_dim = 6, horizon = 64, n_action_steps = 32, num_keypoints = 32;
    bool separate = true;
    std::vector<int> down_dims = {512, 1024, 2048};
    int kernel_size = 5, n_groups = 8, step_embed_dim = 128;
    bool film_scale = true;
    bool ddim = false;
    int num_train_timesteps = 100, num_inference_steps = 100;
    float beta_start = 1e-4f, beta_end = 0.02f;
    std::string beta_schedule = "squaredcos_cap_v2", prediction_type = "epsilon";
    bool clip_sample = true;
    float clip_sample_range = 1.0f, gn_eps = 1e-5f;
    int cam_feature_dim() const { return 2 * num_keypoints; }
    int per_step() const { return state_dim + n_cams * cam_feature_dim(); }
    int global_cond_dim() const { return per_step() * n_obs; }
    int cond_dim() const { return step_embed_dim + global_cond_dim(); }
};

class DpPolicy {
  public:
    ~DpPolicy();
    // max_batch: the most queries one predict may carry (buffers are sized for
    // it). `dir`: a converted directory or a vla.simd GGUF (model_files.h).
    bool load(const std::string& dir, int max_batch = 1);
    const std::string& error() const { return err_; }

    // Host buffers, `batch` queries stacked: frames [batch][n_obs*n_cams][img_h][img_w][3]
    // uint8 (obs-major, then camera), state [batch][n_obs][state_dim], noise
    // [batch][1 + steps][horizon][action_dim] or null (zeros), actions
    // [batch][chunk][action_dim]. Synchronous.
    cudaError_t predict(int batch, const uint8_t* frames, const float* state, const float* noise, bool unnormalize,
                        float* actions);

    // Device-side batch for benchmarks: inputs already in the device buffers,
    // enqueue the graph on `st` (no host copies, no sync).
    cudaError_t enqueue(int batch, cudaStream_t st, bool unnormalize);
    uint8_t* device_frames() { return d_frames_; }
    float* device_state() { return d_state_; }
    float* device_noise() { return d_noise_; }
    const float* device_actions() const { return d_actions_; }

    const DpConfigDev& config() const { return cfg_; }
    int num_steps() const { return static_cast<int>(timesteps_.size()); }
    int max_batch() const { return max_batch_; }
    int int8_layers() const { return n_int8_; }
    int kernels_per_step() const { return kernels_per_step_; }
    int device() const { return device_; }
    size_t frame_bytes() const { return (size_t)cfg_.n_obs * cfg_.n_cams * cfg_.img_h * cfg_.img_w * 3; }
    size_t noise_floats() const { return (size_t)(1 + timesteps_.size()) * cfg_.horizon * cfg_.action_dim; }

    // Eager (uncaptured) forward of `batch` queries.
    cudaError_t forward(int batch, cudaStream_t st, bool unnormalize);

    // Parity taps (host copies, after a predict): the global conditioning
    // [batch][n_obs * (state_dim + n_cams * 2K)] of the last query batch, and,
    // when VLA_DP_DEBUG_STAGE = s was set at load, the first encoder run's map
    // after backbone stage s (0 stem + GroupNorm, 1 max-pool, 2 + i block i),
    // [frames][H][W][C]. Return the element count, or -1.
    long long global_cond(float* out, long long cap);
    long long debug_map(float* out, long long cap);

  private:
    bool load_meta(const ModelFiles& files);
    bool init_schedule();
    bool load_encoder(const ModelFiles& files, int idx, bool int8);
    bool load_unet(const ModelFiles& files, bool int8);
    bool load_stats(const ModelFiles& files);
    bool alloc_buffers();
    bool step_features();
    cudaError_t run_encoder(const DpEncoderDev& e, const float* img, int F, unsigned int* slots, float* feat,
                            bool tap, cudaStream_t st);
    cudaError_t tap_stage(int stage, const float* map, size_t n, cudaStream_t st);
    cudaError_t run_gn_conv(const DpGnConv& c, const float* in, int F, int H, int W, float* out, int epi,
                            const float* res, const unsigned int* amax_in, unsigned int* amax_out, cudaStream_t st);
    unsigned int* res_block(const DpResBlockDev& rb, const float* x, const unsigned int* rm_x, int B, int T,
                            int step, float* out, cudaStream_t st, cudaError_t* err);
    cudaError_t unet(int B, int step, cudaStream_t st);
    cudaError_t gemm_rows(const DevLinear& l, const int8_t* q, const float* qs, const float* xf, int M, float* out,
                          const DpSplitWs& ws, cudaStream_t st);
    cudaError_t im2col_gemm(const DevLinear& l, const float* x, const unsigned int* rm_x, int B, int T, int C, int k,
                            int stride, int pad, int Tout, float* out, unsigned int* rm_out, cudaStream_t st,
                            bool side = false);
    unsigned int* rm_take(long long n);
    cudaStream_t fork(cudaStream_t st);
    cudaError_t join(cudaStream_t st);
    template <class T> T* dalloc(size_t n);
    void fail(const std::string& m) { if (err_.empty()) err_ = m; }

    std::string err_;
    DpConfigDev cfg_;
    int device_ = 0;
    int max_batch_ = 1;
    int n_int8_ = 0;
    int kernels_per_step_ = 0;
    float i8_clip_ = 1.0f;
    bool explicit_convs_ = false;

    // scheduler (host, double, as DPNoiseScheduler::init)
    std::vector<double> alphas_cumprod_;
    std::vector<int> timesteps_;

    std::vector<DpEncoderDev> enc_;
    DevLinear step1_, step2_, cond_all_, final_conv_;
    std::vector<DpDownDev> down_;
    DpResBlockDev mid1_, mid2_;
    std::vector<DpUpDev> up_;
    DpConvBlockDev final_block_;
    long long film_cols_ = 0;

    // stats
    float *d_smin_ = nullptr, *d_smax_ = nullptr, *d_amin_ = nullptr, *d_amax_ = nullptr;
    float *d_img_mean_ = nullptr, *d_img_std_ = nullptr;

    // inputs (one device buffer: frames | state | noise) and outputs
    uint8_t* d_in_ = nullptr;
    uint8_t* d_frames_ = nullptr;
    float* d_state_ = nullptr;
    float* d_noise_ = nullptr;
    size_t in_bytes_ = 0, state_off_ = 0, noise_off_ = 0;
    float* d_actions_ = nullptr;

    // observation encoders
    float* d_img_f_ = nullptr;
    float *d_ba_ = nullptr, *d_bb_ = nullptr, *d_bc_ = nullptr, *d_bres_ = nullptr;
    float *d_gnA_ = nullptr, *d_gnB_ = nullptr;
    ConvScratch conv_s_;
    unsigned int* d_slots_ = nullptr;
    int n_slots_ = 0;
    unsigned int* d_rowmax_ = nullptr;   // U-Net per-row absmax arena, follows d_slots_
    long long rm_cap_ = 0, rm_used_ = 0;
    bool rm_overflow_ = false;
    float *d_kp_ = nullptr, *d_feat_ = nullptr;

    // conditioning
    float* d_stepfeat_ = nullptr;   // [steps][D]
    float* d_gcond_ = nullptr;      // [B][global_cond_dim]
    float* d_gm_ = nullptr;         // [steps*B][cond_dim]
    float* d_film_ = nullptr;       // [steps*B][film_cols_]

    // U-Net
    float* d_sample_ = nullptr;     // [B][horizon][A]
    float* d_eps_ = nullptr;
    std::vector<float*> d_skip_;
    float *d_x_ = nullptr, *d_a_ = nullptr, *d_b_ = nullptr, *d_cat_ = nullptr, *d_h_ = nullptr, *d_o_ = nullptr,
          *d_r_ = nullptr, *d_colf_ = nullptr;
    // split-K workspaces of the skinny U-Net GEMMs: one per stream (the
    // residual conv on the side stream runs beside the main chain)
    DpSplitWs ws_main_, ws_side_;
    int8_t *d_q_ = nullptr, *d_q2_ = nullptr;
    float *d_qs_ = nullptr, *d_qs2_ = nullptr;

    // Mish's scalar tail of the cond input (CD % 8 values per query, all from
    // the global conditioning), computed on the device with the host C
    // library's float functions restated (libm_f32.h), which the reference's
    // values depend on.
    int tail_n_ = 0;
    float* d_tail_ = nullptr;

    int debug_stage_ = -1;
    float* d_debug_ = nullptr;
    size_t debug_n_ = 0, debug_cap_ = 0;
    int last_batch_ = 0;

    std::vector<void*> allocs_;
    float* h_pinned_ = nullptr;     // actions staging
    int* h_status_pinned_ = nullptr;
    int* d_status_ = nullptr;
    cudaStream_t stream_ = nullptr;
    cudaStream_t side_ = nullptr;
    cudaEvent_t ev_fork_ = nullptr, ev_join_ = nullptr;
    std::vector<cudaGraphExec_t> graphs_;   // [batch-1][unnormalize]
    bool use_graph_ = true;
};

}  // namespace vsb
