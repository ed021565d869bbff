// Host-side interface of the Octo kernels (octo.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vsb {

// SmallStem input of F frames [F][npx][3] uint8 -> [F][npx][6] fp32: the
// observation v/127.5 - 1 and an all -1 goal image (src/models/octo/small_stem.cpp:103-113);
// per-frame absmax (float bits) into amax[f] for the first int8 conv.
cudaError_t octo_stem_input(const uint8_t* img, int F, long long npx, float* out, unsigned int* amax,
                            cudaStream_t st);

// T5 token embeddings x [n][D] = emb[ids[t]] (zeros for an id outside [0, vocab)),
// and the per-head additive attention bias [NH][n][n] = key is a real token
// (ids != pad) ? rel[bucket[j - i + n - 1]][h] : lowest (src/nn/t5_encoder.cpp:94-118).
cudaError_t t5_embed(const int* ids, int n, const float* emb, int vocab, int D, int pad_id, const float* rel,
                     const int* bucket, int NH, float* x, float* bias, cudaStream_t st);

// T5 self-attention with a per-head bias, the reference's mha_attention_bias
// (src/hal/common/attn.cpp:43-111): Q/K/V/out [n][NH*hd]; hd % 8 == 0, n <= 256.
cudaError_t t5_attention(const float* Q, const float* K, const float* V, const float* bias, int n, int NH, int hd,
                         float scale, float* out, cudaStream_t st);

// Token sequence of B queries x [B][total][d] (src/models/octo/octo_transformer.cpp:153-185):
// [task (n_task) | per step t: primary (P) | wrist (Wr) | task again | readout (R)],
// each projection output plus its learned position embedding; the wrist rows
// are zero without a wrist camera (wrist == null). task [B][n_task][d] is the
// task projection (pos_task [n_task][d] is added here, for both copies);
// prim [B*wnd*P][d], wrist [B*wnd*Wr][d].
#ifdef __CUDACC__
#define VSB_OCTO_HD __host__ __device__
#else
#define VSB_OCTO_HD
#endif
struct OctoSeq {
    int B, wnd, n_task, P, Wr, R, d;
    VSB_OCTO_HD int total() const { return n_task + wnd * (P + Wr + n_task + R); }
};
cudaError_t octo_assemble(const OctoSeq& s, const float* task, const float* pos_task, const float* prim,
                          const float* pos_prim,
                          const float* wrist, const float* pos_wrist, const float* pos_readout, float* x,
                          cudaStream_t st);

// Additive block-causal masks [B][total][total] (0 = attend, lowest = blocked)
// from the per-query timestep masks tmask [B][wnd] (src/models/octo/octo_transformer.cpp:104-139).
cudaError_t octo_mask(const OctoSeq& s, const uint8_t* tmask, bool wrist, float* mask, cudaStream_t st);

// Rows of n_rows queries: dst[b][0..n) = src[slot[b]][0..n) (the cached T5 outputs).
cudaError_t gather_rows(const float* src, const int* slot, int n_rows, long long n, float* dst, cudaStream_t st);

// Per-row activation then int8 quantization (quantize_act_i8's scale and
// codes) of x [M][K]: kind is an lm_ops kAct* kind, or kActSiluLibm (silu with
// the C library's expf). keep: also write the activation back into x.
enum : int { kActSiluLibm = 100 };
cudaError_t act_rows_q(int kind, float* x, int M, int K, bool keep, int8_t* q, long long ldq, float* scale,
                       cudaStream_t st);

// The tail of one score-net evaluation of B queries, fused: silu(h) ->
// eps = out_proj (fp32, the reference's dense_linear order) -> DDPM update of
// sample (a1, a2, sb as octo_ddpm_step; z [B][z_stride] or null) -> the next
// step's input row [cond_next | emb | x] (in_f32 [B][IN] when set) and its
// int8 quantization (q [B][ldq], qscale [B]) when q is set. With h null and
// x0 set: sample = x0 and the first input row only.
struct OctoHeadTail {
    int B = 0, H = 0, FL = 0, TD = 0, E = 0;
    const float* h = nullptr;      // [B][H] the score net's last hidden state (pre-silu)
    const float* x0 = nullptr;     // [B][FL] initial noise (first call)
    const float* W = nullptr;      // out_proj [FL][H]
    const float* bias = nullptr;
    float* sample = nullptr;       // [B][FL]
    const float* z = nullptr;
    long long z_stride = 0;
    float a1 = 0, a2 = 0, sb = 0, max_action = 0;
    const float* cond_next = nullptr;   // [TD] or null (last step)
    const float* emb = nullptr;         // [B][E]
    float* in_f32 = nullptr;
    int8_t* q = nullptr;
    long long ldq = 0;
    float* qscale = nullptr;
};
cudaError_t octo_head_tail(const OctoHeadTail& a, cudaStream_t st);

// x[i] = x[i] / (1 + expf(-x[i])) with the C library's expf (src/hal/common/eltwise.cpp:59-66).
cudaError_t silu_exact(float* x, long long n, cudaStream_t st);

// Score-net input rows of B queries: in [B][TD + E + FL] = [cond[t] (TD) | emb[b] (E) | x[b] (FL)]
// (src/models/octo/diffusion_head.cpp:159-170).
cudaError_t octo_head_input(const float* cond_t, int TD, const float* emb, int E, const float* x, int FL, int B,
                            float* in, cudaStream_t st);

// One DDPM step on x [B][FL] from eps (src/models/octo/diffusion_head.cpp:172-191):
// x = clamp(fma(fma(-a2, eps, x), a1, sb * z), +-max_action); z [B][z_stride] or null (zeros).
cudaError_t octo_ddpm_step(float* x, const float* eps, const float* z, long long z_stride, int B, int FL, float a1,
                           float a2, float sb, float max_action, cudaStream_t st);

// actions [B][FL] = x, with fma(v, std[a], mean[a]) where mask[a] > 0 when
// unnormalize (src/models/octo/octo_model.cpp:215-221); A = action_dim.
cudaError_t octo_actions(const float* x, int B, int FL, int A, const float* mean, const float* stdv,
                         const float* mask, bool unnormalize, float* out, cudaStream_t st);

}  // namespace vsb
