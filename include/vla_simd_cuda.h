/*
 * vla_simd_cuda.h - op-level C ABI of libvla_simd_b200.so: the B200 kernels
 * behind the reference's portable op API (src/ops/quant_ops.h, lm_ops.h,
 * conv_ops.h), so a TCPU_HAL_CUDA backend of the reference can define its
 * tcpu:: functions on top of these.
 *
 * Two families:
 *   vla_cuda_*  DEVICE pointers, an explicit cudaStream_t (passed as void*),
 *               asynchronous; return vla_status (vla_simd.h).
 *   vla_tcpu_*  HOST pointers with exactly the reference's tcpu:: argument
 *               lists; synchronous (copy in, compute on the GPU, copy out).
 *
 * Device layout. Quantized activations and weights are row-major int8 with a
 * leading dimension (bytes) that is a multiple of 16 (the TMA stride rule);
 * vla_cuda_i8_ld(K) gives the smallest one. Bytes past K in a row are ignored
 * by the GEMMs. The reference's CPU panel layout [N/16][Kp/4][16][4] exists
 * only in the vla_tcpu_* shims.
 *
 * Numerics (all bit-identical to the reference CPU code on identical inputs):
 *   scale = amax > 0 ? max(amax/127, FLT_MIN) : 1;  q = clamp(rne(x/scale*...), +-127)
 *   out   = fma((float)acc * wscale[n], ascale[m], bias[n])
 */

#ifndef VLA_SIMD_CUDA_H
#define VLA_SIMD_CUDA_H

#include <stdint.h>
#include "vla_simd.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Epilogue modes of vla_cuda_gemm_i8 (bit flags). */
#define VLA_EPI_RELU      1   /* v < 0 ? 0 : v                       (tcpu::relu) */
#define VLA_EPI_ADD       2   /* out = res + v                        (residual add) */
#define VLA_EPI_ADD_RELU  4   /* v = v + res; v > 0 ? v : 0           (ResNet block tail) */
#define VLA_EPI_ACC       8   /* write the raw int32 accumulators (out is int32_t*) */

/* Smallest valid int8 row stride for K columns: K rounded up to 16. */
VLA_API int64_t vla_cuda_i8_ld(int32_t K);

/* Read and clear the device status word: 0 OK, 1 a kernel's bounded wait ran
 * out (the kernel returned early), <0 the word could not be read. */
VLA_API int32_t vla_cuda_device_status(void);

/* replaces tcpu::quantize_act_i8 (src/ops/quant_ops.h:76):
 * x [seq][K] fp32 -> xq [seq][ldq] int8 (zero past K) + ascale [seq]. */
VLA_API int32_t vla_cuda_quantize_act_i8(const float* x, int8_t* xq, float* ascale,
                                         int32_t seq, int32_t K, int64_t ldq, void* stream);

/* replaces tcpu::quantize_span_i8 (src/ops/quant_ops.h:80; gemm_i8.cpp:177-207):
 * q[i] = rne(clamp(x[i] * inv, -127, 127)) for n elements, one shared scale
 * (the conv per-tensor quantizer's arithmetic). */
VLA_API int32_t vla_cuda_quantize_span_i8(const float* x, int8_t* q, int64_t n, float inv, void* stream);

/* replaces tcpu::pack_weights_i8 (src/ops/quant_ops.h:58) in the device layout:
 * W [N][K] fp32 (device) -> Wq [N][ldw] int8 + wscale [N]. Same per-row math as
 * the activation quantizer. */
VLA_API int32_t vla_cuda_pack_weights_i8(const float* W, int8_t* Wq, float* wscale,
                                         int32_t N, int32_t K, int64_t ldw, void* stream);

/* replaces tcpu::dense_linear_i8_pre (src/ops/quant_ops.h:83-85):
 * out [seq][N] = dequant(xq [seq][ldx] . Wq [N][ldw]^T) + bias. */
VLA_API int32_t vla_cuda_dense_linear_i8_pre(float* out, const int8_t* xq, const float* ascale,
                                             const int8_t* Wq, const float* wscale, const float* bias,
                                             int32_t seq, int32_t N, int32_t K,
                                             int64_t ldx, int64_t ldw, void* stream);

/* replaces tcpu::dense_linear_i8 (src/ops/quant_ops.h:69-71): quantize x per
 * token into the caller-owned scratch (xq [seq][vla_cuda_i8_ld(K)], ascale
 * [seq]), then the W8A8 GEMM. */
VLA_API int32_t vla_cuda_dense_linear_i8(float* out, const float* x, const int8_t* Wq,
                                         const float* wscale, const float* bias,
                                         int32_t seq, int32_t N, int32_t K, int64_t ldw,
                                         int8_t* xq_scratch, float* ascale_scratch, void* stream);

/* No counterpart in the reference: this backend's addition for callers that
 * cannot allocate device memory (a real-time control loop, where cudaMalloc /
 * cudaFree may synchronize the device and stall for an unbounded time, or a
 * host framework that owns all GPU memory through its own pool). Same result
 * as vla_cuda_dense_linear_i8, but the quantization scratch is a fixed 2 MiB
 * array in GPU global memory that the library reserves on every GPU it runs on
 * until the process exits; nothing is allocated or freed. Limit:
 * seq * ceil16(K) rounded up to 256 bytes, plus 4 * seq, at most 2 MiB (e.g.
 * 602 x 3200); larger calls return VLA_ERR_SHAPE with a message on stderr.
 * The first call on each device looks up the array's device address, so make
 * that first call before any stream capture (inside a capture it prints the
 * reason and returns VLA_ERR_DEVICE). The address is valid per CUDA context:
 * after cudaDeviceReset, or under another context made current through the
 * driver API, the next call looks it up again. All calls share the one array:
 * calls that overlap on the GPU (different streams, or different host threads
 * on the same device) race; serialize them. */
VLA_API int32_t vla_cuda_dense_linear_i8_noalloc(float* out, const float* x, const int8_t* Wq,
                                                 const float* wscale, const float* bias,
                                                 int32_t seq, int32_t N, int32_t K, int64_t ldw,
                                                 void* stream);

/* The W8A8 GEMM with every option exposed (nn::Linear::forward / forward_add
 * and the conv epilogues, src/nn/linear.cpp:121-185). ascale_per_row = 0 uses
 * ascale[0] for every row. res/ldr feed VLA_EPI_ADD / VLA_EPI_ADD_RELU (res
 * may alias out). amax (optional, zeroed by the caller) receives atomicMax of
 * |out| as float bits, slot m / amax_rows. force_simt = 1 takes the CUDA-core
 * kernel instead of the tensor-core one (same results). */
VLA_API int32_t vla_cuda_gemm_i8(void* out, int64_t ldo, const int8_t* xq, int64_t ldx,
                                 const float* ascale, int32_t ascale_per_row,
                                 const int8_t* Wq, int64_t ldw, const float* wscale,
                                 const float* bias, const float* res, int64_t ldr,
                                 int32_t M, int32_t N, int32_t K, int32_t mode,
                                 uint32_t* amax, int32_t amax_rows, int32_t force_simt,
                                 void* stream);

/* replaces tcpu::conv2d_i8 (src/ops/conv_ops.h, src/hal/common/conv.cpp:468-526)
 * for F NHWC frames at once: per-frame per-tensor activation scale
 * (absmax * clip / 127, TCPU_I8_CLIP semantics), int8 im2col, W8A8 GEMM.
 * Wq [Cout][ldw] with K = k*k*Cin in (ky, kx, ci) order. Scratch (caller-owned):
 * col [F*Ho*Wo][ldw] int8, rscale [F*Ho*Wo], amax [F] (zeroed here).
 * mode/res as vla_cuda_gemm_i8 (ld of res = Cout). */
VLA_API int32_t vla_cuda_conv2d_i8(float* out, const float* x, int32_t F, int32_t H, int32_t W,
                                   int32_t Cin, const int8_t* Wq, int64_t ldw, const float* wscale,
                                   const float* bias, int32_t Cout, int32_t k, int32_t stride,
                                   int32_t pad, float clip, int32_t mode, const float* res,
                                   int8_t* col_scratch, float* rscale_scratch, uint32_t* amax_scratch,
                                   void* stream);

/* replaces tcpu::layernorm (src/hal/common/norms.cpp:69-97); out may alias x. */
VLA_API int32_t vla_cuda_layernorm(float* out, const float* x, const float* w, const float* b,
                                   int32_t seq, int32_t hidden, float eps, void* stream);

/* replaces tcpu::gqa_attention_masked / gqa_attention_dense (src/ops/lm_ops.h:21-35):
 * Q [seq_q][n_q*head_dim], K/V [seq_k][n_kv*head_dim], out [seq_q][n_q*head_dim];
 * mask [seq_q][seq_k] additive or NULL (dense). head_dim must be 64. */
VLA_API int32_t vla_cuda_gqa_attention(float* out, const float* Q, const float* K, const float* V,
                                       int32_t seq_q, int32_t seq_k, int32_t n_q, int32_t n_kv,
                                       int32_t head_dim, float scale, const float* mask, void* stream);

/* The same attention on the tensor cores (tcgen05 kind::tf32, QK^T and PV each
 * as three split-precision MMAs, online softmax): fp32-level accuracy but not
 * the reference's summation order, so not bit-identical. The policies use it
 * only when VLA_ATT_TC=1 is set before they load. Same arguments and rules
 * (additive mask, fully blocked row -> mean of V). */
VLA_API int32_t vla_cuda_gqa_attention_tc(float* out, const float* Q, const float* K, const float* V,
                                          int32_t seq_q, int32_t seq_k, int32_t n_q, int32_t n_kv,
                                          int32_t head_dim, float scale, const float* mask, void* stream);

/* replaces tcpu::dense_linear (src/ops/lm_ops.h, src/hal/avx2/gemm.cpp:98-122) for
 * the small fp32 layers a policy keeps out of int8 (ACT's state projection and
 * action head), in the reference's exact summation order:
 * out [seq][N] = x [seq][K] . W [N][K]^T + bias. */
VLA_API int32_t vla_cuda_dense_linear_f32(float* out, const float* x, const float* W, const float* bias,
                                          int32_t seq, int32_t N, int32_t K, void* stream);

/* replaces tcpu::maxpool2d_relu (src/hal/common/conv.cpp:192-225), F frames. */
VLA_API int32_t vla_cuda_maxpool2d_relu(float* out, const float* x, int32_t F, int32_t H, int32_t W,
                                        int32_t C, int32_t k, int32_t stride, int32_t pad, void* stream);

/* ---------------- lm / conv ops of the other policy families (device pointers)
 * The reference's formulas in its order (see the notes per op): bit-identical
 * where it is deterministic fp arithmetic, within its own tests' tolerances
 * where it calls libm. */

/* replaces tcpu::rmsnorm (src/ops/lm_ops.h:21; src/hal/common/norms.cpp:19-35):
 * x, out [seq][hidden], w [hidden]; hidden <= 6144. Bit-identical. */
VLA_API int32_t vla_cuda_rmsnorm(float* out, const float* x, const float* w, int32_t seq, int32_t hidden,
                                 float eps, void* stream);

/* replaces tcpu::rope_neox (src/ops/lm_ops.h:26; norms.cpp:37-67), in place:
 * x [seq][n_heads][head_dim], pos [seq] int32 (device). Double trig. */
VLA_API int32_t vla_cuda_rope_neox(float* x, const int32_t* pos, int32_t seq, int32_t n_heads,
                                   int32_t head_dim, float base, void* stream);

/* replace tcpu::silu_gate / silu / gelu_tanh / gelu_erf / relu / mish
 * (src/ops/lm_ops.h:55-79; src/hal/common/eltwise.cpp): the reference's SIMD
 * bodies with its Cephes exp for every element. out may alias x (in place). */
VLA_API int32_t vla_cuda_silu_gate(float* out, const float* g, const float* u, int64_t n, void* stream);
VLA_API int32_t vla_cuda_silu(float* out, const float* x, int64_t n, void* stream);
VLA_API int32_t vla_cuda_gelu_tanh(float* out, const float* x, int64_t n, void* stream);
VLA_API int32_t vla_cuda_gelu_erf(float* out, const float* x, int64_t n, void* stream);
VLA_API int32_t vla_cuda_relu(float* out, const float* x, int64_t n, void* stream);
VLA_API int32_t vla_cuda_mish(float* out, const float* x, int64_t n, void* stream);

/* replaces tcpu::groupnorm (src/ops/conv_ops.h:91; src/hal/common/conv.cpp:227-318):
 * x, out [n_pixels][C] (channels last), scale/bias [C], C % groups == 0.
 * scratch: vla_cuda_groupnorm_scratch_bytes(C) caller-owned device bytes, 8-byte aligned. */
VLA_API uint64_t vla_cuda_groupnorm_scratch_bytes(int32_t C);
VLA_API int32_t vla_cuda_groupnorm(float* out, const float* x, const float* scale, const float* bias,
                                   int32_t n_pixels, int32_t C, int32_t groups, float eps, int32_t fuse_relu,
                                   void* scratch, void* stream);

/* replaces tcpu::spatial_softmax (src/ops/conv_ops.h:83; conv.cpp:397-422):
 * x [n_pixels][C], grid [n_pixels][2] -> out [C][2] expected coordinates. */
VLA_API int32_t vla_cuda_spatial_softmax(float* out, const float* x, const float* grid, int32_t n_pixels,
                                         int32_t C, void* stream);

/* replaces tcpu::im2col1d (src/ops/conv_ops.h:65; conv.cpp:334-347):
 * x [T][Cin] -> col [Tout][k*Cin] (caller-owned). */
VLA_API int32_t vla_cuda_im2col1d(float* col, const float* x, int32_t T, int32_t Cin, int32_t k,
                                  int32_t stride, int32_t pad, int32_t Tout, void* stream);

/* replaces tcpu::conv_transpose1d (src/ops/conv_ops.h:74; conv.cpp:349-395):
 * x [T][Cin], W [Cin][k][Cout], bias [Cout] or NULL -> out [(T-1)*stride-2*pad+k][Cout].
 * Bit-identical (the reference's accumulation order per output). */
VLA_API int32_t vla_cuda_conv_transpose1d(float* out, const float* x, const float* W, const float* bias,
                                          int32_t T, int32_t Cin, int32_t Cout, int32_t k, int32_t stride,
                                          int32_t pad, void* stream);

/* ------------------------------------------------ host-pointer tcpu shims */

VLA_API int32_t vla_tcpu_int8_gemm_available(void);          /* src/ops/quant_ops.h:41 */
VLA_API int32_t vla_tcpu_i8_kpad(int32_t K);                 /* :45 */
VLA_API uint64_t vla_tcpu_packed_i8_words(int32_t N, int32_t K); /* :57 */
/* :58, the reference's CPU panel layout + int32 row sums (quantized and packed
 * on the device, copied back) */
VLA_API int32_t vla_tcpu_pack_weights_i8(const float* W, int8_t* Wq, float* wscale, int32_t N, int32_t K);
/* :64, the row-sum table pack_weights_i8 stores after the panels */
VLA_API const int32_t* vla_tcpu_i8_rowsums(const int8_t* Wq, int32_t N, int32_t K);
/* :80, on the device */
VLA_API int32_t vla_tcpu_quantize_span_i8(const float* x, int8_t* q, uint64_t n, float inv);
/* :76 */
VLA_API int32_t vla_tcpu_quantize_act_i8(const float* x, int8_t* xq, float* ascale, int32_t seq, int32_t K);
/* :83-85, Wq in the panel layout */
VLA_API int32_t vla_tcpu_dense_linear_i8_pre(float* out, const int8_t* xq, const float* ascale,
                                             const int8_t* Wq, const float* wscale, const float* bias,
                                             int32_t seq, int32_t N, int32_t K);
/* :69-71 */
VLA_API int32_t vla_tcpu_dense_linear_i8(float* out, const float* x, const int8_t* Wq, const float* wscale,
                                         const float* bias, int32_t seq, int32_t N, int32_t K,
                                         int8_t* xq_scratch, float* ascale_scratch);
/* :90-92, the backend's own reference for the same call: the CUDA-core
 * (dp4a) kernel with the same epilogue, independent of the tensor-core path */
VLA_API int32_t vla_tcpu_dense_linear_i8_ref(float* out, const int8_t* xq, const float* ascale,
                                             const int8_t* Wq, const float* wscale, const float* bias,
                                             int32_t seq, int32_t N, int32_t K);

/* ------------------------------------------- device-resident ACT stepping
 * For throughput runs: inputs written straight into the handle's device
 * buffers, the captured step enqueued on a caller stream, no host copies. */
VLA_API int32_t vla_act_device_buffers(void* h, uint8_t** images, float** state, const float** actions);
VLA_API int32_t vla_act_enqueue(void* h, void* stream, int32_t unnormalize);
/* kernels in one captured step (0 before the first predict/enqueue) */
VLA_API int32_t vla_act_kernels_per_step(void* h);
VLA_API int32_t vla_act_int8_layers(void* h);

/* The W8A8 GEMM of vla_cuda_gemm_i8 (same epilogues, same results) for at
 * most 128 rows and a long K, with K split over independent CTAs whose int32
 * partial tiles are summed in a caller workspace: ws (ws_elems int32) and
 * counters (n_counters, zero before the first call; every call leaves them
 * zero). Weight-streaming shapes - a batch-1 policy's layers - spread over all
 * SMs this way. Shapes that gain nothing take the ordinary kernels. Calls that
 * may overlap on the GPU need separate workspaces. No counterpart in the
 * reference (its GEMM is one CPU kernel, src/hal/avx2/gemm_i8.cpp:123-159). */
VLA_API int32_t vla_cuda_gemm_i8_splitk(void* out, int64_t ldo, const int8_t* xq, int64_t ldx,
                                        const float* ascale, const int8_t* Wq, int64_t ldw,
                                        const float* wscale, const float* bias, const float* res,
                                        int64_t ldr, int32_t M, int32_t N, int32_t K, int32_t mode,
                                        int32_t* ws, int64_t ws_elems, uint32_t* counters,
                                        int32_t n_counters, void* stream);

/* The W8A8 GEMM (+ ReLU when relu != 0) writing its output already quantized
 * per row for the next W8A8 GEMM: q [M][ldq] int8 (ldq == N) and qscale [M],
 * exactly what vla_cuda_gemm_i8 followed by vla_cuda_quantize_act_i8 of its
 * fp32 output produce (the reference's dense_linear_i8 then quantize_act_i8,
 * src/hal/common/gemm_i8.cpp:209-278), without the fp32 output. Caller-owned
 * qamax [M] and qsync [2 * ceil(M / 128)] uint32, zero before the first call;
 * every call leaves them zero; calls that may overlap on the GPU need separate
 * ones. Shapes that are not one wave of slab CTAs (N % 32 != 0, K > 1024, too
 * many rows) return VLA_ERR_SHAPE (vla_cuda_gemm_i8_rowq_supported says
 * which). No counterpart in the reference. */
VLA_API int32_t vla_cuda_gemm_i8_rowq_supported(int32_t M, int32_t N, int32_t K);
VLA_API int32_t vla_cuda_gemm_i8_rowq(int8_t* q, int64_t ldq, float* qscale, const int8_t* xq, int64_t ldx,
                                      const float* ascale, const int8_t* Wq, int64_t ldw,
                                      const float* wscale, const float* bias, int32_t M, int32_t N,
                                      int32_t K, int32_t relu, uint32_t* qamax, uint32_t* qsync,
                                      void* stream);

/* ------------------------------------------- batched Diffusion Policy
 * No counterpart in the reference, whose vla_diffusion_predict serves one query
 * (src/models/diffusion/diffusion_capi.cpp:57-72): a handle loaded with
 * max_batch serves up to that many independent queries in one call, each
 * with its own GroupNorm statistics and quantization scales, so every query's
 * actions equal a single-query predict of it. Arrays gain a leading batch axis:
 * frames [batch][n_obs_steps*n_cams][img_h][img_w][3], state [batch][n_obs_steps][state_dim],
 * noise [batch][1 + num_steps][horizon][action_dim] or NULL, actions [batch][chunk][action_dim]. */
VLA_API void* vla_diffusion_load_batch(const char* model_dir, int32_t max_batch);
VLA_API int32_t vla_diffusion_predict_batch(void* h, int32_t batch, const uint8_t* frames, const float* state,
                                            int32_t unnormalize, float* actions, const float* noise);
/* device-resident stepping for throughput runs (as vla_act_device_buffers / vla_act_enqueue) */
VLA_API int32_t vla_diffusion_device_buffers(void* h, uint8_t** frames, float** state, float** noise,
                                             const float** actions);
VLA_API int32_t vla_diffusion_enqueue(void* h, int32_t batch, void* stream, int32_t unnormalize);
VLA_API int32_t vla_diffusion_kernels_per_step(void* h);
VLA_API int32_t vla_diffusion_int8_layers(void* h);
/* Parity taps, no counterpart in the reference's ABI (its intermediates are
 * not exposed): after a predict, copy to `out` (capacity `cap` floats) the last
 * batch's global conditioning vector [batch][n_obs_steps*(state_dim + n_cams*2*keypoints)],
 * or, for a handle loaded with VLA_DP_DEBUG_STAGE = s, the first encoder's map
 * after ResNet stage s (0 stem + GroupNorm, 1 max-pool, 2 + i block i) for all
 * of its frames. Return the element count, or -1. */
VLA_API int64_t vla_diffusion_global_cond(void* h, float* out, int64_t cap);
VLA_API int64_t vla_diffusion_debug_map(void* h, float* out, int64_t cap);

/* --------------------------------------------------------- batched Octo
 * No counterpart in the reference, whose vla_octo_predict_ex serves one query
 * (src/models/octo/octo_capi.cpp:40-58): a handle loaded with max_batch serves
 * up to that many queries of one window length in one call, each with its own
 * instruction, timestep mask and noise; every query's actions equal a
 * single-query predict of it. primary [batch][wnd][256][256][3], wrist
 * [batch][wnd][128][128][3] or NULL (for all queries), timestep_mask
 * [batch][wnd], instructions[batch]; noise [batch][horizon*action_dim] and z
 * [batch][steps][horizon*action_dim], or both NULL with seeds[batch];
 * actions [batch][horizon][action_dim]. */
VLA_API void* vla_octo_load_batch(const char* model_dir, const char* tok_dir, int32_t max_batch);
VLA_API int32_t vla_octo_predict_batch(void* h, int32_t batch, const uint8_t* primary, const uint8_t* wrist,
                                       int32_t wnd, const uint8_t* timestep_mask,
                                       const char* const* instructions, const float* noise, const float* z,
                                       const uint64_t* seeds, int32_t unnormalize, float* actions);
VLA_API int32_t vla_octo_num_steps(void* h);
VLA_API int32_t vla_octo_embed_dim(void* h);
VLA_API int32_t vla_octo_int8_layers(void* h);
VLA_API int32_t vla_octo_kernels_per_step(void* h);
/* how many distinct instructions the T5 encoder has run for (the cache's misses) */
VLA_API int32_t vla_octo_t5_runs(void* h);
/* device-resident stepping for throughput runs: the input buffers (sized for
 * max_batch x max_window), vla_octo_set_instruction for query slot b, then
 * vla_octo_enqueue of one graph on `stream` (no copies, no sync). */
VLA_API int32_t vla_octo_device_buffers(void* h, uint8_t** primary, uint8_t** wrist, uint8_t** timestep_mask,
                                        float** noise, float** z, const float** actions);
VLA_API int32_t vla_octo_set_instruction(void* h, int32_t b, const char* instruction);
VLA_API int32_t vla_octo_enqueue(void* h, int32_t batch, int32_t wnd, int32_t wrist, void* stream,
                                 int32_t unnormalize);
/* Parity tap: the last batch's readout embeddings [batch][embed_dim] (after the
 * final LayerNorm, the diffusion head's input). Returns the element count, or -1. */
VLA_API int64_t vla_octo_readout(void* h, float* out, int64_t cap);
/* The host tokenizer Octo's handles use (no device work): ids [max_len] of
 * `text` under the vocab.txt contents `vocab_text`, pieces truncated to
 * max_len - 1, then </s>, then <pad> (src/tokenizer/t5_tokenizer.cpp:131-155). */
VLA_API int32_t vla_t5_tokenize(const char* vocab_text, const char* text, int32_t max_len, int32_t* ids);

/* --------------------------------------------------------- batched SmolVLA
 * No counterpart in the reference, whose vla_smolvla_predict_rtc serves one
 * query (src/models/smolvla/smolvla_capi.cpp:116-165): a handle loaded with
 * max_batch serves up to that many queries of one frame size per call, each
 * with its own prompt, state, noise (or seeds[b]) and guidance; every query's
 * actions equal a single-query predict of it. frames [batch][n_views][h][w][3],
 * lang tokens / mask [batch][n_lang], state [batch][state_dim], noise
 * [batch][chunk][32] or NULL, prev [batch][n_prev][action_dim], weights
 * [batch][chunk], actions [batch][chunk][action_dim]. */
VLA_API void* vla_smolvla_load_batch(const char* model_dir, const char* tok_dir, int32_t max_batch);
VLA_API int32_t vla_smolvla_predict_batch(void* h, int32_t batch, const uint8_t* frames, int32_t n_views,
                                          int32_t height, int32_t width, const int32_t* lang_tokens,
                                          const int32_t* lang_mask, int32_t n_lang, const float* state,
                                          const float* noise, const uint64_t* seeds, float* actions,
                                          const float* prev, int32_t n_prev, const float* weights,
                                          float max_guidance);
VLA_API int32_t vla_smolvla_int8_layers(void* h);
VLA_API int32_t vla_smolvla_kernels_per_step(void* h);
/* The byte-level BPE tokenizer SmolVLA's handles use (host code, no device
 * work): ids of `text` (at most cap written; ids may be NULL when cap is 0)
 * under the vocab.txt / merges.txt contents; returns the full token count. */
VLA_API int32_t vla_bpe_tokenize(const char* vocab_text, const char* merges_text, const char* text, int32_t* ids,
                                 int32_t cap);

#ifdef __cplusplus
}
#endif

#endif /* VLA_SIMD_CUDA_H */
