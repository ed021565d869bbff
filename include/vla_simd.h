/*
 * vla_simd.h - model-level C ABI of libvla_simd_b200.so, the B200 (sm_100a)
 * backend of vla.simd. Same symbols, argument order and contracts as the
 * reference's include/vla_simd.h, so its ctypes callers
 * (vla_simd/policy_server.py:181-262, ActEngine at :276-307) load this library
 * unchanged.
 *
 * Ownership
 *   vla_act_load pairs with vla_act_free. Every other pointer - frames, state,
 *   the actions output - is caller-owned HOST memory, borrowed for the duration
 *   of the call. Weights live on the GPU from load to free.
 *
 * Errors
 *   Fallible calls return vla_status (0 == VLA_OK); _load returns NULL. C++
 *   exceptions never cross the boundary. CUDA failures (including a kernel's
 *   bounded wait running out) are reported as VLA_ERR_DEVICE, a code this
 *   backend appends after the reference's three.
 *
 * Threading
 *   One handle is one inference at a time (it owns a stream, scratch buffers
 *   and a captured CUDA graph). Load one handle per GPU for data parallelism;
 *   VLA_CUDA_DEVICE (or the calling thread's current device) picks the GPU.
 *
 * Precision
 *   ACT_INT8 selects the W8A8 layers exactly as in the reference
 *   (1 enc attention, 2 enc w1, 4 enc w2, 8 image projection, 16 decoder,
 *   32 backbone convs; ACT_I8_CONV_FROM / ACT_I8_CONV_TO, TCPU_I8_CLIP).
 */

#ifndef VLA_SIMD_H
#define VLA_SIMD_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VLA_API __attribute__((visibility("default")))

/* Kept at the reference's value: the additions below are new codes only, so a
 * caller that checks vla_abi_version() == 1 (the reference server does) binds. */
#define VLA_ABI_VERSION 1

typedef enum {
    VLA_OK            =  0,
    VLA_ERR_ARG       = -1,  /* NULL handle, NULL buffer, or an out-of-range dimension */
    VLA_ERR_SHAPE     = -2,  /* an argument disagrees with the loaded checkpoint */
    VLA_ERR_EXCEPTION = -3,  /* a C++ exception was caught at the boundary */
    VLA_ERR_DEVICE    = -4   /* a CUDA call or kernel failed (this backend only) */
} vla_status;

/* replaces reference include/vla_simd.h:60-62 (src/capi_version.cpp:14-15) */
VLA_API int32_t vla_abi_version(void);
VLA_API const char* vla_backend_name(void);   /* "cuda-sm100a" */
VLA_API int32_t vla_int8_available(void);      /* 1 when an sm_100 device is visible */

/* ---------------------------------------------------------------- ACT -----
 * replaces reference include/vla_simd.h:66-81 (src/models/act/act_capi.cpp:20-54).
 * model_dir: a converter directory (config.txt, backbone.meta/.bin, act.meta/.bin,
 * stats.bin) as written by the reference's tools/convert_act.py. */

VLA_API void* vla_act_load(const char* model_dir);
VLA_API void  vla_act_free(void* h);

/* 0 on a NULL handle. */
VLA_API int32_t vla_act_chunk(void* h);
VLA_API int32_t vla_act_action_dim(void* h);
VLA_API int32_t vla_act_state_dim(void* h);
VLA_API int32_t vla_act_n_cams(void* h);
VLA_API int32_t vla_act_img_h(void* h);
VLA_API int32_t vla_act_img_w(void* h);

/* images: n_cams frames back to back, uint8 HWC at img_h x img_w, in the
 * checkpoint's camera order. state [state_dim] in raw robot units.
 * actions out [chunk*action_dim]. */
VLA_API int32_t vla_act_predict(void* h, const uint8_t* images, const float* state,
                                int32_t unnormalize, float* actions);

/* ---------------------------------------------------- Diffusion Policy -----
 * replaces reference include/vla_simd.h:258-280 (src/models/diffusion/diffusion_capi.cpp:23-72).
 * model_dir: a converter directory (diffusion.meta, rgb_encoder{i}_backbone.meta/.bin,
 * rgb_encoder{i}.bin, unet.bin, stats.bin) as written by tools/convert_diffusion.py.
 * DIFFUSION_INT8 (bit 1 U-Net GEMMs, bit 2 backbone convs), DP_STEPS and
 * DP_SCHEDULER keep the reference's meaning. */
VLA_API void* vla_diffusion_load(const char* model_dir);
VLA_API void  vla_diffusion_free(void* h);

VLA_API int32_t vla_diffusion_chunk(void* h);        /* n_action_steps */
VLA_API int32_t vla_diffusion_horizon(void* h);
VLA_API int32_t vla_diffusion_action_dim(void* h);
VLA_API int32_t vla_diffusion_state_dim(void* h);
VLA_API int32_t vla_diffusion_n_cams(void* h);
VLA_API int32_t vla_diffusion_n_obs_steps(void* h);
VLA_API int32_t vla_diffusion_img_h(void* h);
VLA_API int32_t vla_diffusion_img_w(void* h);
VLA_API int32_t vla_diffusion_num_steps(void* h);
VLA_API int32_t vla_diffusion_is_ddim(void* h);

/* frames [n_obs_steps, n_cams, img_h, img_w, 3] uint8, oldest first; state
 * [n_obs_steps, state_dim]; noise [1 + num_steps, horizon, action_dim] or NULL
 * (the sampler then starts from zeros); actions out [chunk, action_dim]. */
VLA_API int32_t vla_diffusion_predict(void* h, const uint8_t* frames, const float* state,
                                      int32_t unnormalize, float* actions,
                                      const float* noise);

/* -------------------------------------------------------------- SmolVLA -----
 * replaces reference include/vla_simd.h:83-117 (src/models/smolvla/smolvla_capi.cpp:66-180).
 * model_dir: a converter directory (vit / vlm / aex / heads .meta + .bin,
 * emb.bin, stats_{state,action}_{mean,std}.bin, config.txt) as written by
 * tools/convert_hf_safetensors.py, or its vla.simd GGUF; tok_dir holds the
 * byte-level BPE tokenizer (vocab.txt, merges.txt). SMOLVLA_INT8 (1 vision
 * q/k/v/o, 2 fc1, 4 fc2, 8 patch embedding + connector, 16 text tower, 32
 * action expert) and SMOLVLA_NUM_STEPS keep the reference's meaning. */
VLA_API void* vla_smolvla_load(const char* model_dir, const char* tok_dir);
VLA_API void  vla_smolvla_free(void* h);

VLA_API int32_t vla_smolvla_chunk(void* h);
VLA_API int32_t vla_smolvla_action_dim(void* h);
VLA_API int32_t vla_smolvla_state_dim(void* h);
VLA_API int32_t vla_smolvla_n_views(void* h);
VLA_API int32_t vla_smolvla_img_size(void* h);
VLA_API int32_t vla_smolvla_tok_maxlen(void* h);

/* ids / mask [tok_maxlen] of the instruction (a newline appended, the last
 * tok_maxlen tokens kept, then pad); returns the token count. */
VLA_API int32_t vla_smolvla_tokenize(void* h, const char* text, int32_t* ids, int32_t* mask);

/* frames [n_views, height, width, 3] uint8 at the camera's resolution
 * (resize-with-pad happens inside); lang tokens / mask [n_lang] from
 * vla_smolvla_tokenize; state [state_dim] raw; noise [chunk, 32] or NULL
 * (drawn from seed); actions out [chunk, action_dim]. */
VLA_API int32_t vla_smolvla_predict(void* h, const uint8_t* frames, int32_t n_views,
                                    int32_t height, int32_t width,
                                    const int32_t* lang_tokens, const int32_t* lang_mask, int32_t n_lang,
                                    const float* state, const float* noise, uint64_t seed,
                                    float* actions);

/* As vla_smolvla_predict with real-time-chunking guidance toward the previous
 * chunk's first n_prev rows prev [n_prev, action_dim], weights [chunk],
 * max_guidance > 0. */
VLA_API int32_t vla_smolvla_predict_rtc(void* h, const uint8_t* frames, int32_t n_views,
                                        int32_t height, int32_t width,
                                        const int32_t* lang_tokens, const int32_t* lang_mask, int32_t n_lang,
                                        const float* state, const float* noise, uint64_t seed,
                                        float* actions, const float* prev, int32_t n_prev,
                                        const float* weights, float max_guidance);

/* ----------------------------------------------------------------- Octo -----
 * replaces reference include/vla_simd.h:121-144 (src/models/octo/octo_capi.cpp:19-58).
 * model_dir: a converter directory (t5.meta/.bin, stem_primary.meta/.bin,
 * stem_wrist.meta/.bin, octo.meta/.bin, head.meta/.bin,
 * stats_action_{mean,std,mask}.bin) as written by tools/convert_octo.py, or
 * its vla.simd GGUF; tok_dir holds the tokenizer's vocab.txt
 * (tools/convert_t5_tokenizer.py). OCTO_INT8 (1 q/k/v/o, 2 MLP w1, 4 MLP w2,
 * 8 token projections + stem embeddings, 16 stem convs, 32 diffusion head)
 * keeps the reference's meaning. */
VLA_API void* vla_octo_load(const char* model_dir, const char* tok_dir);
VLA_API void  vla_octo_free(void* h);

VLA_API int32_t vla_octo_horizon(void* h);
VLA_API int32_t vla_octo_action_dim(void* h);
VLA_API int32_t vla_octo_max_window(void* h);

/* primary [wnd,256,256,3] and wrist [wnd,128,128,3] (or NULL) uint8 HWC;
 * timestep_mask [wnd] (1 = real, 0 = history padding); wnd in
 * [1, vla_octo_max_window]. The DDPM noise is drawn from `seed` as the
 * reference draws it. actions out [horizon*action_dim]. */
VLA_API int32_t vla_octo_predict(void* h, const uint8_t* primary, const uint8_t* wrist,
                                 int32_t wnd, const uint8_t* timestep_mask,
                                 const char* instruction, uint64_t seed,
                                 int32_t unnormalize, float* actions);

/* As vla_octo_predict with the noise supplied: noise [horizon*action_dim] is
 * the initial x, z [steps*horizon*action_dim] the per-step draws. Both or neither. */
VLA_API int32_t vla_octo_predict_ex(void* h, const uint8_t* primary, const uint8_t* wrist,
                                    int32_t wnd, const uint8_t* timestep_mask,
                                    const char* instruction, const float* noise,
                                    const float* z, uint64_t seed,
                                    int32_t unnormalize, float* actions);

#ifdef __cplusplus
}
#endif

#endif /* VLA_SIMD_H */
