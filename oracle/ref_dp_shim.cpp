// TEST INFRASTRUCTURE ONLY. Intermediate taps of the reference's own Diffusion
// Policy (vla.simd src/models/diffusion), for locating a parity difference:
// the global conditioning vector a query builds (DiffusionModel::predict,
// src/models/diffusion/diffusion_model.cpp:190-240) and one ResNet stage map of
// one frame (ResNetBackbone::forward, src/models/act/resnet_backbone.cpp:211-315).
// Compiled with the reference's sources into oracle/_ref/libvla_ref.so; the
// model's members are opened to this file only, to call its private preprocess.
#define private public
#include "models/diffusion/diffusion_model.h"
#undef private
#include "ops/conv_ops.h"
#include "ops/lm_ops.h"

#include <cstdint>
#include <cstring>
#include <vector>

using tcpu::DiffusionModel;

extern "C" {

// gcond [n_obs * (state_dim + n_cams * 2K)] of one query; returns 0 on success
int ref_dp_global_cond(const char* dir, const uint8_t* frames, const float* state, float* gcond) {
    DiffusionModel m;
    if (!m.load(dir)) return -1;
    const tcpu::DPConfig& c = m.cfg;
    const int S = c.n_obs_steps, N = c.n_cams, F = 2 * c.num_keypoints, per = c.state_dim + N * F;
    const int oh = c.crop_h > 0 ? c.crop_h : c.img_h, ow = c.crop_w > 0 ? c.crop_w : c.img_w;
    std::vector<float> img((size_t)oh * ow * 3);
    const size_t px = (size_t)c.img_h * c.img_w * 3;
    for (int s = 0; s < S; ++s) {
        float* g = gcond + (size_t)s * per;
        for (int i = 0; i < c.state_dim; ++i) {
            const float den = m.state_max[i] - m.state_min[i];
            const float d = den == 0.0f ? 1e-8f : den;
            g[i] = 2.0f * (state[(size_t)s * c.state_dim + i] - m.state_min[i]) / d - 1.0f;
        }
        for (int cam = 0; cam < N; ++cam) {
            m.preprocess(frames + ((size_t)s * N + cam) * px, cam, img.data());
            const tcpu::DPRgbEncoder& e = m.encoders[c.separate_encoder_per_camera ? cam : 0];
            e.forward(img.data(), m.scratch, g + c.state_dim + (size_t)cam * F);
        }
    }
    return 0;
}

// The map after stage `stage` (0 stem + GroupNorm, 1 max-pool, 2 + i block i)
// of encoder `cam` on frame (s, cam); returns its element count, or -1.
long long ref_dp_backbone_stage(const char* dir, const uint8_t* frames, int s, int cam, int stage, float* out,
                                long long cap) {
    DiffusionModel m;
    if (!m.load(dir)) return -1;
    const tcpu::DPConfig& c = m.cfg;
    const int oh = c.crop_h > 0 ? c.crop_h : c.img_h, ow = c.crop_w > 0 ? c.crop_w : c.img_w;
    std::vector<float> x((size_t)oh * ow * 3);
    const size_t px = (size_t)c.img_h * c.img_w * 3;
    m.preprocess(frames + ((size_t)s * c.n_cams + cam) * px, cam, x.data());
    const tcpu::ResNetBackbone& b = m.encoders[c.separate_encoder_per_camera ? cam : 0].backbone;
    const tcpu::ResNetConfig& bc = b.cfg;
    const int gs = bc.gn_group_size;
    auto conv_out = [](int in, int k, int st, int p) { return (in + 2 * p - k) / st + 1; };
    auto emit = [&](const std::vector<float>& v, size_t n) -> long long {
        if ((long long)n > cap) return -1;
        std::memcpy(out, v.data(), n * sizeof(float));
        return (long long)n;
    };
    int h = conv_out(oh, bc.stem_k, bc.stem_stride, bc.stem_pad), w = conv_out(ow, bc.stem_k, bc.stem_stride, bc.stem_pad);
    std::vector<float> a((size_t)h * w * bc.stem_out);
    b.stem.forward(a.data(), x.data(), oh, ow, bc.stem_stride, bc.stem_pad);
    if (gs) tcpu::groupnorm(a.data(), a.data(), b.stem_gn[0], b.stem_gn[1], h * w, bc.stem_out, bc.stem_out / gs, 1e-5f, false);
    if (stage == 0) return emit(a, a.size());
    const int ph = conv_out(h, bc.pool_k, bc.pool_stride, bc.pool_pad), pw = conv_out(w, bc.pool_k, bc.pool_stride, bc.pool_pad);
    std::vector<float> cur((size_t)ph * pw * bc.stem_out);
    tcpu::maxpool2d_relu(cur.data(), a.data(), h, w, bc.stem_out, bc.pool_k, bc.pool_stride, bc.pool_pad);
    h = ph; w = pw;
    if (stage == 1) return emit(cur, cur.size());
    for (size_t i = 0; i < b.blocks.size(); ++i) {
        const tcpu::BasicBlock& blk = b.blocks[i];
        const int h2 = conv_out(h, 3, blk.stride, 1), w2 = conv_out(w, 3, blk.stride, 1);
        const size_t n = (size_t)h2 * w2 * blk.cout;
        std::vector<float> idn = cur, r(n), t(n), c2(n);
        if (blk.has_down) {
            blk.down.forward(r.data(), cur.data(), h, w, blk.stride, 0);
            if (gs) tcpu::groupnorm(r.data(), r.data(), blk.gnd[0], blk.gnd[1], h2 * w2, blk.cout, blk.cout / gs, 1e-5f, false);
            idn = r;
        }
        blk.conv1.forward(t.data(), cur.data(), h, w, blk.stride, 1);
        if (gs) tcpu::groupnorm(t.data(), t.data(), blk.gn1[0], blk.gn1[1], h2 * w2, blk.cout, blk.cout / gs, 1e-5f, true);
        else tcpu::relu(t.data(), (int)n);
        blk.conv2.forward(c2.data(), t.data(), h2, w2, 1, 1);
        if (gs) tcpu::groupnorm(c2.data(), c2.data(), blk.gn2[0], blk.gn2[1], h2 * w2, blk.cout, blk.cout / gs, 1e-5f, false);
        for (size_t j = 0; j < n; ++j) {
            const float v = c2[j] + idn[j];
            c2[j] = v > 0.0f ? v : 0.0f;
        }
        cur.swap(c2);
        h = h2; w = w2;
        if (stage == (int)(2 + i)) return emit(cur, cur.size());
    }
    return -1;
}

}  // extern "C"
