// TEST INFRASTRUCTURE ONLY. Taps of the reference's own Octo (vla.simd
// src/models/octo) and T5 tokenizer, for parity tests that look inside a
// query: the token ids of an instruction (T5Tokenizer::encode,
// src/tokenizer/t5_tokenizer.cpp:131-155) and the readout embedding the
// diffusion head reads (OctoModel::predict, src/models/octo/octo_model.cpp:166-197,
// up to the transformer's final LayerNorm). Compiled with the reference's
// sources into oracle/_ref/libvla_ref.so.
#include "models/octo/octo_model.h"
#include "io/files.h"
#include "tokenizer/t5_tokenizer.h"

#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

extern "C" {

// ids [max_len] of `text` under the vocab.txt in tok_dir; returns 0 on success
int ref_t5_tokenize(const char* tok_dir, const char* text, int max_len, int32_t* ids) {
    tcpu::T5Tokenizer tok;
    if (!tok.load(tok_dir)) return -1;
    const std::vector<int> v = tok.encode(text, max_len);
    if ((int)v.size() != max_len) return -2;
    for (int i = 0; i < max_len; ++i) ids[i] = v[i];
    return 0;
}

// readout [d] of the last step of one query; returns 0 on success
int ref_octo_readout(const char* dir, const char* tok_dir, const uint8_t* primary, const uint8_t* wrist, int wnd,
                     const uint8_t* tmask, const char* instruction, float* readout) {
    tcpu::OctoModel m;
    if (!m.load(dir, tok_dir)) return -1;
    const int NT = m.tf.cfg.n_task, D = m.tf.cfg.d;
    std::vector<int> ids = m.tok.encode(instruction, NT), am(NT);
    for (int i = 0; i < NT; ++i) am[i] = ids[i] != m.tok.pad_id;
    std::vector<float> t5((size_t)NT * m.t5.cfg.d_model);
    m.t5.encode(ids.data(), am.data(), NT, t5.data());
    const size_t PB = (size_t)256 * 256 * 3, WB = (size_t)128 * 128 * 3;
    const size_t SP = (size_t)m.tf.cfg.tok_primary * m.tf.cfg.stem_dim, SW = (size_t)m.tf.cfg.tok_wrist * m.tf.cfg.stem_dim;
    std::vector<float> sp((size_t)wnd * SP), sw(wrist ? (size_t)wnd * SW : 0);
    for (int t = 0; t < wnd; ++t) {
        m.stem_primary.encode(primary + t * PB, 256, 256, sp.data() + t * SP);
        if (wrist) m.stem_wrist.encode(wrist + t * WB, 128, 128, sw.data() + t * SW);
    }
    std::vector<float> out((size_t)m.tf.total_tokens(wnd) * D);
    m.tf.forward(t5.data(), sp.data(), wrist ? sw.data() : nullptr, wnd, tmask, out.data());
    std::memcpy(readout, out.data() + (size_t)m.tf.readout_index(wnd, wnd - 1) * D, sizeof(float) * D);
    return 0;
}

}  // extern "C"
