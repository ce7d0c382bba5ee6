// Golden-vector generator for the KV append (fp32 -> truncated fp16 encode +
// page-slot scatter), built against the reference's own
// cottus::GenericTransformer (cottus/csrc/generic_transformer.cpp) by
// `make -C oracle engine`.
//
// TEST INFRASTRUCTURE ONLY, used here (where the reference tree exists) by
// tests/golden/make_golden.py.  It runs forwardToken on the CPU device for a
// one-layer model and, next to it, recomputes the rotated k and the v that
// forwardToken encodes (same reference primitives, same order as
// generic_transformer.cpp:150-202), so the fixture pins the restated encoder
// and scatter against the real code bit for bit.
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "compute_primitives_cpu.h"
#include "engine.h"
#include "generic_transformer.h"
#include "page_table.h"

extern "C" int ref_forward_token_kv(int32_t vocab, int32_t hidden, int32_t num_heads, int32_t num_kv_heads,
                                    int32_t head_dim, int32_t inter, int32_t block_size, float theta,
                                    float eps, const float *embed, const float *attn_norm, const float *wq,
                                    const float *wk, const float *wv, const float *wo, const float *w1,
                                    const float *w2, const float *w3, const float *ffn_norm,
                                    const float *out_norm, const float *lm_head, int32_t token, int32_t pos,
                                    const int32_t *table, int32_t ntable, uint16_t *kv_cache,
                                    float *k_rot_out, float *v_out) {
    try {
        cottus::EngineConfig cfg{};
        cfg.vocabSize = vocab;
        cfg.hiddenDim = hidden;
        cfg.numLayers = 1;
        cfg.numHeads = num_heads;
        cfg.numKvHeads = num_kv_heads;
        cfg.headDim = head_dim;
        cfg.intermediateDim = inter;
        cfg.maxSeqLen = ntable * block_size;
        cfg.blockSize = block_size;
        cfg.ropeTheta = theta;
        cfg.normEpsilon = eps;
        cfg.device = "cpu";
        cfg.dtype = "float32";
        auto p = [](const float *x) { return reinterpret_cast<uintptr_t>(x); };
        std::unordered_map<std::string, uintptr_t> w{
            {"model.embed_tokens.weight", p(embed)},
            {"model.norm.weight", p(out_norm)},
            {"lm_head.weight", p(lm_head)},
            {"model.layers.0.self_attn.q_proj.weight", p(wq)},
            {"model.layers.0.self_attn.k_proj.weight", p(wk)},
            {"model.layers.0.self_attn.v_proj.weight", p(wv)},
            {"model.layers.0.self_attn.o_proj.weight", p(wo)},
            {"model.layers.0.mlp.gate_proj.weight", p(w1)},
            {"model.layers.0.mlp.down_proj.weight", p(w2)},
            {"model.layers.0.mlp.up_proj.weight", p(w3)},
            {"model.layers.0.input_layernorm.weight", p(attn_norm)},
            {"model.layers.0.post_attention_layernorm.weight", p(ffn_norm)},
        };
        cottus::GenericTransformer tf(cfg, w);
        cottus::PageTable pt(block_size);
        for (int32_t i = 0; i < ntable; ++i) pt.appendBlock(table[i]);

        // The k and v that forwardToken encodes for layer 0.
        std::vector<float> x(embed + static_cast<int64_t>(token) * hidden,
                             embed + static_cast<int64_t>(token + 1) * hidden);
        cottus::rmsnormCPU(x.data(), x.data(), attn_norm, hidden, eps);
        cottus::gemmCPU(k_rot_out, x.data(), wk, 1, num_kv_heads * head_dim, hidden);
        cottus::gemmCPU(v_out, x.data(), wv, 1, num_kv_heads * head_dim, hidden);
        cottus::ropeCPU(k_rot_out, k_rot_out, pos, num_kv_heads, head_dim, theta);

        tf.forwardToken(token, pos, pt, reinterpret_cast<uintptr_t>(kv_cache), "cpu");
        return 0;
    } catch (...) {
        return -3;
    }
}
