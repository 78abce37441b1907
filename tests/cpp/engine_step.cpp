// Drives ec::gpu::KVCache the way InferenceEngine::forward drives its cache:
// for every token, every layer runs attention over that layer's cached tokens
// and then appends the token's K/V (src/inference.cpp:301-415), here through
// step_host() with host buffers, as the reference engine keeps them.  Every
// output is checked against the oracle's decode attention (liboracle.so, the
// CPU restatement of src/inference.cpp:321-392) over an independently
// quantized host copy of the cache.  Exit status 0 = all steps within the
// attention bar (max-abs <= 2e-3 and |err| <= 2e-3 + 1e-3*|ref|).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <random>
#include <vector>

#include "ec_kv_cache.hpp"

extern "C" {
void oracle_quantize_per_token_symmetric(const float* in, int8_t* out, float* scales,
                                         uint32_t num_tokens, uint32_t num_elements);
void oracle_decode_attention(const int8_t* keys, const int8_t* values, const float* kscales,
                             const float* vscales, uint32_t kv_len, const float* q, float* out,
                             uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim,
                             float softmax_scale, int scale_mode, float* scratch);
}

// the reference's ModelConfig (include/config.h:6-24), field for field
struct ModelConfig {
    uint32_t vocab_size, hidden_dim, num_heads, num_kv_heads, head_dim, num_layers;
    uint32_t ffn_hidden_dim, max_seq_len;
    int32_t ffn_type, norm_type, pos_encoding;
    bool use_kv_quantization;
};

int main() {
    const uint32_t H = 16, HKV = 4, D = 128, LAYERS = 3, TOKENS = 40;
    ModelConfig cfg{1000, H * D, H, HKV, D, LAYERS, 4 * H * D, 64, 0, 0, 0, true};
    ec::gpu::KVCache cache(cfg);
    const float scale = 1.0f / std::sqrt((float)D);
    std::mt19937 rng(7);
    std::normal_distribution<float> nd(0.f, 1.f);
    const uint32_t nkv = HKV * D;
    std::vector<std::vector<int8_t>> kq(LAYERS), vq(LAYERS);
    std::vector<std::vector<float>> ks(LAYERS), vs(LAYERS);
    std::vector<float> q(H * D), k(nkv), v(nkv), out(H * D), want(H * D), scratch(TOKENS + 1);
    double worst = 0;
    for (uint32_t t = 0; t < TOKENS; ++t) {
        for (uint32_t l = 0; l < LAYERS; ++l) {
            for (auto& x : q) x = nd(rng);
            for (auto& x : k) x = nd(rng);
            for (auto& x : v) x = nd(rng);
            cache.step_host(l, q.data(), k.data(), v.data(), out.data(), scale);
            // oracle: attention over the t tokens cached before this one
            if (t == 0) {
                for (float w : out)
                    if (w != 0.f) { std::printf("FAIL: empty layer gave nonzero\n"); return 1; }
            } else {
                oracle_decode_attention(kq[l].data(), vq[l].data(), ks[l].data(), vs[l].data(), t,
                                        q.data(), want.data(), H, HKV, D, scale, 0, scratch.data());
                for (uint32_t i = 0; i < H * D; ++i) {
                    const double err = std::fabs((double)out[i] - want[i]);
                    worst = std::max(worst, err);
                    if (!(err <= 2e-3 && err <= 2e-3 + 1e-3 * std::fabs(want[i]))) {
                        std::printf("FAIL: token %u layer %u elem %u got %g want %g\n", t, l, i,
                                    out[i], want[i]);
                        return 1;
                    }
                }
            }
            // this token joins the host copy, quantized per head as KVCache::append does
            kq[l].resize((t + 1) * nkv); vq[l].resize((t + 1) * nkv);
            ks[l].resize((t + 1) * HKV); vs[l].resize((t + 1) * HKV);
            oracle_quantize_per_token_symmetric(k.data(), kq[l].data() + t * nkv,
                                                ks[l].data() + t * HKV, HKV, D);
            oracle_quantize_per_token_symmetric(v.data(), vq[l].data() + t * nkv,
                                                vs[l].data() + t * HKV, HKV, D);
        }
    }
    if (cache.seq_len() != TOKENS) { std::printf("FAIL: seq_len %u\n", cache.seq_len()); return 1; }
    // the device cache holds the same codes as the host copy
    for (uint32_t l = 0; l < LAYERS; ++l)
        if (cache.layer(l).seq_len != TOKENS) { std::printf("FAIL: layer length\n"); return 1; }
    cache.reset();
    if (cache.seq_len() != 0) { std::printf("FAIL: reset\n"); return 1; }
    std::printf("engine_step ok: %u tokens x %u layers, worst abs err %.3g\n", TOKENS, LAYERS, worst);
    return 0;
}
