// ec_kv_cache.hpp -- C++ face of the C ABI, shaped like echo-core's KVCache.
//
// echo-core's engine holds a `std::unique_ptr<KVCache>` and calls
// KVCache(const ModelConfig&), layer(i), append(i, k, v), seq_len(), reset()
// (include/kv_cache.h:21-48), then runs its attention loop over the layer's
// buffers (src/inference.cpp:321-406).  ec::gpu::KVCache keeps those names
// and argument meanings with the storage in HBM:
//   - the constructor takes the reference's ModelConfig unchanged (layout is
//     checked at compile time against ec_model_config);
//   - layer(i) returns a KVCacheLayer view with device pointers, as a
//     reference that binds to the reference's own `KVCacheLayer&` (so
//     `KVCacheLayer& cache_layer = kv_cache_->layer(layer_idx);` of
//     src/inference.cpp:331 compiles unchanged) or to ec_kv_layer&;
//   - append(i, k, v) takes device pointers to the token's fp32 K/V
//     projections and quantizes them on the GPU;
//   - attention(i, q, out) is the KV half of InferenceEngine::attention;
//   - step / step_host(i, q, k, v, attn_out) are InferenceEngine::attention
//     without its weight matvecs: attention, then the token's append.
// Errors throw std::runtime_error carrying ec_last_error(); the reference
// used assert (compiled out) and std::runtime_error (src/inference.cpp:22).
#pragma once

#include <cstddef>
#include <stdexcept>
#include <string>
#include <vector>

#include "ec_kv.h"

namespace ec {
namespace gpu {

inline void check(int status) {
    if (status != EC_OK)
        throw std::runtime_error(std::string("ec: ") + ec_status_string(status) + ": " +
                                 ec_last_error());
}

// One layer's view: ec_kv_layer plus a conversion to any struct laid out like
// it, the reference's KVCacheLayer (include/kv_cache.h:7-18) included.  The
// view is refreshed from the cache by every KVCache::layer() call; writing to
// it does not change the cache (append() and reset() do).
struct LayerView : ec_kv_layer {
    template <class KVCacheLayerT>
    operator KVCacheLayerT&() {
        static_assert(sizeof(KVCacheLayerT) == sizeof(ec_kv_layer) &&
                          alignof(KVCacheLayerT) == alignof(ec_kv_layer),
                      "KVCacheLayer layout differs from ec_kv_layer");
        return *reinterpret_cast<KVCacheLayerT*>(static_cast<ec_kv_layer*>(this));
    }
    template <class KVCacheLayerT>
    operator const KVCacheLayerT&() const {
        static_assert(sizeof(KVCacheLayerT) == sizeof(ec_kv_layer) &&
                          alignof(KVCacheLayerT) == alignof(ec_kv_layer),
                      "KVCacheLayer layout differs from ec_kv_layer");
        return *reinterpret_cast<const KVCacheLayerT*>(static_cast<const ec_kv_layer*>(this));
    }
};
static_assert(sizeof(LayerView) == 64 && alignof(LayerView) == 64,
              "KVCacheLayer is 64 bytes, 64-byte aligned");

class KVCache {
public:
    // Any struct laid out like ModelConfig (include/config.h:6-24) is accepted,
    // the reference's own type included.
    template <class ModelConfigT>
    explicit KVCache(const ModelConfigT& config, ec_scale_mode mode = EC_SCALE_PER_HEAD) {
        static_assert(sizeof(ModelConfigT) == sizeof(ec_model_config),
                      "ModelConfig layout differs from ec_model_config");
        check(ec_kv_cache_create(reinterpret_cast<const ec_model_config*>(&config), mode, &h_));
        views_.resize(config.num_layers);
    }
    ~KVCache() { ec_kv_cache_destroy(h_); }
    KVCache(const KVCache&) = delete;
    KVCache& operator=(const KVCache&) = delete;

    // KVCache::layer (src/kv_cache.cpp:79-87): the layer's buffers and length.
    LayerView& layer(uint32_t layer_idx) {
        refresh(layer_idx);
        return views_[layer_idx];
    }
    const LayerView& layer(uint32_t layer_idx) const {
        refresh(layer_idx);
        return views_[layer_idx];
    }
    void append(uint32_t layer_idx, const float* k_proj, const float* v_proj,
                ec_stream_t stream = nullptr) {
        check(ec_kv_cache_append(h_, layer_idx, k_proj, v_proj, stream));
    }
    uint32_t seq_len() const { return ec_kv_cache_seq_len(h_); }
    void reset() { check(ec_kv_cache_reset(h_)); }
    void attention(uint32_t layer_idx, const float* q, float* out, float softmax_scale,
                   ec_stream_t stream = nullptr) {
        check(ec_kv_cache_attention(h_, layer_idx, q, out, softmax_scale, stream));
    }
    // One token of InferenceEngine::attention without its weight matvecs
    // (src/inference.cpp:321-414): attend over the layer's cached tokens, then
    // append this token's k/v.  Device pointers, asynchronous.
    void step(uint32_t layer_idx, const float* q_proj, const float* k_proj, const float* v_proj,
              float* attn_out, float softmax_scale, ec_stream_t stream = nullptr) {
        check(ec_kv_cache_step(h_, layer_idx, q_proj, k_proj, v_proj, attn_out, softmax_scale,
                               stream));
    }
    // The same for host buffers (the reference engine's q_proj_, k_proj_,
    // v_proj_, attn_out_); synchronous.
    void step_host(uint32_t layer_idx, const float* q_proj, const float* k_proj,
                   const float* v_proj, float* attn_out, float softmax_scale) {
        check(ec_kv_cache_step_host(h_, layer_idx, q_proj, k_proj, v_proj, attn_out,
                                    softmax_scale));
    }
    ec_kv_cache* handle() const { return h_; }

private:
    void refresh(uint32_t layer_idx) const {
        check(ec_kv_cache_layer(h_, layer_idx, static_cast<ec_kv_layer*>(&views_.at(layer_idx))));
    }
    ec_kv_cache* h_ = nullptr;
    mutable std::vector<LayerView> views_;
};

}  // namespace gpu
}  // namespace ec
