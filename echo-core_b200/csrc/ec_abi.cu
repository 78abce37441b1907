// ec_abi.cu -- host side of the C ABI declared in include/ec_kv.h.
//
// Validates arguments, translates the reference's object model (KVCache,
// KVCacheLayer, ModelConfig) onto device memory, picks the split plan and
// launches the kernels.  No exception crosses the ABI; every failure returns
// an ec_status and records a one-line reason for ec_last_error().
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "ec_common.cuh"
#include "ec_internal.h"
#include "ec_kv.h"

namespace {

thread_local char g_last_error[256] = "";

int fail(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return status;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(EC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms_current() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
}

// The fp32-cache kernel: any num_kv_heads, query groups of 1, 2, 4 or 8.
bool f32_shape_supported(uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim) {
    if (head_dim != 128 || num_kv_heads == 0 || num_heads == 0 || num_heads % num_kv_heads)
        return false;
    const uint32_t g = num_heads / num_kv_heads;
    return g == 1 || g == 2 || g == 4 || g == 8;
}

cudaStream_t as_stream(ec_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace

int ec::set_last_error(int status, const char* msg) { return fail(status, "%s", msg); }

bool ec::decode_shape_supported(uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim) {
    if ((head_dim != 128 && head_dim != 256) || num_kv_heads == 0 || num_kv_heads > 8) return false;
    if (num_heads == 0 || num_heads % num_kv_heads || num_heads / num_kv_heads > 32) return false;
    return ec::decode_variant((int)num_kv_heads, (int)(num_heads / num_kv_heads), (int)head_dim).hc != 0;
}

using ec::decode_shape_supported;

struct ec_kv_cache {
    ec_model_config cfg;
    int scale_mode;
    int device;
    void* slab;
    size_t slab_bytes;
    std::vector<ec_kv_layer> layers;
    void* ws;
    size_t ws_bytes;
    ec::DecodePlan plan;
    float* stage;        // device staging of the host-pointer step: q | k | v | out
};

extern "C" {

int ec_abi_version(void) { return EC_KV_ABI_VERSION; }

const char* ec_status_string(int status) {
    switch (status) {
        case EC_OK: return "ok";
        case EC_ERR_INVALID_ARGUMENT: return "invalid argument";
        case EC_ERR_MISALIGNED: return "device pointer not 16-byte aligned";
        case EC_ERR_CAPACITY: return "cache capacity exceeded";
        case EC_ERR_UNSUPPORTED: return "shape outside the supported envelope";
        case EC_ERR_CUDA: return "CUDA error";
        case EC_ERR_WORKSPACE: return "workspace missing or too small";
        case EC_ERR_DEVICE_CHECK: return "a kernel flagged bad input";
        default: return "unknown status";
    }
}

const char* ec_last_error(void) { return g_last_error; }

int ec_device_error(int32_t* err_word, ec_stream_t stream, int32_t* code) {
    if (!code) return fail(EC_ERR_INVALID_ARGUMENT, "ec_device_error: code is NULL");
    cudaStream_t st = as_stream(stream);
    int32_t zero = 0, host = 0;
    cudaError_t e;
    if (err_word) {
        e = cudaMemcpyAsync(&host, err_word, sizeof(host), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(err_word, &zero, sizeof(zero), cudaMemcpyHostToDevice, st);
    } else {
        e = cudaMemcpyFromSymbolAsync(&host, ec::g_error_word, sizeof(host), 0, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(ec::g_error_word, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st);
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "ec_device_error");
    *code = host;
    return EC_OK;
}

int ec_quantize_per_token_symmetric(const float* input, int8_t* output, float* scales,
                                    uint32_t num_tokens, uint32_t num_elements,
                                    ec_stream_t stream) {
    if (num_tokens == 0) return EC_OK;
    if (!input || !output || !scales || num_elements == 0)
        return fail(EC_ERR_INVALID_ARGUMENT, "quantize: null pointer or num_elements == 0");
    cudaError_t e = ec::launch_quantize_rows(input, output, scales, num_tokens, num_elements,
                                             as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "quantize launch");
}

int ec_fused_dequant_dot_int8(const float* query, const int8_t* key_cache, const float* scales,
                              float* scores, uint32_t dim, uint32_t seq_len, ec_stream_t stream) {
    if (seq_len == 0) return EC_OK;
    if (!query || !key_cache || !scales || !scores || dim == 0)
        return fail(EC_ERR_INVALID_ARGUMENT, "fused_dequant_dot: null pointer or dim == 0");
    cudaError_t e = ec::launch_fused_dequant_dot(query, key_cache, scales, scores, dim, seq_len,
                                                 as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "fused_dequant_dot launch");
}

// ---------------------------------------------------------------- KVCache
int ec_kv_cache_create(const ec_model_config* config, int scale_mode, ec_kv_cache** out) {
    if (!config || !out) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_create: null argument");
    *out = nullptr;
    if (scale_mode != EC_SCALE_PER_HEAD && scale_mode != EC_SCALE_ROW)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_create: bad scale_mode %d", scale_mode);
    const ec_model_config& c = *config;
    if (c.num_kv_heads == 0 || c.head_dim == 0)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_create: num_kv_heads and head_dim must be > 0");
    if ((uint64_t)c.max_seq_len > 0x7fffffffull)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_create: max_seq_len too large");
    ec_kv_cache* kc = new (std::nothrow) ec_kv_cache();
    if (!kc) return fail(EC_ERR_CUDA, "kv_cache_create: host allocation failed");
    kc->cfg = c;
    kc->scale_mode = scale_mode;
    kc->slab = nullptr;
    kc->ws = nullptr;
    kc->ws_bytes = 0;
    kc->plan = ec::DecodePlan{32, 1};
    kc->stage = nullptr;
    cudaGetDevice(&kc->device);
    kc->layers.assign(c.num_layers, ec_kv_layer{});

    // Same partition as src/kv_cache.cpp:24-71; every sub-buffer is rounded
    // up to 256 B so the kernels' 16-byte vector and bulk accesses stay aligned.
    auto r256 = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t row = (size_t)c.num_kv_heads * c.head_dim;
    const size_t max_seq = c.max_seq_len;
    size_t per_layer;
    if (c.use_kv_quantization) {
        per_layer = 2 * r256(max_seq * row) + 2 * r256(max_seq * c.num_kv_heads * sizeof(float));
    } else {
        per_layer = 2 * r256(max_seq * row * sizeof(float));
    }
    kc->slab_bytes = per_layer * c.num_layers;
    if (kc->slab_bytes) {
        cudaError_t e = cudaMalloc(&kc->slab, kc->slab_bytes);
        if (e == cudaSuccess) e = cudaMemset(kc->slab, 0, kc->slab_bytes);
        if (e != cudaSuccess) {
            cudaFree(kc->slab);
            delete kc;
            return cuda_fail(e, "kv_cache_create: device slab");
        }
        uint8_t* p = static_cast<uint8_t*>(kc->slab);
        for (uint32_t l = 0; l < c.num_layers; ++l) {
            ec_kv_layer& L = kc->layers[l];
            if (c.use_kv_quantization) {
                L.keys_int8 = reinterpret_cast<int8_t*>(p); p += r256(max_seq * row);
                L.values_int8 = reinterpret_cast<int8_t*>(p); p += r256(max_seq * row);
                L.key_scales = reinterpret_cast<float*>(p); p += r256(max_seq * c.num_kv_heads * 4);
                L.val_scales = reinterpret_cast<float*>(p); p += r256(max_seq * c.num_kv_heads * 4);
            } else {
                L.keys_fp32 = reinterpret_cast<float*>(p); p += r256(max_seq * row * 4);
                L.values_fp32 = reinterpret_cast<float*>(p); p += r256(max_seq * row * 4);
            }
        }
    }
    if (!c.use_kv_quantization && c.num_layers > 0 &&
        f32_shape_supported(c.num_heads, c.num_kv_heads, c.head_dim)) {
        kc->ws_bytes = ec::f32_decode_workspace_bytes((int)c.max_seq_len, (int)c.num_kv_heads,
                                                       (int)c.num_heads);
        if (kc->ws_bytes) {
            cudaError_t e = cudaMalloc(&kc->ws, kc->ws_bytes);
            if (e != cudaSuccess) {
                cudaFree(kc->slab);
                delete kc;
                return cuda_fail(e, "kv_cache_create: decode workspace");
            }
        }
    }
    if (c.use_kv_quantization && c.num_layers > 0 &&
        decode_shape_supported(c.num_heads, c.num_kv_heads, c.head_dim)) {
        kc->plan = ec::plan_decode(1, (int)c.max_seq_len, num_sms_current(), 0,
                                   (int)c.num_kv_heads, (int)c.num_heads, (int)c.head_dim);
        kc->ws_bytes = ec::decode_workspace_bytes(kc->plan, 1, (int)c.num_heads, (int)c.head_dim);
        if (kc->ws_bytes) {
            cudaError_t e = cudaMalloc(&kc->ws, kc->ws_bytes);
            if (e != cudaSuccess) {
                cudaFree(kc->slab);
                delete kc;
                return cuda_fail(e, "kv_cache_create: decode workspace");
            }
        }
    }
    *out = kc;
    return EC_OK;
}

void ec_kv_cache_destroy(ec_kv_cache* cache) {
    if (!cache) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(cache->device);
    cudaDeviceSynchronize();
    cudaFree(cache->slab);
    cudaFree(cache->ws);
    cudaFree(cache->stage);
    cudaSetDevice(prev);
    delete cache;
}

int ec_kv_cache_layer(const ec_kv_cache* cache, uint32_t layer_idx, ec_kv_layer* out) {
    if (!cache || !out) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_layer: null argument");
    if (layer_idx >= cache->cfg.num_layers)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_layer: layer %u >= num_layers %u", layer_idx,
                    cache->cfg.num_layers);
    *out = cache->layers[layer_idx];
    return EC_OK;
}

int ec_kv_cache_append(ec_kv_cache* cache, uint32_t layer_idx, const float* k_proj,
                       const float* v_proj, ec_stream_t stream) {
    if (!cache || !k_proj || !v_proj) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_append: null argument");
    if (layer_idx >= cache->cfg.num_layers)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_append: layer %u out of range", layer_idx);
    ec_kv_layer& L = cache->layers[layer_idx];
    const ec_model_config& c = cache->cfg;
    if (L.seq_len >= c.max_seq_len)
        return fail(EC_ERR_CAPACITY, "kv_cache_append: layer %u is full (%u tokens)", layer_idx,
                    c.max_seq_len);
    const size_t row = (size_t)c.num_kv_heads * c.head_dim;
    const size_t pos = L.seq_len;
    cudaStream_t st = as_stream(stream);
    cudaError_t e;
    if (!c.use_kv_quantization) {
        e = cudaMemcpyAsync(L.keys_fp32 + pos * row, k_proj, row * 4, cudaMemcpyDeviceToDevice, st);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(L.values_fp32 + pos * row, v_proj, row * 4, cudaMemcpyDeviceToDevice, st);
    } else if ((c.head_dim == 128 || c.head_dim == 256) && aligned16(k_proj) && aligned16(v_proj) &&
               (c.num_kv_heads == 1 || c.num_kv_heads == 2 || c.num_kv_heads == 4 || c.num_kv_heads == 8)) {
        ec::AppendArgs a{};
        a.k = k_proj;
        a.v = v_proj;
        a.keys = L.keys_int8;
        a.values = L.values_int8;
        a.key_scales = L.key_scales;
        a.val_scales = L.val_scales;
        a.host_offset = 0;
        a.host_capacity = (int32_t)c.max_seq_len;
        a.host_length = (int32_t)pos;
        a.err = nullptr;
        a.total_slots = c.max_seq_len;
        a.num_seqs = 1;
        a.n_new = 1;
        a.head_dim = (int)c.head_dim;
        e = ec::launch_append(a, (int)c.num_kv_heads, cache->scale_mode == EC_SCALE_ROW, st);
    } else if (cache->scale_mode == EC_SCALE_ROW) {
        e = ec::launch_quantize_rows(k_proj, L.keys_int8 + pos * row, L.key_scales + pos, 1, (uint32_t)row, st);
        if (e == cudaSuccess)
            e = ec::launch_quantize_rows(v_proj, L.values_int8 + pos * row, L.val_scales + pos, 1, (uint32_t)row, st);
    } else {
        e = ec::launch_quantize_rows(k_proj, L.keys_int8 + pos * row, L.key_scales + pos * c.num_kv_heads,
                                     c.num_kv_heads, c.head_dim, st);
        if (e == cudaSuccess)
            e = ec::launch_quantize_rows(v_proj, L.values_int8 + pos * row, L.val_scales + pos * c.num_kv_heads,
                                         c.num_kv_heads, c.head_dim, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "kv_cache_append");
    L.seq_len++;
    return EC_OK;
}

uint32_t ec_kv_cache_seq_len(const ec_kv_cache* cache) {
    if (!cache || cache->cfg.num_layers == 0) return 0;
    return cache->layers[0].seq_len;
}

int ec_kv_cache_reset(ec_kv_cache* cache) {
    if (!cache) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_reset: null cache");
    for (auto& L : cache->layers) L.seq_len = 0;
    return EC_OK;
}

int ec_kv_cache_attention(ec_kv_cache* cache, uint32_t layer_idx, const float* q, float* out,
                          float softmax_scale, ec_stream_t stream) {
    if (!cache || !q || !out) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_attention: null argument");
    const ec_model_config& c = cache->cfg;
    if (layer_idx >= c.num_layers) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_attention: layer out of range");
    if (!c.use_kv_quantization) {
        // FP32 mode (src/inference.cpp:346-358, 386-393)
        if (!f32_shape_supported(c.num_heads, c.num_kv_heads, c.head_dim))
            return fail(EC_ERR_UNSUPPORTED, "kv_cache_attention (fp32 cache): needs head_dim 128 and num_heads / num_kv_heads in {1, 2, 4, 8}");
        if (!aligned16(q) || !aligned16(out)) return fail(EC_ERR_MISALIGNED, "kv_cache_attention: q/out not 16-byte aligned");
        const ec_kv_layer& L = cache->layers[layer_idx];
        cudaError_t e = ec::launch_decode_f32(L.keys_fp32, L.values_fp32, (int)c.num_kv_heads,
                                              (int)c.num_heads, (int)L.seq_len, q, softmax_scale,
                                              out, cache->ws, as_stream(stream));
        return e == cudaSuccess ? EC_OK : cuda_fail(e, "kv_cache_attention (fp32 cache) launch");
    }
    if (!decode_shape_supported(c.num_heads, c.num_kv_heads, c.head_dim))
        return fail(EC_ERR_UNSUPPORTED, "kv_cache_attention: needs head_dim 128|256, num_kv_heads 1|2|4|8 and num_heads a multiple of it by at most 32");
    if (!aligned16(q) || !aligned16(out)) return fail(EC_ERR_MISALIGNED, "kv_cache_attention: q/out not 16-byte aligned");
    const ec_kv_layer& L = cache->layers[layer_idx];
    ec::DecodeArgs a{};
    a.keys = L.keys_int8;
    a.values = L.values_int8;
    a.key_scales = L.key_scales;
    a.val_scales = L.val_scales;
    a.host_offset = 0;
    a.host_capacity = (int32_t)c.max_seq_len;
    a.host_length = (int32_t)L.seq_len;
    a.err = nullptr;
    a.total_slots = c.max_seq_len;
    a.q = q;
    a.out = out;
    a.q_mul = softmax_scale;
    a.num_seqs = 1;
    a.num_heads = (int)c.num_heads;
    a.head_dim = (int)c.head_dim;
    a.row_scales = cache->scale_mode == EC_SCALE_ROW;
    a.mode = ec::kOut;
    cudaError_t e = ec::launch_decode(a, (int)c.num_kv_heads, cache->plan, cache->ws, as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "kv_cache_attention launch");
}

int ec_kv_cache_step(ec_kv_cache* cache, uint32_t layer_idx, const float* q, const float* k_proj,
                     const float* v_proj, float* attn_out, float softmax_scale, ec_stream_t stream) {
    if (!cache) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_step: null cache");
    if (layer_idx >= cache->cfg.num_layers)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_step: layer %u out of range", layer_idx);
    // full layer: refuse before attending, so a failed step changes nothing
    if (cache->layers[layer_idx].seq_len >= cache->cfg.max_seq_len)
        return fail(EC_ERR_CAPACITY, "kv_cache_step: layer %u is full (%u tokens)", layer_idx,
                    cache->cfg.max_seq_len);
    // attention over the cache as it stands, then this token's append: the
    // order of src/inference.cpp:330-414
    int rc = ec_kv_cache_attention(cache, layer_idx, q, attn_out, softmax_scale, stream);
    if (rc != EC_OK) return rc;
    return ec_kv_cache_append(cache, layer_idx, k_proj, v_proj, stream);
}

int ec_kv_cache_step_host(ec_kv_cache* cache, uint32_t layer_idx, const float* q,
                          const float* k_proj, const float* v_proj, float* attn_out,
                          float softmax_scale) {
    if (!cache || !q || !k_proj || !v_proj || !attn_out)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_step_host: null argument");
    const ec_model_config& c = cache->cfg;
    const size_t nq = (size_t)c.num_heads * c.head_dim;
    const size_t nkv = (size_t)c.num_kv_heads * c.head_dim;
    // four 256-byte-aligned slots: q, k, v, out
    auto r64 = [](size_t n) { return (n + 63) & ~size_t(63); };
    const size_t oq = 0, ok = r64(nq), ov = ok + r64(nkv), oo = ov + r64(nkv), total = oo + r64(nq);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(cache->device);
    cudaError_t e = cudaSuccess;
    if (!cache->stage) e = cudaMalloc(&cache->stage, total * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(cache->stage + oq, q, nq * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(cache->stage + ok, k_proj, nkv * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(cache->stage + ov, v_proj, nkv * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaSetDevice(prev);
        return cuda_fail(e, "kv_cache_step_host: staging");
    }
    int rc = ec_kv_cache_step(cache, layer_idx, cache->stage + oq, cache->stage + ok,
                              cache->stage + ov, cache->stage + oo, softmax_scale, nullptr);
    if (rc == EC_OK) {
        e = cudaMemcpy(attn_out, cache->stage + oo, nq * 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = cuda_fail(e, "kv_cache_step_host: read back");
    }
    cudaSetDevice(prev);
    return rc;
}

// ------------------------------------------------------------ snapshots
// Host image of a cache object's contents: a header (magic, version, shape,
// scale mode, per-layer lengths) followed, per layer, by the used prefix of
// each buffer: int8 K and V codes plus K and V scales ([len][num_kv_heads],
// or [len] for ROW scales), or the fp32 K and V rows.  Little-endian, packed.
namespace {
constexpr char kSnapMagic[8] = {'E', 'C', 'K', 'V', 'S', 'N', 'A', 'P'};
constexpr uint32_t kSnapVersion = 1;
struct SnapHeader {
    char magic[8];
    uint32_t version, num_heads, num_kv_heads, head_dim, num_layers, max_seq_len;
    uint32_t use_kv_quantization, scale_mode;
};
struct LayerBytes { size_t codes, scales, fp32; };
LayerBytes layer_bytes(const ec_kv_cache* c, uint32_t len) {
    const size_t row = (size_t)c->cfg.num_kv_heads * c->cfg.head_dim;
    const size_t ns = c->scale_mode == EC_SCALE_ROW ? 1 : c->cfg.num_kv_heads;
    if (c->cfg.use_kv_quantization) return {len * row, len * ns * sizeof(float), 0};
    return {0, 0, len * row * sizeof(float)};
}
size_t snapshot_bytes(const ec_kv_cache* c) {
    size_t b = sizeof(SnapHeader) + (size_t)c->cfg.num_layers * sizeof(uint32_t);
    for (const auto& L : c->layers) {
        const LayerBytes lb = layer_bytes(c, L.seq_len);
        b += 2 * (lb.codes + lb.scales + lb.fp32);
    }
    return b;
}
}  // namespace

size_t ec_kv_cache_snapshot_size(const ec_kv_cache* cache) {
    return cache ? snapshot_bytes(cache) : 0;
}

int ec_kv_cache_snapshot(const ec_kv_cache* cache, void* host, size_t bytes) {
    if (!cache || !host) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_snapshot: null argument");
    const size_t need = snapshot_bytes(cache);
    if (bytes < need)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_snapshot: buffer of %zu bytes, need %zu", bytes, need);
    uint8_t* p = static_cast<uint8_t*>(host);
    SnapHeader h;
    std::memcpy(h.magic, kSnapMagic, 8);
    h.version = kSnapVersion;
    h.num_heads = cache->cfg.num_heads;
    h.num_kv_heads = cache->cfg.num_kv_heads;
    h.head_dim = cache->cfg.head_dim;
    h.num_layers = cache->cfg.num_layers;
    h.max_seq_len = cache->cfg.max_seq_len;
    h.use_kv_quantization = cache->cfg.use_kv_quantization ? 1u : 0u;
    h.scale_mode = (uint32_t)cache->scale_mode;
    std::memcpy(p, &h, sizeof h);
    p += sizeof h;
    for (const auto& L : cache->layers) {
        std::memcpy(p, &L.seq_len, sizeof(uint32_t));
        p += sizeof(uint32_t);
    }
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(cache->device);
    cudaError_t e = cudaDeviceSynchronize();   // appends in flight land first
    for (size_t l = 0; e == cudaSuccess && l < cache->layers.size(); ++l) {
        const ec_kv_layer& L = cache->layers[l];
        const LayerBytes lb = layer_bytes(cache, L.seq_len);
        const void* src[4] = {L.keys_int8, L.values_int8, L.key_scales, L.val_scales};
        const size_t len[4] = {lb.codes, lb.codes, lb.scales, lb.scales};
        const void* srcf[2] = {L.keys_fp32, L.values_fp32};
        for (int i = 0; e == cudaSuccess && i < 4 && cache->cfg.use_kv_quantization; ++i) {
            if (len[i]) e = cudaMemcpy(p, src[i], len[i], cudaMemcpyDeviceToHost);
            p += len[i];
        }
        for (int i = 0; e == cudaSuccess && i < 2 && !cache->cfg.use_kv_quantization; ++i) {
            if (lb.fp32) e = cudaMemcpy(p, srcf[i], lb.fp32, cudaMemcpyDeviceToHost);
            p += lb.fp32;
        }
    }
    cudaSetDevice(prev);
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "kv_cache_snapshot");
}

int ec_kv_cache_restore(ec_kv_cache* cache, const void* host, size_t bytes) {
    if (!cache || !host) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_restore: null argument");
    const uint8_t* p = static_cast<const uint8_t*>(host);
    SnapHeader h;
    if (bytes < sizeof h) return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_restore: truncated header");
    std::memcpy(&h, p, sizeof h);
    p += sizeof h;
    if (std::memcmp(h.magic, kSnapMagic, 8) != 0 || h.version != kSnapVersion)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_restore: not a version-%u cache snapshot", kSnapVersion);
    const ec_model_config& c = cache->cfg;
    if (h.num_heads != c.num_heads || h.num_kv_heads != c.num_kv_heads || h.head_dim != c.head_dim ||
        h.num_layers != c.num_layers || h.use_kv_quantization != (c.use_kv_quantization ? 1u : 0u) ||
        h.scale_mode != (uint32_t)cache->scale_mode)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_restore: snapshot shape or mode differs from the cache's");
    if (bytes < sizeof h + (size_t)h.num_layers * sizeof(uint32_t))
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_restore: truncated length table");
    std::vector<uint32_t> lens(h.num_layers);
    std::memcpy(lens.data(), p, lens.size() * sizeof(uint32_t));
    p += lens.size() * sizeof(uint32_t);
    size_t need = sizeof h + lens.size() * sizeof(uint32_t);
    for (uint32_t n : lens) {
        if (n > c.max_seq_len)
            return fail(EC_ERR_CAPACITY, "kv_cache_restore: a layer holds %u tokens, the cache %u", n, c.max_seq_len);
        const LayerBytes lb = layer_bytes(cache, n);
        need += 2 * (lb.codes + lb.scales + lb.fp32);
    }
    if (bytes < need)
        return fail(EC_ERR_INVALID_ARGUMENT, "kv_cache_restore: %zu bytes, the header describes %zu", bytes, need);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(cache->device);
    cudaError_t e = cudaDeviceSynchronize();
    for (size_t l = 0; e == cudaSuccess && l < cache->layers.size(); ++l) {
        ec_kv_layer& L = cache->layers[l];
        const LayerBytes lb = layer_bytes(cache, lens[l]);
        void* dst[4] = {L.keys_int8, L.values_int8, L.key_scales, L.val_scales};
        const size_t len[4] = {lb.codes, lb.codes, lb.scales, lb.scales};
        void* dstf[2] = {L.keys_fp32, L.values_fp32};
        for (int i = 0; e == cudaSuccess && i < 4 && c.use_kv_quantization; ++i) {
            if (len[i]) e = cudaMemcpy(dst[i], p, len[i], cudaMemcpyHostToDevice);
            p += len[i];
        }
        for (int i = 0; e == cudaSuccess && i < 2 && !c.use_kv_quantization; ++i) {
            if (lb.fp32) e = cudaMemcpy(dstf[i], p, lb.fp32, cudaMemcpyHostToDevice);
            p += lb.fp32;
        }
        if (e == cudaSuccess) L.seq_len = lens[l];
    }
    cudaSetDevice(prev);
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "kv_cache_restore");
}

// ------------------------------------------------- context-parallel comm
struct ec_cp_comm {
    int world, rank, num_seqs, num_heads, device;
    float* local;                        // this rank's receive buffer
    float* peers[ec::kCpMaxWorld];       // opened IPC mappings (own slot = local)
    uint32_t* epoch_dev;                 // device epochs per (sequence, head, split) (calls with epoch 0)
    int epoch_mode;                      // 0 none yet, 1 caller epochs, 2 device epochs
    bool opened;
};

int ec_cp_comm_create(uint32_t world, uint32_t rank, uint32_t num_seqs, uint32_t num_heads,
                      ec_cp_comm** out, void* ipc_handle) {
    if (!out || !ipc_handle) return fail(EC_ERR_INVALID_ARGUMENT, "cp_comm_create: null argument");
    if (world == 0 || world > (uint32_t)ec::kCpMaxWorld || rank >= world)
        return fail(EC_ERR_INVALID_ARGUMENT, "cp_comm_create: world %u / rank %u (world at most %d)",
                    world, rank, ec::kCpMaxWorld);
    if (num_seqs == 0 || num_heads == 0 || (uint64_t)num_seqs * num_heads > 148u * 16u)
        return fail(EC_ERR_UNSUPPORTED, "cp_comm_create: num_seqs * num_heads must be in 1..2368");
    ec_cp_comm* c = new (std::nothrow) ec_cp_comm();
    if (!c) return fail(EC_ERR_CUDA, "cp_comm_create: host allocation failed");
    c->world = (int)world;
    c->rank = (int)rank;
    c->num_seqs = (int)num_seqs;
    c->num_heads = (int)num_heads;
    c->opened = false;
    c->epoch_mode = 0;
    c->local = nullptr;
    c->epoch_dev = nullptr;
    cudaGetDevice(&c->device);
    const size_t bytes = ec::cp_exchange_buffer_bytes(c->world, c->num_seqs, c->num_heads);
    cudaError_t e = cudaMalloc(&c->local, bytes);
    if (e == cudaSuccess) e = cudaMemset(c->local, 0, bytes);   // flags start below epoch 1
    const size_t ebytes = (size_t)num_seqs * num_heads * ec::kCpSplitMax * sizeof(uint32_t);
    if (e == cudaSuccess) e = cudaMalloc(&c->epoch_dev, ebytes);
    if (e == cudaSuccess) e = cudaMemset(c->epoch_dev, 0, ebytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
    if (e != cudaSuccess) {
        cudaFree(c->local);
        cudaFree(c->epoch_dev);
        delete c;
        return cuda_fail(e, "cp_comm_create: receive buffer");
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == EC_CP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(ipc_handle, &h, sizeof h);
    for (auto& p : c->peers) p = nullptr;
    c->peers[c->rank] = c->local;
    *out = c;
    return EC_OK;
}

int ec_cp_comm_open(ec_cp_comm* c, const void* handles) {
    if (!c || !handles) return fail(EC_ERR_INVALID_ARGUMENT, "cp_comm_open: null argument");
    if (c->opened) return fail(EC_ERR_INVALID_ARGUMENT, "cp_comm_open: already open");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    const uint8_t* hp = static_cast<const uint8_t*>(handles);
    cudaError_t e = cudaSuccess;
    int r = 0;
    for (; r < c->world && e == cudaSuccess; ++r) {
        if (r == c->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, hp + (size_t)r * EC_CP_HANDLE_BYTES, sizeof h);
        void* p = nullptr;
        e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        c->peers[r] = static_cast<float*>(p);
    }
    if (e != cudaSuccess) {
        for (int q = 0; q < c->world; ++q)
            if (q != c->rank && c->peers[q]) { cudaIpcCloseMemHandle(c->peers[q]); c->peers[q] = nullptr; }
        cudaSetDevice(prev);
        return cuda_fail(e, "cp_comm_open: cudaIpcOpenMemHandle of a peer's buffer");
    }
    c->opened = true;
    cudaSetDevice(prev);
    return EC_OK;
}

void ec_cp_comm_destroy(ec_cp_comm* c) {
    if (!c) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    for (int r = 0; r < c->world; ++r)
        if (r != c->rank && c->peers[r]) cudaIpcCloseMemHandle(c->peers[r]);
    cudaFree(c->local);
    cudaFree(c->epoch_dev);
    cudaSetDevice(prev);
    delete c;
}

// Checks a comm for a step with the given epoch and fills the exchange
// arguments common to both exchange entry points.
static int cp_step_args(ec_cp_comm* c, uint32_t epoch, float* out, const char* who,
                        ec::CpExchangeArgs& a) {
    if (!c->opened && c->world > 1) return fail(EC_ERR_INVALID_ARGUMENT, "%s: comm not opened", who);
    const int mode = epoch == 0 ? 2 : 1;
    if (c->epoch_mode != 0 && c->epoch_mode != mode)
        return fail(EC_ERR_INVALID_ARGUMENT,
                    "%s: a comm uses caller epochs or device epochs (0), not both", who);
    c->epoch_mode = mode;
    a = ec::CpExchangeArgs{};
    for (int r = 0; r < c->world; ++r) a.peer_base[r] = c->peers[r];
    a.out = out;
    a.err = nullptr;
    a.world = c->world;
    a.rank = c->rank;
    a.num_seqs = c->num_seqs;
    a.num_heads = c->num_heads;
    a.epoch = epoch;
    a.epoch_dev = mode == 2 ? c->epoch_dev : nullptr;
    return EC_OK;
}

int ec_cp_exchange_combine(ec_cp_comm* c, const float* part_o, const float* part_ml,
                           uint32_t epoch, float* out, ec_stream_t stream) {
    if (!c || !part_o || !part_ml || !out)
        return fail(EC_ERR_INVALID_ARGUMENT, "cp_exchange_combine: null argument");
    if (!c->opened && c->world > 1)
        return fail(EC_ERR_INVALID_ARGUMENT, "cp_exchange_combine: comm not opened");
    const int mode = epoch == 0 ? 2 : 1;
    if (c->epoch_mode != 0 && c->epoch_mode != mode)
        return fail(EC_ERR_INVALID_ARGUMENT,
                    "cp_exchange_combine: a comm uses caller epochs or device epochs (0), not both");
    c->epoch_mode = mode;
    ec::CpExchangeArgs a{};
    for (int r = 0; r < c->world; ++r) a.peer_base[r] = c->peers[r];
    a.part_o = part_o;
    a.part_ml = part_ml;
    a.out = out;
    a.err = nullptr;
    a.world = c->world;
    a.rank = c->rank;
    a.num_seqs = c->num_seqs;
    a.num_heads = c->num_heads;
    a.epoch = epoch;
    a.epoch_dev = mode == 2 ? c->epoch_dev : nullptr;
    cudaError_t e = ec::launch_cp_exchange(a, as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "cp_exchange_combine launch");
}

size_t ec_cp_decode_workspace_size(const ec_kv_batch* b, uint32_t num_heads) {
    if (!b) return 0;
    const ec::DecodePlan p = ec::plan_decode((int)b->num_seqs, (int)b->max_seq_len,
                                             num_sms_current(), b->total_tokens_hint,
                                             (int)b->num_kv_heads, (int)num_heads,
                                             (int)b->head_dim, false);
    const int chunks = p.max_chunks > 1 ? p.max_chunks : 1;
    return (size_t)b->num_seqs * chunks * num_heads * (b->head_dim + 2) * sizeof(float);
}

int ec_cp_decode_exchange(ec_cp_comm* c, const ec_kv_batch* b, const float* q,
                          uint32_t num_heads, float softmax_scale, void* workspace,
                          size_t workspace_bytes, uint32_t epoch, float* out,
                          ec_stream_t stream) {
    const char* who = "cp_decode_exchange";
    if (!c) return fail(EC_ERR_INVALID_ARGUMENT, "%s: comm is NULL", who);
    int rc = ec::check_batch(b, who);
    if (rc) return rc;
    if (!q || !out || !workspace) return fail(EC_ERR_INVALID_ARGUMENT, "%s: q/out/workspace NULL", who);
    if (b->num_seqs != (uint32_t)c->num_seqs || num_heads != (uint32_t)c->num_heads)
        return fail(EC_ERR_INVALID_ARGUMENT, "%s: batch of %u sequences x %u heads, comm made for %d x %d",
                    who, b->num_seqs, num_heads, c->num_seqs, c->num_heads);
    if (b->head_dim != 128 || !decode_shape_supported(num_heads, b->num_kv_heads, b->head_dim))
        return fail(EC_ERR_UNSUPPORTED, "%s: needs head_dim 128 and a decode-kernel GQA shape", who);
    if (!aligned16(q) || !aligned16(out) || !aligned16(workspace))
        return fail(EC_ERR_MISALIGNED, "%s: q/out/workspace not 16-byte aligned", who);
    const ec::DecodePlan plan = ec::plan_decode((int)b->num_seqs, (int)b->max_seq_len,
                                                num_sms_current(), b->total_tokens_hint,
                                                (int)b->num_kv_heads, (int)num_heads, 128, false);
    const size_t need = ec_cp_decode_workspace_size(b, num_heads);
    if (workspace_bytes < need)
        return fail(EC_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", who, need,
                    workspace_bytes);
    ec::CpExchangeArgs x;
    if ((rc = cp_step_args(c, epoch, out, who, x)) != EC_OK) return rc;
    ec::DecodeArgs a{};
    a.keys = b->keys;
    a.values = b->values;
    a.key_scales = b->key_scales;
    a.val_scales = b->val_scales;
    a.seq_offset = b->seq_offset;
    a.seq_capacity = b->seq_capacity;
    a.seq_len = b->seq_len;
    a.err = b->error_word;
    a.total_slots = b->total_slots;
    a.pages = ec::page_map_of(b);
    a.q = q;
    a.out = out;
    a.q_mul = softmax_scale;
    a.num_seqs = (int)b->num_seqs;
    a.num_heads = (int)num_heads;
    a.head_dim = 128;
    a.row_scales = b->scale_mode == EC_SCALE_ROW;
    a.mode = ec::kChunks;
    cudaStream_t st = as_stream(stream);
    cudaError_t e = ec::launch_decode(a, (int)b->num_kv_heads, plan, workspace, st);
    if (e != cudaSuccess) return cuda_fail(e, who);
    x.part_o = static_cast<const float*>(workspace);
    x.part_ml = x.part_o + (size_t)b->num_seqs * plan.max_chunks * num_heads * 128;
    x.err = b->error_word;
    x.seq_len = b->seq_len;
    x.chunk_tokens = plan.chunk_tokens;
    x.max_chunks = plan.max_chunks;
    e = ec::launch_cp_exchange(x, st);
    return e == cudaSuccess ? EC_OK : cuda_fail(e, who);
}

// ------------------------------------------------------------ batched cache
}  // extern "C"

int ec::check_batch(const ec_kv_batch* b, const char* who) {
    if (!b) return fail(EC_ERR_INVALID_ARGUMENT, "%s: batch is NULL", who);
    if (!b->keys || !b->values || !b->key_scales || !b->val_scales ||
        (!b->seq_offset && !b->page_table) || !b->seq_capacity || !b->seq_len)
        return fail(EC_ERR_INVALID_ARGUMENT, "%s: null buffer in batch", who);
    if (b->page_table) {
        const uint32_t p = b->page_tokens;
        if (p < 128 || (p & (p - 1)) || p > (1u << 24))
            return fail(EC_ERR_INVALID_ARGUMENT, "%s: page_tokens must be a power of two >= 128", who);
        if (b->max_pages == 0 || b->total_slots < p || b->total_slots % p)
            return fail(EC_ERR_INVALID_ARGUMENT, "%s: paged batch needs max_pages > 0 and total_slots a non-zero multiple of page_tokens", who);
        if ((uint64_t)b->max_pages * p > 0x7fffffffull)
            return fail(EC_ERR_INVALID_ARGUMENT, "%s: max_pages * page_tokens must fit int32", who);
    }
    if (b->scale_mode != EC_SCALE_PER_HEAD && b->scale_mode != EC_SCALE_ROW)
        return fail(EC_ERR_INVALID_ARGUMENT, "%s: bad scale_mode", who);
    if (!aligned16(b->keys) || !aligned16(b->values) || !aligned16(b->key_scales) ||
        !aligned16(b->val_scales))
        return fail(EC_ERR_MISALIGNED, "%s: cache buffers must be 16-byte aligned", who);
    if (b->num_seqs > 65535u) return fail(EC_ERR_UNSUPPORTED, "%s: more than 65535 sequences", who);
    if (b->total_slots >= (1ull << 31))
        return fail(EC_ERR_UNSUPPORTED, "%s: total_slots must be below 2^31", who);
    if (b->max_seq_len > 0x7fffffffu) return fail(EC_ERR_INVALID_ARGUMENT, "%s: max_seq_len too large", who);
    return EC_OK;
}

using ec::check_batch;

extern "C" {

int ec_kv_batch_append(const ec_kv_batch* b, const float* k, const float* v,
                       uint32_t tokens_per_seq, ec_stream_t stream) {
    int rc = check_batch(b, "kv_batch_append");
    if (rc) return rc;
    if (tokens_per_seq == 0 || b->num_seqs == 0) return EC_OK;
    if (!k || !v) return fail(EC_ERR_INVALID_ARGUMENT, "kv_batch_append: k/v NULL");
    if ((b->head_dim != 128 && b->head_dim != 256) ||
        !(b->num_kv_heads == 1 || b->num_kv_heads == 2 || b->num_kv_heads == 4 || b->num_kv_heads == 8))
        return fail(EC_ERR_UNSUPPORTED, "kv_batch_append: needs head_dim 128|256 and num_kv_heads 1|2|4|8");
    if (!aligned16(k) || !aligned16(v)) return fail(EC_ERR_MISALIGNED, "kv_batch_append: k/v not 16-byte aligned");
    if ((uint64_t)b->num_seqs * tokens_per_seq > 0x7fffffffull)
        return fail(EC_ERR_UNSUPPORTED, "kv_batch_append: too many tokens in one call");
    ec::AppendArgs a{};
    a.k = k;
    a.v = v;
    a.keys = b->keys;
    a.values = b->values;
    a.key_scales = b->key_scales;
    a.val_scales = b->val_scales;
    a.seq_offset = b->seq_offset;
    a.seq_capacity = b->seq_capacity;
    a.seq_len = b->seq_len;
    a.err = b->error_word;
    a.total_slots = b->total_slots;
    a.pages = ec::page_map_of(b);
    a.num_seqs = (int)b->num_seqs;
    a.n_new = (int)tokens_per_seq;
    a.head_dim = (int)b->head_dim;
    cudaError_t e = ec::launch_append(a, (int)b->num_kv_heads, b->scale_mode == EC_SCALE_ROW,
                                      as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "kv_batch_append launch");
}

// 1 / base^(i/d), i = 0, 2, .., d - 2 (echo-core-zig src/inference/engine.zig:
// 477-478: freq = 1.0 / pow(f32, base, i / head_dim), all in fp32)
static void rope_inv_freq(float base, uint32_t head_dim, float* out) {
    for (uint32_t i = 0; i < head_dim; i += 2)
        out[i / 2] = 1.0f / std::pow(base, static_cast<float>(i) / static_cast<float>(head_dim));
}

int ec_kv_batch_append_rope(const ec_kv_batch* b, const float* k, const float* v,
                            uint32_t tokens_per_seq, const ec_rope_desc* k_desc,
                            ec_stream_t stream) {
    int rc = check_batch(b, "kv_batch_append_rope");
    if (rc) return rc;
    if (!k_desc) return fail(EC_ERR_INVALID_ARGUMENT, "kv_batch_append_rope: rope descriptor NULL");
    if (tokens_per_seq == 0 || b->num_seqs == 0) return EC_OK;
    if (!k || !v) return fail(EC_ERR_INVALID_ARGUMENT, "kv_batch_append_rope: k/v NULL");
    if ((b->head_dim != 128 && b->head_dim != 256) ||
        !(b->num_kv_heads == 1 || b->num_kv_heads == 2 || b->num_kv_heads == 4 || b->num_kv_heads == 8))
        return fail(EC_ERR_UNSUPPORTED, "kv_batch_append_rope: needs head_dim 128|256 and num_kv_heads 1|2|4|8");
    if (!aligned16(k) || !aligned16(v)) return fail(EC_ERR_MISALIGNED, "kv_batch_append_rope: k/v not 16-byte aligned");
    if (k_desc->norm_weight && (reinterpret_cast<uintptr_t>(k_desc->norm_weight) & 7))
        return fail(EC_ERR_MISALIGNED, "kv_batch_append_rope: norm weight not 8-byte aligned");
    if ((uint64_t)b->num_seqs * tokens_per_seq > 0x7fffffffull)
        return fail(EC_ERR_UNSUPPORTED, "kv_batch_append_rope: too many tokens in one call");
    ec::AppendArgs a{};
    a.k = k;
    a.v = v;
    a.keys = b->keys;
    a.values = b->values;
    a.key_scales = b->key_scales;
    a.val_scales = b->val_scales;
    a.seq_offset = b->seq_offset;
    a.seq_capacity = b->seq_capacity;
    a.seq_len = b->seq_len;
    a.err = b->error_word;
    a.total_slots = b->total_slots;
    a.pages = ec::page_map_of(b);
    a.num_seqs = (int)b->num_seqs;
    a.n_new = (int)tokens_per_seq;
    a.head_dim = (int)b->head_dim;
    a.k_norm_w = k_desc->norm_weight;
    a.rope = k_desc->rope_base > 0.0f;
    if (a.rope) rope_inv_freq(k_desc->rope_base, b->head_dim, a.inv_freq);
    cudaError_t e = ec::launch_append_rope(a, (int)b->num_kv_heads, b->scale_mode == EC_SCALE_ROW,
                                           as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "kv_batch_append_rope launch");
}

int ec_rope_rows(float* x, uint32_t rows, uint32_t num_heads, uint32_t head_dim,
                 const int32_t* positions, const ec_rope_desc* desc, ec_stream_t stream) {
    if (!x || !desc) return fail(EC_ERR_INVALID_ARGUMENT, "rope_rows: null argument");
    if (rows == 0 || num_heads == 0) return EC_OK;
    if (head_dim != 128 && head_dim != 256)
        return fail(EC_ERR_UNSUPPORTED, "rope_rows: needs head_dim 128 or 256");
    const bool rope = desc->rope_base > 0.0f;
    if (rope && !positions) return fail(EC_ERR_INVALID_ARGUMENT, "rope_rows: positions NULL");
    if (!aligned16(x)) return fail(EC_ERR_MISALIGNED, "rope_rows: x not 16-byte aligned");
    if (desc->norm_weight && (reinterpret_cast<uintptr_t>(desc->norm_weight) & 7))
        return fail(EC_ERR_MISALIGNED, "rope_rows: norm weight not 8-byte aligned");
    float inv_freq[ec::kMaxHeadDim / 2] = {};
    if (rope) rope_inv_freq(desc->rope_base, head_dim, inv_freq);
    cudaError_t e = ec::launch_rope_rows(x, rows, num_heads, head_dim, positions, desc->norm_weight,
                                         rope ? 1 : 0, inv_freq, as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "rope_rows launch");
}

size_t ec_decode_workspace_size(uint32_t num_seqs, uint32_t num_heads, uint32_t head_dim,
                                uint32_t max_seq_len) {
    // the plan depends on num_kv_heads, which this query does not take: the
    // largest workspace over every num_kv_heads a kernel covers for num_heads
    const int sms = num_sms_current();
    size_t most = 0;
    for (uint32_t hkv = 1; hkv <= 8; hkv *= 2) {
        if (!num_heads || num_heads % hkv || !decode_shape_supported(num_heads, hkv, head_dim)) continue;
        const ec::DecodePlan p = ec::plan_decode((int)num_seqs, (int)max_seq_len, sms, 0, (int)hkv,
                                                 (int)num_heads, (int)head_dim);
        const size_t b = ec::decode_workspace_bytes(p, (int)num_seqs, (int)num_heads, (int)head_dim);
        if (b > most) most = b;
    }
    return most;
}

size_t ec_decode_workspace_size_batch(const ec_kv_batch* b, uint32_t num_heads) {
    if (!b) return 0;
    ec::DecodePlan p = ec::plan_decode((int)b->num_seqs, (int)b->max_seq_len, num_sms_current(),
                                       b->total_tokens_hint, (int)b->num_kv_heads, (int)num_heads,
                                       (int)b->head_dim);
    return ec::decode_workspace_bytes(p, (int)b->num_seqs, (int)num_heads, (int)b->head_dim);
}

static int decode_common(const ec_kv_batch* b, const float* q, float* out, float* out_ml,
                         uint32_t num_heads, float softmax_scale, void* ws, size_t ws_bytes,
                         int mode, ec_stream_t stream, const char* who) {
    int rc = check_batch(b, who);
    if (rc) return rc;
    if (b->num_seqs == 0) return EC_OK;
    if (!q || !out || (mode == ec::kPartial && !out_ml))
        return fail(EC_ERR_INVALID_ARGUMENT, "%s: q/out NULL", who);
    if (!decode_shape_supported(num_heads, b->num_kv_heads, b->head_dim))
        return fail(EC_ERR_UNSUPPORTED, "%s: needs head_dim 128|256, num_kv_heads 1|2|4|8 and num_heads a multiple of it by at most 32", who);
    if (!aligned16(q) || !aligned16(out)) return fail(EC_ERR_MISALIGNED, "%s: q/out not 16-byte aligned", who);
    ec::DecodePlan plan = ec::plan_decode((int)b->num_seqs, (int)b->max_seq_len, num_sms_current(),
                                          b->total_tokens_hint, (int)b->num_kv_heads, (int)num_heads,
                                          (int)b->head_dim);
    const size_t need = ec::decode_workspace_bytes(plan, (int)b->num_seqs, (int)num_heads,
                                                   (int)b->head_dim);
    if (need > 0 && (!ws || ws_bytes < need))
        return fail(EC_ERR_WORKSPACE, "%s: workspace of %zu bytes needed, %zu given", who, need, ws_bytes);
    if (need > 0 && !aligned16(ws)) return fail(EC_ERR_MISALIGNED, "%s: workspace not 16-byte aligned", who);
    ec::DecodeArgs a{};
    a.keys = b->keys;
    a.values = b->values;
    a.key_scales = b->key_scales;
    a.val_scales = b->val_scales;
    a.seq_offset = b->seq_offset;
    a.seq_capacity = b->seq_capacity;
    a.seq_len = b->seq_len;
    a.err = b->error_word;
    a.total_slots = b->total_slots;
    a.pages = ec::page_map_of(b);
    a.q = q;
    a.out = out;
    a.out_ml = out_ml;
    a.q_mul = softmax_scale;
    a.num_seqs = (int)b->num_seqs;
    a.num_heads = (int)num_heads;
    a.head_dim = (int)b->head_dim;
    a.row_scales = b->scale_mode == EC_SCALE_ROW;
    a.mode = mode;
    cudaError_t e = ec::launch_decode(a, (int)b->num_kv_heads, plan, ws, as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, who);
}

int ec_decode_attention(const ec_kv_batch* b, const float* q, float* out, uint32_t num_heads,
                        float softmax_scale, void* workspace, size_t workspace_bytes,
                        ec_stream_t stream) {
    return decode_common(b, q, out, nullptr, num_heads, softmax_scale, workspace, workspace_bytes,
                         ec::kOut, stream, "decode_attention");
}

int ec_decode_attention_partial(const ec_kv_batch* b, const float* q, float* part_o,
                                float* part_ml, uint32_t num_heads, float softmax_scale,
                                void* workspace, size_t workspace_bytes, ec_stream_t stream) {
    return decode_common(b, q, part_o, part_ml, num_heads, softmax_scale, workspace,
                         workspace_bytes, ec::kPartial, stream, "decode_attention_partial");
}

int ec_prefill_attention(const ec_kv_batch* b, const float* q, float* out, uint32_t n_new,
                         uint32_t num_heads, float softmax_scale, ec_stream_t stream) {
    int rc = check_batch(b, "prefill_attention");
    if (rc) return rc;
    if (b->num_seqs == 0 || n_new == 0) return EC_OK;
    if (!q || !out) return fail(EC_ERR_INVALID_ARGUMENT, "prefill_attention: q/out NULL");
    if (b->head_dim != 128 || b->num_kv_heads == 0 || num_heads == 0 || num_heads % b->num_kv_heads)
        return fail(EC_ERR_UNSUPPORTED, "prefill_attention: needs head_dim 128 and num_heads a multiple of num_kv_heads");
    if (!aligned16(q) || !aligned16(out)) return fail(EC_ERR_MISALIGNED, "prefill_attention: q/out not 16-byte aligned");
    if (n_new > 0x7fffffffu / 128u) return fail(EC_ERR_UNSUPPORTED, "prefill_attention: n_new too large");
    ec::PrefillArgs a{};
    a.keys = b->keys;
    a.values = b->values;
    a.key_scales = b->key_scales;
    a.val_scales = b->val_scales;
    a.seq_offset = b->seq_offset;
    a.seq_capacity = b->seq_capacity;
    a.seq_len = b->seq_len;
    a.err = b->error_word;
    a.total_slots = b->total_slots;
    a.pages = ec::page_map_of(b);
    a.q = q;
    a.out = out;
    a.num_seqs = (int)b->num_seqs;
    a.num_heads = (int)num_heads;
    a.num_kv_heads = (int)b->num_kv_heads;
    a.n_new = (int)n_new;
    a.row_scales = b->scale_mode == EC_SCALE_ROW;
    a.qk_mul = softmax_scale * 1.4426950408889634f;
    cudaError_t e = ec::launch_prefill(a, as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "prefill_attention launch");
}

int ec_lse_combine(const float* part_o, const float* part_ml, uint32_t num_parts,
                   uint32_t num_seqs, uint32_t num_heads, uint32_t head_dim, float* out,
                   ec_stream_t stream) {
    if (!part_o || !part_ml || !out) return fail(EC_ERR_INVALID_ARGUMENT, "lse_combine: null argument");
    if (head_dim != 128 && head_dim != 256)
        return fail(EC_ERR_UNSUPPORTED, "lse_combine: head_dim must be 128 or 256");
    if (num_parts == 0 || num_seqs == 0 || num_heads == 0) return EC_OK;
    if (num_seqs > 0x7fffffffu || num_heads > 65535u)
        return fail(EC_ERR_UNSUPPORTED, "lse_combine: grid too large");
    cudaError_t e = ec::launch_lse_combine(part_o, part_ml, (int)num_parts, (int)num_seqs,
                                           (int)num_heads, (int)head_dim, out, as_stream(stream));
    return e == cudaSuccess ? EC_OK : cuda_fail(e, "lse_combine launch");
}

}  // extern "C"
