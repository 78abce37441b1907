// decode_noalloc.cu -- decode attention for callers that cannot allocate.
//
// ec_decode_attention needs a device workspace for its split-K partials and
// leaves it to the caller to provide one.  Some callers have no way to get
// device memory at the point where they run decode: code that runs where
// cudaMalloc is off limits (a host callback or an interrupt-like hook, where
// a blocking, device-synchronising allocator call would stall or deadlock),
// a runtime whose memory was carved up once at start-up and may not grow, or
// a plugin host that forbids device allocations after initialisation.  For
// them this file provides ec_decode_attention_noalloc, which takes its
// workspace from a fixed array compiled into the library instead.
//
// The array is kNoAllocScratchBytes (16 MiB) of device memory that every GPU
// which loads this library keeps until the process exits.  The first call on
// each device looks up the array's device address with cudaGetSymbolAddress
// (with that device current) and remembers it; make that first call before
// any stream capture.  All calls share the one array and nothing in it needs
// to start at zero: every partial the combine step reads is written earlier
// by the same call.  Two calls whose kernels overlap on the GPU (different
// streams, no ordering) race on the array and corrupt each other's results.
#include <cstdio>
#include <mutex>

#include "ec_common.cuh"
#include "ec_internal.h"
#include "ec_kv.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch for each device ordinal, looked up once.
void* scratch_address(int device, cudaError_t* err) {
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[device]) {
        void* p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (*err != cudaSuccess) return nullptr;
        addr[device] = p;
    }
    *err = cudaSuccess;
    return addr[device];
}

int reject(int status, const char* msg) {
    char line[256];
    snprintf(line, sizeof(line), "decode_attention_noalloc: %s", msg);
    return ec::set_last_error(status, line);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int ec_decode_attention_noalloc(const ec_kv_batch* b, const float* q, float* out,
                                uint32_t num_heads, float softmax_scale, ec_stream_t stream) {
    if (!b || !q || !out) return reject(EC_ERR_INVALID_ARGUMENT, "null argument");
    if (!b->keys || !b->values || !b->key_scales || !b->val_scales || !b->seq_offset ||
        !b->seq_capacity || !b->seq_len)
        return reject(EC_ERR_INVALID_ARGUMENT, "null buffer in batch");
    if (b->scale_mode != EC_SCALE_PER_HEAD && b->scale_mode != EC_SCALE_ROW)
        return reject(EC_ERR_INVALID_ARGUMENT, "bad scale_mode");
    if (!aligned16(b->keys) || !aligned16(b->values) || !aligned16(b->key_scales) ||
        !aligned16(b->val_scales) || !aligned16(q) || !aligned16(out))
        return reject(EC_ERR_MISALIGNED, "buffers must be 16-byte aligned");
    if (b->num_seqs == 0) return EC_OK;
    if (b->num_seqs > 65535u || b->total_slots >= (1ull << 31) || b->max_seq_len > 0x7fffffffu)
        return reject(EC_ERR_UNSUPPORTED, "batch too large (num_seqs <= 65535, total_slots < 2^31)");
    const uint32_t hkv = b->num_kv_heads;
    if (b->head_dim != 128 || (hkv != 4 && hkv != 8) || num_heads == 0 || num_heads % hkv ||
        (num_heads / hkv != 1 && num_heads / hkv != 2 && num_heads / hkv != 4))
        return reject(EC_ERR_UNSUPPORTED,
                      "needs head_dim 128, num_kv_heads 4|8, num_heads/num_kv_heads 1|2|4");

    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return reject(EC_ERR_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return reject(EC_ERR_UNSUPPORTED, "device ordinal >= 64");

    const ec::DecodePlan plan = ec::plan_decode((int)b->num_seqs, (int)b->max_seq_len, sms,
                                                b->total_tokens_hint);
    const size_t need = ec::decode_workspace_bytes(plan, (int)b->num_seqs, (int)num_heads);
    if (need > kNoAllocScratchBytes) {
        char msg[200];
        snprintf(msg, sizeof(msg),
                 "this batch needs %zu bytes of split-K scratch, above the fixed %zu-byte array; "
                 "use ec_decode_attention with a caller-provided workspace",
                 need, kNoAllocScratchBytes);
        return reject(EC_ERR_WORKSPACE, msg);
    }
    void* scratch = scratch_address(dev, &e);
    if (!scratch) return reject(EC_ERR_CUDA, cudaGetErrorString(e));

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
    a.row_scales = b->scale_mode == EC_SCALE_ROW;
    a.mode = ec::kOut;
    e = ec::launch_decode(a, (int)hkv, plan, scratch, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return reject(EC_ERR_CUDA, cudaGetErrorString(e));
    return EC_OK;
}

}  // extern "C"
