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
// (with that device current) and remembers it together with the device's
// current CUDA context; make that first call before any stream capture.  A
// later call that finds a different context current on the device (after
// cudaDeviceReset, the module is loaded again and the array may move) looks
// the address up again instead of using the stale one.  All calls share the
// one array and nothing in it needs to start at zero: every partial the
// combine step reads is written earlier by the same call.  Two calls whose
// kernels overlap on the GPU (different streams, no ordering) race on the
// array and corrupt each other's results.
//
// Argument checking is the main entry point's own (ec::check_batch and
// ec::decode_shape_supported), so the two accept and refuse the same batches,
// paged ones included.
#include <cstdio>
#include <mutex>

#include "ec_common.cuh"
#include "ec_internal.h"
#include "ec_kv.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (no libcuda link).
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    return fn;
}

// Device address of g_noalloc_scratch for each device ordinal, looked up once
// per CUDA context of that device (the caller has made the device current).
void* scratch_address(int device, cudaError_t* err) {
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    static CUcontext ctx_of[kMaxDevices] = {};
    CtxGetCurrentFn get_ctx = ctx_get_current();
    CUcontext ctx = nullptr;
    if (!get_ctx || get_ctx(&ctx) != CUDA_SUCCESS || !ctx) {
        *err = cudaErrorInvalidDeviceFunction;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[device] || ctx_of[device] != ctx) {
        void* p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (*err != cudaSuccess) return nullptr;
        addr[device] = p;
        ctx_of[device] = ctx;
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
    // the same checks, in the same order, as ec_decode_attention
    const int rc = ec::check_batch(b, "decode_attention_noalloc");
    if (rc != EC_OK) return rc;
    if (b->num_seqs == 0) return EC_OK;
    if (!q || !out) return reject(EC_ERR_INVALID_ARGUMENT, "q/out NULL");
    const uint32_t hkv = b->num_kv_heads;
    if (!ec::decode_shape_supported(num_heads, hkv, b->head_dim))
        return reject(EC_ERR_UNSUPPORTED, "shape outside the decode kernel's envelope");
    if (!aligned16(q) || !aligned16(out)) return reject(EC_ERR_MISALIGNED, "q/out not 16-byte aligned");

    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return reject(EC_ERR_CUDA, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return reject(EC_ERR_UNSUPPORTED, "device ordinal >= 64");

    const ec::DecodePlan plan = ec::plan_decode((int)b->num_seqs, (int)b->max_seq_len, sms,
                                                b->total_tokens_hint, (int)hkv, (int)num_heads,
                                                (int)b->head_dim);
    const size_t need = ec::decode_workspace_bytes(plan, (int)b->num_seqs, (int)num_heads,
                                                   (int)b->head_dim);
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
    a.head_dim = (int)b->head_dim;
    a.row_scales = b->scale_mode == EC_SCALE_ROW;
    a.mode = ec::kOut;
    e = ec::launch_decode(a, (int)hkv, plan, scratch, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return reject(EC_ERR_CUDA, cudaGetErrorString(e));
    return EC_OK;
}

}  // extern "C"
