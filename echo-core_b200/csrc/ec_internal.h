// ec_internal.h -- launch arguments and launchers shared by the .cu files.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "ec_kv.h"

namespace ec {

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device
// ordinal (one bit each in `done`; devices past 63 set it on every call).
// Safe to call from several host threads: a repeated set is harmless.
inline cudaError_t ensure_smem_limit(const void* kernel, int bytes,
                                     std::atomic<unsigned long long>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_release);
    return e;
}

// Launch with programmatic stream serialization: the kernel's CTAs may be
// scheduled while the previous kernel on the stream drains; the kernel itself
// waits for it (pdl_wait) before touching global memory.
template <typename... P, typename... A>
inline cudaError_t launch_pdl(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, A&&... args) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
}

// Optional paged layout of a batch (device page table; null: contiguous slabs
// addressed by seq_offset).  Page size 1 << shift tokens, a multiple of 128.
struct PageMap {
    const int32_t* table;   // [num_seqs][max_pages] page ids into the slot pool
    int shift;
    int max_pages;
};

inline PageMap page_map_of(const ec_kv_batch* b) {
    PageMap m{nullptr, 0, 0};
    if (b->page_table) {
        int sh = 0;
        while ((1u << sh) < b->page_tokens) ++sh;
        m = PageMap{b->page_table, sh, (int)b->max_pages};
    }
    return m;
}

constexpr int kMaxHeadDim = 256;   // head_dim 128 or 256 (append, decode)

struct AppendArgs {
    const float* k;
    const float* v;
    int8_t* keys;
    int8_t* values;
    float* key_scales;
    float* val_scales;
    const int32_t* seq_offset;    // null: host_offset for every sequence
    const int32_t* seq_capacity;  // null: host_capacity
    int32_t* seq_len;             // null: host_length, and no length update
    int32_t host_offset, host_capacity, host_length;
    int32_t* err;
    uint64_t total_slots;
    int num_seqs;
    int n_new;
    int head_dim;                 // 128 or 256
    PageMap pages;
    // K pre-processing of echo-core-zig (src/inference/engine.zig): per-head
    // RMS norm with an fp16 weight (:521-532), then RoPE (:466-518).  Used by
    // the rope variant of the append kernel only.
    const uint16_t* k_norm_w;     // fp16 [head_dim] or null: no norm
    int rope;                     // 0: no rotation
    float inv_freq[kMaxHeadDim / 2];   // 1 / base^(2i/head_dim), computed on the host
};

struct DecodeArgs {
    const int8_t* keys;       // [total_slots][num_kv_heads][head_dim]
    const int8_t* values;
    const float* key_scales;
    const float* val_scales;
    const int32_t* seq_offset;
    const int32_t* seq_capacity;
    const int32_t* seq_len;
    int32_t host_offset, host_capacity, host_length;
    int32_t* err;
    uint64_t total_slots;
    const float* q;       // [num_seqs][num_heads][head_dim]
    float* out;           // final output (normalised) when mode == kOut
    float* out_ml;        // (m, l) per (seq, head) when mode == kPartial
    float* part_o;        // [num_seqs*max_chunks][num_heads][head_dim]
    float* part_ml;       // [num_seqs*max_chunks][num_heads][2]
    float q_mul;          // softmax scale (applied to q first, as the reference does)
    int num_seqs;
    int num_heads;
    int num_kv_heads;     // query head h reads KV head h % num_kv_heads
    int head_dim;         // 128 or 256
    int sk_ctas;          // > 0: stream-K grid of this many CTAs per head block (0: chunked)
    int32_t* sk_prefix;   // stream-K: [num_seqs + 1] tiles before each sequence, then the total
    int max_chunks;
    int chunk_tokens;
    int row_scales;       // 1: EC_SCALE_ROW
    int mode;             // kOut or kPartial
    PageMap pages;
};

// kOut: normalised output; kPartial: (m, l, O) per (sequence, head);
// kChunks: every chunk's (m, l, O) left in the workspace (unsplit plans too),
// for the exchange kernel to merge.
enum { kOut = 0, kPartial = 1, kChunks = 2 };

cudaError_t launch_quantize_rows(const float* in, int8_t* out, float* scales, uint32_t rows,
                                 uint32_t n, cudaStream_t st);
cudaError_t launch_append(const AppendArgs& a, int num_kv_heads, bool row_mode, cudaStream_t st);
cudaError_t launch_append_rope(const AppendArgs& a, int num_kv_heads, bool row_mode, cudaStream_t st);
// In-place per-head RMS norm (fp16 weight, may be null) and RoPE of rows of
// num_heads * head_dim floats (head_dim 128 or 256), row r at position
// positions[r]; inv_freq has head_dim / 2 entries.
cudaError_t launch_rope_rows(float* x, uint32_t rows, uint32_t num_heads, uint32_t head_dim,
                             const int32_t* positions, const uint16_t* norm_w, int rope,
                             const float* inv_freq, cudaStream_t st);
cudaError_t launch_fused_dequant_dot(const float* q, const int8_t* k, const float* s, float* out,
                                     uint32_t dim, uint32_t seq_len, cudaStream_t st);

// Split policy shared by the workspace query and the launch.
// Chunked plan (sk_ctas == 0): max_chunks chunks of chunk_tokens tokens per
// sequence.  Stream-K plan (sk_ctas > 0): sk_ctas CTAs per head block share
// the batch's tiles evenly; chunk_tokens then only bounds the lengths.
struct DecodePlan {
    int chunk_tokens;
    int max_chunks;
    int sk_ctas;
};
// The compiled decode kernel for a shape: hc KV heads per CTA, qw quads of
// query heads per KV head, scw = num_kv_heads, dv = head_dim / 128, and its
// resident CTAs per SM.  hc == 0: no kernel covers the shape.
struct DecodeVariant {
    int hc, qw, scw, dv, ctas_per_sm;
};
DecodeVariant decode_variant(int num_kv_heads, int group, int head_dim);
// total_tokens: host estimate of the batch's cached tokens (0: unknown, every
// sequence is assumed to be max_seq_len long).  The kernel variant of
// (num_kv_heads, num_heads, head_dim) sets how many CTAs fit on the GPU at once.
// allow_stream false: a chunked plan (the context-parallel exchange merges
// a sequence's chunks itself).
DecodePlan plan_decode(int num_seqs, int max_seq_len, int num_sms, uint64_t total_tokens,
                       int num_kv_heads, int num_heads, int head_dim, bool allow_stream = true);
size_t decode_workspace_bytes(const DecodePlan& p, int num_seqs, int num_heads, int head_dim);
// Returns cudaErrorInvalidValue for a shape outside the envelope.
cudaError_t launch_decode(DecodeArgs a, int num_kv_heads, const DecodePlan& plan, void* ws,
                          cudaStream_t st);
// Tensor map over [total_slots][hkv * 128] int8 codes with a 128-byte x
// box_rows-token box, 128-byte swizzle.
cudaError_t make_f32_row_map(CUtensorMap* m, const float* base, int hkv, uint64_t rows,
                             int box_rows);
cudaError_t make_code_map(CUtensorMap* m, const int8_t* base, int hkv, uint64_t total_slots,
                          int box_rows);

struct PrefillArgs {
    const int8_t* keys;
    const int8_t* values;
    const float* key_scales;
    const float* val_scales;
    const int32_t* seq_offset;
    const int32_t* seq_capacity;
    const int32_t* seq_len;   // lengths after the chunk's append
    int32_t* err;
    uint64_t total_slots;
    const float* q;           // [num_seqs][n_new][num_heads][128] fp32 (cast to bf16 on load)
    float* out;               // same shape, fp32
    int num_seqs, num_heads, num_kv_heads, n_new, row_scales;
    float qk_mul;             // softmax scale * log2(e)
    PageMap pages;
};
cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t st);
// Records `msg` as the calling thread's ec_last_error() text; returns status.
int set_last_error(int status, const char* msg);
// Host-side validation of a batch descriptor shared by every entry point that
// takes one: null buffers, the paged-layout fields (page_tokens a power of two
// >= 128, max_pages > 0, total_slots a multiple of page_tokens), scale mode,
// 16-byte alignment and the int32 index limits.  EC_OK, or a status with
// ec_last_error() set to "<who>: <reason>".
int check_batch(const ec_kv_batch* b, const char* who);
// The (num_heads, num_kv_heads, head_dim) shapes the int8 decode kernel covers.
bool decode_shape_supported(uint32_t num_heads, uint32_t num_kv_heads, uint32_t head_dim);
cudaError_t launch_lse_combine(const float* part_o, const float* part_ml, int num_parts,
                               int num_seqs, int num_heads, int head_dim, float* out,
                               cudaStream_t st);

// Context-parallel exchange + merge over peer memory (cp_exchange.cu).
// CTAs per (sequence, head) of a split-K merge (the decode's merge kernel and
// the context-parallel exchange), each taking a slice of the head's dims:
// more when the batch has few pairs (one long sequence: 16 pairs on 148 SMs).
int merge_splits(int pairs);

constexpr int kCpMaxWorld = 8;
constexpr int kCpSplitMax = 8;       // dims splits of a (sequence, head) in the exchange kernel
struct CpExchangeArgs {
    float* peer_base[kCpMaxWorld];   // every rank's receive buffer, this rank's own included
    const float* part_o;             // this rank's partial O [num_seqs][num_heads][128]
    const float* part_ml;            // and (m, l) [num_seqs][num_heads][2]
    float* out;                      // merged output [num_seqs][num_heads][128]
    int32_t* err;
    int world, rank, num_seqs, num_heads;
    uint32_t epoch;
    uint32_t* epoch_dev;             // non-null: [num_seqs][num_heads][kCpSplitMax] device epochs
    // max_chunks > 0: part_o / part_ml are the decode kernel's split-K chunk
    // partials of this rank's slice ([num_seqs*max_chunks][num_heads][..]),
    // merged in the exchange kernel; sequence s has ceil(seq_len[s] /
    // chunk_tokens) of them
    const int32_t* seq_len;
    int chunk_tokens, max_chunks;
};
size_t cp_exchange_buffer_bytes(int world, int num_seqs, int num_heads);
cudaError_t launch_cp_exchange(const CpExchangeArgs& a, cudaStream_t st);

// Decode attention over the fp32 cache mode (use_kv_quantization = false):
// keys / values [len][num_kv_heads][128] fp32, q [num_heads][128] unscaled,
// out [num_heads][128].  Split-K over chunks of at least kF32ChunkTokens
// tokens; the workspace holds (m, l, O) per (chunk, head).
constexpr int kF32ChunkTokens = 256;   // minimum tokens per CTA
int f32_decode_chunks(int len, int num_kv_heads);
size_t f32_decode_workspace_bytes(int max_len, int num_kv_heads, int num_heads);
cudaError_t launch_decode_f32(const float* keys, const float* values, int num_kv_heads,
                              int num_heads, int len, const float* q, float q_mul, float* out,
                              void* ws, cudaStream_t st);

}  // namespace ec
