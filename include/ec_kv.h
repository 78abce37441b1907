/*
 * ec_kv.h -- C ABI of the B200 (sm_100a) INT8 KV-cache path of echo-core.
 *
 * Three kernels sit behind this boundary:
 *   1. quantize-on-append: per-token symmetric int8 with an fp32 scale,
 *      bit-exact with the reference's quantize_per_token_symmetric;
 *   2. split-K grouped-query decode attention over the int8 cache;
 *   3. causal chunked-prefill attention over the same cache.
 *
 * Conventions
 *   - Every pointer argument documented "device" must be device memory of the
 *     current CUDA device.  Host pointers are accepted only where stated.
 *   - Calls are asynchronous on `stream` (a cudaStream_t; NULL = legacy
 *     default stream) unless documented otherwise.
 *   - Every entry point returns an ec_status.  No exception crosses the ABI.
 *     ec_last_error() gives a one-line reason for the last failure on the
 *     calling thread.
 *   - Kernels never trap.  A bad length/offset table entry, an append past a
 *     sequence's capacity or a device-side wait that runs out of time writes
 *     a non-zero code into the batch's error word (or the library's own word
 *     when none is given) and skips the offending work; ec_device_error()
 *     reads and clears it.
 *
 * Cache layout (identical to the reference's KVCacheLayer, include/kv_cache.h:7-18):
 *   codes   [slot][num_kv_heads][head_dim]  int8   (keys and values separately)
 *   scales  [slot][num_kv_heads]            fp32   (EC_SCALE_PER_HEAD)
 *           [slot]                          fp32   (EC_SCALE_ROW)
 */
#ifndef EC_KV_H
#define EC_KV_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EC_KV_ABI_VERSION 4  /* 4: ec_kv_layer is 64-byte aligned (64 bytes), as KVCacheLayer */

#if defined(__GNUC__)
#define EC_API __attribute__((visibility("default")))
#else
#define EC_API
#endif

typedef void* ec_stream_t; /* cudaStream_t */

typedef enum ec_status {
    EC_OK = 0,
    EC_ERR_INVALID_ARGUMENT = 1, /* null pointer, zero or inconsistent size     */
    EC_ERR_MISALIGNED = 2,       /* device pointer not 16-byte aligned          */
    EC_ERR_CAPACITY = 3,         /* append past max_seq_len / capacity          */
    EC_ERR_UNSUPPORTED = 4,      /* shape outside the kernels' envelope         */
    EC_ERR_CUDA = 5,             /* CUDA runtime or launch failure              */
    EC_ERR_WORKSPACE = 6,        /* workspace missing or too small              */
    EC_ERR_DEVICE_CHECK = 7      /* a kernel flagged bad input (see above)      */
} ec_status;

/* Where a token's scales live.  PER_HEAD is what the reference's decode loop
 * reads (src/inference.cpp:347,387) and what its scale buffer is sized for
 * (include/kv_cache.h:11-12).  ROW reproduces KVCache::append literally
 * (src/kv_cache.cpp:101,105): one scale over the whole token row, at [slot]. */
typedef enum ec_scale_mode { EC_SCALE_PER_HEAD = 0, EC_SCALE_ROW = 1 } ec_scale_mode;

/* Device-side error codes written into an error word. */
enum {
    EC_DEVERR_NONE = 0,
    EC_DEVERR_BAD_TABLE = 1,    /* offset/length/capacity entry out of range */
    EC_DEVERR_OVERFLOW = 2,     /* append would pass a sequence's capacity   */
    EC_DEVERR_TIMEOUT = 3,      /* a bounded device wait ran out             */
    EC_DEVERR_RANGE = 4         /* a value outside a kernel's supported range
                                   (no current kernel raises it)            */
};

EC_API int ec_abi_version(void);
EC_API const char* ec_status_string(int status);
EC_API const char* ec_last_error(void);

/* Reads (and resets to 0) the device error word `err_word` (device int32), or
 * the library's own word for the current device when err_word is NULL.
 * Synchronises `stream`.  Returns EC_OK and stores the code in *code. */
EC_API int ec_device_error(int32_t* err_word, ec_stream_t stream, int32_t* code);

/* ------------------------------------------------------------------------
 * Kernel-level entry points (device pointers)
 * ---------------------------------------------------------------------- */

/* Replaces quantize_per_token_symmetric (include/kernels/quant.h:8-14,
 * src/kernels/quant.cpp:18-98).  input [num_tokens*num_elements] fp32,
 * output int8 and scales [num_tokens] fp32, all device.  Bit-exact with the
 * reference for finite input, including the scalar tail for
 * num_elements % 8 != 0. */
EC_API int ec_quantize_per_token_symmetric(const float* input, int8_t* output, float* scales,
                                    uint32_t num_tokens, uint32_t num_elements,
                                    ec_stream_t stream);

/* Replaces fused_dequant_dot_int8 (include/kernels/quant.h:19-26,
 * src/kernels/quant.cpp:100-144): scores[pos] = dot(query, key_cache[pos]*scales[pos]). */
EC_API int ec_fused_dequant_dot_int8(const float* query, const int8_t* key_cache, const float* scales,
                              float* scores, uint32_t dim, uint32_t seq_len, ec_stream_t stream);

/* ------------------------------------------------------------------------
 * Single-sequence cache object: the reference's KVCache (include/kv_cache.h:21-48)
 * with its storage in HBM.
 * ---------------------------------------------------------------------- */

/* Field-for-field mirror of ModelConfig (include/config.h:6-24); a C++ caller
 * may pass its ModelConfig by reinterpret_cast (the C++ wrapper in
 * ec_kv_cache.hpp static_asserts the layout). */
typedef struct ec_model_config {
    uint32_t vocab_size;
    uint32_t hidden_dim;
    uint32_t num_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    uint32_t num_layers;
    uint32_t ffn_hidden_dim;
    uint32_t max_seq_len;
    int32_t ffn_type;
    int32_t norm_type;
    int32_t pos_encoding;
    bool use_kv_quantization;
} ec_model_config;

/* Mirror of KVCacheLayer (include/kv_cache.h:7-18), including its 64-byte
 * alignment (64 bytes in all); pointers are device pointers into the cache's
 * HBM slab. */
#if defined(__cplusplus)
#define EC_ALIGN64 alignas(64)
#elif defined(__GNUC__)
#define EC_ALIGN64 __attribute__((aligned(64)))
#else
#define EC_ALIGN64 _Alignas(64)
#endif
typedef struct EC_ALIGN64 ec_kv_layer {
    int8_t* keys_int8;
    int8_t* values_int8;
    float* key_scales;
    float* val_scales;
    float* keys_fp32;
    float* values_fp32;
    uint32_t seq_len;
} ec_kv_layer;

typedef struct ec_kv_cache ec_kv_cache;

/* KVCache::KVCache (src/kv_cache.cpp:6-72): one zeroed device slab on the
 * current device, partitioned per layer exactly as the reference partitions
 * its host slab.  scale_mode selects PER_HEAD (default) or ROW scales. */
EC_API int ec_kv_cache_create(const ec_model_config* config, int scale_mode, ec_kv_cache** out);
/* KVCache::~KVCache (src/kv_cache.cpp:74-77).  Synchronises the device. */
EC_API void ec_kv_cache_destroy(ec_kv_cache* cache);
/* KVCache::layer (src/kv_cache.cpp:79-87). */
EC_API int ec_kv_cache_layer(const ec_kv_cache* cache, uint32_t layer_idx, ec_kv_layer* out);
/* KVCache::append (src/kv_cache.cpp:89-113): quantizes one token's K and V
 * ([num_kv_heads*head_dim] fp32 each, device) into the next slot of layer
 * layer_idx and advances that layer's length.  EC_ERR_CAPACITY instead of the
 * reference's assert when the layer is full (src/kv_cache.cpp:91). */
EC_API int ec_kv_cache_append(ec_kv_cache* cache, uint32_t layer_idx, const float* k_proj,
                       const float* v_proj, ec_stream_t stream);
/* KVCache::seq_len (src/kv_cache.cpp:115-118): layer 0's length. */
EC_API uint32_t ec_kv_cache_seq_len(const ec_kv_cache* cache);
/* KVCache::reset (src/kv_cache.cpp:120-124): zeroes every layer's length. */
EC_API int ec_kv_cache_reset(ec_kv_cache* cache);
/* The KV part of InferenceEngine::attention (src/inference.cpp:321-406) for
 * one decode step of layer layer_idx over that layer's own length:
 * q [num_heads*head_dim] fp32 (unscaled; softmax_scale is applied to q first,
 * as src/inference.cpp:322-325 does), out [num_heads*head_dim] fp32, both
 * device.  Q head h reads KV head h % num_kv_heads (src/inference.cpp:335).
 * A layer of length 0 gives zeros (src/inference.cpp:331). */
EC_API int ec_kv_cache_attention(ec_kv_cache* cache, uint32_t layer_idx, const float* q, float* out,
                          float softmax_scale, ec_stream_t stream);
/* One token of one layer of InferenceEngine::attention minus its weight
 * matvecs (src/inference.cpp:321-414): attention of q over the layer's cached
 * tokens (the cache before this token, as :330-392 read it), then the append
 * of this token's k/v (:414).  q [num_heads*head_dim], k_proj / v_proj
 * [num_kv_heads*head_dim], attn_out [num_heads*head_dim]: device pointers,
 * asynchronous on the stream.  EC_ERR_CAPACITY (and nothing done) when the
 * layer is full. */
EC_API int ec_kv_cache_step(ec_kv_cache* cache, uint32_t layer_idx, const float* q,
                            const float* k_proj, const float* v_proj, float* attn_out,
                            float softmax_scale, ec_stream_t stream);
/* ec_kv_cache_step for an engine whose buffers live in host memory, as the
 * reference's q_proj_ / k_proj_ / v_proj_ / attn_out_ do (include/inference.h:
 * 21-27): copies q/k/v to a device staging area owned by the cache, runs the
 * step and copies attn_out back.  Synchronous. */
EC_API int ec_kv_cache_step_host(ec_kv_cache* cache, uint32_t layer_idx, const float* q,
                                 const float* k_proj, const float* v_proj, float* attn_out,
                                 float softmax_scale);

/* Cache snapshots (persistence; the reference keeps its cache only in
 * process memory).  ec_kv_cache_snapshot writes the cache's contents into a
 * host buffer of ec_kv_cache_snapshot_size() bytes: a header (magic
 * "ECKVSNAP", version, shape, scale mode, per-layer lengths) and, per layer,
 * the used prefix of each buffer.  ec_kv_cache_restore loads such an image
 * into a cache of the same shape and mode, replacing its contents and
 * lengths; a mismatched or truncated image gives EC_ERR_INVALID_ARGUMENT (or
 * EC_ERR_CAPACITY for a layer longer than max_seq_len) and changes nothing.
 * Both synchronise the device. */
EC_API size_t ec_kv_cache_snapshot_size(const ec_kv_cache* cache);
EC_API int ec_kv_cache_snapshot(const ec_kv_cache* cache, void* host, size_t bytes);
EC_API int ec_kv_cache_restore(ec_kv_cache* cache, const void* host, size_t bytes);

/* ------------------------------------------------------------------------
 * Batched ragged cache: per-sequence contiguous slabs inside caller-owned
 * device buffers, addressed through an int32 offset / capacity / length
 * table.  Sequence s owns slots [seq_offset[s], seq_offset[s]+seq_capacity[s])
 * and holds seq_len[s] tokens.
 * ---------------------------------------------------------------------- */
typedef struct ec_kv_batch {
    int8_t* keys;                /* [total_slots][num_kv_heads][head_dim]          */
    int8_t* values;              /* same                                           */
    float* key_scales;           /* [total_slots][num_kv_heads] or [total_slots]   */
    float* val_scales;           /* same                                           */
    const int32_t* seq_offset;   /* [num_seqs] first slot of each sequence         */
    const int32_t* seq_capacity; /* [num_seqs] slots owned by each sequence        */
    int32_t* seq_len;            /* [num_seqs] cached tokens (append advances it)  */
    int32_t* error_word;         /* device int32 or NULL (library word)            */
    uint64_t total_slots;        /* slots in keys/values (bounds every table entry)*/
    uint32_t num_seqs;
    uint32_t num_kv_heads;
    uint32_t head_dim;
    int32_t scale_mode;          /* ec_scale_mode                                  */
    uint32_t max_seq_len;        /* host-side bound on every seq_len (sizes grids) */
    /* Paged layout (optional; all zero = contiguous slabs).  With page_table
     * set, seq_offset is ignored (it may be NULL) and token t of sequence s
     * lives in slot page_table[s*max_pages + t/page_tokens]*page_tokens +
     * t%page_tokens; seq_capacity[s] is the tokens its pages hold (at most
     * max_pages*page_tokens).  Pages are taken from a pool of total_slots
     * slots; a sequence grows past any initial size by receiving more pages
     * (the reference's cache stops at max_seq_len, src/main.cpp:304).  A page
     * id outside the pool is flagged EC_DEVERR_BAD_TABLE, never dereferenced. */
    const int32_t* page_table;   /* [num_seqs][max_pages] device int32            */
    uint32_t page_tokens;        /* power of two, multiple of 128                  */
    uint32_t max_pages;          /* row stride of page_table                       */
    /* Optional host-side estimate of the batch's cached tokens (the sum of
     * seq_len) at the decode, 0 if unknown.  A ragged batch whose sequences
     * are mostly shorter than max_seq_len gets a split-K plan sized for its
     * actual tokens; size the workspace with ec_decode_workspace_size_batch.
     * The estimate only steers the plan: results do not depend on it. */
    uint64_t total_tokens_hint;
} ec_kv_batch;

/* Batched KVCache::append: quantizes tokens_per_seq new tokens of every
 * sequence, k/v [num_seqs][tokens_per_seq][num_kv_heads*head_dim] fp32 device,
 * into slots seq_offset[s]+seq_len[s]+i, then advances seq_len[s].  A
 * sequence that would pass its capacity is skipped whole and flags
 * EC_DEVERR_OVERFLOW. */
EC_API int ec_kv_batch_append(const ec_kv_batch* batch, const float* k, const float* v,
                       uint32_t tokens_per_seq, ec_stream_t stream);

/* K pre-processing of echo-core-zig before the cache append
 * (src/inference/engine.zig:544-559): a per-head RMS norm with an fp16 weight
 * (:521-532; rms = sqrt(sum x^2 / d + 1e-6) summed in dimension order,
 * x = x * (1/rms) * w), then rotary position embedding over interleaved pairs
 * (:466-518; angle = pos * freq_i, freq_i = 1 / rope_base^(i/d); (x0, x1) ->
 * (x0 cos - x1 sin, x0 sin + x1 cos)), d = head_dim (128 or 256).  Every
 * product and sum is rounded on its own in that order; cos and sin are the
 * fp32 roundings of their double-precision values.  rope_base <= 0 skips the
 * rotation, a NULL norm_weight (device, fp16 [head_dim], 8-byte aligned)
 * skips the norm. */
typedef struct ec_rope_desc {
    float rope_base;                /* 10000 in echo-core-zig */
    const uint16_t* norm_weight;
} ec_rope_desc;

/* ec_kv_batch_append with K normed and rotated at each new token's position
 * (its sequence's length before the call, plus its index in the chunk) before
 * quantization; V as ec_kv_batch_append. */
EC_API int ec_kv_batch_append_rope(const ec_kv_batch* batch, const float* k_new,
                                   const float* v_new, uint32_t tokens_per_seq,
                                   const ec_rope_desc* k_desc, ec_stream_t stream);
/* The same norm and rotation in place on rows of num_heads * head_dim floats
 * (the queries), row r at position positions[r] (device int32; may be NULL
 * when rope_base <= 0). */
EC_API int ec_rope_rows(float* x, uint32_t rows, uint32_t num_heads, uint32_t head_dim,
                        const int32_t* positions, const ec_rope_desc* desc, ec_stream_t stream);

/* Workspace (device bytes) ec_decode_attention needs for this batch shape on
 * the current device: the largest over the num_kv_heads values the kernels
 * cover for num_heads (the split plan depends on num_kv_heads, which this
 * query does not take); ec_decode_workspace_size_batch gives the exact size. */
EC_API size_t ec_decode_workspace_size(uint32_t num_seqs, uint32_t num_heads, uint32_t head_dim,
                                uint32_t max_seq_len);
/* The same for a batch descriptor, taking its total_tokens_hint into account
 * (equals ec_decode_workspace_size when the hint is 0). */
EC_API size_t ec_decode_workspace_size_batch(const ec_kv_batch* batch, uint32_t num_heads);

/* Decode attention for every sequence of the batch (the loop of
 * src/inference.cpp:321-392 per sequence):
 * q [num_seqs][num_heads][head_dim] fp32, out same shape fp32, device.
 * Supported envelope: head_dim 128 or 256, num_kv_heads 1, 2, 4 or 8, and
 * num_heads any multiple of num_kv_heads up to 32 times it (query head h
 * reads KV head h % num_kv_heads, src/inference.cpp:335). */
EC_API int ec_decode_attention(const ec_kv_batch* batch, const float* q, float* out,
                        uint32_t num_heads, float softmax_scale, void* workspace,
                        size_t workspace_bytes, ec_stream_t stream);

/* Context parallelism.  ec_decode_attention_partial computes, for every
 * (sequence, head), the unnormalised partial state over this batch's tokens:
 *   part_o  [num_seqs][num_heads][head_dim]  sum_t 2^(s_t*log2e - m) * v_t
 *   part_ml [num_seqs][num_heads][2]         (m, l): m = max_t s_t*log2e,
 *                                            l = sum_t 2^(s_t*log2e - m)
 * (m = -inf, l = 0, o = 0 for an empty shard).  ec_lse_combine merges
 * num_parts such states, stacked [num_parts][...] in a fixed part order, into
 * the normalised output [num_seqs][num_heads][head_dim]. */
EC_API int ec_decode_attention_partial(const ec_kv_batch* batch, const float* q, float* part_o,
                                float* part_ml, uint32_t num_heads, float softmax_scale,
                                void* workspace, size_t workspace_bytes, ec_stream_t stream);
EC_API int ec_lse_combine(const float* part_o, const float* part_ml, uint32_t num_parts,
                   uint32_t num_seqs, uint32_t num_heads, uint32_t head_dim, float* out,
                   ec_stream_t stream);

/* Context parallelism with the exchange and the merge in one kernel over
 * NVLink peer memory, instead of an all-gather plus ec_lse_combine.  One
 * process per GPU.  Each rank creates a comm (a receive buffer on its
 * current device, double-buffered by step parity) and gets its 64-byte CUDA
 * IPC handle; the ranks exchange handles (any host channel, e.g. a
 * torch.distributed all-gather of the bytes, in rank order) and open them.
 * Per step every rank calls ec_cp_exchange_combine with its partial state
 * from ec_decode_attention_partial and the same epoch (1, 2, 3, ...): its
 * partial is stored into every rank's buffer, and the merged output (rank
 * order, as ec_lse_combine) is written once every rank's partial for that
 * epoch has arrived.  Waits are bounded (about 1 s); a rank that never
 * arrives makes the others flag EC_DEVERR_TIMEOUT and write zeros.
 * epoch 0 instead keeps the epochs in device memory (one per sequence and
 * head) and advances them inside the kernel, so the call can be captured into
 * a CUDA graph and replayed; a comm uses caller epochs or device epochs, not
 * both
 * (EC_ERR_INVALID_ARGUMENT on a switch).
 * world <= 8; num_seqs * num_heads <= 2368.  A CTA waits only for the words
 * of the same CTA (sequence, head, dims split) on the other ranks. */
#define EC_CP_HANDLE_BYTES 64
typedef struct ec_cp_comm ec_cp_comm;
EC_API int ec_cp_comm_create(uint32_t world, uint32_t rank, uint32_t num_seqs,
                             uint32_t num_heads, ec_cp_comm** out, void* ipc_handle);
EC_API int ec_cp_comm_open(ec_cp_comm* comm, const void* handles);
EC_API int ec_cp_exchange_combine(ec_cp_comm* comm, const float* part_o, const float* part_ml,
                                  uint32_t epoch, float* out, ec_stream_t stream);
EC_API void ec_cp_comm_destroy(ec_cp_comm* comm);

/* One context-parallel decode step in two launches per rank: the decode
 * kernel over this rank's slice (batch: the comm's num_seqs sequences, each
 * holding this rank's contiguous share of its tokens), leaving its split-K
 * chunk partials in `workspace`, then the exchange kernel, which merges those
 * chunks into this rank's (m, l, O), stores it into every rank's buffer and
 * merges the world's states in rank order into out [num_seqs][num_heads][128]
 * -- the output ec_decode_attention_partial + ec_cp_exchange_combine give,
 * without their separate chunk-merge launch.  head_dim 128; num_heads must
 * be the comm's; epoch as ec_cp_exchange_combine (0: device epochs).
 * workspace: device, ec_cp_decode_workspace_size bytes. */
EC_API size_t ec_cp_decode_workspace_size(const ec_kv_batch* batch, uint32_t num_heads);
EC_API int ec_cp_decode_exchange(ec_cp_comm* comm, const ec_kv_batch* batch, const float* q,
                                 uint32_t num_heads, float softmax_scale, void* workspace,
                                 size_t workspace_bytes, uint32_t epoch, float* out,
                                 ec_stream_t stream);

/* Chunked-prefill attention.  The reference has no chunked prefill: it feeds
 * a prompt one token at a time (src/main.cpp:404-405), each token running the
 * decode loop of src/inference.cpp:321-392 over the cache as it stands after
 * that token's append.  This computes the same attention for a whole chunk at
 * once.  For every sequence the chunk is the last n_new cached tokens (slots
 * [len - n_new, len) after ec_kv_batch_append), and query row i attends to
 * slots [0, len - n_new + i].  q [num_seqs][n_new][num_heads][128] fp32 is cast
 * to bf16 on load (bf16-cast queries); out has the same shape, fp32.  Runs on
 * the tcgen05 tensor cores; head_dim 128, any num_kv_heads dividing num_heads.
 * Any finite v-scale is in range: p' = p * v_scale is carried in f16 under a
 * power of two per query row, set from the largest v-scale of the row's
 * causal range. */
EC_API int ec_prefill_attention(const ec_kv_batch* batch, const float* q, float* out,
                                uint32_t n_new, uint32_t num_heads, float softmax_scale,
                                ec_stream_t stream);

/* No counterpart in the reference (which has no device memory at all): this
 * entry point exists for callers that cannot allocate device memory when they
 * run decode -- code running where cudaMalloc is not allowed (a host callback
 * or hook, where a blocking, device-synchronising allocation would stall or
 * deadlock), or a runtime that carved up its memory once at start-up and may
 * not grow it.  Same inputs, outputs and results as ec_decode_attention, but
 * the split-K workspace is a fixed 16 MiB array built into the library, so
 * the caller passes none and no allocation happens.  Every GPU that loads the
 * library holds that array until the process exits.  A batch whose workspace
 * would exceed 16 MiB (ec_decode_workspace_size) is rejected with
 * EC_ERR_WORKSPACE and a message in ec_last_error(); nothing is launched.
 * The first call on each device looks up the array's address, so make it
 * before any stream capture.  All calls share the array: calls whose kernels
 * can overlap on the GPU (different streams, no ordering between them) race
 * and corrupt each other's results. */
EC_API int ec_decode_attention_noalloc(const ec_kv_batch* batch, const float* q, float* out,
                                       uint32_t num_heads, float softmax_scale,
                                       ec_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* EC_KV_H */
