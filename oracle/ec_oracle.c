/*
 * ec_oracle.c -- CPU restatement of echo-core's INT8 KV-cache hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, the
 * smoke check and the bench's CPU-baseline leg compare the CUDA kernels
 * against.  Nothing in the shipped library links, loads or calls it.
 *
 * Each function restates one piece of the reference (void0x14/echo-core)
 * operation for operation; citations are path:line inside that project.
 * The restatement is pinned two ways (see tests/test_oracle.py):
 *   - against the reference's own known-answer tests
 *     (src/kernels/quant.cpp:403-521, src/kv_cache.cpp:158-300), and
 *   - against the reference's own compiled code (oracle/_ref, built from the
 *     reference sources by oracle/Makefile) on seeded inputs, with the
 *     outputs committed as golden fixtures under tests/golden/.
 *
 * Build flags follow the reference's CMakeLists.txt:9-10,21
 * (-O3 -mavx2 -mfma -mf16c) so that floating-point contraction matches.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

enum { ORACLE_SCALE_PER_HEAD = 0, ORACLE_SCALE_ROW = 1 };

/* x86 cvtps2dq / cvttss2si return INT32_MIN for NaN and out-of-range input. */
static int32_t x86_cvt_i32(float v) {
    if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
    return (int32_t)v;
}

static int8_t sat_i8(int32_t v) {           /* packs_epi32 then packs_epi16 */
    if (v > 127) return 127;
    if (v < -128) return -128;
    return (int8_t)v;
}

/*
 * quantize_per_token_symmetric -- src/kernels/quant.cpp:18-98.
 *   pass 1 (:29-60): row absmax (sign-mask AND + max); scalar tail (:56-59).
 *   scale (:63): max_abs / 127.0f, or 1.0f for an all-zero row.
 *   pass 2, 8-wide body (:70-88): q = sat8(RNE(x * (1.0f/scale))).
 *   pass 2, scalar tail (:91-96): q = clamp(+-127, round_half_away(x / scale)).
 */
void oracle_quantize_per_token_symmetric(const float* input, int8_t* output,
                                         float* scales, uint32_t num_tokens,
                                         uint32_t num_elements) {
    for (uint32_t t = 0; t < num_tokens; ++t) {
        const float* row = input + (size_t)t * num_elements;
        int8_t* out = output + (size_t)t * num_elements;
        const uint32_t vec_end = num_elements - (num_elements % 8u);

        /* 8 lanes of MAXPS(acc, |x|): MAXPS returns the second operand
         * when the compare fails, so a NaN element is carried forward. */
        float lane_max[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (uint32_t i = 0; i < vec_end; ++i) {
            float a = fabsf(row[i]);
            float* m = &lane_max[i % 8u];
            *m = (*m > a) ? *m : a;
        }
        /* horizontal max (:49-53): max(lo,hi) then movehl then shuffle, each
         * MAXPS(a, b) = a > b ? a : b */
        float m4[4];
        for (int k = 0; k < 4; ++k) m4[k] = lane_max[k] > lane_max[k + 4] ? lane_max[k] : lane_max[k + 4];
        float m2[2];
        for (int k = 0; k < 2; ++k) m2[k] = m4[k] > m4[k + 2] ? m4[k] : m4[k + 2];
        float max_abs = m2[0] > m2[1] ? m2[0] : m2[1];
        for (uint32_t i = vec_end; i < num_elements; ++i) {
            float a = fabsf(row[i]);
            if (a > max_abs) max_abs = a;
        }

        const float scale = (max_abs > 0.0f) ? (max_abs / 127.0f) : 1.0f;
        scales[t] = scale;
        const float inv = 1.0f / scale;

        for (uint32_t i = 0; i < vec_end; ++i) {
            float v = nearbyintf(row[i] * inv);     /* round-to-nearest-even */
            out[i] = sat_i8(x86_cvt_i32(v));
        }
        for (uint32_t i = vec_end; i < num_elements; ++i) {
            int32_t v = x86_cvt_i32(roundf(row[i] / scale));
            if (v > 127) v = 127;
            if (v < -127) v = -127;
            out[i] = (int8_t)v;
        }
    }
}

/*
 * fused_dequant_dot_int8 -- src/kernels/quant.cpp:100-144.
 * 8 accumulator lanes, 16 elements per step (two FMAs of dequantised K
 * against q), horizontal sum (hsum256_ps, :9-16), scalar tail (:138-140).
 */
void oracle_fused_dequant_dot_int8(const float* query, const int8_t* key_cache,
                                   const float* scales, float* scores,
                                   uint32_t dim, uint32_t seq_len) {
    for (uint32_t pos = 0; pos < seq_len; ++pos) {
        const int8_t* key = key_cache + (size_t)pos * dim;
        const float s = scales[pos];
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        uint32_t k = 0;
        for (; k + 16 <= dim; k += 16) {
            for (int j = 0; j < 8; ++j) acc[j] = fmaf((float)key[k + j] * s, query[k + j], acc[j]);
            for (int j = 0; j < 8; ++j) acc[j] = fmaf((float)key[k + 8 + j] * s, query[k + 8 + j], acc[j]);
        }
        /* hsum256_ps: (hi + lo) then two hadds */
        float h4[4];
        for (int j = 0; j < 4; ++j) h4[j] = acc[j + 4] + acc[j];
        float a0 = h4[0] + h4[1], a1 = h4[2] + h4[3];
        float score = a0 + a1;
        /* The reference build keeps this tail uncontracted: the product is
         * rounded before the add (verified against oracle/_ref). */
        for (; k < dim; ++k) {
            volatile float prod = (float)key[k] * scales[pos] * query[k];
            score += prod;
        }
        scores[pos] = score;
    }
}

/*
 * KVCache::append for the int8 cache -- src/kv_cache.cpp:89-113.
 * ROW mode is the literal reference (:101,:105): one scale over the whole
 * num_kv_heads*head_dim token row, stored at scales[pos].
 * PER_HEAD mode quantizes each kv head's head_dim slice with its own scale,
 * stored at scales[pos*num_kv_heads + head], which is the index the decode
 * loop reads (src/inference.cpp:347,387) and the size the buffer has
 * (include/kv_cache.h:11-12).
 */
void oracle_kv_append_token(int8_t* keys, int8_t* values, float* key_scales,
                            float* val_scales, uint32_t pos, const float* k_proj,
                            const float* v_proj, uint32_t num_kv_heads,
                            uint32_t head_dim, int scale_mode) {
    const uint32_t row = num_kv_heads * head_dim;
    if (scale_mode == ORACLE_SCALE_ROW) {
        oracle_quantize_per_token_symmetric(k_proj, keys + (size_t)pos * row, &key_scales[pos], 1, row);
        oracle_quantize_per_token_symmetric(v_proj, values + (size_t)pos * row, &val_scales[pos], 1, row);
    } else {
        oracle_quantize_per_token_symmetric(k_proj, keys + (size_t)pos * row,
                                            &key_scales[(size_t)pos * num_kv_heads], num_kv_heads, head_dim);
        oracle_quantize_per_token_symmetric(v_proj, values + (size_t)pos * row,
                                            &val_scales[(size_t)pos * num_kv_heads], num_kv_heads, head_dim);
    }
}

/*
 * Decode attention over the int8 cache -- src/inference.cpp:321-392.
 *   q *= 1/sqrt(d) element-wise (:322-325; here `softmax_scale`).
 *   per Q head h: kv_head = h % num_kv_heads (:335);
 *   score[pos] = sum_d q[d] * float(k8[d]) * k_scale (:343-352);
 *   softmax: max, exp(s - max) with running sum, multiply by 1/sum (:367-379);
 *   out[d] = sum_pos p[pos] * (float(v8[d]) * v_scale) (:383-392).
 * kv_len replaces kv_cache_->seq_len() (:307), which is layer 0's count;
 * callers pass the attended layer's own length.
 * Scale index is pos*num_kv_heads + kv_head (PER_HEAD, :347,:387) or pos
 * (ROW: the scale KVCache::append writes, :101).
 * `q` is not modified; `scores` is caller scratch of kv_len floats.
 */
void oracle_decode_attention(const int8_t* keys, const int8_t* values,
                             const float* key_scales, const float* val_scales,
                             uint32_t kv_len, const float* q, float* out,
                             uint32_t num_heads, uint32_t num_kv_heads,
                             uint32_t head_dim, float softmax_scale,
                             int scale_mode, float* scores) {
    const uint32_t kv_dim = num_kv_heads * head_dim;
    float* qs = (float*)malloc(sizeof(float) * (size_t)num_heads * head_dim);
    for (uint32_t i = 0; i < num_heads * head_dim; ++i) qs[i] = q[i] * softmax_scale;
    memset(out, 0, sizeof(float) * (size_t)num_heads * head_dim);
    if (kv_len == 0) { free(qs); return; }

    for (uint32_t h = 0; h < num_heads; ++h) {
        const uint32_t kv_head = h % num_kv_heads;
        const float* head_q = qs + (size_t)h * head_dim;
        for (uint32_t pos = 0; pos < kv_len; ++pos) {
            float score = 0.0f;
            const int8_t* key_head = keys + (size_t)pos * kv_dim + (size_t)kv_head * head_dim;
            const float k_scale = scale_mode == ORACLE_SCALE_ROW
                                      ? key_scales[pos]
                                      : key_scales[(size_t)pos * num_kv_heads + kv_head];
            for (uint32_t d = 0; d < head_dim; ++d)
                score += head_q[d] * (float)key_head[d] * k_scale;
            scores[pos] = score;
        }
        float max_score = scores[0];
        for (uint32_t i = 1; i < kv_len; ++i)
            if (scores[i] > max_score) max_score = scores[i];
        float sum = 0.0f;
        for (uint32_t i = 0; i < kv_len; ++i) {
            scores[i] = expf(scores[i] - max_score);
            sum += scores[i];
        }
        const float inv_sum = 1.0f / sum;
        for (uint32_t i = 0; i < kv_len; ++i) scores[i] *= inv_sum;

        float* head_out = out + (size_t)h * head_dim;
        for (uint32_t pos = 0; pos < kv_len; ++pos) {
            const int8_t* val_head = values + (size_t)pos * kv_dim + (size_t)kv_head * head_dim;
            const float v_scale = scale_mode == ORACLE_SCALE_ROW
                                      ? val_scales[pos]
                                      : val_scales[(size_t)pos * num_kv_heads + kv_head];
            for (uint32_t d = 0; d < head_dim; ++d)
                head_out[d] += scores[pos] * ((float)val_head[d] * v_scale);
        }
    }
    free(qs);
}

/*
 * FP32 cache mode of the same loop (use_kv_quantization = false): scores over
 * keys_fp32 (src/inference.cpp:346-358), the softmax of :361-375 and P.V over
 * values_fp32 (:386-393); layout [pos][num_kv_heads][head_dim] fp32
 * (src/kv_cache.cpp:59-70).  Same operation order as the int8 restatement.
 */
void oracle_decode_attention_f32(const float* keys, const float* values, uint32_t kv_len,
                                 const float* q, float* out, uint32_t num_heads,
                                 uint32_t num_kv_heads, uint32_t head_dim, float softmax_scale,
                                 float* scores) {
    const uint32_t kv_dim = num_kv_heads * head_dim;
    float* qs = (float*)malloc(sizeof(float) * (size_t)num_heads * head_dim);
    for (uint32_t i = 0; i < num_heads * head_dim; ++i) qs[i] = q[i] * softmax_scale;
    memset(out, 0, sizeof(float) * (size_t)num_heads * head_dim);
    if (kv_len == 0) { free(qs); return; }
    for (uint32_t h = 0; h < num_heads; ++h) {
        const uint32_t kv_head = h % num_kv_heads;
        const float* head_q = qs + (size_t)h * head_dim;
        for (uint32_t pos = 0; pos < kv_len; ++pos) {
            float score = 0.0f;
            const float* key_head = keys + (size_t)pos * kv_dim + (size_t)kv_head * head_dim;
            for (uint32_t d = 0; d < head_dim; ++d) score += head_q[d] * key_head[d];
            scores[pos] = score;
        }
        float max_score = scores[0];
        for (uint32_t i = 1; i < kv_len; ++i)
            if (scores[i] > max_score) max_score = scores[i];
        float sum = 0.0f;
        for (uint32_t i = 0; i < kv_len; ++i) {
            scores[i] = expf(scores[i] - max_score);
            sum += scores[i];
        }
        const float inv_sum = 1.0f / sum;
        for (uint32_t i = 0; i < kv_len; ++i) scores[i] *= inv_sum;
        float* head_out = out + (size_t)h * head_dim;
        for (uint32_t pos = 0; pos < kv_len; ++pos) {
            const float* val_head = values + (size_t)pos * kv_dim + (size_t)kv_head * head_dim;
            for (uint32_t d = 0; d < head_dim; ++d) head_out[d] += scores[pos] * val_head[d];
        }
    }
    free(qs);
}

/*
 * K pre-processing of echo-core-zig before its cache append
 * (src/inference/engine.zig:544-559): per-head RMS norm with an fp16 weight
 * (applyHeadNorm, :521-532) then RoPE over interleaved pairs (applyRoPE,
 * :466-518).  x: [num_heads][head_dim] fp32 in place; norm_w: head_dim fp32
 * values of the fp16 weight, or NULL; rope_base <= 0: no rotation.  Every
 * product and sum is rounded on its own (volatile), as the Zig code evaluates
 * them without contraction, in the Zig code's order:
 *   :525-526  rms += x[i] * x[i], i = 0 .. head_dim-1 in sequence
 *   :527      rms = sqrt(rms / head_dim + 1e-6)
 *   :528      inv_rms = 1 / rms
 *   :530      x[i] = x[i] * inv_rms * w[i]        (left to right)
 *   :477      freq = 1 / pow(base, i / head_dim)  (fp32 throughout)
 *   :478      angle = pos * freq
 *   :479-480  cos(angle), sin(angle)
 *   :483-484  x0' = x0 cos - x1 sin;  x1' = x0 sin + x1 cos
 * The Zig code's @cos/@sin/pow are fp32 library functions that this container
 * cannot run (no Zig toolchain); this restatement takes cos and sin as the
 * fp32 rounding of the double-precision values at the fp32 angle (the
 * correctly rounded fp32 result but for double-rounding cases) and pow as
 * the C library's powf.  The restatement is therefore pinned to no Zig
 * output; the GPU kernels are bit-exact with it.
 */
void oracle_norm_rope(float* x, uint32_t num_heads, uint32_t head_dim, uint32_t pos,
                      const float* norm_w, float rope_base) {
    for (uint32_t h = 0; h < num_heads; ++h) {
        float* p = x + (size_t)h * head_dim;
        if (norm_w) {
            float rms = 0.0f;
            for (uint32_t i = 0; i < head_dim; ++i) {
                volatile float sq = p[i] * p[i];
                rms += sq;
            }
            rms = sqrtf(rms / (float)head_dim + 1e-6f);
            const float inv_rms = 1.0f / rms;
            for (uint32_t i = 0; i < head_dim; ++i) {
                volatile float t = p[i] * inv_rms;
                p[i] = t * norm_w[i];
            }
        }
        if (rope_base > 0.0f) {
            for (uint32_t i = 0; i < head_dim; i += 2) {
                const float freq = 1.0f / powf(rope_base, (float)i / (float)head_dim);
                volatile float angle = (float)pos * freq;
                const float c = (float)cos((double)angle), s = (float)sin((double)angle);
                const float x0 = p[i], x1 = p[i + 1];
                volatile float a = x0 * c, b = x1 * s, d = x0 * s, e = x1 * c;
                p[i] = a - b;
                p[i + 1] = d + e;
            }
        }
    }
}

/*
 * Chunked-prefill attention.  The reference has no chunked prefill: it feeds
 * a prompt one token at a time (src/main.cpp:404-405), each token running the
 * decode loop above over the cache as it stands after that token's append
 * (append-then-attend, the order echo-core-zig/src/inference/engine.zig:560-561
 * uses).  So query row i of an n_new-token chunk appended after past_len
 * cached tokens attends to kv positions [0, past_len + i].
 * q: [n_new][num_heads][head_dim]; out: same shape.
 */
void oracle_prefill_attention(const int8_t* keys, const int8_t* values,
                              const float* key_scales, const float* val_scales,
                              uint32_t past_len, uint32_t n_new, const float* q,
                              float* out, uint32_t num_heads, uint32_t num_kv_heads,
                              uint32_t head_dim, float softmax_scale, int scale_mode,
                              float* scores) {
    const size_t qrow = (size_t)num_heads * head_dim;
    for (uint32_t i = 0; i < n_new; ++i)
        oracle_decode_attention(keys, values, key_scales, val_scales, past_len + i + 1,
                                q + i * qrow, out + i * qrow, num_heads, num_kv_heads,
                                head_dim, softmax_scale, scale_mode, scores);
}
