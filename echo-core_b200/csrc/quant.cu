// quant.cu -- quantize-on-append kernels (sm_100a).
//
// Rounding contract, bit-exact with quantize_per_token_symmetric
// (src/kernels/quant.cpp:18-98) for finite input:
//   amax  = max |x| over the row                       (:29-60)
//   scale = amax / 127.0f, or 1.0f when amax == 0       (:63)  -- IEEE division
//   body  (first n - n%8 elements):  q = sat8(RNE(x * (1.0f/scale)))   (:70-88)
//   tail  (last n%8 elements):       q = clamp127(round_half_away(x / scale)) (:91-96)
// with x86's conversion of a NaN or out-of-range value to INT32_MIN, which a
// subnormal scale (reciprocal inf) reaches for finite input.
// Every operation uses an explicitly IEEE-rounded intrinsic; this file must
// not be compiled with fast-math.
#include <cstdint>

#include <cuda_fp16.h>

#include "ec_common.cuh"
#include "ec_internal.h"

namespace ec {

__device__ int32_t g_error_word = 0;

__device__ __forceinline__ float warp_max(float v, unsigned width = 32) {
    for (unsigned o = width / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o, width));
    return v;
}

__device__ __forceinline__ float scale_of(float amax) {
    return amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1.0f;
}

// x86 CVTPS2DQ semantics: a value that is NaN or outside the int32 range
// converts to INT32_MIN ("integer indefinite"), which the saturating packs
// then turn into -128 (body) or the clamp into -127 (tail).  Finite input
// reaches this only through a subnormal scale, whose reciprocal overflows.
__device__ __forceinline__ int32_t q_body(float x, float inv) {
    const float v = __fmul_rn(x, inv);
    if (!(fabsf(v) < 2147483648.0f)) return -128;
    return max(-128, min(127, __float2int_rn(v)));
}

__device__ __forceinline__ int32_t q_tail(float x, float scale) {
    const float v = roundf(__fdiv_rn(x, scale));
    if (!(fabsf(v) < 2147483648.0f)) return -127;
    return max(-127, min(127, (int32_t)v));
}

// ---------------------------------------------------------------- generic
// One warp per row, any row length.  Used by ec_quantize_per_token_symmetric
// and by the single-sequence cache when head_dim is not 128.
__global__ void quantize_rows_kernel(const float* __restrict__ in, int8_t* __restrict__ out,
                                     float* __restrict__ scales, uint32_t num_rows,
                                     uint32_t n) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t warps_per_grid = (gridDim.x * blockDim.x) >> 5;
    const uint32_t vec_end = n - (n % 8u);
    for (uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < num_rows;
         row += warps_per_grid) {
        const float* x = in + (size_t)row * n;
        int8_t* o = out + (size_t)row * n;
        float amax = 0.0f;
        for (uint32_t i = lane; i < n; i += 32) amax = fmaxf(amax, fabsf(x[i]));
        amax = warp_max(amax);
        const float scale = scale_of(amax);
        const float inv = __fdiv_rn(1.0f, scale);
        for (uint32_t i = lane; i < n; i += 32) {
            const float v = x[i];
            o[i] = (int8_t)(i < vec_end ? q_body(v, inv) : q_tail(v, scale));
        }
        if (lane == 0) scales[row] = scale;
    }
}

// ------------------------------------------------------------ batched append
// One warp per (sequence, new token).  head_dim is 128: lane l holds float4
// number l of every head's 128-wide slice, so each load and each store of the
// warp is one contiguous 512 B / 128 B run.  PER_HEAD reduces the absmax per
// head across the warp; ROW reduces it over the whole token row.
struct TableView {
    const int32_t* offset;
    const int32_t* capacity;
    const int32_t* length;
    int32_t host_offset, host_capacity, host_length;  // used when the pointers are null
    uint64_t total_slots;
    PageMap pages;

    // Loads and checks one entry; false (and a flagged error) for a bad one.
    __device__ __forceinline__ bool load(int s, int32_t* err, int32_t& off, int32_t& cap,
                                         int32_t& len) const {
        off = offset ? offset[s] : host_offset;
        cap = capacity ? capacity[s] : host_capacity;
        len = length ? length[s] : host_length;
        return page_entry_ok(pages, off, cap, len, total_slots);
    }
};

// Quantizes one token's K and V rows held as xs[t][g * DV + dv] (lane l holds
// float4 l of the dv-th 128-float block of head g; head_dim = 128 * DV) and
// stores codes and scales at `slot`.
//
// The 2 x HKV absmaxes (2 for ROW) are reduced with a butterfly
// reduce-scatter: after it, lane l holds the full absmax of value
// k = l >> (5 - log2(NV)), replicated over 32 / NV lanes.  That lane alone
// computes k's scale and reciprocal (two IEEE divisions per lane instead of
// one per value per lane); shuffles broadcast the reciprocals back.
//
// Codes: v = RN(x * inv) is below 127.5 in magnitude whenever the scale is a
// normal float (|x| <= amax, and scale and inv each carry one rounding of
// 2^-24), so sat8(RNE(v)) is the low byte of RN(v + 1.5 * 2^23): adding the
// even integer 1.5 * 2^23 rounds v to an integer with ties to even, and the
// sum's mantissa is 2^22 + RNE(v).  A subnormal scale (absmax below about
// 1.5e-36) takes the exact path, uniformly across the warp.
template <int HKV, bool ROW, int DV>
__device__ __forceinline__ void quantize_store(const float4 (&xs)[2][HKV * DV], const AppendArgs& a,
                                               int64_t slot, int lane) {
    constexpr int D = 128 * DV;
    constexpr int NV = ROW ? 2 : 2 * HKV;           // values to reduce: (t, g) or t
    constexpr int LB = NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : 4;   // log2(NV)
    constexpr int SH = 5 - LB;                      // lane >> SH = the value a lane ends with
    static_assert(NV == (1 << LB) && NV <= 16, "HKV must be 1, 2, 4 or 8");
    float v[NV];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
#pragma unroll
        for (int g = 0; g < HKV; ++g) {
            float m = 0.0f;
#pragma unroll
            for (int dv = 0; dv < DV; ++dv) {
                const float4 x = xs[t][g * DV + dv];
                m = fmaxf(m, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
            }
            if (ROW) v[t] = g == 0 ? m : fmaxf(v[t], m);
            else v[t * HKV + g] = m;
        }
    }
    // reduce-scatter: each step halves the values a lane keeps
#pragma unroll
    for (int step = 0, half = NV / 2; half >= 1; ++step, half >>= 1) {
        const int o = 16 >> step;
        const bool upper = lane & o;
#pragma unroll
        for (int j = 0; j < half; ++j) {
            const float send = upper ? v[j] : v[j + half];
            const float keep = upper ? v[j + half] : v[j];
            v[j] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, o));
        }
    }
    // all-reduce across the 32 / NV lanes that share a value
#pragma unroll
    for (int o = (16 >> LB); o > 0; o >>= 1) v[0] = fmaxf(v[0], __shfl_xor_sync(0xffffffffu, v[0], o));
    const float scale = scale_of(v[0]);
    const float inv_own = __fdiv_rn(1.0f, scale);
    const uint32_t sub = __ballot_sync(0xffffffffu, scale < 1.17549435e-38f);
    if ((lane & ((1 << SH) - 1)) == 0) {
        const int k = lane >> SH;
        const int t = k / (NV / 2), g = k % (NV / 2);
        float* sc = t == 0 ? a.key_scales : a.val_scales;
        if (ROW) sc[slot] = scale;
        else sc[(size_t)slot * HKV + g] = scale;
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {
        int8_t* dst = (t == 0 ? a.keys : a.values) + (size_t)slot * (HKV * D);
#pragma unroll
        for (int g = 0; g < HKV; ++g) {
            const int src = (ROW ? t : t * HKV + g) << SH;
            const float inv = __shfl_sync(0xffffffffu, inv_own, src);
#pragma unroll
            for (int dv = 0; dv < DV; ++dv) {
                const float4 x = xs[t][g * DV + dv];
                uint32_t word;
                if (!((sub >> src) & 1u)) {
                    constexpr float kRound = 12582912.0f;   // 1.5 * 2^23
                    const uint32_t b0 = __float_as_uint(__fadd_rn(__fmul_rn(x.x, inv), kRound));
                    const uint32_t b1 = __float_as_uint(__fadd_rn(__fmul_rn(x.y, inv), kRound));
                    const uint32_t b2 = __float_as_uint(__fadd_rn(__fmul_rn(x.z, inv), kRound));
                    const uint32_t b3 = __float_as_uint(__fadd_rn(__fmul_rn(x.w, inv), kRound));
                    word = __byte_perm(__byte_perm(b0, b1, 0x0040u), __byte_perm(b2, b3, 0x0040u), 0x5410u);
                } else {
                    word = (uint32_t)(q_body(x.x, inv) & 0xff) | ((uint32_t)(q_body(x.y, inv) & 0xff) << 8) |
                           ((uint32_t)(q_body(x.z, inv) & 0xff) << 16) |
                           ((uint32_t)(q_body(x.w, inv) & 0xff) << 24);
                }
                reinterpret_cast<uint32_t*>(dst + g * D + dv * 128)[lane] = word;
            }
        }
    }
}

// With one new token per sequence, the sequence's only warp advances its
// length itself once every lane has read the old one; with more, a separate
// launch does it after all of a sequence's warps have read it.
__device__ __forceinline__ void bump_own_length(const AppendArgs& a, int s, int32_t len, int lane) {
    if (a.n_new != 1 || a.seq_len == nullptr) return;
    __syncwarp();
    if (lane == 0) a.seq_len[s] = len + 1;
}

template <int HKV, bool ROW, int DV>
__global__ void __launch_bounds__(256) append_kernel(AppendArgs a) {
    constexpr int D = 128 * DV;
    pdl_wait();  // k / v and the table may come from the previous kernel
    pdl_trigger();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int s = warp / a.n_new;
    const int i = warp - s * a.n_new;
    if (s >= a.num_seqs) return;
    // The K and V rows do not depend on the table: all 2 x HKV float4 loads of
    // the lane are issued first, so that they and the table load are in
    // flight together.
    const size_t src_row = ((size_t)s * a.n_new + i) * (HKV * D);
    float4 xs[2][HKV * DV];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int gd = 0; gd < HKV * DV; ++gd)
            xs[t][gd] = __ldcs(reinterpret_cast<const float4*>((t == 0 ? a.k : a.v) + src_row) +
                               gd * 32 + lane);
    TableView tv{a.seq_offset, a.seq_capacity, a.seq_len, a.host_offset, a.host_capacity,
                 a.host_length, a.total_slots, a.pages};
    int32_t off, cap, len;
    if (!tv.load(s, a.err, off, cap, len)) {
        if (i == 0 && lane == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        return;
    }
    if ((int64_t)len + a.n_new > cap) {
        if (i == 0 && lane == 0) flag_error(a.err, EC_DEVERR_OVERFLOW);
        return;
    }
    int64_t slot;
    if (!page_slot(a.pages, s, off, len + i, a.total_slots, slot)) {
        if (lane == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        return;
    }

    quantize_store<HKV, ROW, DV>(xs, a, slot, lane);
    bump_own_length(a, s, len, lane);
}

__global__ void bump_lengths_kernel(AppendArgs a) {
    pdl_wait();
    pdl_trigger();
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= a.num_seqs || a.seq_len == nullptr) return;
    TableView tv{a.seq_offset, a.seq_capacity, a.seq_len, 0, 0, 0, a.total_slots, a.pages};
    int32_t off, cap, len;
    if (!tv.load(s, a.err, off, cap, len)) return;  // already flagged by append_kernel
    if ((int64_t)len + a.n_new > cap) return;
    a.seq_len[s] = len + a.n_new;
}

// ------------------------------------------------- head norm + RoPE on K
// echo-core-zig applies, to each token's K before it enters the cache, a
// per-head RMS norm (src/inference/engine.zig:521-532: rms = sqrt(sum k^2 / d
// + 1e-6); k = k * (1/rms) * w) and rotary position embedding over
// interleaved pairs (:466-518: angle = pos * freq_i, freq_i = 1/base^(i/d);
// (k0, k1) -> (k0 cos - k1 sin, k0 sin + k1 cos)).  Products and sums are
// rounded one at a time (no contraction) and in the Zig code's order -- the
// sum of squares runs over the head's dims in sequence (:525-526), not as a
// tree -- so the results are bit-identical to the CPU restatement; the sines
// and cosines are the double-precision values rounded to fp32.
struct PairRot { float c0, s0, c1, s1; };

__device__ __forceinline__ PairRot pair_rotation(int pos, int lane, const float* inv_freq,
                                                 int dv = 0) {
    // lane holds dims 128*dv + 4*lane .. +3: pairs 64*dv + 2*lane and +1
    const float a0 = __fmul_rn((float)pos, inv_freq[64 * dv + 2 * lane]);
    const float a1 = __fmul_rn((float)pos, inv_freq[64 * dv + 2 * lane + 1]);
    double s0, c0, s1, c1;
    sincos((double)a0, &s0, &c0);
    sincos((double)a1, &s1, &c1);
    return {(float)c0, (float)s0, (float)c1, (float)s1};
}

__device__ __forceinline__ float4 rotate(float4 x, const PairRot& r) {
    float4 y;
    y.x = __fsub_rn(__fmul_rn(x.x, r.c0), __fmul_rn(x.y, r.s0));
    y.y = __fadd_rn(__fmul_rn(x.x, r.s0), __fmul_rn(x.y, r.c0));
    y.z = __fsub_rn(__fmul_rn(x.z, r.c1), __fmul_rn(x.w, r.s1));
    y.w = __fadd_rn(__fmul_rn(x.z, r.s1), __fmul_rn(x.w, r.c1));
    return y;
}

// per-head RMS norm of one head of 128 * DV floats held as DV float4 per lane
// (lane l: dims 128*dv + 4l .. +3).  The squares are summed in dimension
// order, one rounding per addition, as src/inference/engine.zig:525-526 sums
// them: every lane runs the same chain over squares broadcast by shuffle.
template <int DV>
__device__ __forceinline__ void head_rms_norm(float4 (&x)[DV], const uint16_t* w, int lane) {
    constexpr float kD = 128.0f * DV;
    float ss = 0.0f;
#pragma unroll
    for (int dv = 0; dv < DV; ++dv) {
        const float q0 = __fmul_rn(x[dv].x, x[dv].x), q1 = __fmul_rn(x[dv].y, x[dv].y);
        const float q2 = __fmul_rn(x[dv].z, x[dv].z), q3 = __fmul_rn(x[dv].w, x[dv].w);
#pragma unroll 8
        for (int l = 0; l < 32; ++l) {
            ss = __fadd_rn(ss, __shfl_sync(0xffffffffu, q0, l));
            ss = __fadd_rn(ss, __shfl_sync(0xffffffffu, q1, l));
            ss = __fadd_rn(ss, __shfl_sync(0xffffffffu, q2, l));
            ss = __fadd_rn(ss, __shfl_sync(0xffffffffu, q3, l));
        }
    }
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, kD), 1e-6f));
    const float inv = __fdiv_rn(1.0f, rms);
#pragma unroll
    for (int dv = 0; dv < DV; ++dv) {
        const ushort4 wb = reinterpret_cast<const ushort4*>(w)[dv * 32 + lane];
        x[dv].x = __fmul_rn(__fmul_rn(x[dv].x, inv), __half2float(__ushort_as_half(wb.x)));
        x[dv].y = __fmul_rn(__fmul_rn(x[dv].y, inv), __half2float(__ushort_as_half(wb.y)));
        x[dv].z = __fmul_rn(__fmul_rn(x[dv].z, inv), __half2float(__ushort_as_half(wb.z)));
        x[dv].w = __fmul_rn(__fmul_rn(x[dv].w, inv), __half2float(__ushort_as_half(wb.w)));
    }
}

// append_kernel with K normed and rotated at its cache position before
// quantization (one warp per (sequence, new token), as append_kernel)
template <int HKV, bool ROW, int DV>
__global__ void __launch_bounds__(256) append_rope_kernel(AppendArgs a) {
    constexpr int D = 128 * DV;
    pdl_wait();  // k / v and the table may come from the previous kernel
    pdl_trigger();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int s = warp / a.n_new;
    const int i = warp - s * a.n_new;
    if (s >= a.num_seqs) return;
    TableView tv{a.seq_offset, a.seq_capacity, a.seq_len, a.host_offset, a.host_capacity,
                 a.host_length, a.total_slots, a.pages};
    int32_t off, cap, len;
    if (!tv.load(s, a.err, off, cap, len)) {
        if (i == 0 && lane == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        return;
    }
    if ((int64_t)len + a.n_new > cap) {
        if (i == 0 && lane == 0) flag_error(a.err, EC_DEVERR_OVERFLOW);
        return;
    }
    const int pos = len + i;                  // the token's position in its sequence
    int64_t slot;
    if (!page_slot(a.pages, s, off, pos, a.total_slots, slot)) {
        if (lane == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        return;
    }
    const size_t src_row = ((size_t)s * a.n_new + i) * (HKV * D);
    PairRot rot[DV];
    if (a.rope) {
#pragma unroll
        for (int dv = 0; dv < DV; ++dv) rot[dv] = pair_rotation(pos, lane, a.inv_freq, dv);
    }
    float4 xs[2][HKV * DV];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int g = 0; g < HKV; ++g) {
            float4 x[DV];
#pragma unroll
            for (int dv = 0; dv < DV; ++dv)
                x[dv] = __ldcs(reinterpret_cast<const float4*>((t == 0 ? a.k : a.v) + src_row) +
                               (g * DV + dv) * 32 + lane);
            if (t == 0) {
                if (a.k_norm_w) head_rms_norm<DV>(x, a.k_norm_w, lane);
                if (a.rope) {
#pragma unroll
                    for (int dv = 0; dv < DV; ++dv) x[dv] = rotate(x[dv], rot[dv]);
                }
            }
#pragma unroll
            for (int dv = 0; dv < DV; ++dv) xs[t][g * DV + dv] = x[dv];
        }
    quantize_store<HKV, ROW, DV>(xs, a, slot, lane);
    bump_own_length(a, s, len, lane);
}

struct RopeRowsArgs {
    float* x;
    const int32_t* positions;
    const uint16_t* norm_w;
    uint32_t rows, num_heads;
    int rope;
    float inv_freq[kMaxHeadDim / 2];
};

// one warp per (row, head): the Q side of the same pre-processing
template <int DV>
__global__ void __launch_bounds__(256) rope_rows_kernel(RopeRowsArgs a) {
    const uint64_t w = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= (uint64_t)a.rows * a.num_heads) return;
    const uint32_t r = (uint32_t)(w / a.num_heads);
    float4* p = reinterpret_cast<float4*>(a.x + w * 128 * DV) + lane;
    float4 x[DV];
#pragma unroll
    for (int dv = 0; dv < DV; ++dv) x[dv] = p[32 * dv];
    if (a.norm_w) head_rms_norm<DV>(x, a.norm_w, lane);
#pragma unroll
    for (int dv = 0; dv < DV; ++dv) {
        if (a.rope) x[dv] = rotate(x[dv], pair_rotation(a.positions[r], lane, a.inv_freq, dv));
        p[32 * dv] = x[dv];
    }
}

// ---------------------------------------------------------------- launchers
using AppendFn = void (*)(AppendArgs);

// One warp per (sequence, new token); lengths bumped in place for n_new == 1,
// by a second kernel otherwise.
static cudaError_t launch_append_with(AppendFn fn, const AppendArgs& a, cudaStream_t st) {
    const int64_t warps = (int64_t)a.num_seqs * a.n_new;
    if (warps == 0) return cudaSuccess;
    if (fn == nullptr) return cudaErrorInvalidValue;
    const int threads = 256;
    const int64_t blocks = (warps * 32 + threads - 1) / threads;
    if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
    cudaError_t e = launch_pdl(fn, dim3((unsigned)blocks), dim3(threads), 0, st, a);
    if (e == cudaSuccess && a.seq_len != nullptr && a.n_new > 1)
        e = launch_pdl(bump_lengths_kernel, dim3((a.num_seqs + 127) / 128), dim3(128), 0, st, a);
    return e;
}

#define EC_PICK_APPEND_DV(K, DV)                                             \
    switch (num_kv_heads) {                                                  \
        case 1: return row_mode ? K<1, true, DV> : K<1, false, DV>;          \
        case 2: return row_mode ? K<2, true, DV> : K<2, false, DV>;          \
        case 4: return row_mode ? K<4, true, DV> : K<4, false, DV>;          \
        case 8: return row_mode ? K<8, true, DV> : K<8, false, DV>;          \
        default: return nullptr;                                             \
    }
#define EC_PICK_APPEND(K)                                                    \
    if (head_dim == 128) { EC_PICK_APPEND_DV(K, 1) }                         \
    if (head_dim == 256) { EC_PICK_APPEND_DV(K, 2) }                         \
    return nullptr;
static AppendFn pick_append(int num_kv_heads, int head_dim, bool row_mode) {
    EC_PICK_APPEND(append_kernel)
}
static AppendFn pick_append_rope(int num_kv_heads, int head_dim, bool row_mode) {
    EC_PICK_APPEND(append_rope_kernel)
}
#undef EC_PICK_APPEND
#undef EC_PICK_APPEND_DV

cudaError_t launch_append_rope(const AppendArgs& a, int num_kv_heads, bool row_mode, cudaStream_t st) {
    return launch_append_with(pick_append_rope(num_kv_heads, a.head_dim, row_mode), a, st);
}

cudaError_t launch_rope_rows(float* x, uint32_t rows, uint32_t num_heads, uint32_t head_dim,
                             const int32_t* positions, const uint16_t* norm_w, int rope,
                             const float* inv_freq, cudaStream_t st) {
    const uint64_t warps = (uint64_t)rows * num_heads;
    if (warps == 0) return cudaSuccess;
    if (head_dim != 128 && head_dim != 256) return cudaErrorInvalidValue;
    RopeRowsArgs a{};
    a.x = x;
    a.positions = positions;
    a.norm_w = norm_w;
    a.rows = rows;
    a.num_heads = num_heads;
    a.rope = rope;
    for (uint32_t i = 0; i < head_dim / 2; ++i) a.inv_freq[i] = inv_freq[i];
    const uint64_t blocks = (warps * 32 + 255) / 256;
    if (blocks > 0x7fffffffull) return cudaErrorInvalidConfiguration;
    if (head_dim == 128)
        rope_rows_kernel<1><<<(unsigned)blocks, 256, 0, st>>>(a);
    else
        rope_rows_kernel<2><<<(unsigned)blocks, 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const float* in, int8_t* out, float* scales, uint32_t rows,
                                 uint32_t n, cudaStream_t st) {
    if (rows == 0) return cudaSuccess;
    const uint32_t threads = 256, warps_per_block = threads / 32;
    uint32_t blocks = (rows + warps_per_block - 1) / warps_per_block;
    if (blocks > 65535u * 8u) blocks = 65535u * 8u;
    quantize_rows_kernel<<<blocks, threads, 0, st>>>(in, out, scales, rows, n);
    return cudaGetLastError();
}

cudaError_t launch_append(const AppendArgs& a, int num_kv_heads, bool row_mode, cudaStream_t st) {
    return launch_append_with(pick_append(num_kv_heads, a.head_dim, row_mode), a, st);
}

// ------------------------------------------------------ fused dequant dot
// scores[pos] = sum_d query[d] * (key[pos][d] * scale[pos]); one warp per pos.
__global__ void fused_dequant_dot_kernel(const float* __restrict__ q, const int8_t* __restrict__ k,
                                         const float* __restrict__ s, float* __restrict__ out,
                                         uint32_t dim, uint32_t seq_len) {
    const uint32_t lane = threadIdx.x & 31;
    const uint32_t pos = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (pos >= seq_len) return;
    const int8_t* row = k + (size_t)pos * dim;
    const float sc = s[pos];
    float acc = 0.0f;
    for (uint32_t d = lane; d < dim; d += 32) acc = fmaf((float)row[d] * sc, q[d], acc);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) out[pos] = acc;
}

cudaError_t launch_fused_dequant_dot(const float* q, const int8_t* k, const float* s, float* out,
                                     uint32_t dim, uint32_t seq_len, cudaStream_t st) {
    if (seq_len == 0) return cudaSuccess;
    const uint32_t threads = 256;
    const uint64_t blocks = ((uint64_t)seq_len * 32 + threads - 1) / threads;
    if (blocks > 0x7fffffffull) return cudaErrorInvalidConfiguration;
    fused_dequant_dot_kernel<<<(unsigned)blocks, threads, 0, st>>>(q, k, s, out, dim, seq_len);
    return cudaGetLastError();
}

}  // namespace ec
