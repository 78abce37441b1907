// decode.cu -- split-K grouped-query decode attention over the int8 KV cache
// (sm_100a), and the log-sum-exp combine of split partials.
//
// Semantics follow the decode loop of InferenceEngine::attention
// (src/inference.cpp:321-392): q is multiplied by the softmax scale first
// (:322-325); Q head h reads KV head h % num_kv_heads (:335); scores are
// q . (code * k_scale) (:343-352); softmax (:367-379); output is
// sum_t p_t * (code * v_scale) (:383-392).  The softmax runs online in base 2
// (log2(e) folded into q), with the maximum carried per split.
//
// Work decomposition.  One CTA owns one (sequence, chunk of tokens) and all
// num_kv_heads heads of it, so each K/V tile it stages is one contiguous run
// of [tokens][num_kv_heads][128] int8 codes: a single 1-D bulk copy (TMA,
// no multicast) per tile per tensor, plus one for each scale array.  A
// producer warp streams tiles through a kStages-deep shared-memory ring
// guarded by mbarriers; 8 consumer warps each own one KV head (and its
// GROUP query heads) for a 16-token slice of every tile.  Every K and V
// byte is read from HBM exactly once per step.
//
// Consumer inner loops, per lane:
//   QK: 8 lanes share one token row (16 codes each).  Codes become fp32 with
//       a byte-permute into the mantissa of 2^23 and one packed subtract;
//       dots use packed fp32 FMA (fma.rn.f32x2); a transposing butterfly
//       leaves each lane with one head's full dot.
//   PV: the same lanes own 16 output dims of every head and accumulate
//       p'(t) * code(t) with packed FMA, p' = p * v_scale (fused scale).
// Online softmax rescales the accumulators only when a head's running
// maximum grows by more than 2^8 (exact: numerator and denominator always
// share the same reference maximum).
#include <cmath>
#include <cstdint>

#include "ec_common.cuh"
#include "ec_internal.h"

namespace ec {
namespace {

constexpr int D = 128;
constexpr int kPairs = 8;                          // QK warp + PV warp pairs
constexpr int kQkWarps = kPairs;
constexpr int kConsumerWarps = 2 * kPairs;         // QK warps 0..7, PV warps 8..15
constexpr int kThreads = kConsumerWarps * 32;      // 16 warps: 4 per SM sub-partition
constexpr int kStages = 5;
constexpr int kPBufs = 2;                          // P tiles in flight per pair
// QK warp 0 also issues the bulk copies.  At its tile i it issues tile
// i + kPrefetch, whose stage was last used by tile i - kPBufs: every warp has
// released that stage by the time warp 0 holds the P buffer of tile i.
constexpr int kPrefetch = kStages - kPBufs;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyRescale = 8.0f;
constexpr unsigned kFull = 0xffffffffu;

template <int HKV>
struct Geo {
    static constexpr int T = 128 / HKV;                 // tokens per tile
    static constexpr int WPH = kPairs / HKV;            // pairs per KV head
    static constexpr int ROWB = HKV * D;                // code bytes per token row
    static constexpr int KV_TILE = T * ROWB;            // 16 KB
    static constexpr int SC_TILE = T * HKV * 4;         // 512 B
    static constexpr int STAGE = 2 * KV_TILE + 2 * SC_TILE;
    // per pair and P buffer: P'[16 tokens][4 heads] then corr[4]
    static constexpr int PSLOT = 16 * 4 + 4;
    static constexpr int PBUF = kPairs * kPBufs * PSLOT * 4;
    static constexpr int NBARS = 2 * kStages + 2 * kPairs * kPBufs;
    static constexpr int SMEM = kStages * STAGE + PBUF + NBARS * 8;
    static_assert(T == WPH * 16, "each pair owns 16 tokens of a tile");
};

__device__ __forceinline__ void consumer_barrier() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

template <int N>
__device__ __forceinline__ float pick(const float (&v)[N], int i) {
    float r = v[0];
#pragma unroll
    for (int k = 1; k < N; ++k) r = (i == k) ? v[k] : r;
    return r;
}

// Within an 8-lane token group (c = lane & 7), each lane ends the score
// reduction holding the dot of head head_of_lane(c).  To make the reduction a
// plain butterfly, the lane keeps its GROUP per-head partial dots in the slot
// order slot k <-> head k ^ head_of_lane(c); the q registers are loaded in
// that order once, so no select is needed per token.
template <int GROUP>
__device__ __forceinline__ int head_of_lane(int c) {
    if constexpr (GROUP == 4) return ((c >> 2) & 1) * 2 + ((c >> 1) & 1);
    else if constexpr (GROUP == 2) return (c >> 2) & 1;
    else return 0;
}
template <int GROUP>
__device__ __forceinline__ int lane_of_head(int j) {
    if constexpr (GROUP == 4) return (j >> 1) * 4 + (j & 1) * 2;
    else if constexpr (GROUP == 2) return j * 4;
    else return 0;
}
template <int GROUP>
__device__ __forceinline__ bool writer_lane(int c) {
    if constexpr (GROUP == 4) return (c & 1) == 0;
    else if constexpr (GROUP == 2) return (c & 3) == 0;
    else return c == 0;
}

template <int GROUP>
__device__ __forceinline__ float butterfly(float (&v)[GROUP]) {
    if constexpr (GROUP == 4) {
        v[0] += __shfl_xor_sync(kFull, v[2], 4);
        v[1] += __shfl_xor_sync(kFull, v[3], 4);
        v[0] += __shfl_xor_sync(kFull, v[1], 2);
    } else if constexpr (GROUP == 2) {
        v[0] += __shfl_xor_sync(kFull, v[1], 4);
        v[0] += __shfl_xor_sync(kFull, v[0], 2);
    } else {
        v[0] += __shfl_xor_sync(kFull, v[0], 4);
        v[0] += __shfl_xor_sync(kFull, v[0], 2);
    }
    v[0] += __shfl_xor_sync(kFull, v[0], 1);
    return v[0];
}

__device__ __forceinline__ void codes16_to_f2(const uint4 w, float2 (&f)[8]) {
    i8x4_to_f2x2(w.x, f[0], f[1]);
    i8x4_to_f2x2(w.y, f[2], f[3]);
    i8x4_to_f2x2(w.z, f[4], f[5]);
    i8x4_to_f2x2(w.w, f[6], f[7]);
}

__device__ __forceinline__ bool load_entry(const DecodeArgs& a, int s, int32_t& off, int32_t& cap,
                                           int32_t& len) {
    off = a.seq_offset ? a.seq_offset[s] : a.host_offset;
    cap = a.seq_capacity ? a.seq_capacity[s] : a.host_capacity;
    len = a.seq_len ? a.seq_len[s] : a.host_length;
    // len is also bounded by the tokens the grid covers (max_chunks chunks),
    // which the host sized from its max_seq_len bound.
    return off >= 0 && cap >= 0 && len >= 0 && len <= cap &&
           (uint64_t)off + (uint64_t)cap <= a.total_slots &&
           (int64_t)len <= (int64_t)a.max_chunks * a.chunk_tokens;
}

// Writes the result of a sequence with no cached token: zeros (kOut, as the
// reference's memset at src/inference.cpp:328) or an empty partial state.
__device__ void write_empty(const DecodeArgs& a, int seq) {
    for (int o = threadIdx.x; o < a.num_heads * D; o += blockDim.x) {
        a.out[(size_t)seq * a.num_heads * D + o] = 0.0f;
        if (a.mode == kPartial && (o % D) == 0) {
            const int h = o / D;
            a.out_ml[((size_t)seq * a.num_heads + h) * 2] = -INFINITY;
            a.out_ml[((size_t)seq * a.num_heads + h) * 2 + 1] = 0.0f;
        }
    }
}

// Bounded wait shared by all 32 lanes of a warp; the outcome is warp-uniform.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
    return __all_sync(kFull, mbar_wait(bar, parity));
}

// Issues tile j of the chunk into stage j % kStages (warp-collective; lane 0
// drives the bulk copies).  Waits, bounded, until every consumer warp has
// released the stage's previous tile.  Returns false on a timeout.
template <int HKV>
__device__ __forceinline__ bool issue_tile(const DecodeArgs& a, uint8_t* stages, uint64_t* full,
                                           uint64_t* empty, int j, int n, size_t slot0,
                                           uint64_t pol, int lane) {
    using G = Geo<HKV>;
    const int s = j % kStages;
    bool ok = true;
    if (lane == 0 && j >= kStages) ok = mbar_wait(&empty[s], ((j / kStages) - 1) & 1);
    ok = __shfl_sync(kFull, ok, 0);
    if (!ok) return false;
    const int ntok = min(G::T, n - j * G::T);
    const size_t slot = slot0 + (size_t)j * G::T;
    uint8_t* st = stages + s * G::STAGE;
    const uint32_t kvb = (uint32_t)ntok * G::ROWB;
    if (!a.row_scales) {
        if (lane == 0) {
            const uint32_t scb = (uint32_t)ntok * HKV * 4;
            mbar_arrive_expect_tx(&full[s], 2 * kvb + 2 * scb);
            bulk_g2s_hint(st, a.keys + slot * G::ROWB, kvb, &full[s], pol);
            bulk_g2s_hint(st + G::KV_TILE, a.values + slot * G::ROWB, kvb, &full[s], pol);
            bulk_g2s_hint(st + 2 * G::KV_TILE, a.key_scales + slot * HKV, scb, &full[s], pol);
            bulk_g2s_hint(st + 2 * G::KV_TILE + G::SC_TILE, a.val_scales + slot * HKV, scb,
                          &full[s], pol);
        }
    } else {
        // ROW scales: one fp32 per token, broadcast into the per-head tile
        // layout with plain loads; the arrive releases them to the consumers.
        if (lane == 0) {
            mbar_expect_tx(&full[s], 2 * kvb);
            bulk_g2s_hint(st, a.keys + slot * G::ROWB, kvb, &full[s], pol);
            bulk_g2s_hint(st + G::KV_TILE, a.values + slot * G::ROWB, kvb, &full[s], pol);
        }
        float* ks = reinterpret_cast<float*>(st + 2 * G::KV_TILE);
        float* vs = ks + G::T * HKV;
        for (int t = lane; t < ntok; t += 32) {
            const float kv = a.key_scales[slot + t];
            const float vv = a.val_scales[slot + t];
#pragma unroll
            for (int g = 0; g < HKV; ++g) {
                ks[t * HKV + g] = kv;
                vs[t * HKV + g] = vv;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
    }
    return true;
}

template <int HKV, int GROUP>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const DecodeArgs a) {
    using G = Geo<HKV>;
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ int fail_flag;
    uint8_t* stages = smem;
    float* pbuf = reinterpret_cast<float*>(smem + kStages * G::STAGE);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * G::STAGE + G::PBUF);
    uint64_t* full = bars;                           // [kStages]  TMA -> consumers
    uint64_t* empty = full + kStages;                // [kStages]  consumers -> producer
    uint64_t* p_full = empty + kStages;              // [kPairs][kPBufs]  QK -> PV
    uint64_t* p_empty = p_full + kPairs * kPBufs;    // [kPairs][kPBufs]  PV -> QK

    const int seq = blockIdx.y;
    const int chunk = blockIdx.x;
    const bool direct = a.max_chunks == 1;
    int32_t off, cap, len;
    if (!load_entry(a, seq, off, cap, len)) {
        if (chunk == 0 && threadIdx.x == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        return;
    }
    const int t0 = chunk * a.chunk_tokens;
    if (t0 >= len) {
        if (direct && chunk == 0) write_empty(a, seq);
        return;
    }
    const int n = min(a.chunk_tokens, len - t0);
    const int ntiles = (n + G::T - 1) / G::T;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        for (int i = 0; i < kPairs * kPBufs; ++i) {
            mbar_init(&p_full[i], 1);
            mbar_init(&p_empty[i], 1);
        }
        fail_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    const int pair = warp % kPairs;
    const bool is_qk = warp < kQkWarps;
    const int g = pair / G::WPH;      // KV head
    const int sw = pair % G::WPH;     // which 16-token slice of each tile
    const int c = lane & 7;           // 16-byte column of the 128-byte head row
    const int tq = lane >> 3;         // token within a 4-token pass / PV row group
    const int hsel = head_of_lane<GROUP>(c);
    float* pslots = pbuf + pair * kPBufs * G::PSLOT;
    bool failed = false;
    float* mo = reinterpret_cast<float*>(stages);                 // merge area, [8][GROUP][128]
    float* mm = mo + kPairs * GROUP * D;                           // [8][GROUP]
    float* ml = mm + kPairs * GROUP;                               // [8][GROUP]

    if (is_qk) {
        // ======================================================== QK warps
        // Scores of this pair's 16 tokens x GROUP query heads on the tensor
        // cores: mma.sync m16n8k32 with the int8 K codes as A (rows = tokens,
        // unconverted) and q as B, split exactly into three digits
        // q_int = 65536*d0 + 256*d1 + d2 (d0 signed, d1/d2 unsigned bytes) of a
        // per-head 24-bit fixed-point scale.  Integer accumulation is exact;
        // the digits are recombined in fp32.  The contraction order over the
        // 128 dims is permuted (thread t4 holds dims [32*t4, 32*t4+32) of its
        // rows), identically for A and B.
        const bool producer = warp == 0;
        const size_t slot0 = (size_t)off + t0;
        const uint64_t pol = l2_policy_evict_first();
        if (producer) {
            for (int j = 0; j < kPrefetch && j < ntiles; ++j)
                issue_tile<HKV>(a, stages, full, empty, j, n, slot0, pol, lane);
        }
        const int gid = lane >> 2;    // mma group: token row gid (and gid + 8)
        const int t4 = lane & 3;      // thread in group: query head t4's column pair
        // --- q digits as B fragments (n = gid <-> (head gid>>1, digit))
        uint32_t b_hi[4][2], b_lo[4][2];   // n-tile 0: d0 (s8); n-tile 1: d1 | d2 (u8)
        float sq_own;                      // dequant scale of head gid>>1
        {
            const int hq = gid >> 1;
            const bool live = hq < GROUP;
            float qv[32];
            float amax = 0.0f;
            const float* qp = a.q + ((size_t)seq * a.num_heads + g + HKV * (live ? hq : 0)) * D + 32 * t4;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float4 v = reinterpret_cast<const float4*>(qp)[e];
                qv[4 * e + 0] = __fmul_rn(__fmul_rn(v.x, a.q_mul), kLog2e);
                qv[4 * e + 1] = __fmul_rn(__fmul_rn(v.y, a.q_mul), kLog2e);
                qv[4 * e + 2] = __fmul_rn(__fmul_rn(v.z, a.q_mul), kLog2e);
                qv[4 * e + 3] = __fmul_rn(__fmul_rn(v.w, a.q_mul), kLog2e);
            }
#pragma unroll
            for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(qv[e]));
            amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
            const float kQMax = 8323072.0f;  // 2^23 - 2^16 keeps d0 in [-128, 127]
            const float inv = amax > 0.0f ? __fdiv_rn(kQMax, amax) : 0.0f;
            sq_own = amax > 0.0f ? __fdiv_rn(amax, kQMax) : 0.0f;
            const bool odd = gid & 1;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t w0 = 0, w1 = 0;
#pragma unroll
                    for (int x = 0; x < 4; ++x) {
                        const int qi = __float2int_rn(qv[8 * j + 4 * half + x] * inv);
                        const uint32_t d0 = (uint32_t)(qi >> 16) & 0xffu;
                        const uint32_t r = (uint32_t)qi & 0xffffu;
                        const uint32_t dl = odd ? (r & 0xffu) : (r >> 8);
                        w0 |= (live && !odd ? d0 : 0u) << (8 * x);
                        w1 |= (live ? dl : 0u) << (8 * x);
                    }
                    b_hi[j][half] = w0;
                    b_lo[j][half] = w1;
                }
            }
        }
        // scale of the head this thread's accumulator columns belong to (t4)
        const float sq = __shfl_sync(kFull, sq_own, (2 * t4) << 2);
        const bool head_live = t4 < GROUP;
        const float c16 = 65536.0f * sq, c8 = 256.0f * sq;
        float m_run = -INFINITY;      // running max of head t4 (log2 units)
        float l_part = 0.0f;          // this thread's share of head t4's sum

        for (int i = 0; i < ntiles; ++i) {
            const int s = i % kStages;
            const int b = i % kPBufs;
            if (!warp_wait(&full[s], (i / kStages) & 1)) { failed = true; break; }
            const uint8_t* st = stages + s * G::STAGE;
            const int8_t* kt = reinterpret_cast<const int8_t*>(st);
            const float* kst = reinterpret_cast<const float*>(st + 2 * G::KV_TILE);
            const float* vst = kst + G::T * HKV;
            const int valid = n - i * G::T;

            const int8_t* r0 = kt + (sw * 16 + gid) * G::ROWB + g * D + 32 * t4;
            const int8_t* r1 = r0 + 8 * G::ROWB;
            const uint4 a00 = *reinterpret_cast<const uint4*>(r0);
            const uint4 a01 = *reinterpret_cast<const uint4*>(r0 + 16);
            const uint4 a10 = *reinterpret_cast<const uint4*>(r1);
            const uint4 a11 = *reinterpret_cast<const uint4*>(r1 + 16);
            const uint32_t w0[8] = {a00.x, a00.y, a00.z, a00.w, a01.x, a01.y, a01.z, a01.w};
            const uint32_t w1[8] = {a10.x, a10.y, a10.z, a10.w, a11.x, a11.y, a11.z, a11.w};
            int acc_hi[4] = {0, 0, 0, 0}, acc_lo[4] = {0, 0, 0, 0};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                asm volatile(
                    "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
                    "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                    : "+r"(acc_hi[0]), "+r"(acc_hi[1]), "+r"(acc_hi[2]), "+r"(acc_hi[3])
                    : "r"(w0[2 * j]), "r"(w1[2 * j]), "r"(w0[2 * j + 1]), "r"(w1[2 * j + 1]),
                      "r"(b_hi[j][0]), "r"(b_hi[j][1]));
                asm volatile(
                    "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 "
                    "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                    : "+r"(acc_lo[0]), "+r"(acc_lo[1]), "+r"(acc_lo[2]), "+r"(acc_lo[3])
                    : "r"(w0[2 * j]), "r"(w1[2 * j]), "r"(w0[2 * j + 1]), "r"(w1[2 * j + 1]),
                      "r"(b_lo[j][0]), "r"(b_lo[j][1]));
            }
            // accumulator (row, col): c0 (gid, 2*t4) c1 (gid, 2*t4+1) c2/c3 rows gid+8
            const int tA = sw * 16 + gid, tB = tA + 8;
            float sA = fmaf((float)acc_hi[0], c16, fmaf((float)acc_lo[0], c8, (float)acc_lo[1] * sq));
            float sB = fmaf((float)acc_hi[2], c16, fmaf((float)acc_lo[2], c8, (float)acc_lo[3] * sq));
            sA = (head_live && tA < valid) ? sA * kst[tA * HKV + g] : -INFINITY;
            sB = (head_live && tB < valid) ? sB * kst[tB * HKV + g] : -INFINITY;

            // online softmax of head t4, base 2, lazy rescale
            float tm = fmaxf(sA, sB);
            tm = fmaxf(tm, __shfl_xor_sync(kFull, tm, 4));
            tm = fmaxf(tm, __shfl_xor_sync(kFull, tm, 8));
            tm = fmaxf(tm, __shfl_xor_sync(kFull, tm, 16));
            float corr = 1.0f;
            if (tm > m_run + kLazyRescale) {
                corr = exp2f(m_run - tm);
                m_run = tm;
            }
            l_part *= corr;
            const float pA = sA == -INFINITY ? 0.0f : exp2f(sA - m_run);
            const float pB = sB == -INFINITY ? 0.0f : exp2f(sB - m_run);
            l_part += pA + pB;

            if (i >= kPBufs && !warp_wait(&p_empty[pair * kPBufs + b], ((i / kPBufs) - 1) & 1)) {
                failed = true;
                break;
            }
            if (producer && i + kPrefetch < ntiles &&
                !issue_tile<HKV>(a, stages, full, empty, i + kPrefetch, n, slot0, pol, lane)) {
                failed = true;
                break;
            }
            float* pw = pslots + b * G::PSLOT;
            if (head_live) {
                pw[gid * 4 + t4] = pA == 0.0f ? 0.0f : pA * vst[tA * HKV + g];
                pw[(gid + 8) * 4 + t4] = pB == 0.0f ? 0.0f : pB * vst[tB * HKV + g];
                if (gid == 0) pw[64 + t4] = corr;
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&p_full[pair * kPBufs + b]);
                mbar_arrive(&empty[s]);
            }
        }
        l_part += __shfl_xor_sync(kFull, l_part, 4);
        l_part += __shfl_xor_sync(kFull, l_part, 8);
        l_part += __shfl_xor_sync(kFull, l_part, 16);
        consumer_barrier();   // every warp is done with the stage ring
        if (failed) {
            if (lane == 0) fail_flag = 1;
        } else if (gid == 0 && head_live) {
            mm[pair * GROUP + t4] = m_run;
            ml[pair * GROUP + t4] = l_part;
        }
    } else {
        // ======================================================== PV warps
        float2 acc_o[GROUP][8];
#pragma unroll
        for (int j = 0; j < GROUP; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) acc_o[j][e] = make_float2(0.f, 0.f);

        for (int i = 0; i < ntiles; ++i) {
            const int s = i % kStages;
            const int b = i % kPBufs;
            if (!warp_wait(&p_full[pair * kPBufs + b], (i / kPBufs) & 1)) { failed = true; break; }
            if (!warp_wait(&full[s], (i / kStages) & 1)) { failed = true; break; }
            const int8_t* vt = reinterpret_cast<const int8_t*>(stages + s * G::STAGE) + G::KV_TILE;
            const float* pw = pslots + b * G::PSLOT;
            float corr[GROUP];
            bool resc = false;
#pragma unroll
            for (int j = 0; j < GROUP; ++j) {
                corr[j] = pw[64 + j];
                resc |= corr[j] != 1.0f;
            }
            if (resc) {
#pragma unroll
                for (int j = 0; j < GROUP; ++j) {
                    const float2 cj = make_float2(corr[j], corr[j]);
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc_o[j][e] = __fmul2_rn(acc_o[j][e], cj);
                }
            }
#pragma unroll
            for (int it = 0; it < 4; ++it) {
                const int tw = it * 4 + tq;
                const int tt = sw * 16 + tw;
                float pp[4];
                if constexpr (GROUP == 4) {
                    const float4 p4 = *reinterpret_cast<const float4*>(pw + tw * 4);
                    pp[0] = p4.x; pp[1] = p4.y; pp[2] = p4.z; pp[3] = p4.w;
                } else if constexpr (GROUP == 2) {
                    const float2 p2 = *reinterpret_cast<const float2*>(pw + tw * 4);
                    pp[0] = p2.x; pp[1] = p2.y;
                } else {
                    pp[0] = pw[tw * 4];
                }
                const uint4 w = *reinterpret_cast<const uint4*>(vt + tt * G::ROWB + g * D + 16 * c);
                float2 vf[8];
                codes16_to_f2(w, vf);
#pragma unroll
                for (int j = 0; j < GROUP; ++j) {
                    const float2 pj = make_float2(pp[j], pp[j]);
#pragma unroll
                    for (int e = 0; e < 8; ++e) acc_o[j][e] = __ffma2_rn(pj, vf[e], acc_o[j][e]);
                }
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&p_empty[pair * kPBufs + b]);
                mbar_arrive(&empty[s]);
            }
        }
        // reduce the four row groups of the warp
#pragma unroll
        for (int j = 0; j < GROUP; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                float2 v = acc_o[j][e];
                v.x += __shfl_xor_sync(kFull, v.x, 8);
                v.y += __shfl_xor_sync(kFull, v.y, 8);
                v.x += __shfl_xor_sync(kFull, v.x, 16);
                v.y += __shfl_xor_sync(kFull, v.y, 16);
                acc_o[j][e] = v;
            }
        consumer_barrier();   // every warp is done with the stage ring
        if (failed) {
            if (lane == 0) fail_flag = 1;
        } else if (tq == 0) {
#pragma unroll
            for (int j = 0; j < GROUP; ++j)
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    *reinterpret_cast<float2*>(mo + (pair * GROUP + j) * D + 16 * c + 2 * e) = acc_o[j][e];
        }
    }
    consumer_barrier();
    if (fail_flag) return;

    // ---- merge the WPH pairs of each KV head and write the result
    const int H = a.num_heads;
    for (int o = threadIdx.x; o < HKV * GROUP * D; o += kConsumerWarps * 32) {
        const int d = o % D;
        const int hl = o / D;
        const int g2 = hl / GROUP, j = hl % GROUP;
        float M = -INFINITY;
#pragma unroll
        for (int w2 = 0; w2 < G::WPH; ++w2) M = fmaxf(M, mm[(g2 * G::WPH + w2) * GROUP + j]);
        float so = 0.0f, sl = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < G::WPH; ++w2) {
            const int w = g2 * G::WPH + w2;
            const float mw = mm[w * GROUP + j];
            const float f = mw == -INFINITY ? 0.0f : exp2f(mw - M);
            so += f * mo[(w * GROUP + j) * D + d];
            sl += f * ml[w * GROUP + j];
        }
        const int h = g2 + HKV * j;
        if (direct) {
            const size_t oi = ((size_t)seq * H + h) * D + d;
            if (a.mode == kOut) {
                a.out[oi] = __fdiv_rn(so, sl);
            } else {
                a.out[oi] = so;
                if (d == 0) {
                    a.out_ml[((size_t)seq * H + h) * 2] = M;
                    a.out_ml[((size_t)seq * H + h) * 2 + 1] = sl;
                }
            }
        } else {
            const size_t pidx = ((size_t)seq * a.max_chunks + chunk) * H + h;
            a.part_o[pidx * D + d] = so;
            if (d == 0) {
                a.part_ml[pidx * 2] = M;
                a.part_ml[pidx * 2 + 1] = sl;
            }
        }
    }
}

// Merges the chunk partials of one (sequence, head); one thread per dim.
__global__ void __launch_bounds__(D) combine_kernel(const DecodeArgs a) {
    const int seq = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const int H = a.num_heads;
    int32_t off, cap, len;
    if (!load_entry(a, seq, off, cap, len)) return;  // flagged by decode_kernel
    const int nch = (len + a.chunk_tokens - 1) / a.chunk_tokens;
    const size_t base = (size_t)seq * a.max_chunks * H + h;
    float M = -INFINITY;
    for (int c = 0; c < nch; ++c) M = fmaxf(M, a.part_ml[(base + (size_t)c * H) * 2]);
    float so = 0.0f, sl = 0.0f;
    for (int c = 0; c < nch; ++c) {
        const size_t p = base + (size_t)c * H;
        const float mc = a.part_ml[p * 2];
        const float f = mc == -INFINITY ? 0.0f : exp2f(mc - M);
        so += f * a.part_o[p * D + d];
        sl += f * a.part_ml[p * 2 + 1];
    }
    const size_t oi = ((size_t)seq * H + h) * D + d;
    if (a.mode == kOut) {
        a.out[oi] = nch ? __fdiv_rn(so, sl) : 0.0f;
    } else {
        a.out[oi] = so;
        if (d == 0) {
            a.out_ml[((size_t)seq * H + h) * 2] = nch ? M : -INFINITY;
            a.out_ml[((size_t)seq * H + h) * 2 + 1] = sl;
        }
    }
}

// Merges num_parts partial states stacked [part][seq][head] (context shards).
__global__ void __launch_bounds__(D) lse_merge_kernel(const float* __restrict__ part_o,
                                                      const float* __restrict__ part_ml,
                                                      int num_parts, int num_seqs, int H,
                                                      float* __restrict__ out) {
    const int seq = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const size_t stride = (size_t)num_seqs * H;
    const size_t sh = (size_t)seq * H + h;
    float M = -INFINITY;
    for (int p = 0; p < num_parts; ++p) M = fmaxf(M, part_ml[(p * stride + sh) * 2]);
    float so = 0.0f, sl = 0.0f;
    for (int p = 0; p < num_parts; ++p) {
        const size_t i = p * stride + sh;
        const float mp = part_ml[i * 2];
        const float f = mp == -INFINITY ? 0.0f : exp2f(mp - M);
        so += f * part_o[i * D + d];
        sl += f * part_ml[i * 2 + 1];
    }
    out[sh * D + d] = sl > 0.0f ? __fdiv_rn(so, sl) : 0.0f;
}

template <int HKV, int GROUP>
cudaError_t launch_decode_t(const DecodeArgs& a, const DecodePlan& plan, cudaStream_t st) {
    using G = Geo<HKV>;
    static unsigned long long attr_done = 0;  // one bit per device ordinal
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
    if (!bit || !(attr_done & bit)) {
        e = cudaFuncSetAttribute(decode_kernel<HKV, GROUP>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
        if (e != cudaSuccess) return e;
        attr_done |= bit;
    }
    dim3 grid(plan.max_chunks, a.num_seqs);
    decode_kernel<HKV, GROUP><<<grid, kThreads, G::SMEM, st>>>(a);
    return cudaGetLastError();
}

}  // namespace

DecodePlan plan_decode(int num_seqs, int max_seq_len, int num_sms) {
    DecodePlan best{32, 1};
    if (max_seq_len <= 0 || num_seqs <= 0) return best;
    const int gran = 32;
    const int tiles = (max_seq_len + gran - 1) / gran;
    double best_cost = 1e300;
    const int kmax = tiles < 256 ? tiles : 256;
    for (int k = 1; k <= kmax; ++k) {
        const int chunk = ((tiles + k - 1) / k) * gran;
        const int kk = (max_seq_len + chunk - 1) / chunk;
        const long long ctas = (long long)num_seqs * kk;
        const long long waves = (ctas + num_sms - 1) / num_sms;
        // per-CTA time ~ its tokens plus a fixed prologue; a combine pass when split
        const double cost = (double)waves * (chunk + 48) + (kk > 1 ? 64.0 : 0.0);
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = DecodePlan{chunk, kk};
        }
    }
    return best;
}

size_t decode_workspace_bytes(const DecodePlan& p, int num_seqs, int num_heads) {
    if (p.max_chunks <= 1) return 0;
    return (size_t)num_seqs * p.max_chunks * num_heads * (D + 2) * sizeof(float);
}

cudaError_t launch_decode(DecodeArgs a, int num_kv_heads, const DecodePlan& plan, void* ws,
                          cudaStream_t st) {
    a.chunk_tokens = plan.chunk_tokens;
    a.max_chunks = plan.max_chunks;
    if (plan.max_chunks > 1) {
        a.part_o = static_cast<float*>(ws);
        a.part_ml = a.part_o + (size_t)a.num_seqs * plan.max_chunks * a.num_heads * D;
    }
    const int group = a.num_heads / num_kv_heads;
    cudaError_t e = cudaErrorInvalidValue;
#define EC_DEC(H, GR) \
    if (num_kv_heads == H && group == GR) e = launch_decode_t<H, GR>(a, plan, st);
    EC_DEC(4, 4) EC_DEC(4, 2) EC_DEC(4, 1) EC_DEC(8, 4) EC_DEC(8, 2) EC_DEC(8, 1)
#undef EC_DEC
    if (e != cudaSuccess || plan.max_chunks <= 1) return e;
    combine_kernel<<<dim3(a.num_seqs, a.num_heads), D, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_lse_combine(const float* part_o, const float* part_ml, int num_parts,
                               int num_seqs, int num_heads, float* out, cudaStream_t st) {
    lse_merge_kernel<<<dim3(num_seqs, num_heads), D, 0, st>>>(part_o, part_ml, num_parts, num_seqs,
                                                              num_heads, out);
    return cudaGetLastError();
}

}  // namespace ec
