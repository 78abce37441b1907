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
// KV heads of it.  Tiles of 32 tokens stream through a shared-memory ring:
// per KV head one 2-D TMA copy of the K codes and one of the V codes (a
// [32 tokens x 128 B] box of the [slot][head][128] cache, 128-byte swizzled),
// plus one 1-D bulk copy per scale array.  No multicast.  Each KV head has
// one QK warp and one PV warp; they hand tiles of p' = p * v_scale to each
// other through a double-buffered slot guarded by mbarriers.  Every K and V
// byte is read from HBM exactly once per step.
//
// Both contractions run on the tensor cores as int8 mma.sync m16n8k32 with
// exact integer accumulation:
//   scores  S[t][h] = K_codes[t][:] . q_h      A = K codes (unconverted),
//           B = q_h split exactly into digits q_int = 65536*d0 + 256*d1 + d2
//           of a 24-bit per-head fixed-point scale (d0 signed, d1/d2 bytes);
//   output  O[h][d] += sum_t p'[h][t] * V_codes[t][d]
//                                              A = V codes transposed by
//           ldmatrix.trans.b8, B = p' per (head, tile) split into two bytes of
//           a 15-bit power-of-two scale.
// Integer sums are recombined in fp32.  The online softmax rescales only when
// a head's running maximum grows by more than 2^8 (exact: numerator and
// denominator always share the same reference maximum).
#include <cmath>
#include <cstdint>

#include <cuda.h>

#include "ec_common.cuh"
#include "ec_internal.h"

namespace ec {
namespace {

constexpr int D = 128;
constexpr int T = 32;                              // tokens per tile
constexpr int kPBufs = 2;                          // p' tiles in flight per head
constexpr int kDecodeCtasPerSm = 2;                // decode_kernel residency, HKV <= 4
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyRescale = 8.0f;
constexpr unsigned kFull = 0xffffffffu;

template <int HKV>
struct Geo {
    static constexpr int kWarps = 2 * HKV;                  // QK warps 0..HKV-1, PV warps HKV..
    static constexpr int kConsumerThreads = kWarps * 32;
    static constexpr int kThreads = kConsumerThreads + 32;   // + one producer warp
    static constexpr int HEAD_TILE = T * D;                 // 4 KB: one head's [32][128] box
    static constexpr int KV_TILE = HKV * HEAD_TILE;
    static constexpr int SC_TILE = T * HKV * 4;
    static constexpr int STAGE = 2 * KV_TILE + 2 * SC_TILE; // multiple of 1024
    // Two CTAs per SM for HKV <= 4 (three stages each, ~105 KB): one CTA's
    // prologue, pipeline fill and epilogue overlap the other's streaming.
    static constexpr int kCtasPerSm = HKV <= 4 ? kDecodeCtasPerSm : 1;
    static constexpr int kStages = 3;
    static constexpr int PSLOT = 4 * T + 4;                 // p'[4 heads][32 tokens], corr[4]
    static constexpr int PBUF = HKV * kPBufs * PSLOT * 4;
    static constexpr int NBARS = 2 * kStages + 2 * HKV * kPBufs;
    static constexpr int SMEM = 1024 /*alignment slack*/ + kStages * STAGE + PBUF + NBARS * 8;
    static_assert(STAGE % 1024 == 0, "swizzled boxes need 1024-byte aligned stages");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(kCtasPerSm * (SMEM + 1024) <= 228 * 1024, "resident CTAs per SM");
};

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// 2-D tiled TMA load (no multicast) with an L2 eviction hint.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Byte offset of 16-byte chunk `c` of row `r` inside a 128-byte-swizzled box.
__device__ __forceinline__ int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16x16 int8 block, rows = tokens, transposed: lane (g, t) gets the bytes of
// rows 4t..4t+3 at columns g (r0) and g + 8 (r1).
__device__ __forceinline__ void ldmatrix_t_b8(uint32_t& r0, uint32_t& r1, const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m16n16.x1.trans.shared.b8 {%0, %1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(smem_addr(row_addr)));
}

__device__ __forceinline__ bool load_entry(const DecodeArgs& a, int s, int32_t& off, int32_t& cap,
                                           int32_t& len) {
    off = a.seq_offset ? a.seq_offset[s] : a.host_offset;
    cap = a.seq_capacity ? a.seq_capacity[s] : a.host_capacity;
    len = a.seq_len ? a.seq_len[s] : a.host_length;
    // len is also bounded by the tokens the grid covers (max_chunks chunks),
    // which the host sized from its max_seq_len bound.
    return page_entry_ok(a.pages, off, cap, len, a.total_slots) &&
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

__device__ __forceinline__ void consumer_barrier(int threads) {
    asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// Issues tile j of the chunk into stage j % kStages (warp-collective; lane 0
// drives the copies).  Waits, bounded, until every consumer warp has released
// the stage's previous tile.  Returns false on a timeout.
template <int HKV>
__device__ __forceinline__ bool issue_tile(const DecodeArgs& a, const CUtensorMap* tk,
                                           const CUtensorMap* tv, uint8_t* stages, uint64_t* full,
                                           uint64_t* empty, int j, int n, int seq, int32_t off,
                                           int t0, uint64_t pol, int lane) {
    using G = Geo<HKV>;
    const int s = j % G::kStages;
    bool ok = true;
    if (lane == 0 && j >= G::kStages) ok = mbar_wait(&empty[s], ((j / G::kStages) - 1) & 1);
    ok = __shfl_sync(kFull, ok, 0);
    if (!ok) return false;
    const int ntok = min(T, n - j * T);
    // a tile never crosses a page (pages are multiples of 128 tokens); a bad
    // page id is flagged and slot 0 read instead, so that the pipeline still
    // completes and nothing outside the pool is touched
    int64_t slot;
    if (!page_slot(a.pages, seq, off, t0 + j * T, a.total_slots, slot)) {
        if (lane == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        slot = 0;
    }
    uint8_t* st = stages + s * G::STAGE;
    // the boxes always land whole (rows past the tensor are zero-filled)
    const uint32_t kvb = 2u * G::KV_TILE;
    if (!a.row_scales) {
        if (lane == 0) {
            const uint32_t scb = (uint32_t)ntok * HKV * 4;
            mbar_arrive_expect_tx(&full[s], kvb + 2 * scb);
#pragma unroll
            for (int g = 0; g < HKV; ++g) {
                tma_load_2d(st + g * G::HEAD_TILE, tk, g * D, (int)slot, &full[s], pol);
                tma_load_2d(st + G::KV_TILE + g * G::HEAD_TILE, tv, g * D, (int)slot, &full[s], pol);
            }
            bulk_g2s_hint(st + 2 * G::KV_TILE, a.key_scales + slot * HKV, scb, &full[s], pol);
            bulk_g2s_hint(st + 2 * G::KV_TILE + G::SC_TILE, a.val_scales + slot * HKV, scb, &full[s],
                          pol);
        }
    } else {
        // ROW scales: one fp32 per token, broadcast into the per-head tile
        // layout with plain loads; the arrive releases them to the consumers.
        if (lane == 0) {
            mbar_expect_tx(&full[s], kvb);
#pragma unroll
            for (int g = 0; g < HKV; ++g) {
                tma_load_2d(st + g * G::HEAD_TILE, tk, g * D, (int)slot, &full[s], pol);
                tma_load_2d(st + G::KV_TILE + g * G::HEAD_TILE, tv, g * D, (int)slot, &full[s], pol);
            }
        }
        float* ks = reinterpret_cast<float*>(st + 2 * G::KV_TILE);
        float* vs = ks + T * HKV;
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
__global__ void __launch_bounds__(Geo<HKV>::kThreads, Geo<HKV>::kCtasPerSm)
    decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                  const __grid_constant__ CUtensorMap tmap_v, const DecodeArgs a) {
    using G = Geo<HKV>;
    constexpr int S = G::kStages;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int fail_flag;
    uint8_t* stages = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* pbuf = reinterpret_cast<float*>(stages + S * G::STAGE);
    uint64_t* bars = reinterpret_cast<uint64_t*>(stages + S * G::STAGE + G::PBUF);
    uint64_t* full = bars;                           // [S]        TMA -> warps
    uint64_t* empty = full + S;                      // [S]        warps -> producer
    uint64_t* p_full = empty + S;                    // [HKV][kPBufs]  QK -> PV
    uint64_t* p_empty = p_full + HKV * kPBufs;       // [HKV][kPBufs]  PV -> QK

    const int seq = blockIdx.y;
    const int chunk = blockIdx.x;
    const bool direct = a.max_chunks == 1;
    pdl_wait();  // the append before this kernel writes the lengths and the codes
    pdl_trigger();
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
    const int ntiles = (n + T - 1) / T;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], G::kWarps);
        }
        for (int i = 0; i < HKV * kPBufs; ++i) {
            mbar_init(&p_full[i], 1);
            mbar_init(&p_empty[i], 1);
        }
        fail_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == G::kWarps) {
        // ============================================================ producer
        // Keeps the ring full: refills a stage as soon as every consumer warp
        // has released it, independent of the consumers' own progress.
        const uint64_t pol = l2_policy_evict_first();
        for (int j = 0; j < ntiles; ++j) {
            if (!issue_tile<HKV>(a, &tmap_k, &tmap_v, stages, full, empty, j, n, seq, off, t0, pol, lane)) {
                if (lane == 0) flag_error(a.err, EC_DEVERR_TIMEOUT);
                break;
            }
        }
        return;
    }

    const bool is_qk = warp < HKV;
    const int g = is_qk ? warp : warp - HKV;        // KV head of this warp
    const int gid = lane >> 2;
    const int t4 = lane & 3;
    const bool head_live = t4 < GROUP;              // accumulator columns belong to head t4
    float* pslots = pbuf + g * kPBufs * G::PSLOT;
    bool failed = false;
    // merge area (reused stage memory) for the final (m, l, O) per head
    float* mo = reinterpret_cast<float*>(stages);    // [HKV][GROUP][128]
    float* mm = mo + HKV * GROUP * D;                // [HKV][GROUP]
    float* ml = mm + HKV * GROUP;                    // [HKV][GROUP]

    if (is_qk) {
        // ================================================================ QK
        // q as B fragments: column n = gid <-> (head gid >> 1, digit), thread
        // t4 holds dims [32*t4, 32*t4 + 32), k-step j covers 8 of them.
        uint32_t b_hi[4][2], b_lo[4][2];
        float sq_own;
        {
            const int hq = gid >> 1;
            const bool live = hq < GROUP;
            const float* qp =
                a.q + ((size_t)seq * a.num_heads + g + HKV * (live ? hq : 0)) * D + 32 * t4;
            float qv[32];
            float amax = 0.0f;
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
            for (int j = 0; j < 4; ++j)
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
        const float sq = __shfl_sync(kFull, sq_own, (2 * t4) << 2);
        const float c16 = 65536.0f * sq, c8 = 256.0f * sq;
        float m_run = -INFINITY;      // running max of head t4 (log2 units)
        float l_part = 0.0f;          // this thread's share of head t4's sum

        for (int i = 0; i < ntiles; ++i) {
            const int s = i % S;
            const int b = i % kPBufs;
            if (!warp_wait(&full[s], (i / S) & 1)) { failed = true; break; }
            const uint8_t* st = stages + s * G::STAGE;
            const uint8_t* kt = st + g * G::HEAD_TILE;
            const float* kst = reinterpret_cast<const float*>(st + 2 * G::KV_TILE);
            const float* vst = kst + T * HKV;
            const int valid = n - i * T;

            float sc[4];   // tokens gid, gid+8, 16+gid, 24+gid of head t4
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const int ra = mt * 16 + gid, rb = ra + 8;
                const uint4 a00 = *reinterpret_cast<const uint4*>(kt + swz(ra, 2 * t4));
                const uint4 a01 = *reinterpret_cast<const uint4*>(kt + swz(ra, 2 * t4 + 1));
                const uint4 a10 = *reinterpret_cast<const uint4*>(kt + swz(rb, 2 * t4));
                const uint4 a11 = *reinterpret_cast<const uint4*>(kt + swz(rb, 2 * t4 + 1));
                const uint32_t w0[8] = {a00.x, a00.y, a00.z, a00.w, a01.x, a01.y, a01.z, a01.w};
                const uint32_t w1[8] = {a10.x, a10.y, a10.z, a10.w, a11.x, a11.y, a11.z, a11.w};
                int hi[4] = {0, 0, 0, 0}, lo[4] = {0, 0, 0, 0};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    mma_s8s8(hi, w0[2 * j], w1[2 * j], w0[2 * j + 1], w1[2 * j + 1], b_hi[j][0], b_hi[j][1]);
                    mma_s8u8(lo, w0[2 * j], w1[2 * j], w0[2 * j + 1], w1[2 * j + 1], b_lo[j][0], b_lo[j][1]);
                }
                // accumulator (row, col): [0] (ra, 2*t4) [1] (ra, 2*t4+1) [2]/[3] row rb
                const float sa = fmaf((float)hi[0], c16, fmaf((float)lo[0], c8, (float)lo[1] * sq));
                const float sb = fmaf((float)hi[2], c16, fmaf((float)lo[2], c8, (float)lo[3] * sq));
                sc[2 * mt] = (head_live && ra < valid) ? sa * kst[ra * HKV + g] : -INFINITY;
                sc[2 * mt + 1] = (head_live && rb < valid) ? sb * kst[rb * HKV + g] : -INFINITY;
            }

            // online softmax of head t4, base 2, lazy rescale
            float tm = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
            tm = fmaxf(tm, __shfl_xor_sync(kFull, tm, 4));
            tm = fmaxf(tm, __shfl_xor_sync(kFull, tm, 8));
            tm = fmaxf(tm, __shfl_xor_sync(kFull, tm, 16));
            float corr = 1.0f;
            if (tm > m_run + kLazyRescale) {
                corr = exp2f(m_run - tm);
                m_run = tm;
            }
            l_part *= corr;
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                p[e] = sc[e] == -INFINITY ? 0.0f : exp2f(sc[e] - m_run);
                l_part += p[e];
            }

            if (i >= kPBufs && !warp_wait(&p_empty[g * kPBufs + b], ((i / kPBufs) - 1) & 1)) {
                failed = true;
                break;
            }
            float* pw = pslots + b * G::PSLOT;   // p'[head][token], then corr[head]
            if (head_live) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int tok = (e >> 1) * 16 + (e & 1) * 8 + gid;
                    pw[t4 * T + tok] = p[e] == 0.0f ? 0.0f : p[e] * vst[tok * HKV + g];
                }
                if (gid == 0) pw[4 * T + t4] = corr;
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&p_full[g * kPBufs + b]);
                mbar_arrive(&empty[s]);
            }
        }
        l_part += __shfl_xor_sync(kFull, l_part, 4);
        l_part += __shfl_xor_sync(kFull, l_part, 8);
        l_part += __shfl_xor_sync(kFull, l_part, 16);
        consumer_barrier(G::kConsumerThreads);   // every warp is done with the stage ring
        if (failed) {
            if (lane == 0) fail_flag = 1;
        } else if (gid == 0 && head_live) {
            mm[g * GROUP + t4] = m_run;
            ml[g * GROUP + t4] = l_part;
        }
    } else {
        // ================================================================ PV
        // O^T[dim][col] += V^T[dim][token] . P[token][col], col = (head, digit)
        float acc[8][2];   // head t4, dims 16*mt + gid (+8)
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) acc[mt][0] = acc[mt][1] = 0.0f;
        const int hp = gid >> 1;           // head whose p' digits this thread supplies
        const bool p_live = hp < GROUP;
        const bool lo_digit = gid & 1;

        for (int i = 0; i < ntiles; ++i) {
            const int s = i % S;
            const int b = i % kPBufs;
            if (!warp_wait(&p_full[g * kPBufs + b], (i / kPBufs) & 1)) { failed = true; break; }
            if (!warp_wait(&full[s], (i / S) & 1)) { failed = true; break; }
            const uint8_t* vt = stages + s * G::STAGE + G::KV_TILE + g * G::HEAD_TILE;
            const float* pw = pslots + b * G::PSLOT;

            // p' digits as B fragments: tokens 4*t4.. (b0) and 16 + 4*t4.. (b1)
            float4 pa = make_float4(0.f, 0.f, 0.f, 0.f), pb = pa;
            if (p_live) {
                pa = *reinterpret_cast<const float4*>(pw + hp * T + 4 * t4);
                pb = *reinterpret_cast<const float4*>(pw + hp * T + 16 + 4 * t4);
            }
            float pmax = fmaxf(fmaxf(fmaxf(pa.x, pa.y), fmaxf(pa.z, pa.w)),
                               fmaxf(fmaxf(pb.x, pb.y), fmaxf(pb.z, pb.w)));
            pmax = fmaxf(pmax, __shfl_xor_sync(kFull, pmax, 1));
            pmax = fmaxf(pmax, __shfl_xor_sync(kFull, pmax, 2));
            // power-of-two scale putting the head's largest p' in [2^14, 2^15);
            // a tile whose p' all lie below 2^-100 (far under the running max,
            // with l >= 1) contributes nothing representable and is dropped.
            if (!(pmax >= 0x1p-100f)) {
                pa = make_float4(0.f, 0.f, 0.f, 0.f);
                pb = pa;
                pmax = 0.0f;
            }
            const int e = pmax > 0.0f ? ((__float_as_int(pmax) >> 23) & 0xff) - 127 : 0;
            const float up = __int_as_float((127 + 14 - e) << 23);
            const float down = __int_as_float((127 - 14 + e) << 23);
            uint32_t bw0 = 0, bw1 = 0;
            {
                const float va[4] = {pa.x, pa.y, pa.z, pa.w};
                const float vb[4] = {pb.x, pb.y, pb.z, pb.w};
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                    const uint32_t qa = (uint32_t)__float2int_rn(va[x] * up);
                    const uint32_t qb = (uint32_t)__float2int_rn(vb[x] * up);
                    bw0 |= (lo_digit ? (qa & 0xffu) : (qa >> 8)) << (8 * x);
                    bw1 |= (lo_digit ? (qb & 0xffu) : (qb >> 8)) << (8 * x);
                }
            }
            const float sp = __shfl_sync(kFull, down, (2 * t4) << 2);
            float corr = 1.0f;
            if (head_live) corr = pw[4 * T + t4];
            if (__any_sync(kFull, corr != 1.0f)) {
#pragma unroll
                for (int mt = 0; mt < 8; ++mt) {
                    acc[mt][0] *= corr;
                    acc[mt][1] *= corr;
                }
            }
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                // 16x16 blocks of V (tokens x dims 16*mt..): rows from lanes 0-15
                const int r = lane & 15;
                uint32_t x0, x1, y0, y1;
                ldmatrix_t_b8(x0, x1, vt + swz(r, mt));
                ldmatrix_t_b8(y0, y1, vt + swz(16 + r, mt));
                int d[4] = {0, 0, 0, 0};
                mma_s8u8(d, x0, x1, y0, y1, bw0, bw1);
                // d: (dim 16mt+gid, col 2t4 = hi digit of head t4), (.., lo), rows +8
                acc[mt][0] = fmaf((float)(d[0] * 256 + d[1]), sp, acc[mt][0]);
                acc[mt][1] = fmaf((float)(d[2] * 256 + d[3]), sp, acc[mt][1]);
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&p_empty[g * kPBufs + b]);
                mbar_arrive(&empty[s]);
            }
        }
        consumer_barrier(G::kConsumerThreads);   // every warp is done with the stage ring
        if (failed) {
            if (lane == 0) fail_flag = 1;
        } else if (head_live) {
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                mo[(g * GROUP + t4) * D + 16 * mt + gid] = acc[mt][0];
                mo[(g * GROUP + t4) * D + 16 * mt + gid + 8] = acc[mt][1];
            }
        }
    }
    consumer_barrier(G::kConsumerThreads);
    if (fail_flag) return;

    // ---- write the chunk's state (or the final output when unsplit)
    const int H = a.num_heads;
    for (int o = threadIdx.x; o < HKV * GROUP * D; o += G::kConsumerThreads) {
        const int d = o % D;
        const int hl = o / D;                 // g2 * GROUP + j
        const int g2 = hl / GROUP, j = hl % GROUP;
        const float M = mm[hl];
        const float so = mo[hl * D + d];
        const float sl = ml[hl];
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

// Merges the chunk partials of one (sequence, head).  4 warps per dim group:
// the chunk weights 2^(m_c - M) are computed once into shared memory, then
// each of kCombineSplit thread groups sums a quarter of the chunks for every
// dim (independent loads, so a long chunk list is not one serial chain).
constexpr int kCombineSplit = 4;
static_assert(D * kCombineSplit >= 256, "one thread per chunk: the plan allows 256 chunks");
__global__ void __launch_bounds__(D * kCombineSplit) combine_kernel(const DecodeArgs a) {
    const int seq = blockIdx.x, h = blockIdx.y;
    const int d = threadIdx.x % D, part = threadIdx.x / D;
    const int H = a.num_heads;
    pdl_wait();  // the partials of decode_kernel
    pdl_trigger();
    int32_t off, cap, len;
    if (!load_entry(a, seq, off, cap, len)) return;  // flagged by decode_kernel
    const int nch = (len + a.chunk_tokens - 1) / a.chunk_tokens;
    const size_t base = (size_t)seq * a.max_chunks * H + h;
    __shared__ float s_f[256], s_l[256], s_red[D * kCombineSplit];
    __shared__ float s_M;
    // chunk maxima -> M (the plan keeps nch <= 256 < the block's threads, so
    // thread c holds chunk c's (m, l) from the one load)
    const bool has_c = threadIdx.x < nch;
    float2 mlc = make_float2(-INFINITY, 0.0f);
    if (has_c) mlc = *reinterpret_cast<const float2*>(a.part_ml + (base + (size_t)threadIdx.x * H) * 2);
    float m = mlc.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float M = -INFINITY;
        for (int w = 0; w < D * kCombineSplit / 32; ++w) M = fmaxf(M, s_red[w]);
        s_M = M;
    }
    __syncthreads();
    const float M = s_M;
    if (has_c) {
        const float f = mlc.x == -INFINITY ? 0.0f : exp2f(mlc.x - M);
        s_f[threadIdx.x] = f;
        s_l[threadIdx.x] = f * mlc.y;
    }
    __syncthreads();
    float so = 0.0f;
#pragma unroll 4
    for (int c = part; c < nch; c += kCombineSplit)
        so += s_f[c] * a.part_o[(base + (size_t)c * H) * D + d];
    s_red[part * D + d] = so;
    __syncthreads();
    if (part != 0) return;
    so = 0.0f;
#pragma unroll
    for (int q = 0; q < kCombineSplit; ++q) so += s_red[q * D + d];
    float sl = 0.0f;
    for (int c = 0; c < nch; ++c) sl += s_l[c];
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
    static std::atomic<unsigned long long> attr_done{0};
    cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(decode_kernel<HKV, GROUP>),
                                      G::SMEM, attr_done);
    if (e != cudaSuccess) return e;
    CUtensorMap mk, mv;
    if ((e = make_code_map(&mk, a.keys, HKV, a.total_slots, T)) != cudaSuccess) return e;
    if ((e = make_code_map(&mv, a.values, HKV, a.total_slots, T)) != cudaSuccess) return e;
    dim3 grid(plan.max_chunks, a.num_seqs);
    return launch_pdl(decode_kernel<HKV, GROUP>, grid, dim3(G::kThreads), G::SMEM, st, mk, mv, a);
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// Tensor map over [total_slots][hkv * 128] int8 codes; box = one head's 128
// bytes x box_rows tokens, 128-byte swizzle.
cudaError_t make_code_map(CUtensorMap* m, const int8_t* base, int hkv, uint64_t total_slots,
                          int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)hkv * D, (cuuint64_t)total_slots};
    const cuuint64_t strides[1] = {(cuuint64_t)hkv * D};
    const cuuint32_t box[2] = {D, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Tensor map over [rows][hkv * 128] fp32 (the fp32 cache mode); box = one
// head's 128 floats x box_rows tokens, no swizzle.
cudaError_t make_f32_row_map(CUtensorMap* m, const float* base, int hkv, uint64_t rows,
                             int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {(cuuint64_t)hkv * D, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)hkv * D * sizeof(float)};
    const cuuint32_t box[2] = {D, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

DecodePlan plan_decode(int num_seqs, int max_seq_len, int num_sms, uint64_t total_tokens) {
    const int slots = num_sms * kDecodeCtasPerSm;  // resident CTAs (exact for HKV <= 4)
    DecodePlan best{T, 1};
    if (max_seq_len <= 0 || num_seqs <= 0) return best;
    const int tiles = (max_seq_len + T - 1) / T;
    double best_cost = 1e300;
    const int kmax = tiles < 256 ? tiles : 256;
    // with a token count below the all-full batch, the CTAs that find work
    // are about total / chunk plus half a chunk per sequence; the others exit
    // at once (about 16 tokens' worth of time each)
    const bool ragged = total_tokens > 0 && total_tokens < (uint64_t)num_seqs * max_seq_len;
    for (int k = 1; k <= kmax; ++k) {
        const int chunk = ((tiles + k - 1) / k) * T;
        const int kk = (max_seq_len + chunk - 1) / chunk;
        const long long ctas = (long long)num_seqs * kk;
        long long busy = ctas;
        if (ragged) {
            const double est = (double)total_tokens / chunk + 0.5 * num_seqs;
            busy = est < (double)ctas ? (long long)est + 1 : ctas;
        }
        const long long waves = (busy + slots - 1) / slots;
        // per-CTA time ~ its tokens plus a fixed prologue; a combine pass when
        // split, growing with the number of chunks it merges
        const double cost = (double)waves * (chunk + 48) + 16.0 * (double)(ctas - busy) / slots +
                            (kk > 1 ? 64.0 + 0.5 * kk : 0.0);
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
    return launch_pdl(combine_kernel, dim3(a.num_seqs, a.num_heads), dim3(D * kCombineSplit), 0, st, a);
}

cudaError_t launch_lse_combine(const float* part_o, const float* part_ml, int num_parts,
                               int num_seqs, int num_heads, float* out, cudaStream_t st) {
    lse_merge_kernel<<<dim3(num_seqs, num_heads), D, 0, st>>>(part_o, part_ml, num_parts, num_seqs,
                                                              num_heads, out);
    return cudaGetLastError();
}

}  // namespace ec
