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
// Work decomposition.  One CTA owns one (head block, chunk of tokens,
// sequence): HC consecutive KV heads of the sequence (all of them unless a
// large query group or head_dim 256 splits the heads over several CTAs).  The
// unit of work is a (KV head, quad of up to 4 of its query heads); a CTA
// holds HC * QW units, QW = ceil(group / 4).  Tiles of 32 tokens stream
// through a shared-memory ring: per KV head and 128-dim block one 2-D TMA copy
// of the K codes and one of the V codes (a [32 tokens x 128 B] box of the
// [slot][head][head_dim] cache, 128-byte swizzled), plus the tile's per-token
// scales (one 1-D bulk copy per scale array, or 4-byte cp.async copies when a
// token's scale row is not 16-byte sized).  No multicast.  Each unit has one
// QK warp and one PV warp; they hand tiles of p' = p * v_scale to each other
// through a double-buffered slot guarded by mbarriers.  Every K and V byte is
// read from HBM once per step by the CTA that owns its KV head.
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
#include <mutex>

#include <cuda.h>

#include "ec_common.cuh"
#include "ec_internal.h"

namespace ec {
namespace {

// Prefetch a __grid_constant__ tensor map (kernel parameter space) into the
// tensor-map cache ahead of the first TMA that uses it.
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

constexpr int D = 128;                             // dims per 128-byte box (one block)
constexpr int T = 32;                              // tokens per tile
constexpr int kPBufs = 2;                          // p' tiles in flight per head
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyRescale = 8.0f;
constexpr unsigned kFull = 0xffffffffu;

constexpr int kMaxChunks = 1024;                   // split-K chunks (or pieces) per sequence, at most
constexpr int kStreamMaxSeqs = 1024;               // stream-K plans: batches up to this size
constexpr int kStreamMinSeqs = 32;                 // ... and from this size

constexpr int kResidentSmem = 228 * 1024;   // shared memory per SM
constexpr int kCtaReservedSmem = 1024;      // reserved by the system per resident CTA

// HC KV heads per CTA, QW query-head quads per KV head, SCW scale words per
// token in a tile's scale arrays (the cache's num_kv_heads), DV 128-dim
// blocks per head (head_dim = 128 * DV).
template <int HC, int QW, int SCW, int DV>
struct Geo {
    static constexpr int DH = D * DV;                       // head_dim
    static constexpr int kUnits = HC * QW;                  // (KV head, query quad)
    static constexpr int kWarps = 2 * kUnits;               // QK warps 0..U-1, PV warps U..
    static constexpr int kConsumerThreads = kWarps * 32;
    static constexpr int kThreads = kConsumerThreads + 32;   // + one producer warp
    static constexpr int BOX = T * D;                       // 4 KB: one [32][128 B] box
    static constexpr int HEAD_TILE = DV * BOX;              // one head's DV boxes
    static constexpr int KV_TILE = HC * HEAD_TILE;
    static constexpr int SC_TILE = ((T * SCW * 4 + 511) / 512) * 512;
    static constexpr int STAGE = 2 * KV_TILE + 2 * SC_TILE; // multiple of 1024
    // Ring depth: three stages when a stage carries 4+ KV heads; a deeper
    // ring for the narrow stages of one or two KV heads, whose few resident
    // CTAs must still keep ~60 KB or more in flight per SM.
    static constexpr int kStages =
        HC >= 4 ? 3 : HC == 2 ? (QW >= 2 ? 4 : 3) : (QW >= 8 ? 8 : QW >= 4 ? 6 : 3);
    static constexpr int PSLOT = 4 * T + 4;                 // p'[4 heads][32 tokens], corr[4]
    static constexpr int PBUF = kUnits * kPBufs * PSLOT * 4;
    static constexpr int NBARS = 2 * kStages + 2 * kUnits * kPBufs;
    static constexpr int SMEM = 1024 /*alignment slack*/ + kStages * STAGE + PBUF + NBARS * 8;
    // Resident CTAs per SM: as many as shared memory and registers allow, at
    // most 8.  With several CTAs per SM one CTA's prologue, pipeline fill and
    // epilogue overlap another's streaming (two for 4 KV heads, ~105 KB each).
    // Registers: the QK and PV warps need about 96 a thread without spilling
    // at head_dim 128, about 112 at 256.
    static constexpr int kBySmem = kResidentSmem / (SMEM + kCtaReservedSmem);
    static constexpr int kByRegs = 65536 / (kThreads * (DV == 1 ? 96 : 112));
    static constexpr int kByRes = kBySmem < kByRegs ? kBySmem : kByRegs;
    static constexpr int kCtasPerSm = kByRes < 8 ? kByRes : 8;
    // SCW >= 4 scale rows are whole multiples of 16 bytes: one bulk copy each
    static constexpr bool kBulkScales = SCW % 4 == 0;
    static_assert(STAGE % 1024 == 0, "swizzled boxes need 1024-byte aligned stages");
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(kCtasPerSm >= 1, "resident CTAs per SM");
    static_assert(kUnits * 4 * (DH + 2) * 4 <= kStages * STAGE, "merge area fits the ring");
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

// 4-byte asynchronous copy global -> shared, and an arrive on `bar` that fires
// once every cp.async this thread issued before it has landed (the pending
// count is raised when this executes and lowered on completion, so the
// barrier's expected count is unchanged).
__device__ __forceinline__ void cp_async_4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
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
    const int dh = a.head_dim;
    for (int o = threadIdx.x; o < a.num_heads * dh; o += blockDim.x) {
        a.out[(size_t)seq * a.num_heads * dh + o] = 0.0f;
        if (a.mode == kPartial && (o % dh) == 0) {
            const int h = o / dh;
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
// the stage's previous tile.  Returns false on a timeout.  The stage holds the
// K and V boxes of KV heads g0 .. g0 + HC - 1 and every KV head's scales of
// the tile's tokens, [token][num_kv_heads].
template <int HC, int QW, int SCW, int DV>
__device__ __forceinline__ void issue_boxes(const CUtensorMap* tk, const CUtensorMap* tv,
                                            uint8_t* st, int g0, int64_t slot, uint64_t* bar,
                                            uint64_t pol) {
    using G = Geo<HC, QW, SCW, DV>;
#pragma unroll
    for (int g = 0; g < HC; ++g)
#pragma unroll
        for (int dv = 0; dv < DV; ++dv) {
            const int x = ((g0 + g) * DV + dv) * D;
            tma_load_2d(st + g * G::HEAD_TILE + dv * G::BOX, tk, x, (int)slot, bar, pol);
            tma_load_2d(st + G::KV_TILE + g * G::HEAD_TILE + dv * G::BOX, tv, x, (int)slot, bar,
                        pol);
        }
}

// The ring slot of a CTA's j-th tile overall is j % kStages: a CTA that
// streams several pieces (stream-K) keeps counting across them.  `tok` is the
// tile's first token in its sequence, ntok its tokens (<= 32).
template <int HC, int QW, int SCW, int DV>
__device__ __forceinline__ bool issue_tile_at(const DecodeArgs& a, const CUtensorMap* tk,
                                              const CUtensorMap* tv, uint8_t* stages,
                                              uint64_t* full, uint64_t* empty, int j, int ntok,
                                              int seq, int32_t off, int tok, int g0, uint64_t pol,
                                              int lane) {
    using G = Geo<HC, QW, SCW, DV>;
    const int s = j % G::kStages;
    bool ok = true;
    if (lane == 0 && j >= G::kStages) ok = mbar_wait(&empty[s], ((j / G::kStages) - 1) & 1);
    ok = __shfl_sync(kFull, ok, 0);
    if (!ok) return false;
    constexpr int hkv = SCW;   // the cache's num_kv_heads: variants are chosen by it
    // a tile never crosses a page (pages are multiples of 128 tokens); a bad
    // page id is flagged and slot 0 read instead, so that the pipeline still
    // completes and nothing outside the pool is touched
    int64_t slot;
    if (!page_slot(a.pages, seq, off, tok, a.total_slots, slot)) {
        if (lane == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        slot = 0;
    }
    uint8_t* st = stages + s * G::STAGE;
    float* ks = reinterpret_cast<float*>(st + 2 * G::KV_TILE);
    float* vs = reinterpret_cast<float*>(st + 2 * G::KV_TILE + G::SC_TILE);
    // the boxes always land whole (rows past the tensor are zero-filled)
    const uint32_t kvb = 2u * G::KV_TILE;
    if (!a.row_scales && G::kBulkScales) {
        if (lane == 0) {
            const uint32_t scb = (uint32_t)ntok * hkv * 4;
            mbar_arrive_expect_tx(&full[s], kvb + 2 * scb);
            issue_boxes<HC, QW, SCW, DV>(tk, tv, st, g0, slot, &full[s], pol);
            bulk_g2s_hint(ks, a.key_scales + slot * hkv, scb, &full[s], pol);
            bulk_g2s_hint(vs, a.val_scales + slot * hkv, scb, &full[s], pol);
        }
    } else if (!a.row_scales) {
        // scale rows of 1 or 2 floats: no 16-byte alignment to rely on, so
        // 4-byte cp.async copies, each lane's tracked by the stage barrier
        // (registered before lane 0's arrive, which the __syncwarp orders)
        const int nsc = ntok * hkv;
        for (int i = lane; i < nsc; i += 32) {
            cp_async_4(ks + i, a.key_scales + slot * hkv + i);
            cp_async_4(vs + i, a.val_scales + slot * hkv + i);
        }
        cp_async_mbar_arrive(&full[s]);
        __syncwarp();
        if (lane == 0) {
            mbar_arrive_expect_tx(&full[s], kvb);
            issue_boxes<HC, QW, SCW, DV>(tk, tv, st, g0, slot, &full[s], pol);
        }
    } else {
        // ROW scales: one fp32 per token, broadcast into the per-head tile
        // layout with plain loads; the arrive releases them to the consumers.
        if (lane == 0) {
            mbar_expect_tx(&full[s], kvb);
            issue_boxes<HC, QW, SCW, DV>(tk, tv, st, g0, slot, &full[s], pol);
        }
        for (int t = lane; t < ntok; t += 32) {
            const float kv = a.key_scales[slot + t];
            const float vv = a.val_scales[slot + t];
            for (int g = 0; g < hkv; ++g) {
                ks[t * hkv + g] = kv;
                vs[t * hkv + g] = vv;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&full[s]);
    }
    return true;
}

template <int HC, int QW, int SCW, int DV>
__device__ __forceinline__ bool issue_tile(const DecodeArgs& a, const CUtensorMap* tk,
                                           const CUtensorMap* tv, uint8_t* stages, uint64_t* full,
                                           uint64_t* empty, int j, int n, int seq, int32_t off,
                                           int t0, int g0, uint64_t pol, int lane) {
    return issue_tile_at<HC, QW, SCW, DV>(a, tk, tv, stages, full, empty, j, min(T, n - j * T),
                                          seq, off, t0 + j * T, g0, pol, lane);
}

// ---------------------------------------------------------- warp roles
// The QK and PV warps' work, shared by the chunked kernel (one piece of one
// sequence per CTA) and the stream-K kernel (a CTA's pieces back to back).
// `i` counts a CTA's tiles overall: it selects the ring stage and the p'
// buffer and their phases, so a CTA may run any number of pieces in a row.

// q of the quad's query heads (gkv + hkv * (jb + h), h < 4) of sequence seq
// as int8 B fragments of a 24-bit per-head fixed-point scale: column n =
// gid <-> (head jb + (gid >> 1), digit), thread t4 holds dims [32*t4, +32)
// of every 128-dim block, k-step j covers 8 of them (block j / 4).  Returns
// the fixed-point step of head jb + t4.
template <int DV>
__device__ __forceinline__ float qk_load_q(const DecodeArgs& a, int seq, int gkv, int jb,
                                           int group, int hkv, int lane,
                                           uint32_t (&b_hi)[4 * DV][2], uint32_t (&b_lo)[4 * DV][2]) {
    constexpr int DH = D * DV;
    const int gid = lane >> 2, t4 = lane & 3;
    float sq_own;
    {
        const int hq = gid >> 1;
        const bool live = jb + hq < group;
        // a quad past the group's end (groups that are not a multiple of
        // 4) reads query head 0 of the group and keeps no column live
        const float* qp =
            a.q + ((size_t)seq * a.num_heads + gkv + hkv * (live ? jb + hq : 0)) * DH + 32 * t4;
        auto scaled = [&](float v) { return __fmul_rn(__fmul_rn(v, a.q_mul), kLog2e); };
        // the head's absmax over all its blocks, then the digits block by
        // block: at head_dim 128 from the values kept in registers, at 256 by
        // loading each block again (L1 hits)
        float amax = 0.0f;
        float qv1[32];
#pragma unroll
        for (int dv = 0; dv < DV; ++dv)
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float4 v = reinterpret_cast<const float4*>(qp + dv * D)[e];
                const float x0 = scaled(v.x), x1 = scaled(v.y), x2 = scaled(v.z), x3 = scaled(v.w);
                if (DV == 1) {
                    qv1[4 * e + 0] = x0;
                    qv1[4 * e + 1] = x1;
                    qv1[4 * e + 2] = x2;
                    qv1[4 * e + 3] = x3;
                }
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x0), fabsf(x1)), fmaxf(fabsf(x2), fabsf(x3))));
            }
        amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, 2));
        const float kQMax = 8323072.0f;  // 2^23 - 2^16 keeps d0 in [-128, 127]
        const float inv = amax > 0.0f ? __fdiv_rn(kQMax, amax) : 0.0f;
        sq_own = amax > 0.0f ? __fdiv_rn(amax, kQMax) : 0.0f;
        const bool odd = gid & 1;
#pragma unroll
        for (int dv = 0; dv < DV; ++dv) {
            float qv[32];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                if (DV == 1) {
                    qv[4 * e + 0] = qv1[4 * e + 0];
                    qv[4 * e + 1] = qv1[4 * e + 1];
                    qv[4 * e + 2] = qv1[4 * e + 2];
                    qv[4 * e + 3] = qv1[4 * e + 3];
                } else {
                    const float4 v = reinterpret_cast<const float4*>(qp + dv * D)[e];
                    qv[4 * e + 0] = scaled(v.x);
                    qv[4 * e + 1] = scaled(v.y);
                    qv[4 * e + 2] = scaled(v.z);
                    qv[4 * e + 3] = scaled(v.w);
                }
            }
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
                    b_hi[4 * dv + j][half] = w0;
                    b_lo[4 * dv + j][half] = w1;
                }
        }
    }
    return __shfl_sync(kFull, sq_own, (2 * t4) << 2);
}

// One tile of a QK warp: the quad's scores of the tile's `valid` tokens,
// the online softmax of head jb + t4 (base 2, lazy rescale) and p' = p *
// v_scale handed to the unit's PV warp.  False when a bounded wait ran out.
template <int HC, int QW, int SCW, int DV>
__device__ __forceinline__ bool qk_tile(const DecodeArgs& a, uint8_t* stages, uint64_t* full,
                                        uint64_t* empty, uint64_t* p_full, uint64_t* p_empty,
                                        float* pslots, int i, int valid, int u, int gl, int gkv,
                                        bool head_live, int lane, const uint32_t (&b_hi)[4 * DV][2],
                                        const uint32_t (&b_lo)[4 * DV][2], float sq, float& m_run,
                                        float& l_part) {
    using G = Geo<HC, QW, SCW, DV>;
    constexpr int S = G::kStages;
    const int gid = lane >> 2, t4 = lane & 3;
    constexpr int hkv = SCW;   // the cache's num_kv_heads: variants are chosen by it
    const float c16 = 65536.0f * sq, c8 = 256.0f * sq;
    const int s = i % S;
    const int b = i % kPBufs;
    if (!warp_wait(&full[s], (i / S) & 1)) return false;
    const uint8_t* st = stages + s * G::STAGE;
    const uint8_t* kt = st + gl * G::HEAD_TILE;
    const float* kst = reinterpret_cast<const float*>(st + 2 * G::KV_TILE);
    const float* vst = reinterpret_cast<const float*>(st + 2 * G::KV_TILE + G::SC_TILE);

    float sc[4];   // tokens gid, gid+8, 16+gid, 24+gid of head jb + t4
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
        const int ra = mt * 16 + gid, rb = ra + 8;
        int hi[4] = {0, 0, 0, 0}, lo[4] = {0, 0, 0, 0};
#pragma unroll
        for (int dv = 0; dv < DV; ++dv) {
            const uint8_t* kb = kt + dv * G::BOX;
            const uint4 a00 = *reinterpret_cast<const uint4*>(kb + swz(ra, 2 * t4));
            const uint4 a01 = *reinterpret_cast<const uint4*>(kb + swz(ra, 2 * t4 + 1));
            const uint4 a10 = *reinterpret_cast<const uint4*>(kb + swz(rb, 2 * t4));
            const uint4 a11 = *reinterpret_cast<const uint4*>(kb + swz(rb, 2 * t4 + 1));
            const uint32_t w0[8] = {a00.x, a00.y, a00.z, a00.w, a01.x, a01.y, a01.z, a01.w};
            const uint32_t w1[8] = {a10.x, a10.y, a10.z, a10.w, a11.x, a11.y, a11.z, a11.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                mma_s8s8(hi, w0[2 * j], w1[2 * j], w0[2 * j + 1], w1[2 * j + 1],
                         b_hi[4 * dv + j][0], b_hi[4 * dv + j][1]);
                mma_s8u8(lo, w0[2 * j], w1[2 * j], w0[2 * j + 1], w1[2 * j + 1],
                         b_lo[4 * dv + j][0], b_lo[4 * dv + j][1]);
            }
        }
        // accumulator (row, col): [0] (ra, 2*t4) [1] (ra, 2*t4+1) [2]/[3] row rb
        const float sa = fmaf((float)hi[0], c16, fmaf((float)lo[0], c8, (float)lo[1] * sq));
        const float sb = fmaf((float)hi[2], c16, fmaf((float)lo[2], c8, (float)lo[3] * sq));
        sc[2 * mt] = (head_live && ra < valid) ? sa * kst[ra * hkv + gkv] : -INFINITY;
        sc[2 * mt + 1] = (head_live && rb < valid) ? sb * kst[rb * hkv + gkv] : -INFINITY;
    }

    // online softmax of head jb + t4, base 2, lazy rescale
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

    if (i >= kPBufs && !warp_wait(&p_empty[u * kPBufs + b], ((i / kPBufs) - 1) & 1)) return false;
    float* pw = pslots + b * G::PSLOT;   // p'[head][token], then corr[head]
    if (head_live) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int tok = (e >> 1) * 16 + (e & 1) * 8 + gid;
            pw[t4 * T + tok] = p[e] == 0.0f ? 0.0f : p[e] * vst[tok * hkv + gkv];
        }
        if (gid == 0) pw[4 * T + t4] = corr;
    }
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(&p_full[u * kPBufs + b]);
        mbar_arrive(&empty[s]);
    }
    return true;
}

// One tile of a PV warp: O^T[dim][col] += V^T[dim][token] . P[token][col],
// col = (head, digit), with the QK warp's rescale factor applied first.
template <int HC, int QW, int SCW, int DV>
__device__ __forceinline__ bool pv_tile(uint8_t* stages, uint64_t* full, uint64_t* empty,
                                        uint64_t* p_full, uint64_t* p_empty, float* pslots, int i,
                                        int u, int gl, int jb, int group, bool head_live, int lane,
                                        float (&acc)[8 * DV][2]) {
    using G = Geo<HC, QW, SCW, DV>;
    constexpr int S = G::kStages;
    const int gid = lane >> 2, t4 = lane & 3;
    const int hp = gid >> 1;           // head (in the quad) whose p' digits this thread supplies
    const bool p_live = jb + hp < group;
    const bool lo_digit = gid & 1;
    const int s = i % S;
    const int b = i % kPBufs;
    if (!warp_wait(&p_full[u * kPBufs + b], (i / kPBufs) & 1)) return false;
    if (!warp_wait(&full[s], (i / S) & 1)) return false;
    const uint8_t* vt = stages + s * G::STAGE + G::KV_TILE + gl * G::HEAD_TILE;
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
        for (int mt = 0; mt < 8 * DV; ++mt) {
            acc[mt][0] *= corr;
            acc[mt][1] *= corr;
        }
    }
#pragma unroll
    for (int mt = 0; mt < 8 * DV; ++mt) {
        // 16x16 blocks of V (tokens x dims 16*mt..): rows from lanes 0-15
        const int r = lane & 15;
        const uint8_t* vb = vt + (mt >> 3) * G::BOX;
        uint32_t x0, x1, y0, y1;
        ldmatrix_t_b8(x0, x1, vb + swz(r, mt & 7));
        ldmatrix_t_b8(y0, y1, vb + swz(16 + r, mt & 7));
        int d[4] = {0, 0, 0, 0};
        mma_s8u8(d, x0, x1, y0, y1, bw0, bw1);
        // d: (dim 16mt+gid, col 2t4 = hi digit of head t4), (.., lo), rows +8
        acc[mt][0] = fmaf((float)(d[0] * 256 + d[1]), sp, acc[mt][0]);
        acc[mt][1] = fmaf((float)(d[2] * 256 + d[3]), sp, acc[mt][1]);
    }
    __syncwarp();
    if (lane == 0) {
        mbar_arrive(&p_empty[u * kPBufs + b]);
        mbar_arrive(&empty[s]);
    }
    return true;
}

// Ring and handoff barriers (thread 0).
template <int HC, int QW, int SCW, int DV>
__device__ __forceinline__ void init_barriers(uint64_t* full, uint64_t* empty, uint64_t* p_full,
                                              uint64_t* p_empty) {
    using G = Geo<HC, QW, SCW, DV>;
    for (int s = 0; s < G::kStages; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], G::kWarps);
    }
    for (int i = 0; i < G::kUnits * kPBufs; ++i) {
        mbar_init(&p_full[i], 1);
        mbar_init(&p_empty[i], 1);
    }
    fence_mbar_init();
}

template <int HC, int QW, int SCW, int DV>
__global__ void __launch_bounds__(Geo<HC, QW, SCW, DV>::kThreads, Geo<HC, QW, SCW, DV>::kCtasPerSm)
    decode_kernel(const __grid_constant__ CUtensorMap tmap_k,
                  const __grid_constant__ CUtensorMap tmap_v, const DecodeArgs a) {
    using G = Geo<HC, QW, SCW, DV>;
    constexpr int DH = G::DH;
    constexpr int S = G::kStages;
    constexpr int U = G::kUnits;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int fail_flag;
    uint8_t* stages = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* pbuf = reinterpret_cast<float*>(stages + S * G::STAGE);
    uint64_t* bars = reinterpret_cast<uint64_t*>(stages + S * G::STAGE + G::PBUF);
    uint64_t* full = bars;                           // [S]        TMA -> warps
    uint64_t* empty = full + S;                      // [S]        warps -> producer
    uint64_t* p_full = empty + S;                    // [U][kPBufs]  QK -> PV
    uint64_t* p_empty = p_full + U * kPBufs;         // [U][kPBufs]  PV -> QK

    const int g0 = blockIdx.x * HC;                  // first KV head of this CTA
    const int chunk = blockIdx.y;
    const int seq = blockIdx.z;
    const bool direct = a.max_chunks == 1 && a.mode != kChunks;
    // shared-memory set-up and the tensor maps' prefetch overlap the kernel
    // before this one: neither reads memory that kernel writes
    if (threadIdx.x == 0) {
        init_barriers<HC, QW, SCW, DV>(full, empty, p_full, p_empty);
        fail_flag = 0;
        prefetch_tensormap(&tmap_k);
        prefetch_tensormap(&tmap_v);
    }
    pdl_wait();  // the append before this kernel writes the lengths and the codes
    pdl_trigger();
    int32_t off, cap, len;
    if (!load_entry(a, seq, off, cap, len)) {
        if (chunk == 0 && blockIdx.x == 0 && threadIdx.x == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        return;
    }
    const int t0 = chunk * a.chunk_tokens;
    if (t0 >= len) {
        if (direct && chunk == 0 && blockIdx.x == 0) write_empty(a, seq);
        return;
    }
    const int n = min(a.chunk_tokens, len - t0);
    const int ntiles = (n + T - 1) / T;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    constexpr int hkv = SCW;   // the cache's num_kv_heads: variants are chosen by it
    const int group = a.num_heads / hkv;
    __syncthreads();   // the barrier inits

    if (warp == G::kWarps) {
        // ============================================================ producer
        // Keeps the ring full: refills a stage as soon as every consumer warp
        // has released it, independent of the consumers' own progress.
        const uint64_t pol = l2_policy_evict_first();
        for (int j = 0; j < ntiles; ++j) {
            if (!issue_tile<HC, QW, SCW, DV>(a, &tmap_k, &tmap_v, stages, full, empty, j, n, seq,
                                             off, t0, g0, pol, lane)) {
                if (lane == 0) flag_error(a.err, EC_DEVERR_TIMEOUT);
                break;
            }
        }
        return;
    }

    const bool is_qk = warp < U;
    const int u = is_qk ? warp : warp - U;           // unit of this warp
    const int gl = u / QW;                           // KV head within the CTA
    const int gkv = g0 + gl;                         // KV head in the cache row
    const int jb = 4 * (u % QW);                     // first query head of the quad in the group
    const int gid = lane >> 2;
    const int t4 = lane & 3;
    const bool head_live = jb + t4 < group;          // accumulator columns belong to head jb + t4
    float* pslots = pbuf + u * kPBufs * G::PSLOT;
    bool failed = false;
    // merge area (reused stage memory) for the final (m, l, O) per head slot
    float* mo = reinterpret_cast<float*>(stages);    // [U][4][head_dim]
    float* mm = mo + U * 4 * DH;                     // [U][4]
    float* ml = mm + U * 4;                          // [U][4]

    if (is_qk) {
        // ================================================================ QK
        uint32_t b_hi[4 * DV][2], b_lo[4 * DV][2];
        const float sq = qk_load_q<DV>(a, seq, gkv, jb, group, hkv, lane, b_hi, b_lo);
        float m_run = -INFINITY;      // running max of head jb + t4 (log2 units)
        float l_part = 0.0f;          // this thread's share of that head's sum
        for (int i = 0; i < ntiles; ++i) {
            if (!qk_tile<HC, QW, SCW, DV>(a, stages, full, empty, p_full, p_empty, pslots, i,
                                          n - i * T, u, gl, gkv, head_live, lane, b_hi, b_lo, sq,
                                          m_run, l_part)) {
                failed = true;
                break;
            }
        }
        l_part += __shfl_xor_sync(kFull, l_part, 4);
        l_part += __shfl_xor_sync(kFull, l_part, 8);
        l_part += __shfl_xor_sync(kFull, l_part, 16);
        consumer_barrier(G::kConsumerThreads);   // every warp is done with the stage ring
        if (failed) {
            if (lane == 0) fail_flag = 1;
        } else if (gid == 0 && head_live) {
            mm[u * 4 + t4] = m_run;
            ml[u * 4 + t4] = l_part;
        }
    } else {
        // ================================================================ PV
        float acc[8 * DV][2];   // head jb + t4, dims 16*mt + gid (+8)
#pragma unroll
        for (int mt = 0; mt < 8 * DV; ++mt) acc[mt][0] = acc[mt][1] = 0.0f;
        for (int i = 0; i < ntiles; ++i) {
            if (!pv_tile<HC, QW, SCW, DV>(stages, full, empty, p_full, p_empty, pslots, i, u, gl,
                                          jb, group, head_live, lane, acc)) {
                failed = true;
                break;
            }
        }
        consumer_barrier(G::kConsumerThreads);   // every warp is done with the stage ring
        if (failed) {
            if (lane == 0) fail_flag = 1;
        } else if (head_live) {
#pragma unroll
            for (int mt = 0; mt < 8 * DV; ++mt) {
                mo[(u * 4 + t4) * DH + 16 * mt + gid] = acc[mt][0];
                mo[(u * 4 + t4) * DH + 16 * mt + gid + 8] = acc[mt][1];
            }
        }
    }
    consumer_barrier(G::kConsumerThreads);
    if (fail_flag) return;

    // ---- write the chunk's state (or the final output when unsplit)
    const int H = a.num_heads;
    for (int o = threadIdx.x; o < U * 4 * DH; o += G::kConsumerThreads) {
        const int d = o % DH;
        const int hl = o / DH;                // u2 * 4 + quad slot
        const int u2 = hl >> 2;
        const int j = 4 * (u2 % QW) + (hl & 3);
        if (j >= group) continue;
        const int h = (g0 + u2 / QW) + hkv * j;
        const float M = mm[hl];
        const float so = mo[hl * DH + d];
        const float sl = ml[hl];
        if (direct) {
            const size_t oi = ((size_t)seq * H + h) * DH + d;
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
            a.part_o[pidx * DH + d] = so;
            if (d == 0) {
                a.part_ml[pidx * 2] = M;
                a.part_ml[pidx * 2 + 1] = sl;
            }
        }
    }
}

// ------------------------------------------------------------ stream-K
// The batch's tiles in sequence order, 0 .. TT-1, are split evenly over the
// grid's first Ce = min(C, TT) CTAs (of every head block): CTA c takes
// [c*TT/Ce, (c+1)*TT/Ce), at least one tile, so every CTA streams the same
// number of tiles whatever the lengths, in one wave.  Its range meets one or more sequences; each (CTA c, sequence s)
// intersection is a piece whose unnormalised (m, l, O) goes to workspace row
// c + s (distinct for distinct non-empty pieces: they are ordered in both c
// and s), and the merge kernel combines a sequence's pieces.

// Tiles of sequence s (0 for an entry outside its bounds: flagged apart).
__device__ __forceinline__ int sk_tiles(const DecodeArgs& a, int s) {
    int32_t off, cap, len;
    if (!load_entry(a, s, off, cap, len)) return 0;
    return (len + T - 1) / T;
}

// The CTA whose range holds global tile t.
__device__ __forceinline__ int sk_cta_of(long long t, long long TT, int C) {
    return (int)(((t + 1) * C - 1) / TT);
}

// Sequences a thread covers in the stream-K table pass: thread t takes
// sequences [t*kSkPerThread, (t+1)*kSkPerThread), so the smallest CTA (96
// threads) covers kStreamMaxSeqs of them.
constexpr int kSkPerThread = 11;
static_assert(kSkPerThread * 96 >= kStreamMaxSeqs, "stream-K table pass covers the batch");

// One block-wide pass over the length table (every thread calls it): the
// batch's tile count TT; the split over Ce = min(C, TT) CTAs, each of which
// then owns at least one tile (the merge counts on every CTA of a sequence's
// range having written its piece); CTA c's tile range [lo, hi) (empty for
// c >= Ce); the sequence holding tile lo and the tiles before it.  With
// `prefix` set, the tiles before every sequence go to prefix[0 ..
// num_seqs - 1] and TT to prefix[num_seqs], for the merge kernel.  Tile
// indices fit int: a batch holds fewer than 2^31 slots.
__device__ void sk_locate(const DecodeArgs& a, int c, int C, int32_t* prefix, int& lo, int& hi,
                          int& s_at, int& p_at) {
    __shared__ long long s_warp[32];
    __shared__ int s_res[2];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int nw = (blockDim.x + 31) >> 5;
    const int s_beg = tid * kSkPerThread;
    int v[kSkPerThread];
    long long mine = 0;
#pragma unroll
    for (int k = 0; k < kSkPerThread; ++k) {
        v[k] = s_beg + k < a.num_seqs ? sk_tiles(a, s_beg + k) : 0;
        mine += v[k];
    }
    if (tid == 0) {
        s_res[0] = -1;
        s_res[1] = 0;
    }
    long long x = mine;                           // inclusive scan over the block
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(kFull, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[wid] = x;
    __syncthreads();
    if (wid == 0) {
        long long w = lane < nw ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const long long y = __shfl_up_sync(kFull, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) s_warp[lane] = w;
    }
    __syncthreads();
    const long long TT = s_warp[nw - 1];
    const int Ce = (int)(TT < C ? TT : C);
    lo = c < Ce ? (int)((long long)c * TT / Ce) : 0;
    hi = c < Ce ? (int)((long long)(c + 1) * TT / Ce) : 0;
    int e = (int)((wid ? s_warp[wid - 1] : 0) + x - mine);   // tiles before s_beg
#pragma unroll
    for (int k = 0; k < kSkPerThread; ++k) {
        if (prefix && s_beg + k < a.num_seqs) prefix[s_beg + k] = e;
        if (lo < hi && v[k] > 0 && e <= lo && lo < e + v[k]) {
            s_res[0] = s_beg + k;
            s_res[1] = e;
        }
        e += v[k];
    }
    if (prefix && tid == 0) prefix[a.num_seqs] = (int32_t)TT;
    __syncthreads();
    s_at = s_res[0];
    p_at = s_res[1];
}

template <int HC, int QW, int SCW, int DV>
__global__ void __launch_bounds__(Geo<HC, QW, SCW, DV>::kThreads, Geo<HC, QW, SCW, DV>::kCtasPerSm)
    decode_sk_kernel(const __grid_constant__ CUtensorMap tmap_k,
                     const __grid_constant__ CUtensorMap tmap_v, const DecodeArgs a) {
    using G = Geo<HC, QW, SCW, DV>;
    constexpr int DH = G::DH;
    constexpr int S = G::kStages;
    constexpr int U = G::kUnits;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* stages = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* pbuf = reinterpret_cast<float*>(stages + S * G::STAGE);
    uint64_t* bars = reinterpret_cast<uint64_t*>(stages + S * G::STAGE + G::PBUF);
    uint64_t* full = bars;
    uint64_t* empty = full + S;
    uint64_t* p_full = empty + S;
    uint64_t* p_empty = p_full + U * kPBufs;

    const int g0 = blockIdx.x * HC;
    const int cta = blockIdx.y, C = a.sk_ctas;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    constexpr int hkv = SCW;   // the cache's num_kv_heads: variants are chosen by it
    const int group = a.num_heads / hkv;
    const int H = a.num_heads;
    if (threadIdx.x == 0) {   // before the wait: reads nothing the previous kernel writes
        init_barriers<HC, QW, SCW, DV>(full, empty, p_full, p_empty);
        prefetch_tensormap(&tmap_k);
        prefetch_tensormap(&tmap_v);
    }
    pdl_wait();  // the append before this kernel writes the lengths and the codes
    pdl_trigger();
    if (cta == 0 && blockIdx.x == 0) {
        for (int s = threadIdx.x; s < a.num_seqs; s += blockDim.x) {
            int32_t off, cap, len;
            if (!load_entry(a, s, off, cap, len)) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        }
    }
    // the table pass (its barriers also publish the barrier inits); CTA 0 of
    // head block 0 leaves the per-sequence tile prefix for the merge kernel
    int32_t* prefix = (cta == 0 && blockIdx.x == 0) ? a.sk_prefix : nullptr;
    int lo, hi, s0, p0;
    sk_locate(a, cta, C, prefix, lo, hi, s0, p0);
    if (lo >= hi) return;

    if (warp == G::kWarps) {
        // ============================================================ producer
        const uint64_t pol = l2_policy_evict_first();
        int gj = 0;
        int p = p0;
        for (int s = s0; s < a.num_seqs && p < hi; ++s) {
            int32_t off, cap, len;
            const int nt = load_entry(a, s, off, cap, len) ? (len + T - 1) / T : 0;
            const int t_lo = max(lo, p), t_hi = min(hi, p + nt);
            for (int t = t_lo; t < t_hi; ++t, ++gj) {
                const int tok = (t - p) * T;
                if (!issue_tile_at<HC, QW, SCW, DV>(a, &tmap_k, &tmap_v, stages, full, empty, gj,
                                                    min(T, len - tok), s, off, tok, g0, pol, lane)) {
                    if (lane == 0) flag_error(a.err, EC_DEVERR_TIMEOUT);
                    return;
                }
            }
            p += nt;
        }
        return;
    }

    const bool is_qk = warp < U;
    const int u = is_qk ? warp : warp - U;
    const int gl = u / QW;
    const int gkv = g0 + gl;
    const int jb = 4 * (u % QW);
    const int gid = lane >> 2;
    const int t4 = lane & 3;
    const bool head_live = jb + t4 < group;
    const int h_out = gkv + hkv * (jb + t4);         // the head this thread's columns belong to
    float* pslots = pbuf + u * kPBufs * G::PSLOT;
    int gi = 0;
    int p = p0;
    for (int s = s0; s < a.num_seqs && p < hi; ++s) {
        int32_t off, cap, len;
        const int nt = load_entry(a, s, off, cap, len) ? (len + T - 1) / T : 0;
        const int t_lo = max(lo, p), t_hi = min(hi, p + nt);
        const int first_tok = (t_lo - p) * T;       // the piece's first token in sequence s
        p += nt;
        if (t_lo >= t_hi) continue;
        const size_t row = (size_t)(cta + s) * H;    // this piece's partial rows
        if (is_qk) {
            uint32_t b_hi[4 * DV][2], b_lo[4 * DV][2];
            const float sq = qk_load_q<DV>(a, s, gkv, jb, group, hkv, lane, b_hi, b_lo);
            float m_run = -INFINITY, l_part = 0.0f;
            for (int t = t_lo, tok = first_tok; t < t_hi; ++t, ++gi, tok += T) {
                if (!qk_tile<HC, QW, SCW, DV>(a, stages, full, empty, p_full, p_empty, pslots, gi,
                                              len - tok, u, gl, gkv, head_live, lane, b_hi, b_lo,
                                              sq, m_run, l_part)) {
                    if (lane == 0) flag_error(a.err, EC_DEVERR_TIMEOUT);
                    return;
                }
            }
            l_part += __shfl_xor_sync(kFull, l_part, 4);
            l_part += __shfl_xor_sync(kFull, l_part, 8);
            l_part += __shfl_xor_sync(kFull, l_part, 16);
            if (gid == 0 && head_live) {
                a.part_ml[(row + h_out) * 2] = m_run;
                a.part_ml[(row + h_out) * 2 + 1] = l_part;
            }
        } else {
            float acc[8 * DV][2];
#pragma unroll
            for (int mt = 0; mt < 8 * DV; ++mt) acc[mt][0] = acc[mt][1] = 0.0f;
            for (int t = t_lo; t < t_hi; ++t, ++gi) {
                if (!pv_tile<HC, QW, SCW, DV>(stages, full, empty, p_full, p_empty, pslots, gi, u,
                                              gl, jb, group, head_live, lane, acc)) {
                    if (lane == 0) flag_error(a.err, EC_DEVERR_TIMEOUT);
                    return;
                }
            }
            if (head_live) {
                float* po = a.part_o + (row + h_out) * DH;
#pragma unroll
                for (int mt = 0; mt < 8 * DV; ++mt) {
                    po[16 * mt + gid] = acc[mt][0];
                    po[16 * mt + gid + 8] = acc[mt][1];
                }
            }
        }
    }
}

// Merges the chunk partials of one (sequence, head): the maximum M of the
// chunk maxima, the weights 2^(m_c - M) (kept in shared memory), L = the
// weighted sum of l, and O = the weighted sum of the chunks' O rows.  The
// head's dims are split over gridDim.z CTAs (8 when the batch has few
// (sequence, head) pairs, so that one long sequence's merge is spread over
// many SMs instead of a few).  A CTA's threads are float4 column groups x
// chunk lanes; each issues its first kBatch O loads together with the (m, l)
// loads, before M is known, so that a merge of a few hundred chunks is two
// dependent global round trips (table entry, then partials) instead of a
// chain.  Reductions run in a fixed order: the result does not depend on
// timing.
// NT threads at up to 64 registers: 256, or 128 for many (sequence, head)
// pairs of one 128-dim block each (eight CTAs an SM, so up to 1,184 pairs run in
// one wave); a CTA's thread count must cover its dims.
constexpr int kCombineBatch = 8;                  // O loads in flight a thread
template <int DV, int NT>
__global__ void __launch_bounds__(NT, 1024 / NT) combine_kernel(const DecodeArgs a) {
    constexpr int kCombineThreads = NT;
    constexpr int kCombineMlPerThread = kMaxChunks / NT;
    static_assert(kMaxChunks % NT == 0, "(m, l) loads cover every chunk");
    constexpr int DH = D * DV;
    constexpr int kWarpsC = kCombineThreads / 32;
    const int seq = blockIdx.x, h = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int H = a.num_heads;
    const int dims = DH / (int)gridDim.z;            // this CTA's dims: [z * dims, (z+1) * dims)
    const int groups = dims / 4;
    const int lanes = kCombineThreads / groups;
    const int z = blockIdx.z;
    pdl_wait();  // the partials of decode_kernel
    pdl_trigger();
    int32_t off, cap, len;
    if (!load_entry(a, seq, off, cap, len)) return;  // flagged by decode_kernel
    // the sequence's partial rows: chunks c of the chunked grid at
    // (seq * max_chunks + c) * H + h, or the stream-K pieces of CTAs
    // c_first .. c_last at (c + seq) * H + h
    int nch;
    size_t base;
    if (a.sk_ctas) {
        // the tile prefix the decode kernel's CTA 0 left (read only when the
        // sequence has tiles, in which case that CTA ran the table pass)
        const int nt = (len + T - 1) / T;
        const long long p_s = a.sk_prefix[seq];     // written by every launch (CTA 0's table pass)
        const long long TT = nt ? a.sk_prefix[a.num_seqs] : 1;
        const int Ce = (int)(TT < a.sk_ctas ? TT : a.sk_ctas);
        const int c_first = nt ? sk_cta_of(p_s, TT, Ce) : 0;
        nch = nt ? sk_cta_of(p_s + nt - 1, TT, Ce) - c_first + 1 : 0;
        base = (size_t)(c_first + seq) * H + h;
    } else {
        nch = (len + a.chunk_tokens - 1) / a.chunk_tokens;
        nch = nch < a.max_chunks ? nch : a.max_chunks;
        base = (size_t)seq * a.max_chunks * H + h;
    }
    nch = nch < kMaxChunks ? nch : kMaxChunks;
    __shared__ float s_f[kMaxChunks];
    __shared__ __align__(16) float s_acc[kCombineThreads * 4];   // [lane][dims]
    __shared__ float s_rm[kWarpsC], s_rl[kWarpsC];
    __shared__ float s_M, s_L;

    // the first batch of O loads: chunk lane cl takes chunks cl, cl + lanes, ...
    const int gi = tid % groups, cl = tid / groups;
    const float4* po = reinterpret_cast<const float4*>(a.part_o + base * DH + z * dims) + gi;
    const size_t cstride = (size_t)H * (DH / 4);    // float4s from chunk to chunk
    float4 v[kCombineBatch];
#pragma unroll
    for (int k = 0; k < kCombineBatch; ++k) {
        const int c = cl + k * lanes;
        v[k] = c < nch ? po[(size_t)c * cstride] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    // (m, l) of chunks tid, tid + 256, ...
    float2 ml[kCombineMlPerThread];
#pragma unroll
    for (int k = 0; k < kCombineMlPerThread; ++k) {
        const int c = tid + k * kCombineThreads;
        ml[k] = c < nch ? *reinterpret_cast<const float2*>(a.part_ml + (base + (size_t)c * H) * 2)
                        : make_float2(-INFINITY, 0.0f);
    }
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < kCombineMlPerThread; ++k) m = fmaxf(m, ml[k].x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_rm[wid] = m;
    __syncthreads();
    if (tid == 0) {
        float M = -INFINITY;
        for (int w = 0; w < kWarpsC; ++w) M = fmaxf(M, s_rm[w]);
        s_M = M;
    }
    __syncthreads();
    const float M = s_M;
    float lsum = 0.0f;
#pragma unroll
    for (int k = 0; k < kCombineMlPerThread; ++k) {
        const int c = tid + k * kCombineThreads;
        const float f = ml[k].x == -INFINITY ? 0.0f : exp2f(ml[k].x - M);
        if (c < nch) s_f[c] = f;
        lsum += f * ml[k].y;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane == 0) s_rl[wid] = lsum;
    __syncthreads();                                  // s_f and s_rl complete
    if (tid == 0) {
        float L = 0.0f;
        for (int w = 0; w < kWarpsC; ++w) L += s_rl[w];
        s_L = L;
    }
    // O: the batch in registers, then any further batches
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < kCombineBatch; ++k) {
        const int c = cl + k * lanes;
        const float f = c < nch ? s_f[c] : 0.0f;
        acc.x += f * v[k].x;
        acc.y += f * v[k].y;
        acc.z += f * v[k].z;
        acc.w += f * v[k].w;
    }
    for (int c0 = cl + kCombineBatch * lanes; c0 < nch; c0 += kCombineBatch * lanes) {
#pragma unroll
        for (int k = 0; k < kCombineBatch; ++k) {
            const int c = c0 + k * lanes;
            v[k] = c < nch ? po[(size_t)c * cstride] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int k = 0; k < kCombineBatch; ++k) {
            const int c = c0 + k * lanes;
            const float f = c < nch ? s_f[c] : 0.0f;
            acc.x += f * v[k].x;
            acc.y += f * v[k].y;
            acc.z += f * v[k].z;
            acc.w += f * v[k].w;
        }
    }
    reinterpret_cast<float4*>(s_acc)[cl * groups + gi] = acc;
    __syncthreads();                                  // s_acc and s_L complete
    if (tid >= dims) return;
    float sum = 0.0f;
    for (int q = 0; q < lanes; ++q) sum += s_acc[q * dims + tid];   // lanes in order
    const float sl = s_L;
    const size_t oi = ((size_t)seq * H + h) * DH + z * dims + tid;
    if (a.mode == kOut) {
        a.out[oi] = nch ? __fdiv_rn(sum, sl) : 0.0f;
    } else {
        a.out[oi] = sum;
        if (z == 0 && tid == 0) {
            a.out_ml[((size_t)seq * H + h) * 2] = nch ? M : -INFINITY;
            a.out_ml[((size_t)seq * H + h) * 2 + 1] = sl;
        }
    }
}


// Merges num_parts partial states stacked [part][seq][head] (context shards);
// one thread per dim of each 128-dim block of the head.
template <int DV>
__global__ void __launch_bounds__(D) lse_merge_kernel(const float* __restrict__ part_o,
                                                      const float* __restrict__ part_ml,
                                                      int num_parts, int num_seqs, int H,
                                                      float* __restrict__ out) {
    constexpr int DH = D * DV;
    const int seq = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const size_t stride = (size_t)num_seqs * H;
    const size_t sh = (size_t)seq * H + h;
    float M = -INFINITY;
    for (int p = 0; p < num_parts; ++p) M = fmaxf(M, part_ml[(p * stride + sh) * 2]);
    float so[DV], sl = 0.0f;
#pragma unroll
    for (int dv = 0; dv < DV; ++dv) so[dv] = 0.0f;
    for (int p = 0; p < num_parts; ++p) {
        const size_t i = p * stride + sh;
        const float mp = part_ml[i * 2];
        const float f = mp == -INFINITY ? 0.0f : exp2f(mp - M);
#pragma unroll
        for (int dv = 0; dv < DV; ++dv) so[dv] += f * part_o[i * DH + dv * D + d];
        sl += f * part_ml[i * 2 + 1];
    }
#pragma unroll
    for (int dv = 0; dv < DV; ++dv)
        out[sh * DH + dv * D + d] = sl > 0.0f ? __fdiv_rn(so[dv], sl) : 0.0f;
}

template <int HC, int QW, int SCW, int DV>
cudaError_t launch_decode_t(const DecodeArgs& a, const DecodePlan& plan, cudaStream_t st) {
    using G = Geo<HC, QW, SCW, DV>;
    static std::atomic<unsigned long long> attr_done{0}, attr_done_sk{0};
    const bool sk = a.sk_ctas > 0;
    cudaError_t e = sk ? ensure_smem_limit(reinterpret_cast<const void*>(decode_sk_kernel<HC, QW, SCW, DV>),
                                           G::SMEM, attr_done_sk)
                       : ensure_smem_limit(reinterpret_cast<const void*>(decode_kernel<HC, QW, SCW, DV>),
                                           G::SMEM, attr_done);
    if (e != cudaSuccess) return e;
    CUtensorMap mk, mv;
    const int hkv = a.num_kv_heads;
    // a row of the code tensor is hkv * DV 128-byte blocks
    if ((e = make_code_map(&mk, a.keys, hkv * DV, a.total_slots, T)) != cudaSuccess) return e;
    if ((e = make_code_map(&mv, a.values, hkv * DV, a.total_slots, T)) != cudaSuccess) return e;
    // head blocks fastest, so that the CTAs sharing a chunk's scale rows run together
    if (sk)
        return launch_pdl(decode_sk_kernel<HC, QW, SCW, DV>, dim3(hkv / HC, a.sk_ctas),
                          dim3(G::kThreads), G::SMEM, st, mk, mv, a);
    dim3 grid(hkv / HC, plan.max_chunks, a.num_seqs);
    return launch_pdl(decode_kernel<HC, QW, SCW, DV>, grid, dim3(G::kThreads), G::SMEM, st, mk, mv,
                      a);
}

// Every compiled (HC, QW, SCW, DV): for num_kv_heads 1, 2, 4, 8 (SCW), query
// groups up to 4, 8, 16, 32 (QW = 1, 2, 4, 8) and head_dim 128 * DV, the CTA
// covers HC KV heads: all of them for groups up to 4 at head_dim 128 (at most
// two at 256), else as many as keep it at 4 units (8 for the largest groups).
#define EC_DECODE_VARIANTS(X)                                                     \
    X(1, 1, 1, 1) X(2, 1, 2, 1) X(4, 1, 4, 1) X(8, 1, 8, 1)                       \
    X(1, 2, 1, 1) X(2, 2, 2, 1) X(2, 2, 4, 1) X(2, 2, 8, 1)                       \
    X(1, 4, 1, 1) X(1, 4, 2, 1) X(1, 4, 4, 1) X(1, 4, 8, 1)                       \
    X(1, 8, 1, 1) X(1, 8, 2, 1) X(1, 8, 4, 1) X(1, 8, 8, 1)                       \
    X(1, 1, 1, 2) X(2, 1, 2, 2) X(2, 1, 4, 2) X(2, 1, 8, 2)                       \
    X(1, 2, 1, 2) X(1, 2, 2, 2) X(1, 2, 4, 2) X(1, 2, 8, 2)                       \
    X(1, 4, 1, 2) X(1, 4, 2, 2) X(1, 4, 4, 2) X(1, 4, 8, 2)                       \
    X(1, 8, 1, 2) X(1, 8, 2, 2) X(1, 8, 4, 2) X(1, 8, 8, 2)

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

DecodeVariant decode_variant(int num_kv_heads, int group, int head_dim) {
    DecodeVariant none{0, 0, 0, 0, 0};
    if (group < 1 || group > 32 || (head_dim != 128 && head_dim != 256)) return none;
    if (num_kv_heads != 1 && num_kv_heads != 2 && num_kv_heads != 4 && num_kv_heads != 8)
        return none;
    const int dv = head_dim / 128;
    const int qw = group <= 4 ? 1 : group <= 8 ? 2 : group <= 16 ? 4 : 8;
    // KV heads per CTA: every head for groups up to 4 (at most two of 256
    // dims), two for groups up to 8 (one of 256 dims), else one
    const int hc_cap = qw == 1 ? (dv == 1 ? 8 : 2) : qw == 2 ? (dv == 1 ? 2 : 1) : 1;
    const int hc = num_kv_heads < hc_cap ? num_kv_heads : hc_cap;
#define EC_VARIANT(HC_, QW_, SCW_, DV_)                                           \
    if (hc == HC_ && qw == QW_ && num_kv_heads == SCW_ && dv == DV_)              \
        return DecodeVariant{HC_, QW_, SCW_, DV_, Geo<HC_, QW_, SCW_, DV_>::kCtasPerSm};
    EC_DECODE_VARIANTS(EC_VARIANT)
#undef EC_VARIANT
    return none;
}

int merge_splits(int pairs) { return pairs <= 64 ? 8 : pairs <= 128 ? 4 : pairs <= 256 ? 2 : 1; }

static DecodePlan plan_decode_uncached(int num_seqs, int max_seq_len, int num_sms,
                                       uint64_t total_tokens, int num_kv_heads, int num_heads,
                                       int head_dim, bool allow_stream);

// The plan is a pure function of its arguments, and a serving loop asks for
// the same one every step (the workspace query, then the launch): the last
// few are kept, since the chunked plan's cost model scans up to 1024 chunk
// counts (about 10 us of host time for one long sequence).
DecodePlan plan_decode(int num_seqs, int max_seq_len, int num_sms, uint64_t total_tokens,
                       int num_kv_heads, int num_heads, int head_dim, bool allow_stream) {
    struct Entry {
        int num_seqs, max_seq_len, num_sms, num_kv_heads, num_heads, head_dim;
        uint64_t total_tokens;
        bool allow_stream, used;
        DecodePlan plan;
    };
    constexpr int kEntries = 16;
    static std::mutex mu;
    static Entry memo[kEntries] = {};
    static int next = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Entry& e : memo)
            if (e.used && e.num_seqs == num_seqs && e.max_seq_len == max_seq_len &&
                e.num_sms == num_sms && e.total_tokens == total_tokens &&
                e.num_kv_heads == num_kv_heads && e.num_heads == num_heads &&
                e.head_dim == head_dim && e.allow_stream == allow_stream)
                return e.plan;
    }
    const DecodePlan p = plan_decode_uncached(num_seqs, max_seq_len, num_sms, total_tokens,
                                              num_kv_heads, num_heads, head_dim, allow_stream);
    std::lock_guard<std::mutex> lock(mu);
    memo[next] = Entry{num_seqs, max_seq_len, num_sms, num_kv_heads, num_heads, head_dim,
                       total_tokens, allow_stream, true, p};
    next = (next + 1) % kEntries;
    return p;
}

static DecodePlan plan_decode_uncached(int num_seqs, int max_seq_len, int num_sms,
                                       uint64_t total_tokens, int num_kv_heads, int num_heads,
                                       int head_dim, bool allow_stream) {
    const DecodeVariant v = num_kv_heads > 0
        ? decode_variant(num_kv_heads, num_heads / num_kv_heads, head_dim) : DecodeVariant{};
    const int slots = num_sms * (v.hc ? v.ctas_per_sm : 2);   // resident CTAs
    const int hblocks = v.hc ? num_kv_heads / v.hc : 1;       // CTAs per (sequence, chunk)
    DecodePlan best{T, 1, 0};
    if (max_seq_len <= 0 || num_seqs <= 0) return best;
    const int tiles = (max_seq_len + T - 1) / T;
    // Stream-K for batches of 32 to 1024 sequences: one wave, every CTA of a
    // head block streams an equal share of the batch's tiles, so no partial
    // last wave (config 3: 1,152 chunks were 3.9 waves), no CTA prologue per
    // chunk, and ragged lengths balance by construction.  Measured on B200
    // against the chunked grid: +1% on 128 x 32k and +2.5% on 64 ragged
    // sequences of 512-8192 tokens, but behind on one sequence (the table
    // pass and the prefix read add to a 15 us step), which keeps the chunked
    // plan.
    if (allow_stream && num_seqs >= kStreamMinSeqs && num_seqs <= kStreamMaxSeqs) {
        // (the merge takes up to kMaxChunks pieces of a sequence, one per CTA)
        const uint64_t tokens = total_tokens > 0 ? total_tokens : (uint64_t)num_seqs * max_seq_len;
        const uint64_t tt = (tokens + T - 1) / T;
        int c = slots / hblocks;
        c = c < 1 ? 1 : c;
        if ((uint64_t)c > tt) c = (int)(tt > 0 ? tt : 1);
        if (c > kMaxChunks) c = kMaxChunks;
        return DecodePlan{tiles * T, 1, c};
    }
    double best_cost = 1e300;
    const int kmax = tiles < kMaxChunks ? tiles : kMaxChunks;
    // with a token count below the all-full batch, the CTAs that find work
    // are about total / chunk plus half a chunk per sequence; the others exit
    // at once (about 16 tokens' worth of time each)
    const bool ragged = total_tokens > 0 && total_tokens < (uint64_t)num_seqs * max_seq_len;
    for (int k = 1; k <= kmax; ++k) {
        const int chunk = ((tiles + k - 1) / k) * T;
        const int kk = (max_seq_len + chunk - 1) / chunk;
        const long long ctas = (long long)num_seqs * kk * hblocks;
        long long busy = ctas;
        if (ragged) {
            const double est = ((double)total_tokens / chunk + 0.5 * num_seqs) * hblocks;
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

size_t decode_workspace_bytes(const DecodePlan& p, int num_seqs, int num_heads, int head_dim) {
    if (p.sk_ctas > 0)   // a row per (CTA, sequence) piece (rows c + s < C + num_seqs), then the tile prefix
        return (size_t)(p.sk_ctas + num_seqs) * num_heads * (head_dim + 2) * sizeof(float) +
               (((size_t)num_seqs + 1) * sizeof(int32_t) + 15) / 16 * 16;
    if (p.max_chunks <= 1) return 0;
    return (size_t)num_seqs * p.max_chunks * num_heads * (head_dim + 2) * sizeof(float);
}

cudaError_t launch_decode(DecodeArgs a, int num_kv_heads, const DecodePlan& plan, void* ws,
                          cudaStream_t st) {
    a.chunk_tokens = plan.chunk_tokens;
    a.max_chunks = plan.max_chunks;
    a.sk_ctas = a.mode == kChunks ? 0 : plan.sk_ctas;
    if (a.mode == kChunks && plan.sk_ctas > 0) return cudaErrorInvalidValue;   // needs a chunked plan
    if (a.sk_ctas > 0) {
        const size_t rows = (size_t)(a.sk_ctas + a.num_seqs) * a.num_heads;
        a.part_o = static_cast<float*>(ws);
        a.part_ml = a.part_o + rows * a.head_dim;
        a.sk_prefix = reinterpret_cast<int32_t*>(a.part_ml + rows * 2);
    } else if (plan.max_chunks > 1 || a.mode == kChunks) {
        a.part_o = static_cast<float*>(ws);
        a.part_ml = a.part_o + (size_t)a.num_seqs * plan.max_chunks * a.num_heads * a.head_dim;
    }
    a.num_kv_heads = num_kv_heads;
    const DecodeVariant v = decode_variant(num_kv_heads, a.num_heads / num_kv_heads, a.head_dim);
    if (!v.hc || a.num_heads % num_kv_heads) return cudaErrorInvalidValue;
    cudaError_t e = cudaErrorInvalidValue;
#define EC_DEC(HC_, QW_, SCW_, DV_)                                               \
    if (v.hc == HC_ && v.qw == QW_ && v.scw == SCW_ && v.dv == DV_)               \
        e = launch_decode_t<HC_, QW_, SCW_, DV_>(a, plan, st);
    EC_DECODE_VARIANTS(EC_DEC)
#undef EC_DEC
    if (e != cudaSuccess || a.mode == kChunks || (plan.max_chunks <= 1 && a.sk_ctas == 0)) return e;
    const int z = merge_splits(a.num_seqs * a.num_heads);
    const dim3 cg(a.num_seqs, a.num_heads, z);
    if (v.dv == 2) return launch_pdl(combine_kernel<2, 256>, cg, dim3(256), 0, st, a);
    return z == 1 ? launch_pdl(combine_kernel<1, 128>, cg, dim3(128), 0, st, a)
                  : launch_pdl(combine_kernel<1, 256>, cg, dim3(256), 0, st, a);
}

cudaError_t launch_lse_combine(const float* part_o, const float* part_ml, int num_parts,
                               int num_seqs, int num_heads, int head_dim, float* out,
                               cudaStream_t st) {
    const dim3 grid(num_seqs, num_heads);
    if (head_dim == 128)
        lse_merge_kernel<1><<<grid, D, 0, st>>>(part_o, part_ml, num_parts, num_seqs, num_heads, out);
    else if (head_dim == 256)
        lse_merge_kernel<2><<<grid, D, 0, st>>>(part_o, part_ml, num_parts, num_seqs, num_heads, out);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace ec
