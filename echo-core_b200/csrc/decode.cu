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
constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyRescale = 8.0f;
constexpr unsigned kFull = 0xffffffffu;

template <int HKV>
struct Geo {
    static constexpr int T = 128 / HKV;                 // tokens per tile
    static constexpr int WPH = kConsumerWarps / HKV;    // consumer warps per KV head
    static constexpr int ROWB = HKV * D;                // code bytes per token row
    static constexpr int KV_TILE = T * ROWB;            // 16 KB
    static constexpr int SC_TILE = T * HKV * 4;         // 512 B
    static constexpr int STAGE = 2 * KV_TILE + 2 * SC_TILE;
    static constexpr int PBUF = kConsumerWarps * 16 * 4 * 4;
    static constexpr int SMEM = kStages * STAGE + PBUF + 2 * kStages * 8;
    static_assert(T == WPH * 16, "each consumer warp owns 16 tokens of a tile");
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

// Lane (within an 8-lane token group) that ends up holding head j's dot.
template <int GROUP>
__device__ __forceinline__ int lane_of_head(int j) {
    if constexpr (GROUP == 4) return (j >> 1) * 4 + (j & 1) * 2;
    else if constexpr (GROUP == 2) return j * 4;
    else return 0;
}
template <int GROUP>
__device__ __forceinline__ int head_of_lane(int c) {
    if constexpr (GROUP == 4) return ((c >> 2) & 1) * 2 + ((c >> 1) & 1);
    else if constexpr (GROUP == 2) return (c >> 2) & 1;
    else return 0;
}
template <int GROUP>
__device__ __forceinline__ bool writer_lane(int c) {
    if constexpr (GROUP == 4) return (c & 1) == 0;
    else if constexpr (GROUP == 2) return (c & 3) == 0;
    else return c == 0;
}

// Sum GROUP per-lane partial dots over the 8 lanes of a token group, leaving
// head head_of_lane(c)'s total in each lane.
template <int GROUP>
__device__ __forceinline__ float transpose_reduce(const float (&v)[GROUP], int c) {
    if constexpr (GROUP == 4) {
        const bool hi = (c & 4) != 0;
        const float s0 = hi ? v[0] : v[2], s1 = hi ? v[1] : v[3];
        float k0 = hi ? v[2] : v[0], k1 = hi ? v[3] : v[1];
        k0 += __shfl_xor_sync(kFull, s0, 4);
        k1 += __shfl_xor_sync(kFull, s1, 4);
        const bool mid = (c & 2) != 0;
        const float s = mid ? k0 : k1;
        float k = mid ? k1 : k0;
        k += __shfl_xor_sync(kFull, s, 2);
        k += __shfl_xor_sync(kFull, k, 1);
        return k;
    } else if constexpr (GROUP == 2) {
        const bool hi = (c & 4) != 0;
        const float s = hi ? v[0] : v[1];
        float k = hi ? v[1] : v[0];
        k += __shfl_xor_sync(kFull, s, 4);
        k += __shfl_xor_sync(kFull, k, 2);
        k += __shfl_xor_sync(kFull, k, 1);
        return k;
    } else {
        float k = v[0];
        k += __shfl_xor_sync(kFull, k, 4);
        k += __shfl_xor_sync(kFull, k, 2);
        k += __shfl_xor_sync(kFull, k, 1);
        return k;
    }
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

template <int HKV, int GROUP>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const DecodeArgs a) {
    using G = Geo<HKV>;
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ int fail_flag;
    uint8_t* stages = smem;
    float* pbuf = reinterpret_cast<float*>(smem + kStages * G::STAGE);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * G::STAGE + G::PBUF);
    uint64_t* empty = full + kStages;

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
        fail_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    // ------------------------------------------------------------ producer
    if (warp == kConsumerWarps) {
        const size_t slot0 = (size_t)off + t0;
        const uint64_t pol = l2_policy_evict_first();
        for (int i = 0; i < ntiles; ++i) {
            const int s = i % kStages;
            bool ok = true;
            if (lane == 0 && i >= kStages) ok = mbar_wait(&empty[s], ((i / kStages) - 1) & 1);
            ok = __shfl_sync(kFull, ok, 0);
            if (!ok) {
                if (lane == 0) flag_error(a.err, EC_DEVERR_TIMEOUT);
                break;
            }
            const int ntok = min(G::T, n - i * G::T);
            const size_t slot = slot0 + (size_t)i * G::T;
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
                // ROW scales: one fp32 per token; broadcast into the per-head
                // tile layout with plain loads, then arrive.
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
        }
        return;
    }

    // ------------------------------------------------------------ consumers
    const int g = warp / G::WPH;      // KV head
    const int sw = warp % G::WPH;     // which 16-token slice of each tile
    const int c = lane & 7;           // 16-byte column of the 128-byte head row
    const int tq = lane >> 3;         // token within a 4-token pass
    const int hsel = head_of_lane<GROUP>(c);

    float2 q2[GROUP][8];
#pragma unroll
    for (int j = 0; j < GROUP; ++j) {
        const int h = g + HKV * j;
        const float4* qp = reinterpret_cast<const float4*>(a.q + ((size_t)seq * a.num_heads + h) * D + 16 * c);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
            const float4 v = qp[k4];
            q2[j][2 * k4] = make_float2(__fmul_rn(__fmul_rn(v.x, a.q_mul), kLog2e),
                                        __fmul_rn(__fmul_rn(v.y, a.q_mul), kLog2e));
            q2[j][2 * k4 + 1] = make_float2(__fmul_rn(__fmul_rn(v.z, a.q_mul), kLog2e),
                                            __fmul_rn(__fmul_rn(v.w, a.q_mul), kLog2e));
        }
    }

    float2 acc_o[GROUP][8];
#pragma unroll
    for (int j = 0; j < GROUP; ++j)
#pragma unroll
        for (int k = 0; k < 8; ++k) acc_o[j][k] = make_float2(0.f, 0.f);
    float m_run[GROUP];
#pragma unroll
    for (int j = 0; j < GROUP; ++j) m_run[j] = -INFINITY;
    float l_part = 0.0f;
    bool failed = false;
    float* pw = pbuf + warp * 64;  // [16 tokens][4 heads]

    for (int i = 0; i < ntiles; ++i) {
        const int s = i % kStages;
        const bool ok = __all_sync(kFull, mbar_wait(&full[s], (i / kStages) & 1));
        if (!ok) {
            if (lane == 0) flag_error(a.err, EC_DEVERR_TIMEOUT);
            failed = true;
            break;
        }
        const uint8_t* st = stages + s * G::STAGE;
        const int8_t* kt = reinterpret_cast<const int8_t*>(st);
        const int8_t* vt = kt + G::KV_TILE;
        const float* kst = reinterpret_cast<const float*>(st + 2 * G::KV_TILE);
        const float* vst = kst + G::T * HKV;
        const int valid = n - i * G::T;  // tokens of this tile that exist (may exceed T)

        // ---- scores
        float sc[4];
#pragma unroll
        for (int ps = 0; ps < 4; ++ps) {
            const int tt = sw * 16 + ps * 4 + tq;
            const uint4 w = *reinterpret_cast<const uint4*>(kt + tt * G::ROWB + g * D + 16 * c);
            float2 kf[8];
            codes16_to_f2(w, kf);
            float v[GROUP];
#pragma unroll
            for (int j = 0; j < GROUP; ++j) {
                float2 a0 = __fmul2_rn(q2[j][0], kf[0]);
                float2 a1 = __fmul2_rn(q2[j][1], kf[1]);
#pragma unroll
                for (int k = 2; k < 8; k += 2) {
                    a0 = __ffma2_rn(q2[j][k], kf[k], a0);
                    a1 = __ffma2_rn(q2[j][k + 1], kf[k + 1], a1);
                }
                v[j] = (a0.x + a0.y) + (a1.x + a1.y);
            }
            const float r = transpose_reduce<GROUP>(v, c) * kst[tt * HKV + g];
            sc[ps] = tt < valid ? r : -INFINITY;
        }

        // ---- online softmax (base 2, lazy rescale)
        float tm = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
        tm = fmaxf(tm, __shfl_xor_sync(kFull, tm, 8));
        tm = fmaxf(tm, __shfl_xor_sync(kFull, tm, 16));
        float mt[GROUP];
        bool resc = false;
#pragma unroll
        for (int j = 0; j < GROUP; ++j) {
            mt[j] = __shfl_sync(kFull, tm, lane_of_head<GROUP>(j));
            resc |= mt[j] > m_run[j] + kLazyRescale;
        }
        if (resc) {
            float corr[GROUP];
#pragma unroll
            for (int j = 0; j < GROUP; ++j) {
                if (mt[j] > m_run[j] + kLazyRescale) {
                    corr[j] = exp2f(m_run[j] - mt[j]);
                    m_run[j] = mt[j];
                } else {
                    corr[j] = 1.0f;
                }
            }
#pragma unroll
            for (int j = 0; j < GROUP; ++j) {
                const float2 cj = make_float2(corr[j], corr[j]);
#pragma unroll
                for (int k = 0; k < 8; ++k) acc_o[j][k] = __fmul2_rn(acc_o[j][k], cj);
            }
            l_part *= pick<GROUP>(corr, hsel);
        }
        const float m_own = pick<GROUP>(m_run, hsel);
#pragma unroll
        for (int ps = 0; ps < 4; ++ps) {
            const float p = sc[ps] == -INFINITY ? 0.0f : exp2f(sc[ps] - m_own);
            l_part += p;
            if (writer_lane<GROUP>(c)) {
                const int tt = sw * 16 + ps * 4 + tq;
                pw[(ps * 4 + tq) * 4 + hsel] = sc[ps] == -INFINITY ? 0.0f : p * vst[tt * HKV + g];
            }
        }
        __syncwarp();

        // ---- P . V
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
                for (int k = 0; k < 8; ++k) acc_o[j][k] = __ffma2_rn(pj, vf[k], acc_o[j][k]);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }

    // ---- reduce the four token groups of the warp
#pragma unroll
    for (int j = 0; j < GROUP; ++j)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float2 v = acc_o[j][k];
            v.x += __shfl_xor_sync(kFull, v.x, 8);
            v.y += __shfl_xor_sync(kFull, v.y, 8);
            v.x += __shfl_xor_sync(kFull, v.x, 16);
            v.y += __shfl_xor_sync(kFull, v.y, 16);
            acc_o[j][k] = v;
        }
    l_part += __shfl_xor_sync(kFull, l_part, 8);
    l_part += __shfl_xor_sync(kFull, l_part, 16);
    float l_run[GROUP];
#pragma unroll
    for (int j = 0; j < GROUP; ++j) l_run[j] = __shfl_sync(kFull, l_part, lane_of_head<GROUP>(j));

    // ---- merge the WPH warps of each KV head through shared memory
    consumer_barrier();  // every warp is done with the stage ring
    float* mo = reinterpret_cast<float*>(stages);                 // [8][GROUP][128]
    float* mm = mo + kConsumerWarps * GROUP * D;                   // [8][GROUP]
    float* ml = mm + kConsumerWarps * GROUP;                       // [8][GROUP]
    if (failed) {
        if (lane == 0) fail_flag = 1;
    } else {
        if (tq == 0) {
#pragma unroll
            for (int j = 0; j < GROUP; ++j)
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    *reinterpret_cast<float2*>(mo + (warp * GROUP + j) * D + 16 * c + 2 * k) = acc_o[j][k];
        }
        if (lane == 0) {
#pragma unroll
            for (int j = 0; j < GROUP; ++j) {
                mm[warp * GROUP + j] = m_run[j];
                ml[warp * GROUP + j] = l_run[j];
            }
        }
    }
    consumer_barrier();
    if (fail_flag) return;

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
