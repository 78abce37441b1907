// decode_f32.cu -- decode attention over the fp32 KV cache (use_kv_quantization
// = false), the reference's FP32 mode of InferenceEngine::attention
// (src/inference.cpp:346-358 scores, :386-393 P.V) over the layout of
// src/kv_cache.cpp:59-70: keys_fp32 / values_fp32 [pos][num_kv_heads][128].
//
// HBM-bound at 4 bytes per element (4 KB per token for 4 KV heads), so the
// math stays on the CUDA cores in fp32.  Grid = (token chunk, KV head); each
// of the 4 warps of a CTA walks a contiguous quarter of the chunk in batches
// of T = 32 / GROUP tokens.  Lane i holds dims 4i..4i+3 of the GROUP query
// heads that read this KV head (h = g + j * num_kv_heads, the h % num_kv_heads
// rule of src/inference.cpp:335), so a token's K or V row is one coalesced
// 512-byte float4 load per warp.  The GROUP x T partial dot products of a
// batch are summed across the warp by a butterfly reduce-scatter (31
// shuffles), after which lane L holds the full score of (head L / T, token
// L % T).  Online softmax in base 2; the CTA merges its warps and writes one
// (m, l, O) partial per (chunk, head); the log-sum-exp merge of the split-K
// chunks is the same kernel the context-parallel path uses.
#include <cmath>
#include <cstdint>

#include "ec_common.cuh"
#include "ec_internal.h"

namespace ec {
namespace {

constexpr int D = 128;
constexpr int kWarps = 4;
constexpr unsigned kFull = 0xffffffffu;

// 2-D tiled TMA load (no multicast) with an L2 eviction hint.
__device__ __forceinline__ void tma_load_2d_f(void* dst, const CUtensorMap* map, int x, int y,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

template <int GROUP>
struct F32Geo {
    static constexpr int T = 32 / GROUP;                   // tokens per batch; GROUP * T = 32
    static constexpr int STAGE = T * 2 * D * 4;            // K and V rows of one batch
    // A multiple of the 4 consumer warps: stage s is always consumed by warp
    // s % 4, whose successive uses of it are then exactly one barrier phase
    // apart (a waiter two phases ahead would alias the parity).
    static constexpr int NST = STAGE <= 8192 ? 8 : 4;
    // + 128: the dynamic region starts after the static merge arrays, at an
    // offset that need not be 128-byte aligned (tensor copies require it)
    static constexpr int SMEM = 128 + NST * STAGE + 2 * NST * 8;
    static_assert(NST % 4 == 0, "stages must be a multiple of the consumer warps");
};

// 4 consumer warps (0-3) and one producer warp (4).  The producer streams the
// chunk's K and V rows batch by batch into a ring of NST shared-memory
// stages with 512-byte bulk copies (one per row, no multicast); consumer warp
// w takes batches w, w+4, w+8, ... and keeps its own online-softmax state.
template <int GROUP>
__global__ void __launch_bounds__((kWarps + 1) * 32)
    decode_f32_kernel(const __grid_constant__ CUtensorMap tmap_k,
                      const __grid_constant__ CUtensorMap tmap_v, int hkv, int len,
                      int chunk_tokens, const float* __restrict__ q, float q_mul,
                      float* __restrict__ part_o, float* __restrict__ part_ml) {
    using G = F32Geo<GROUP>;
    constexpr int T = G::T, NST = G::NST;
    constexpr int LOGT = T == 32 ? 5 : T == 16 ? 4 : T == 8 ? 3 : T == 4 ? 2 : 1;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                               ~uintptr_t(127));
    float* ring = reinterpret_cast<float*>(smem);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * G::STAGE);
    uint64_t* empty = full + NST;
    const int chunk = blockIdx.x, g = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = hkv * GROUP;
    const int c0 = chunk * chunk_tokens;
    const int c1 = min(len, c0 + chunk_tokens);
    const int nb = (c1 - c0 + T - 1) / T;     // batches in this chunk

    if (threadIdx.x == 0) {
        for (int i = 0; i < NST; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    float o[GROUP][4], m_run[GROUP], l_run[GROUP];
#pragma unroll
    for (int j = 0; j < GROUP; ++j) {
        m_run[j] = -INFINITY;
        l_run[j] = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; ++u) o[j][u] = 0.0f;
    }

    if (warp == kWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            int issued = 0;
            for (int b = 0; b < nb; ++b) {
                const int s = b % NST;
                if (b >= NST && !mbar_wait(&empty[s], ((b / NST) - 1) & 1)) {
                    flag_error(nullptr, EC_DEVERR_TIMEOUT);
                    break;
                }
                const int t0 = c0 + b * T;
                // two boxes of [T tokens][128 floats] (rows past the cache read as
                // zeros; rows past the chunk are masked by the consumer)
                mbar_arrive_expect_tx(&full[s], (uint32_t)G::STAGE);
                float* st = ring + (size_t)s * (G::STAGE / 4);
                tma_load_2d_f(st, &tmap_k, g * D, t0, &full[s], pol);
                tma_load_2d_f(st + T * D, &tmap_v, g * D, t0, &full[s], pol);
                issued = b + 1;
            }
            // never leave with copies in flight into this CTA's shared memory
            for (int b = max(0, issued - NST); b < issued; ++b) mbar_wait(&full[b % NST], (b / NST) & 1);
        }
    } else {
        // ------------------------------------------------------------ consumers
        float qr[GROUP][4];   // q of the group's heads, scaled as src/inference.cpp:322-325 does
#pragma unroll
        for (int j = 0; j < GROUP; ++j) {
            const float4 x = reinterpret_cast<const float4*>(q + (size_t)(g + j * hkv) * D)[lane];
            qr[j][0] = x.x * q_mul; qr[j][1] = x.y * q_mul;
            qr[j][2] = x.z * q_mul; qr[j][3] = x.w * q_mul;
        }
        const int mh = lane >> LOGT;          // this lane's head after the reduction
        constexpr float kLog2e = 1.4426950408889634f;
        for (int b = warp; b < nb; b += kWarps) {
            const int s = b % NST;
            if (!mbar_wait(&full[s], (b / NST) & 1)) {
                if (lane == 0) flag_error(nullptr, EC_DEVERR_TIMEOUT);
                break;
            }
            const int t0 = c0 + b * T;
            const float* st = ring + (size_t)s * (G::STAGE / 4);
            // ---- scores: GROUP x T partial dots, then a reduce-scatter
            float v[32];
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const float4 k = reinterpret_cast<const float4*>(st + t * D)[lane];
#pragma unroll
                for (int j = 0; j < GROUP; ++j)
                    v[j * T + t] = fmaf(qr[j][0], k.x, fmaf(qr[j][1], k.y, fmaf(qr[j][2], k.z, qr[j][3] * k.w)));
            }
#pragma unroll
            for (int n = 16; n >= 1; n >>= 1) {       // lane L ends with index L
                const bool up = lane & n;
#pragma unroll
                for (int i = 0; i < n; ++i) {
                    const float keep = up ? v[i + n] : v[i];
                    const float send = up ? v[i] : v[i + n];
                    v[i] = keep + __shfl_xor_sync(kFull, send, n);
                }
            }
            const int mt = lane & (T - 1);
            const float sc = t0 + mt < c1 ? v[0] * kLog2e : -INFINITY;
            // ---- online softmax per head (the T lanes of a head are adjacent)
            float bm = sc;
#pragma unroll
            for (int n = 1; n < T; n <<= 1) bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, n));
#pragma unroll
            for (int j = 0; j < GROUP; ++j) {
                const float mn = fmaxf(m_run[j], __shfl_sync(kFull, bm, j * T));
                const float corr = mn == -INFINITY ? 1.0f : exp2f(m_run[j] - mn);
                l_run[j] *= corr;
#pragma unroll
                for (int u = 0; u < 4; ++u) o[j][u] *= corr;
                m_run[j] = mn;
            }
            float mine = m_run[0];
#pragma unroll
            for (int j = 1; j < GROUP; ++j)
                if (mh == j) mine = m_run[j];
            const float p = sc == -INFINITY ? 0.0f : exp2f(sc - mine);
            float ps = p;
#pragma unroll
            for (int n = 1; n < T; n <<= 1) ps += __shfl_xor_sync(kFull, ps, n);
#pragma unroll
            for (int j = 0; j < GROUP; ++j) l_run[j] += __shfl_sync(kFull, ps, j * T);
            // ---- O += p V (rows past the chunk end are stale shared memory: p = 0,
            // and they are skipped so that a stale NaN cannot leak in)
#pragma unroll
            for (int t = 0; t < T; ++t) {
                if (t0 + t >= c1) break;
                const float4 vv = reinterpret_cast<const float4*>(st + (T + t) * D)[lane];
#pragma unroll
                for (int j = 0; j < GROUP; ++j) {
                    const float pj = __shfl_sync(kFull, p, j * T + t);
                    o[j][0] = fmaf(pj, vv.x, o[j][0]); o[j][1] = fmaf(pj, vv.y, o[j][1]);
                    o[j][2] = fmaf(pj, vv.z, o[j][2]); o[j][3] = fmaf(pj, vv.w, o[j][3]);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
    }

    // ---- merge the CTA's warps, write the chunk's (m, l, O) per head
    __shared__ float s_ml[kWarps][GROUP][2];
    __shared__ __align__(16) float s_o[kWarps][GROUP][D];
    if (warp < kWarps) {
#pragma unroll
        for (int j = 0; j < GROUP; ++j) {
            *reinterpret_cast<float4*>(&s_o[warp][j][4 * lane]) = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
            if (lane == 0) { s_ml[warp][j][0] = m_run[j]; s_ml[warp][j][1] = l_run[j]; }
        }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < GROUP * D; idx += (kWarps + 1) * 32) {
        const int j = idx / D, d = idx % D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_ml[w][j][0]);
        float so = 0.0f, sl = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const float f = s_ml[w][j][0] == -INFINITY ? 0.0f : exp2f(s_ml[w][j][0] - M);
            so += f * s_o[w][j][d];
            sl += f * s_ml[w][j][1];
        }
        const size_t pi = (size_t)chunk * H + g + (size_t)j * hkv;
        part_o[pi * D + d] = so;
        if (d == 0) { part_ml[pi * 2] = M; part_ml[pi * 2 + 1] = sl; }
    }
}

}  // namespace

// Chunking: at least 512 tokens per CTA, and no more chunks than about three
// resident CTAs per SM across the KV heads, so that long contexts run in
// long-lived CTAs and the log-sum-exp merge sees at most a few hundred parts.
static int f32_target_chunks(int num_kv_heads) {
    // the current device's SM count (queried each call: cheap, and right for
    // whichever device the caller has made current)
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        sms = 148;
    const int t = 3 * sms / (num_kv_heads > 0 ? num_kv_heads : 1);
    return t > 0 ? t : 1;
}

static int f32_chunk_tokens(int len, int num_kv_heads) {
    const int target = f32_target_chunks(num_kv_heads);
    int ct = (len + target - 1) / target;
    if (ct < kF32ChunkTokens) ct = kF32ChunkTokens;
    return (ct + 31) & ~31;
}

int f32_decode_chunks(int len, int num_kv_heads) {
    if (len <= 0) return 0;
    const int ct = f32_chunk_tokens(len, num_kv_heads);
    return (len + ct - 1) / ct;
}

size_t f32_decode_workspace_bytes(int max_len, int num_kv_heads, int num_heads) {
    // the chunk count never exceeds the target, nor the count at the minimum chunk
    const int by_len = (max_len + kF32ChunkTokens - 1) / kF32ChunkTokens;
    const int target = f32_target_chunks(num_kv_heads);
    const int chunks = max_len <= 0 ? 0 : (by_len < target ? by_len : target);
    return (size_t)chunks * num_heads * (D + 2) * sizeof(float);
}

cudaError_t launch_decode_f32(const float* keys, const float* values, int num_kv_heads,
                              int num_heads, int len, const float* q, float q_mul, float* out,
                              void* ws, cudaStream_t st) {
    const int group = num_heads / num_kv_heads;
    const int chunks = f32_decode_chunks(len, num_kv_heads);
    const int chunk_tokens = f32_chunk_tokens(len, num_kv_heads);
    if (chunks == 0) return cudaMemsetAsync(out, 0, (size_t)num_heads * D * sizeof(float), st);
    float* part_o = static_cast<float*>(ws);
    float* part_ml = part_o + (size_t)chunks * num_heads * D;
    dim3 grid(chunks, num_kv_heads);
    cudaError_t e = cudaSuccess;
    CUtensorMap mk, mv;
    const int box = 32 / group;   // T of the kernel instance
    if ((e = make_f32_row_map(&mk, keys, num_kv_heads, (uint64_t)len, box)) != cudaSuccess) return e;
    if ((e = make_f32_row_map(&mv, values, num_kv_heads, (uint64_t)len, box)) != cudaSuccess) return e;
#define EC_F32_CASE(GR)                                                                        \
    case GR: {                                                                                 \
        static std::atomic<unsigned long long> done{0};                                       \
        e = ensure_smem_limit(reinterpret_cast<const void*>(decode_f32_kernel<GR>),            \
                              F32Geo<GR>::SMEM, done);                                         \
        if (e != cudaSuccess) return e;                                                        \
        decode_f32_kernel<GR><<<grid, (kWarps + 1) * 32, F32Geo<GR>::SMEM, st>>>(             \
            mk, mv, num_kv_heads, len, chunk_tokens, q, q_mul, part_o, part_ml);              \
        break;                                                                                 \
    }
    switch (group) {
        EC_F32_CASE(1)
        EC_F32_CASE(2)
        EC_F32_CASE(4)
        EC_F32_CASE(8)
        default: return cudaErrorInvalidValue;
    }
#undef EC_F32_CASE
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_lse_combine(part_o, part_ml, chunks, 1, num_heads, 128, out, st);
}

}  // namespace ec
