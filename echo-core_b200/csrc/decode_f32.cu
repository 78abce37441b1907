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

template <int GROUP>
__global__ void __launch_bounds__(kWarps * 32)
    decode_f32_kernel(const float* __restrict__ keys, const float* __restrict__ values, int hkv,
                      int len, int chunk_tokens, const float* __restrict__ q, float q_mul,
                      float* __restrict__ part_o, float* __restrict__ part_ml) {
    constexpr int T = 32 / GROUP;             // tokens per batch; GROUP * T = 32
    constexpr int LOGT = T == 32 ? 5 : T == 16 ? 4 : T == 8 ? 3 : T == 4 ? 2 : 1;
    const int chunk = blockIdx.x, g = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = hkv * GROUP;
    const size_t row = (size_t)hkv * D;       // floats per token

    // q of the group's heads, scaled as src/inference.cpp:322-325 does
    float qr[GROUP][4];
#pragma unroll
    for (int j = 0; j < GROUP; ++j) {
        const float4 x = reinterpret_cast<const float4*>(q + (size_t)(g + j * hkv) * D)[lane];
        qr[j][0] = x.x * q_mul; qr[j][1] = x.y * q_mul;
        qr[j][2] = x.z * q_mul; qr[j][3] = x.w * q_mul;
    }
    float o[GROUP][4], m_run[GROUP], l_run[GROUP];
#pragma unroll
    for (int j = 0; j < GROUP; ++j) {
        m_run[j] = -INFINITY;
        l_run[j] = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; ++u) o[j][u] = 0.0f;
    }

    const int c0 = chunk * chunk_tokens;
    const int c1 = min(len, c0 + chunk_tokens);
    const int per = (c1 - c0 + kWarps - 1) / kWarps;
    const int w0 = c0 + warp * per, w1 = min(c1, w0 + per);
    const int mh = lane >> LOGT;              // this lane's head after the reduction
    constexpr float kLog2e = 1.4426950408889634f;

    for (int t0 = w0; t0 < w1; t0 += T) {
        // ---- the batch's K and V rows, all loads in flight together where the
        // registers allow (groups 2 and 4: 8 or 16 tokens); groups 1 and 8
        // load each row where it is used
        constexpr bool kEarly = GROUP == 2 || GROUP == 4;
        float4 kr[T], vr[T];
#pragma unroll
        for (int t = 0; t < T; ++t) {
            kr[t] = vr[t] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (kEarly && t0 + t < w1) {
                const size_t base = (size_t)(t0 + t) * row + (size_t)g * D;
                kr[t] = __ldcs(reinterpret_cast<const float4*>(keys + base) + lane);
                vr[t] = __ldcs(reinterpret_cast<const float4*>(values + base) + lane);
            }
        }
        // ---- scores: GROUP x T partial dots, then a reduce-scatter
        float v[32];
#pragma unroll
        for (int t = 0; t < T; ++t) {
            float4 k = kr[t];
            if (!kEarly && t0 + t < w1)
                k = __ldcs(reinterpret_cast<const float4*>(keys + (size_t)(t0 + t) * row + (size_t)g * D) + lane);
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
        float s = t0 + mt < w1 ? v[0] * kLog2e : -INFINITY;
        // ---- online softmax per head (the T lanes of a head are adjacent)
        float bm = s;
#pragma unroll
        for (int n = 1; n < T; n <<= 1) bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, n));
        float m_new[GROUP];
#pragma unroll
        for (int j = 0; j < GROUP; ++j) {
            m_new[j] = fmaxf(m_run[j], __shfl_sync(kFull, bm, j * T));
            const float corr = m_new[j] == -INFINITY ? 1.0f : exp2f(m_run[j] - m_new[j]);
            l_run[j] *= corr;
#pragma unroll
            for (int u = 0; u < 4; ++u) o[j][u] *= corr;
            m_run[j] = m_new[j];
        }
        float mine = m_run[0];
#pragma unroll
        for (int j = 1; j < GROUP; ++j)
            if (mh == j) mine = m_run[j];
        const float p = s == -INFINITY ? 0.0f : exp2f(s - mine);
        float ps = p;
#pragma unroll
        for (int n = 1; n < T; n <<= 1) ps += __shfl_xor_sync(kFull, ps, n);
#pragma unroll
        for (int j = 0; j < GROUP; ++j) l_run[j] += __shfl_sync(kFull, ps, j * T);
        // ---- O += p V
#pragma unroll
        for (int t = 0; t < T; ++t) {
            float4 vv = vr[t];
            if (!kEarly && t0 + t < w1)
                vv = __ldcs(reinterpret_cast<const float4*>(values + (size_t)(t0 + t) * row + (size_t)g * D) + lane);
#pragma unroll
            for (int j = 0; j < GROUP; ++j) {
                const float pj = __shfl_sync(kFull, p, j * T + t);
                o[j][0] = fmaf(pj, vv.x, o[j][0]); o[j][1] = fmaf(pj, vv.y, o[j][1]);
                o[j][2] = fmaf(pj, vv.z, o[j][2]); o[j][3] = fmaf(pj, vv.w, o[j][3]);
            }
        }
    }

    // ---- merge the CTA's warps, write the chunk's (m, l, O) per head
    __shared__ float s_ml[kWarps][GROUP][2];
    __shared__ __align__(16) float s_o[kWarps][GROUP][D];
#pragma unroll
    for (int j = 0; j < GROUP; ++j) {
        *reinterpret_cast<float4*>(&s_o[warp][j][4 * lane]) = make_float4(o[j][0], o[j][1], o[j][2], o[j][3]);
        if (lane == 0) { s_ml[warp][j][0] = m_run[j]; s_ml[warp][j][1] = l_run[j]; }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < GROUP * D; idx += kWarps * 32) {
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

int f32_decode_chunks(int len) { return len <= 0 ? 0 : (len + kF32ChunkTokens - 1) / kF32ChunkTokens; }

size_t f32_decode_workspace_bytes(int max_len, int num_heads) {
    return (size_t)f32_decode_chunks(max_len) * num_heads * (D + 2) * sizeof(float);
}

cudaError_t launch_decode_f32(const float* keys, const float* values, int num_kv_heads,
                              int num_heads, int len, const float* q, float q_mul, float* out,
                              void* ws, cudaStream_t st) {
    const int group = num_heads / num_kv_heads;
    const int chunks = f32_decode_chunks(len);
    if (chunks == 0) return cudaMemsetAsync(out, 0, (size_t)num_heads * D * sizeof(float), st);
    float* part_o = static_cast<float*>(ws);
    float* part_ml = part_o + (size_t)chunks * num_heads * D;
    dim3 grid(chunks, num_kv_heads);
    switch (group) {
        case 1: decode_f32_kernel<1><<<grid, kWarps * 32, 0, st>>>(keys, values, num_kv_heads, len, kF32ChunkTokens, q, q_mul, part_o, part_ml); break;
        case 2: decode_f32_kernel<2><<<grid, kWarps * 32, 0, st>>>(keys, values, num_kv_heads, len, kF32ChunkTokens, q, q_mul, part_o, part_ml); break;
        case 4: decode_f32_kernel<4><<<grid, kWarps * 32, 0, st>>>(keys, values, num_kv_heads, len, kF32ChunkTokens, q, q_mul, part_o, part_ml); break;
        case 8: decode_f32_kernel<8><<<grid, kWarps * 32, 0, st>>>(keys, values, num_kv_heads, len, kF32ChunkTokens, q, q_mul, part_o, part_ml); break;
        default: return cudaErrorInvalidValue;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return launch_lse_combine(part_o, part_ml, chunks, 1, num_heads, out, st);
}

}  // namespace ec
