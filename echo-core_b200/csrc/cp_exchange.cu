// cp_exchange.cu -- the context-parallel exchange and merge in one kernel,
// over NVLink peer memory (one process per GPU).
//
// Context parallelism splits one long sequence's cached tokens across ranks;
// each rank computes the unnormalised partial (m, l, O) of its slice per
// (sequence, head) (ec_decode_attention_partial).  Instead of an all-gather
// followed by a merge launch, every CTA of this kernel owns one (sequence,
// head), or one split of its dims: it stores its rank's partial into slot
// [rank] of every other rank's receive buffer with plain peer stores (CUDA
// IPC mappings, no multicast), each value as a 64-bit word that carries the
// step's epoch beside it, then waits, thread by thread, until the words of
// every other rank in its own buffer show this step's epoch, and merges the
// world's partials in rank order.  A word is its own flag, so the exchange
// needs no fence and no separate flag store: one NVLink trip a step.  Receive
// buffers are double-buffered by step parity: a fast rank publishing step e+1
// never overwrites what a slow rank is still merging for step e.  Every wait
// is bounded (about 1 s of clock64 cycles); a wait that runs out records
// EC_DEVERR_TIMEOUT in the error word and the thread writes zero.
//
// The chunked form (CHUNKS) takes the decode kernel's split-K chunk partials
// of this rank's slice straight from its workspace and merges them first, in
// the same CTA, so a context-parallel decode step is two launches per rank:
// the decode kernel and this one (no separate chunk-merge launch).
#include <cstdint>

#include "ec_common.cuh"
#include "ec_internal.h"

namespace ec {
namespace {

constexpr int D = 128;

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

constexpr int kXThreads = 256;                    // threads of the chunked form
constexpr int kMaxChunkMerge = 1024;               // chunks per (sequence, head), at most
constexpr int kXBatch = 8;                         // O loads in flight a thread
constexpr int kXMlPerThread = kMaxChunkMerge / kXThreads;


// This rank's partial of (s, h) merged from its split-K chunks, for the
// CTA's dims [z * dims, (z + 1) * dims): o (dim z * dims + t, for threads
// t < dims), m and l (every thread), the LSE merge of the chunk merge
// kernel.  Threads are float4 column groups x chunk lanes; each issues its
// first kXBatch O loads together with the (m, l) loads, before the maximum
// is known, so the merge is one dependent round trip after the table read.
__device__ void merge_chunks(const CpExchangeArgs& a, int s, int h, int z, int dims, float& o,
                             float& m_out, float& l_out) {
    constexpr int kWarpsX = kXThreads / 32;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int H = a.num_heads;
    const int groups = dims / 4, lanes = kXThreads / groups;
    int len = a.seq_len ? a.seq_len[s] : 0;
    len = len < 0 ? 0 : len;
    int nch = (len + a.chunk_tokens - 1) / a.chunk_tokens;
    nch = nch > a.max_chunks ? a.max_chunks : nch;   // a bad entry is flagged by the decode
    const size_t base = (size_t)s * a.max_chunks * H + h;
    __shared__ float s_f[kMaxChunkMerge];
    __shared__ __align__(16) float s_acc[kXThreads * 4];   // [lane][dims]
    __shared__ float s_rm[kWarpsX], s_rl[kWarpsX];
    __shared__ float s_M, s_L;

    const int gi = tid % groups, cl = tid / groups;
    const float4* po = reinterpret_cast<const float4*>(a.part_o + base * D + z * dims) + gi;
    const size_t cstride = (size_t)H * (D / 4);        // float4s from chunk to chunk
    float4 v[kXBatch];
#pragma unroll
    for (int k = 0; k < kXBatch; ++k) {
        const int c = cl + k * lanes;
        v[k] = c < nch ? po[(size_t)c * cstride] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float2 ml[kXMlPerThread];
#pragma unroll
    for (int k = 0; k < kXMlPerThread; ++k) {
        const int c = tid + k * kXThreads;
        ml[k] = c < nch ? *reinterpret_cast<const float2*>(a.part_ml + (base + (size_t)c * H) * 2)
                        : make_float2(-INFINITY, 0.0f);
    }
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < kXMlPerThread; ++k) m = fmaxf(m, ml[k].x);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) s_rm[wid] = m;
    __syncthreads();
    if (tid == 0) {
        float M = -INFINITY;
        for (int w = 0; w < kWarpsX; ++w) M = fmaxf(M, s_rm[w]);
        s_M = M;
    }
    __syncthreads();
    const float M = s_M;
    float lsum = 0.0f;
#pragma unroll
    for (int k = 0; k < kXMlPerThread; ++k) {
        const int c = tid + k * kXThreads;
        const float f = ml[k].x == -INFINITY ? 0.0f : exp2f(ml[k].x - M);
        if (c < nch) s_f[c] = f;
        lsum += f * ml[k].y;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    if (lane == 0) s_rl[wid] = lsum;
    __syncthreads();                                  // s_f and s_rl complete
    if (tid == 0) {
        float L = 0.0f;
        for (int w = 0; w < kWarpsX; ++w) L += s_rl[w];
        s_L = L;
    }
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < kXBatch; ++k) {
        const int c = cl + k * lanes;
        const float f = c < nch ? s_f[c] : 0.0f;
        acc.x += f * v[k].x;
        acc.y += f * v[k].y;
        acc.z += f * v[k].z;
        acc.w += f * v[k].w;
    }
    for (int c0 = cl + kXBatch * lanes; c0 < nch; c0 += kXBatch * lanes) {
#pragma unroll
        for (int k = 0; k < kXBatch; ++k) {
            const int c = c0 + k * lanes;
            v[k] = c < nch ? po[(size_t)c * cstride] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int k = 0; k < kXBatch; ++k) {
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
    o = 0.0f;
    if (tid < dims)
        for (int q = 0; q < lanes; ++q) o += s_acc[q * dims + tid];   // lanes in order
    m_out = nch ? M : -INFINITY;
    l_out = s_L;
    __syncthreads();
}

// One CTA per (sequence, head, dims split z): gridDim.z = 1 for the plain
// form (partials given), merge_splits() for the chunked form.  Every split
// has its own (m, l) words and device epoch, so the CTAs of a (sequence,
// head) publish, wait and merge independently.
template <bool CHUNKS>
__global__ void __launch_bounds__(CHUNKS ? kXThreads : D) cp_exchange_kernel(CpExchangeArgs a) {
    const int s = blockIdx.x, h = blockIdx.y, z = blockIdx.z, t = threadIdx.x;
    const int S = a.num_seqs, H = a.num_heads, W = a.world;
    const int dims = D / (int)gridDim.z;
    const size_t sh = (size_t)s * H + h;
    const size_t shz = sh * kCpSplitMax + z;
    if (CHUNKS) {
        pdl_wait();   // the decode kernel's chunk partials
        pdl_trigger();
    }
    // device epochs: one counter per (sequence, head, split), advanced by the
    // only CTA that uses it, so every call of a replayed graph runs the next epoch
    __shared__ uint32_t s_epoch;
    if (t == 0) {
        uint32_t e = a.epoch;
        if (a.epoch_dev) {
            e = a.epoch_dev[shz] + 1;
            a.epoch_dev[shz] = e;
        }
        s_epoch = e;
    }
    __syncthreads();
    const uint32_t epoch = s_epoch;
    const int par = epoch & 1;
    // per rank buffer of 64-bit words, each (epoch << 32 | value bits):
    // [2 parities][W ranks][S][H] of O (D words), then [2][W][S][H][kCpSplitMax]
    // of (m, l).  A word carries its own step, so a reader needs no flag and no
    // fence: it waits until the word it reads shows this step's epoch (an
    // aligned 64-bit relaxed store or load is single-copy atomic).
    const size_t n_sh = (size_t)S * H;
    auto o_at = [&](float* base, int p, int r) {
        return reinterpret_cast<uint64_t*>(base) + ((size_t)(p * W + r) * n_sh + sh) * D;
    };
    auto ml_at = [&](float* base, int p, int r) {
        return reinterpret_cast<uint64_t*>(base) + (size_t)2 * W * n_sh * D +
               (((size_t)(p * W + r) * n_sh + sh) * kCpSplitMax + z) * 2;
    };
    auto word = [&](float v) { return (uint64_t)epoch << 32 | __float_as_uint(v); };

    // ---- publish this rank's partial (this split's dims) into slot [rank]
    // of every other rank's buffer
    float o, m_loc, l_loc;
    if (CHUNKS) {
        merge_chunks(a, s, h, z, dims, o, m_loc, l_loc);
    } else {
        o = a.part_o[sh * D + t];
        m_loc = a.part_ml[sh * 2];
        l_loc = a.part_ml[sh * 2 + 1];
    }
    if (t < dims) {
        for (int r = 0; r < W; ++r) {
            if (r == a.rank) continue;
            float* base = a.peer_base[r];
            st_relaxed_sys_u64(o_at(base, par, a.rank) + z * dims + t, word(o));
            if (t < 2) st_relaxed_sys_u64(ml_at(base, par, a.rank) + t, word(t == 0 ? m_loc : l_loc));
        }
    }
    if (t >= dims) return;

    // ---- every other rank's words of this step, from the local buffer
    float* mine = a.peer_base[a.rank];
    bool bad = false;
    auto wait_word = [&](const uint64_t* w, float& v) {
        uint64_t x = ld_relaxed_sys_u64(w);
        if ((uint32_t)(x >> 32) != epoch) {
            const long long t0 = clock64();
            while ((uint32_t)((x = ld_relaxed_sys_u64(w)) >> 32) != epoch) {
                if (clock64() - t0 > kWaitBudgetCycles) {
                    bad = true;
                    return;
                }
                __nanosleep(32);
            }
        }
        v = __uint_as_float((uint32_t)x);
    };
    float rm[kCpMaxWorld], rl[kCpMaxWorld], ro[kCpMaxWorld];
    for (int r = 0; r < W && !bad; ++r) {
        if (r == a.rank) {
            rm[r] = m_loc;
            rl[r] = l_loc;
            ro[r] = o;
            continue;
        }
        wait_word(ml_at(mine, par, r), rm[r]);
        if (!bad) wait_word(ml_at(mine, par, r) + 1, rl[r]);
        if (!bad) wait_word(o_at(mine, par, r) + z * dims + t, ro[r]);
    }
    const size_t oi = sh * D + z * dims + t;
    if (bad) {
        flag_error(a.err, EC_DEVERR_TIMEOUT);
        a.out[oi] = 0.0f;
        return;
    }
    // ---- merge in rank order (the LSE merge of ec_lse_combine)
    float M = -INFINITY;
    for (int r = 0; r < W; ++r) M = fmaxf(M, rm[r]);
    float so = 0.0f, sl = 0.0f;
    for (int r = 0; r < W; ++r) {
        const float f = rm[r] == -INFINITY ? 0.0f : exp2f(rm[r] - M);
        so += f * ro[r];
        sl += f * rl[r];
    }
    a.out[oi] = sl > 0.0f ? __fdiv_rn(so, sl) : 0.0f;
}

}  // namespace

size_t cp_exchange_buffer_bytes(int world, int num_seqs, int num_heads) {
    const size_t n = (size_t)2 * world * num_seqs * num_heads;
    return n * (D + 2 * kCpSplitMax) * sizeof(uint64_t);
}

cudaError_t launch_cp_exchange(const CpExchangeArgs& a, cudaStream_t st) {
    if (a.num_seqs <= 0 || a.num_heads <= 0) return cudaSuccess;
    if (a.max_chunks > 0) {
        if (a.max_chunks > kMaxChunkMerge || a.chunk_tokens <= 0) return cudaErrorInvalidValue;
        const int z = merge_splits(a.num_seqs * a.num_heads);
        return launch_pdl(cp_exchange_kernel<true>, dim3(a.num_seqs, a.num_heads, z),
                          dim3(kXThreads), 0, st, a);
    }
    cp_exchange_kernel<false><<<dim3(a.num_seqs, a.num_heads), D, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace ec
