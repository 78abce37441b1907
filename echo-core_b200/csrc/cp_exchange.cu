// cp_exchange.cu -- the context-parallel exchange and merge in one kernel,
// over NVLink peer memory (one process per GPU).
//
// Context parallelism splits one long sequence's cached tokens across ranks;
// each rank computes the unnormalised partial (m, l, O) of its slice per
// (sequence, head) (ec_decode_attention_partial).  Instead of an all-gather
// followed by a merge launch, every CTA of this kernel owns one (sequence,
// head): it stores its rank's partial into slot [rank] of every rank's
// receive buffer with plain peer stores (CUDA IPC mappings, no multicast),
// publishes a per-(sequence, head) flag with release semantics, waits with
// acquire loads until every rank's flag for this step has arrived in its own
// buffer, and merges the world's partials in rank order.  Receive buffers are
// double-buffered by step parity: a fast rank publishing step e+1 never
// overwrites what a slow rank is still merging for step e.  Every wait is
// bounded (about 1 s of clock64 cycles); a wait that runs out records
// EC_DEVERR_TIMEOUT in the error word and the CTA writes zeros.
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

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

constexpr int kChunkSplit = 4;                     // thread groups of the chunk merge
constexpr int kMaxChunkMerge = 1024;               // chunks per (sequence, head), at most

// This rank's partial of (s, h) merged from its split-K chunks: (o[d] for the
// calling thread's dim, m, l), the LSE merge of the chunk merge kernel.
// Every thread of the block takes part; threads d < D get o.
__device__ void merge_chunks(const CpExchangeArgs& a, int s, int h, float& o, float& m_out,
                             float& l_out) {
    constexpr int NT = D * kChunkSplit;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int d = tid % D, part = tid / D;
    const int H = a.num_heads;
    int len = a.seq_len ? a.seq_len[s] : 0;
    len = len < 0 ? 0 : len;
    int nch = (len + a.chunk_tokens - 1) / a.chunk_tokens;
    nch = nch > a.max_chunks ? a.max_chunks : nch;   // a bad entry is flagged by the decode
    const size_t base = (size_t)s * a.max_chunks * H + h;
    __shared__ float s_f[kMaxChunkMerge], s_red[NT];
    __shared__ float s_M, s_L;
    auto ml_of = [&](int c) {
        return *reinterpret_cast<const float2*>(a.part_ml + (base + (size_t)c * H) * 2);
    };
    float m = -INFINITY;
    for (int c = tid; c < nch; c += NT) m = fmaxf(m, ml_of(c).x);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) s_red[wid] = m;
    __syncthreads();
    if (tid == 0) {
        float M = -INFINITY;
        for (int w = 0; w < NT / 32; ++w) M = fmaxf(M, s_red[w]);
        s_M = M;
    }
    __syncthreads();
    const float M = s_M;
    float lsum = 0.0f;
    for (int c = tid; c < nch; c += NT) {
        const float2 mlc = ml_of(c);
        const float f = mlc.x == -INFINITY ? 0.0f : exp2f(mlc.x - M);
        s_f[c] = f;
        lsum += f * mlc.y;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    __syncthreads();
    if (lane == 0) s_red[wid] = lsum;
    __syncthreads();
    if (tid == 0) {
        float L = 0.0f;
        for (int w = 0; w < NT / 32; ++w) L += s_red[w];
        s_L = L;
    }
    __syncthreads();
    float so = 0.0f;
#pragma unroll 4
    for (int c = part; c < nch; c += kChunkSplit) so += s_f[c] * a.part_o[(base + (size_t)c * H) * D + d];
    s_red[part * D + d] = so;
    __syncthreads();
    o = 0.0f;
    if (part == 0) {
#pragma unroll
        for (int q = 0; q < kChunkSplit; ++q) o += s_red[q * D + d];
    }
    m_out = nch ? M : -INFINITY;
    l_out = s_L;
    __syncthreads();
}

template <bool CHUNKS>
__global__ void __launch_bounds__(CHUNKS ? D * kChunkSplit : D) cp_exchange_kernel(CpExchangeArgs a) {
    const int s = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    const int S = a.num_seqs, H = a.num_heads, W = a.world;
    const size_t sh = (size_t)s * H + h;
    if (CHUNKS) {
        pdl_wait();   // the decode kernel's chunk partials
        pdl_trigger();
    }
    // device epochs: one counter per (sequence, head), advanced by the only
    // CTA that uses it, so every call of a replayed graph runs the next epoch
    __shared__ uint32_t s_epoch;
    if (d == 0) {
        uint32_t e = a.epoch;
        if (a.epoch_dev) {
            e = a.epoch_dev[sh] + 1;
            a.epoch_dev[sh] = e;
        }
        s_epoch = e;
    }
    __syncthreads();
    const uint32_t epoch = s_epoch;
    const int par = epoch & 1;
    // per rank buffer: [2 parities][W ranks][S][H] of O (D floats), ml (2), flag (1)
    const size_t n_sh = (size_t)S * H;
    auto o_at = [&](float* base, int p, int r) { return base + ((size_t)(p * W + r) * n_sh + sh) * D; };
    auto ml_at = [&](float* base, int p, int r) {
        return base + (size_t)2 * W * n_sh * D + ((size_t)(p * W + r) * n_sh + sh) * 2;
    };
    auto flag_at = [&](float* base, int p, int r) {
        return reinterpret_cast<uint32_t*>(base + (size_t)2 * W * n_sh * (D + 2)) +
               (size_t)(p * W + r) * n_sh + sh;
    };

    // ---- publish this rank's partial into slot [rank] of every rank's buffer
    float o, ml;
    if (CHUNKS) {
        float m_loc, l_loc;
        merge_chunks(a, s, h, o, m_loc, l_loc);
        ml = d == 0 ? m_loc : l_loc;
    } else {
        o = a.part_o[sh * D + d];
        ml = d < 2 ? a.part_ml[sh * 2 + d] : 0.0f;
    }
    if (d < D) {
        for (int r = 0; r < W; ++r) {
            float* base = a.peer_base[r];
            o_at(base, par, a.rank)[d] = o;
            if (d < 2) ml_at(base, par, a.rank)[d] = ml;
        }
    }
    __threadfence_system();
    __syncthreads();
    if (d == 0)
        for (int r = 0; r < W; ++r) st_release_sys(flag_at(a.peer_base[r], par, a.rank), epoch);

    // ---- wait for every rank's flag of this step in the local buffer
    __shared__ int s_bad;
    if (d == 0) {
        int bad = 0;
        float* mine = a.peer_base[a.rank];
        for (int r = 0; r < W && !bad; ++r) {
            const uint32_t* f = flag_at(mine, par, r);
            if (ld_acquire_sys(f) == epoch) continue;
            const long long t0 = clock64();
            while (ld_acquire_sys(f) != epoch) {
                if (clock64() - t0 > kWaitBudgetCycles) { bad = 1; break; }
                __nanosleep(64);
            }
        }
        if (bad) flag_error(a.err, EC_DEVERR_TIMEOUT);
        s_bad = bad;
    }
    __syncthreads();
    float* mine = a.peer_base[a.rank];
    if (d >= D) return;
    if (s_bad) {
        a.out[sh * D + d] = 0.0f;
        return;
    }
    // ---- merge in rank order (the LSE merge of ec_lse_combine)
    float M = -INFINITY;
    for (int r = 0; r < W; ++r) M = fmaxf(M, ml_at(mine, par, r)[0]);
    float so = 0.0f, sl = 0.0f;
    for (int r = 0; r < W; ++r) {
        const float* mlr = ml_at(mine, par, r);
        const float f = mlr[0] == -INFINITY ? 0.0f : exp2f(mlr[0] - M);
        so += f * o_at(mine, par, r)[d];
        sl += f * mlr[1];
    }
    a.out[sh * D + d] = sl > 0.0f ? __fdiv_rn(so, sl) : 0.0f;
}

}  // namespace

size_t cp_exchange_buffer_bytes(int world, int num_seqs, int num_heads) {
    const size_t n = (size_t)2 * world * num_seqs * num_heads;
    return n * (D + 2) * sizeof(float) + n * sizeof(uint32_t);
}

cudaError_t launch_cp_exchange(const CpExchangeArgs& a, cudaStream_t st) {
    if (a.num_seqs <= 0 || a.num_heads <= 0) return cudaSuccess;
    if (a.max_chunks > 0) {
        if (a.max_chunks > kMaxChunkMerge || a.chunk_tokens <= 0) return cudaErrorInvalidValue;
        return launch_pdl(cp_exchange_kernel<true>, dim3(a.num_seqs, a.num_heads),
                          dim3(D * kChunkSplit), 0, st, a);
    }
    cp_exchange_kernel<false><<<dim3(a.num_seqs, a.num_heads), D, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace ec
