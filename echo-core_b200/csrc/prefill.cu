// prefill.cu -- causal chunked-prefill attention over the int8 KV cache on the
// 5th-generation tensor cores (tcgen05, sm_100a).
//
// The reference has no chunked prefill: a prompt is fed one token at a time
// (src/main.cpp:404-405), each token running the decode loop of
// InferenceEngine::attention (src/inference.cpp:321-392) over the cache as it
// stands after that token's append.  So query row i of an n_new-token chunk
// appended after `past` cached tokens attends to slots [0, past + i]; this
// kernel computes exactly that for all rows at once.
//
// One CTA owns 128 query rows of one query head of one sequence (query head h
// reads KV head h % num_kv_heads, src/inference.cpp:335).  Warp roles:
//   producer  (warp 12)   2-D TMA of the int8 K and V codes of 128-token
//                         tiles (128-byte swizzle, no multicast), 2 stages;
//   converter (warps 8-11) int8 -> f16 K (K-major) and int8 -> f16 V
//                         (MN-major), both exact, into 128B-swizzled UMMA
//                         operand layouts (K one tile, V two tiles);
//   MMA       (warp 13)   one thread issues tcgen05.mma: S = Q K^T (f16 x
//                         f16 -> fp32) into one of three S/P buffers in TMEM,
//                         one tile ahead of the softmax, then O += P'hi V +
//                         P'lo V with P' read from TMEM (f16 x f16 -> fp32,
//                         accumulated in TMEM);
//   softmax   (warps 0-7) query row r is TMEM lane r; warps w and w+4 share
//                         the lanes of quadrant w and split each tile's 128
//                         columns in halves, exchanging the row maximum
//                         through shared memory.  They scale S by the
//                         per-token k-scale, mask causally, run the online
//                         softmax in base 2 with lazy rescaling of O, and write
//                         p' = p * v_scale (the fused v-scale) as an f16 hi/lo
//                         pair over the S columns they have read.
// Q is cast to bf16 on load (the queries are bf16-cast), then held as f16
// under one power-of-two scale per CTA (exact for the bf16 values); the
// softmax scale, log2(e) and the inverse power of two multiply the fp32
// scores.  K and V codes are exact in f16; p'
// enters the PV product as an f16 pair hi + lo (two MMAs), about 22 bits, so
// the only rounding of consequence is Q's bf16 cast (part of the contract).
// Each query row carries its own power of two 2^-E, fixed before the first
// tile from the largest v-scale of the row's causal range, that keeps every
// p' = p * v_scale * 2^-E below 2^15 (any finite v-scale is in range) and
// puts the row's largest p' near the top of f16's range (its relative
// precision).  It enters the softmax exponent, 2^(s - m - E), so both p'
// and the row sum l carry it and the output O / l needs no correction.
// Every wait is bounded; a timeout raises a CTA-wide abort flag so that every
// role stops, waits for its own in-flight work and the CTA frees its tensor
// memory before returning.  The softmax warps decide together (a barrier
// that ORs their failure flags) so that none is left at a named barrier.
#include <cmath>
#include <cstdint>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ec_common.cuh"
#include "ec_internal.h"

namespace ec {
namespace {

constexpr int D = 128;
constexpr int BM = 128;                    // query rows per CTA (TMEM lanes)
constexpr int BN = 128;                    // kv tokens per tile
// Warp roles:
//   warps 0-7   softmax: warp w owns TMEM lanes 32*(w%4).. (query rows) and
//               columns 64*(w/4).. of every S/P buffer and of O;
//   warps 8-11  converter;
//   warp 12     TMA producer, warp 13 MMA issuer.
// Four warps share an SMSP's 16K registers, so every thread gets 128.
constexpr int kConvWarp0 = 8;
constexpr int kProducerWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kThreads = 14 * 32;
constexpr int kSoftmaxThreads = 256;
constexpr int ATOM = 128 * 128;            // one [128 rows][128 B] swizzled block
constexpr int OFF_Q = 0;                   // f16 Q    : 2 K-blocks (dims 0-63, 64-127)
constexpr int OFF_K = OFF_Q + 2 * ATOM;    // f16 K    : 2 K-blocks (one tile)
constexpr int OFF_V = OFF_K + 2 * ATOM;    // f16  V   : [2 buffers][2 dim halves], MN-major
constexpr int I8_TILE = BN * 128;          // 16 KB of int8 codes
constexpr int OFF_I8 = OFF_V + 4 * ATOM;   // [2 stages][K, V]
constexpr int OFF_SC = OFF_I8 + 2 * 2 * I8_TILE;   // [2 tiles][k-scale*qk_mul [BN], v-scale [BN]]
constexpr int OFF_RED = OFF_SC + 2 * 2 * BN * 4;   // [2 tiles][2 column halves][BM] row exchange
constexpr int OFF_BAR = OFF_RED + 2 * 2 * BM * 4;
enum {
    B_KV_FULL = 0, B_KV_EMPTY = 2, B_KC_FULL = 4, B_KC_FREE = 5, B_VC_FULL = 6, B_VC_FREE = 8,
    B_S_FULL = 10, B_P_FULL = 13, B_PV_BUF = 16, B_Q_FULL = 19, B_DRAIN, NBARS
};
constexpr int OFF_MISC = OFF_BAR + NBARS * 8;      // [0] tmem base, [1] abort flag
constexpr int OFF_EROW = OFF_MISC + 16;            // [BM] each query row's E (float)
constexpr int SMEM = 1024 + OFF_EROW + BM * 4;
static_assert(SMEM <= 227 * 1024, "shared memory budget");

// Tensor memory: three S/P buffers of 128 columns (QK^T scores, overwritten in
// place by p' as f16 hi/lo pairs), then the O accumulator.
constexpr int TMEM_COLS = 512;
constexpr int NSP = 3;
constexpr int TM_O = 384;
constexpr float kLazyRescale = 8.0f;
// E puts a row's v-scales below 2^7 (p <= 2^8 under the lazy rescale, so p'
// < 2^15, inside f16 with its hi/lo split), within [kEMin, 121]: the floor
// (reached only by v-scales below 2^-57) keeps 2^(s - m - E) and the row sum
// finite for any sequence length.
constexpr int kVScaleBits = 7;
constexpr int kEMin = -64;
constexpr unsigned kFull = 0xffffffffu;

// Instruction descriptors (kind::f16, fp32 accumulate, M = 128, N = 128).
constexpr uint32_t kIdescQK = (1u << 4) | (0u << 7) | (0u << 10) | (16u << 17) | (8u << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (0u << 7) | (0u << 10) | (1u << 16) | (16u << 17) | (8u << 24);

struct Smem {
    uint8_t* base;
    __device__ uint64_t* bar(int i) const { return reinterpret_cast<uint64_t*>(base + OFF_BAR) + i; }
    __device__ volatile int* abort_flag() const {
        return reinterpret_cast<volatile int*>(base + OFF_MISC) + 1;
    }
    __device__ uint32_t* tmem_slot() const { return reinterpret_cast<uint32_t*>(base + OFF_MISC); }
};

// Bounded wait that also gives up as soon as another role has aborted.  The
// waiting thread sleeps in try_wait (up to kSuspendNs per round) rather than
// spinning, so idle roles leave the issue slots to the softmax and converter.
constexpr uint32_t kSuspendNs = 100000;
__device__ __forceinline__ bool wait_abortable(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity, kSuspendNs)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kWaitBudgetCycles) {
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ bool warp_wait_abortable(uint64_t* bar, uint32_t parity,
                                                    volatile int* abort_flag) {
    return __all_sync(kFull, wait_abortable(bar, parity, abort_flag));
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 128B-swizzled shared-memory matrix descriptor (sm_100 UMMA format).
__device__ __forceinline__ uint64_t umma_desc(const void* p, uint32_t lbo, uint32_t sbo) {
    const uint32_t a = smem_addr(p);
    return (uint64_t)((a >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                     bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)accumulate), "r"(0u), "r"(0u),
        "r"(0u), "r"(0u));
}

// A operand from tensor memory (rows = lanes, 2 f16 per 32-bit column).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                        uint32_t idesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"((uint32_t)accumulate), "r"(0u),
        "r"(0u), "r"(0u), "r"(0u));
}

// 16-lane tensor-memory shapes.  For a base address at lane L, column C and
// thread t (g = t / 4, q = t % 4):
//   16x256b, repetition n: v[4n+0], v[4n+1] = lane L+g,   columns C+8n+2q, +1
//                          v[4n+2], v[4n+3] = lane L+g+8, the same columns
//   16x128b, repetition r: v[2r+0] = lane L+g, column C+4r+q; v[2r+1] = lane L+g+8
#define EC_R4(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3])
__device__ __forceinline__ void tmem_ld_16x256b_x2(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : EC_R4(0), EC_R4(4) : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : EC_R4(0), EC_R4(4), EC_R4(8), EC_R4(12) : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_16x256b_x8(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : EC_R4(0), EC_R4(4), EC_R4(8), EC_R4(12), EC_R4(16), EC_R4(20), EC_R4(24), EC_R4(28)
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
#undef EC_R4
__device__ __forceinline__ void tmem_st_16x256b_x2(uint32_t taddr, const float (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x256b.x2.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
        ::"r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]),
        "f"(v[7])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_16x128b_x4(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x128b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
        "r"(v[7])
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_addr(bar)) : "memory");
}

// Byte offset of 16-byte chunk c of row r in a [rows][128 B] 128B-swizzled block.
__device__ __forceinline__ int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// int8 code row (a 128-byte swizzled TMA row) -> f16 token row t of a
// [2 dim halves][128 tokens][64 dims] 128B-swizzled operand: the K-major
// layout of K for QK^T and the MN-major layout of V for PV are the same bytes.
__device__ __forceinline__ void convert_row_f16(const uint8_t* src, uint8_t* vs, int t) {
    const __half2 bias = __floats2half2_rn(1152.0f, 1152.0f);  // 1024 + 128
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint4 w = *reinterpret_cast<const uint4*>(src + swz(t, c));
        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
        uint32_t o[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            // biased bytes under the f16 exponent of 1024: 0x64uu = 1024 + u
            const uint32_t b = ww[q] ^ 0x80808080u;
            uint32_t h0 = __byte_perm(b, 0x64646464u, 0x5140);   // bytes 0,1
            uint32_t h1 = __byte_perm(b, 0x64646464u, 0x7362);   // bytes 2,3
            __half2 x0 = __hsub2(*reinterpret_cast<__half2*>(&h0), bias);
            __half2 x1 = __hsub2(*reinterpret_cast<__half2*>(&h1), bias);
            o[2 * q] = *reinterpret_cast<uint32_t*>(&x0);
            o[2 * q + 1] = *reinterpret_cast<uint32_t*>(&x1);
        }
        uint8_t* blk = vs + (c >> 2) * ATOM;
        const int cb = 2 * (c & 3);
        *reinterpret_cast<uint4*>(blk + swz(t, cb)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(blk + swz(t, cb + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

// 2^x on the SFU (ex2.approx: relative error about 2^-22, -inf -> +0).
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// pv - float(h) per half, each a mixed-precision fma (f16 x f16 + f32 -> f32,
// one rounding): h * -1 + pv.  pv - h is exact in f32 when h = f16(pv).
__device__ __forceinline__ float2 minus_f16x2_from_f32x2(__half2 h, float2 pv) {
    float2 d;
    asm("{\n\t.reg .f16 a0, a1, m;\n\t"
        "mov.b32 {a0, a1}, %2;\n\t"
        "mov.b16 m, 0xBC00;\n\t"
        "fma.rn.f32.f16 %0, a0, m, %3;\n\t"
        "fma.rn.f32.f16 %1, a1, m, %4;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "r"(*reinterpret_cast<const uint32_t*>(&h)), "f"(pv.x), "f"(pv.y));
    return d;
}

// max of three (one sm_100 instruction)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ void named_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Named barrier that also ORs a flag over its threads: every participant
// learns whether any of them failed, so all leave a loop at the same point.
__device__ __forceinline__ bool bar_any(int id, int threads, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %3, 0;\n\t"
        "bar.red.or.pred p, %1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(id), "r"(threads), "r"((uint32_t)v)
        : "memory");
    return r != 0;
}



// Output row of query row r of this CTA's block.  Recomputed from the block
// index (read through asm volatile, so the compiler cannot reuse the values
// from the kernel's start): nothing of it stays live through the tile loop,
// whose register pressure is at the limit.
__device__ __forceinline__ float* out_row(const PrefillArgs& a, int r, bool& live) {
    uint32_t bid;
    asm volatile("mov.u32 %0, %%ctaid.x;" : "=r"(bid));
    const int H = a.num_heads, HKV = a.num_kv_heads, GROUP = H / HKV;
    const int nqb = (a.n_new + BM - 1) / BM;
    int idx = (int)bid;
    const int jh = idx % GROUP;  idx /= GROUP;
    const int qb = nqb - 1 - (idx % nqb);  idx /= nqb;
    const int h = idx % HKV + HKV * jh;
    const int seq = idx / HKV;
    const int qpos = qb * BM + r;
    live = qpos < a.n_new;
    return a.out + (((size_t)seq * a.n_new + (live ? qpos : 0)) * H + h) * D;
}

// PAGED: slots through the batch's page table.  Compiled apart so that the
// contiguous kernel carries none of the translation in its softmax loop.
template <bool PAGED>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmap_k,
                   const __grid_constant__ CUtensorMap tmap_v, const PrefillArgs a) {
    extern __shared__ uint8_t smem_raw[];
    Smem S{reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                      ~uintptr_t(1023))};
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- work item: heaviest (latest) query blocks first; the GROUP heads of a
    // KV head and neighbouring blocks are adjacent for L2 reuse of K/V.
    const int H = a.num_heads, HKV = a.num_kv_heads, GROUP = H / HKV;
    const int nqb = (a.n_new + BM - 1) / BM;
    int idx = blockIdx.x;
    const int jh = idx % GROUP;  idx /= GROUP;
    const int qb = nqb - 1 - (idx % nqb);  idx /= nqb;
    const int g = idx % HKV;
    const int seq = idx / HKV;
    const int h = g + HKV * jh;

    const int32_t off = PAGED ? 0 : a.seq_offset[seq];
    const int32_t cap = a.seq_capacity[seq], len = a.seq_len[seq];
    const int past = len - a.n_new;
    const PageMap pm = PAGED ? a.pages : PageMap{nullptr, 0, 0};
    if (!(page_entry_ok(pm, off, cap, len, a.total_slots) && past >= 0)) {
        if (threadIdx.x == 0 && qb == nqb - 1 && jh == 0) flag_error(a.err, EC_DEVERR_BAD_TABLE);
        return;
    }
    const int q0 = qb * BM;
    const int rows = min(BM, a.n_new - q0);
    const int kv_end = past + q0 + rows;              // exclusive
    const int ntiles = (kv_end + BN - 1) / BN;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(S.bar(B_KV_FULL + i), 1);
            mbar_init(S.bar(B_KV_EMPTY + i), 4);
            mbar_init(S.bar(B_VC_FULL + i), 4);
            mbar_init(S.bar(B_VC_FREE + i), 1);
        }
        mbar_init(S.bar(B_KC_FULL), 4);
        mbar_init(S.bar(B_KC_FREE), 1);
        for (int i = 0; i < NSP; ++i) {
            mbar_init(S.bar(B_S_FULL + i), 1);
            mbar_init(S.bar(B_P_FULL + i), 8);
            mbar_init(S.bar(B_PV_BUF + i), 1);
        }
        mbar_init(S.bar(B_Q_FULL), 8);
        mbar_init(S.bar(B_DRAIN), 1);
        *S.abort_flag() = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(S.tmem_slot())), "r"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *S.tmem_slot();
    volatile int* abort_flag = S.abort_flag();
    uint8_t* Qs = S.base + OFF_Q;
    uint8_t* Kc = S.base + OFF_K;
    uint8_t* I8 = S.base + OFF_I8;
    auto Vc = [&](int b) { return S.base + OFF_V + b * 2 * ATOM; };

    if (warp >= kProducerWarp) {
        if (warp == kProducerWarp && lane == 0) {
            // ============================================================ TMA
            const uint64_t pol = l2_policy_evict_first();
            int issued = 0;
            for (int j = 0; j < ntiles; ++j) {
                const int st = j & 1;
                if (j >= 2 && !wait_abortable(S.bar(B_KV_EMPTY + st), ((j >> 1) - 1) & 1, abort_flag))
                    break;
                mbar_arrive_expect_tx(S.bar(B_KV_FULL + st), 2 * I8_TILE);
                // a tile never crosses a page (pages are multiples of 128 tokens);
                // a bad page id is flagged and slot 0 read instead
                int64_t slot = off + j * BN;
                if (PAGED && !page_slot(pm, seq, off, j * BN, a.total_slots, slot)) {
                    flag_error(a.err, EC_DEVERR_BAD_TABLE);
                    slot = 0;
                }
                const int y = (int)slot;
                tma_load_2d(I8 + (2 * st) * I8_TILE, &tmap_k, g * D, y, S.bar(B_KV_FULL + st), pol);
                tma_load_2d(I8 + (2 * st + 1) * I8_TILE, &tmap_v, g * D, y, S.bar(B_KV_FULL + st), pol);
                issued = j + 1;
            }
            // never leave with copies in flight into this CTA's shared memory
            for (int j = max(0, issued - 2); j < issued; ++j) {
                const long long t0 = clock64();
                while (!mbar_try_wait(S.bar(B_KV_FULL + (j & 1)), (j >> 1) & 1) &&
                       clock64() - t0 < kWaitBudgetCycles) {
                }
            }
        } else if (warp == kMmaWarp && lane == 0) {
            // ============================================================ MMA
            bool ok = wait_abortable(S.bar(B_Q_FULL), 0, abort_flag);
            // S = Q K^T of tile j into S/P buffer j % 3
            auto qk = [&](int j) -> bool {
                const int sb = j % NSP;
                if (!wait_abortable(S.bar(B_KC_FULL), j & 1, abort_flag)) return false;
                if (j >= NSP && !wait_abortable(S.bar(B_PV_BUF + sb), ((j / NSP) - 1) & 1, abort_flag))
                    return false;   // PV of tile j - 3 has read its p' out of this buffer
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const int o = (kk >> 2) * ATOM + (kk & 3) * 32;
                    umma(tmem + sb * BN, umma_desc(Qs + o, 16, 1024), umma_desc(Kc + o, 16, 1024),
                         kIdescQK, kk > 0);
                }
                umma_commit(S.bar(B_S_FULL + sb));
                umma_commit(S.bar(B_KC_FREE));
                return true;
            };
            if (ok) ok = qk(0);
            for (int j = 0; ok && j < ntiles; ++j) {
                if (j + 1 < ntiles && !(ok = qk(j + 1))) break;
                const int vb = j & 1, sb = j % NSP;
                ok = wait_abortable(S.bar(B_P_FULL + sb), (j / NSP) & 1, abort_flag) &&
                     wait_abortable(S.bar(B_VC_FULL + vb), (j >> 1) & 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                const uint8_t* vc = Vc(vb);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    // tokens 16kk..16kk+15: p' hi in columns 16kk..16kk+7, lo in
                    // the next 8 (two f16 per column)
                    const uint32_t at = tmem + sb * BN + 16 * kk;
                    const uint64_t vbd = umma_desc(vc + kk * 16 * 128, ATOM, 1024);
                    umma_ts(tmem + TM_O, at, vbd, kIdescPV, j > 0 || kk > 0);
                    umma_ts(tmem + TM_O, at + 8, vbd, kIdescPV, true);
                }
                umma_commit(S.bar(B_PV_BUF + sb));
                umma_commit(S.bar(B_VC_FREE + vb));
            }
            // before the tensor memory is freed, every issued MMA must be done:
            // one more commit tracks all of them
            umma_commit(S.bar(B_DRAIN));
            const long long t0 = clock64();
            while (!mbar_try_wait(S.bar(B_DRAIN), 0) && clock64() - t0 < kWaitBudgetCycles) {
            }
        }
    } else if (warp >= kConvWarp0) {
        // ================================================================ convert
        const int t = threadIdx.x - kConvWarp0 * 32;     // token row of the tile
        for (int j = 0; j < ntiles; ++j) {
            const int st = j & 1;
            if (!warp_wait_abortable(S.bar(B_KV_FULL + st), (j >> 1) & 1, abort_flag)) break;
            // QK of the previous tile has finished reading the converted K
            if (j >= 1 && !warp_wait_abortable(S.bar(B_KC_FREE), (j - 1) & 1, abort_flag)) break;
            convert_row_f16(I8 + (2 * st) * I8_TILE, Kc, t);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(S.bar(B_KC_FULL));
            if (j >= 2 && !warp_wait_abortable(S.bar(B_VC_FREE + st), ((j >> 1) - 1) & 1, abort_flag)) break;
            convert_row_f16(I8 + (2 * st + 1) * I8_TILE, Vc(st), t);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(S.bar(B_VC_FULL + st));
                mbar_arrive(S.bar(B_KV_EMPTY + st));
            }
        }
    } else {
        // ================================================================ softmax
        const int st = threadIdx.x;            // 0..255
        const int half = warp >> 2;            // column half of every tile
        const int c0 = half * 64;
        const int r = (warp & 3) * 32 + lane;  // query row of the block == TMEM lane
        const bool live = r < rows;
        const int qpos = q0 + r;               // row within the appended chunk
        float* scb = reinterpret_cast<float*>(S.base + OFF_SC);
        float* red = reinterpret_cast<float*>(S.base + OFF_RED);

        const int sc_col = st & (BN - 1);         // this thread's tile column
        // scale of kv slot t (< len) from src
        auto scale_of = [&](const float* src, int t) -> float {
            if (PAGED) {
                int64_t slot;
                if (!page_slot(pm, seq, off, t, a.total_slots, slot)) return 0.0f;
                return a.row_scales ? src[slot] : src[(size_t)slot * HKV + g];
            }
            const int slot = off + t;
            return a.row_scales ? src[slot] : src[(size_t)slot * HKV + g];
        };
        // Each row's E, before Q (work placed between Q's arrival and the
        // first tile measured slower).  Every row sees slots [0, past + q0]
        // (the shared part); row r also sees the r slots after it (the band).
        // The 256 threads take the shared part's v-scales 16 x 256 at a time;
        // thread st < 127 also takes band slot st and an exclusive max-scan
        // over the band gives row r its band maximum.
        {
            const int shared_end = past + q0 + 1;           // exclusive
            float vm = 0.0f;
            for (int t0 = st; t0 < shared_end; t0 += 16 * kSoftmaxThreads) {
                float v[16];
#pragma unroll
                for (int u = 0; u < 16; ++u) {
                    const int t = t0 + u * kSoftmaxThreads;
                    v[u] = t < shared_end ? scale_of(a.val_scales, t) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 16; ++u) vm = fmaxf(vm, v[u]);
            }
            float bv = 0.0f;                                 // band slot st
            if (st < BN && shared_end + st < kv_end) bv = scale_of(a.val_scales, shared_end + st);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) vm = fmaxf(vm, __shfl_xor_sync(kFull, vm, o));
            float incl = bv;                                 // inclusive scan in the warp
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float n = __shfl_up_sync(kFull, incl, o);
                if (lane >= o) incl = fmaxf(incl, n);
            }
            // (clear of the Q block's maxima at red[2 * 2 * BM - 8..]; tile
            // 1's exchange is the next to write here)
            float* vmaxw = red + 2 * 2 * BM - 24;
            float* btot = red + 2 * 2 * BM - 16;
            if (lane == 0) vmaxw[warp] = vm;
            if (lane == 31 && warp < 4) btot[warp] = incl;
            named_bar(1, kSoftmaxThreads);
            if (st < BM) {
                float m = 0.0f;
#pragma unroll
                for (int w = 0; w < 8; ++w) m = fmaxf(m, vmaxw[w]);
                for (int w = 0; w < warp; ++w) m = fmaxf(m, btot[w]);   // earlier band warps
                const float prev = __shfl_up_sync(kFull, incl, 1);
                if (lane >= 1) m = fmaxf(m, prev);           // band slots < st
                // m < 2^ev; an infinite v-scale takes the largest E (and the
                // non-finite answer the reference's float loop gives)
                int ev = 0;
                if (m > 3.4028235e38f) ev = 128;
                else if (m > 0.0f) frexpf(m, &ev);
                reinterpret_cast<float*>(S.base + OFF_EROW)[st] =
                    (float)max(kEMin, ev - kVScaleBits);
            }
            // tile 0's bar_any (a barrier of these threads) precedes every read
        }
        // Q: cast to bf16 (the contract), then scaled by 2^qe, one power of two
        // for the whole CTA that brings max |q| into [2^14, 2^15), and stored
        // as f16.  Every bf16 value in range is exact in f16 after that
        // scaling (8 significant bits; only magnitudes below 2^-31 of the CTA
        // maximum lose bits), so QK^T runs f16 x f16 with exact int8 codes as
        // f16 K, and 2^-qe joins the k-scale multiplier.  K-major, swizzled:
        // this thread's 64 dims are K-block `half`.
        float q_inv = 1.0f;
        {
            const float* qp =
                a.q + (((size_t)seq * a.n_new + (live ? qpos : 0)) * H + h) * D + c0;
            float x[64];
            float amax = 0.0f;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
                if (live) v4 = reinterpret_cast<const float4*>(qp)[c];
                x[4 * c] = __bfloat162float(__float2bfloat16_rn(v4.x));
                x[4 * c + 1] = __bfloat162float(__float2bfloat16_rn(v4.y));
                x[4 * c + 2] = __bfloat162float(__float2bfloat16_rn(v4.z));
                x[4 * c + 3] = __bfloat162float(__float2bfloat16_rn(v4.w));
                amax = fmaxf(amax, fmaxf(fmaxf(fabsf(x[4 * c]), fabsf(x[4 * c + 1])),
                                         fmaxf(fabsf(x[4 * c + 2]), fabsf(x[4 * c + 3]))));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(kFull, amax, o));
            float* qmax = red + 2 * 2 * BM - 8;    // first used by tile 1's exchange
            if (lane == 0) qmax[warp] = amax;
            named_bar(1, kSoftmaxThreads);
#pragma unroll
            for (int w = 0; w < 8; ++w) amax = fmaxf(amax, qmax[w]);
            int qe = 0;
            if (amax > 0.0f) {
                int ex;
                frexpf(amax, &ex);                 // amax = f * 2^ex, f in [0.5, 1)
                qe = min(120, max(-120, 15 - ex));   // keeps 2^qe and 2^-qe normal
            }
            const float q_mul = ldexpf(1.0f, qe);
            q_inv = ldexpf(1.0f, -qe);
            uint8_t* blk = Qs + half * ATOM;
#pragma unroll
            for (int c = 0; c < 8; ++c) {   // 8 chunks of 8 dims
                __half2 hq[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    hq[u] = __floats2half2_rn(x[8 * c + 2 * u] * q_mul, x[8 * c + 2 * u + 1] * q_mul);
                *reinterpret_cast<uint4*>(blk + swz(r, c)) = *reinterpret_cast<const uint4*>(hq);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(S.bar(B_Q_FULL));
        }

        // per-token scales of a tile: thread st loads k-scale * qk_mul of column
        // st (st < 128) or v-scale of column st - 128, two tiles ahead
        const float* sc_src = st < BN ? a.key_scales : a.val_scales;
        const float sc_mul = st < BN ? a.qk_mul * q_inv : 1.0f;
        // (raw value: the multiply waits until the next tile, when the load has
        // landed, so the in-order warp does not stall on it here)
        auto load_scale = [&](int j) -> float {
            const int t = j * BN + sc_col;
            return t < len ? scale_of(sc_src, t) : 0.0f;
        };

        const float* erow = reinterpret_cast<const float*>(S.base + OFF_EROW);

        // From here on a thread works in the 16-lane layout: quad g = lane / 4,
        // q = lane % 4.  It owns the rows rw[k] = 32*(warp%4) + 16*(k/2) + g +
        // 8*(k%2) (k = 0..3) and, in every tile, the 16 columns c0 + 8n + 2q,
        // c0 + 8n + 2q + 1 (n = 0..7), so its 32 per-column scales sit in
        // registers for the whole tile.  A row's 64 columns of this half are
        // spread over the four threads of a quad.
        const int gq = lane >> 2, qq = lane & 3;
        int rlim[4];                               // last kv slot each row may see
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int rw = (warp & 3) * 32 + 16 * (k >> 1) + gq + 8 * (k & 1);
            rlim[k] = rw < rows ? past + q0 + rw : -1;
        }
        auto lanes_of = [&](int blk) -> uint32_t {  // TMEM lane field of block blk
            return (uint32_t)((warp & 3) * 32 + 16 * blk) << 16;
        };

        float sc_next = load_scale(0);
        float sc_next2 = ntiles > 1 ? load_scale(1) : 0.0f;   // two tiles ahead
        float m_run[4];
        float2 l_run[4];                           // this thread's even / odd columns
#pragma unroll
        for (int k = 0; k < 4; ++k) { m_run[k] = -INFINITY; l_run[k] = make_float2(0.0f, 0.0f); }
        bool bad = false;                          // a bounded wait of this warp gave up

        int j = 0;
        for (; j < ntiles; ++j) {
            const int sb = j % NSP, par = j & 1;
            float* sck = scb + par * 2 * BN;
            sck[st] = sc_next * sc_mul;
            sc_next = sc_next2;
            if (j + 2 < ntiles) sc_next2 = load_scale(j + 2);
            bad |= !warp_wait_abortable(S.bar(B_S_FULL + sb), (j / NSP) & 1, abort_flag);
            // tile j's scales are visible to all, and all agree whether to go on
            if (bar_any(1, kSoftmaxThreads, bad)) break;
            tc_fence_after();
            float2 ks[8], vs[8];                   // scales of this thread's column pairs
#pragma unroll
            for (int n = 0; n < 8; ++n) {
                ks[n] = *reinterpret_cast<const float2*>(sck + c0 + 8 * n + 2 * qq);
                vs[n] = *reinterpret_cast<const float2*>(sck + BN + c0 + 8 * n + 2 * qq);
            }
            const uint32_t s_col = tmem + sb * BN + c0;
            const int kv0 = j * BN + c0 + 2 * qq;  // kv slot of column c0 + 2q
            // columns past a row's causal limit exist only near the diagonal or
            // in a partial block (rows >= `rows` have limit -1)
            const bool masked_tile = j * BN + BN - 1 > past + q0 || rows < BM;

            // pass 1: row maxima of s = S * k_scale * qk_mul over this half
            float tmax[4];
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                float v[32];
                tmem_ld_16x256b_x8(s_col + lanes_of(blk), v);
                float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    // packed f32x2 multiplies: one instruction per column pair
                    const float2 pa = __fmul2_rn(make_float2(v[4 * n], v[4 * n + 1]), ks[n]);
                    const float2 pb = __fmul2_rn(make_float2(v[4 * n + 2], v[4 * n + 3]), ks[n]);
                    float a0 = pa.x, a1 = pa.y, b0 = pb.x, b1 = pb.y;
                    if (masked_tile) {
                        const int c = kv0 + 8 * n;
                        if (c > rlim[2 * blk]) a0 = -INFINITY;
                        if (c + 1 > rlim[2 * blk]) a1 = -INFINITY;
                        if (c > rlim[2 * blk + 1]) b0 = -INFINITY;
                        if (c + 1 > rlim[2 * blk + 1]) b1 = -INFINITY;
                    }
                    m0 = fmax3(m0, a0, a1);
                    m1 = fmax3(m1, b0, b1);
                }
                tmax[2 * blk] = m0;
                tmax[2 * blk + 1] = m1;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                tmax[k] = fmaxf(tmax[k], __shfl_xor_sync(kFull, tmax[k], 1));
                tmax[k] = fmaxf(tmax[k], __shfl_xor_sync(kFull, tmax[k], 2));
            }
            // row maximum over both halves (every thread of a row computes the
            // same m_run, corr and p scale from it).  The running maximum only
            // moves when some half-row exceeds it by the lazy threshold, which
            // after the first tiles is rare: one barrier that ORs that
            // condition decides whether the halves need to exchange at all.
            bool need = false;
#pragma unroll
            for (int k = 0; k < 4; ++k) need |= tmax[k] > m_run[k] + kLazyRescale;
            float corr[4] = {1.0f, 1.0f, 1.0f, 1.0f};
            bool any_corr = false;
            if (bar_any(1, kSoftmaxThreads, need)) {
                if (qq == 0) {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        red[(par * 2 + half) * BM + (warp & 3) * 32 + 16 * (k >> 1) + gq + 8 * (k & 1)] =
                            tmax[k];
                }
                named_bar(1, kSoftmaxThreads);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float t = fmaxf(
                        tmax[k],
                        red[(par * 2 + (half ^ 1)) * BM + (warp & 3) * 32 + 16 * (k >> 1) + gq + 8 * (k & 1)]);
                    if (t > m_run[k] + kLazyRescale) {
                        corr[k] = fast_exp2(m_run[k] - t);
                        m_run[k] = t;
                        any_corr = true;
                    }
                    l_run[k] = __fmul2_rn(l_run[k], make_float2(corr[k], corr[k]));
                }
            }
            float neg_m[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)                    // -m - E: p' and l carry 2^-E
                neg_m[k] = (m_run[k] == -INFINITY ? 0.0f : -m_run[k]) -
                           erow[(warp & 3) * 32 + 16 * (k >> 1) + gq + 8 * (k & 1)];

            // rescale this half of the O rows only when some row's maximum
            // jumped (rare): O must first hold every earlier tile
            if (j >= 1 && __any_sync(kFull, any_corr)) {
                const int pj = j - 1;
                if (warp_wait_abortable(S.bar(B_PV_BUF + pj % NSP), (pj / NSP) & 1, abort_flag)) {
                    tc_fence_after();
#pragma unroll
                    for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
                        for (int G = 0; G < 4; ++G) {
                            float o[8];
                            const uint32_t oa = tmem + TM_O + c0 + 16 * G + lanes_of(blk);
                            tmem_ld_16x256b_x2(oa, o);
#pragma unroll
                            for (int i = 0; i < 8; i += 4) {
                                o[i] *= corr[2 * blk];
                                o[i + 1] *= corr[2 * blk];
                                o[i + 2] *= corr[2 * blk + 1];
                                o[i + 3] *= corr[2 * blk + 1];
                            }
                            tmem_st_16x256b_x2(oa, o);
                        }
                    }
                } else {
                    bad = true;
                }
            }
            // pass 2: p' = 2^(s - m) * v_scale as an f16 pair hi + lo (hi =
            // f16(p'), lo = f16(p' - hi)), written over the S columns just
            // read.  Tokens 16G..16G+15 of the half keep their hi words (token
            // pairs) in columns 16G..16G+7 and lo words in the next 8.
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
                for (int GG = 0; GG < 2; ++GG) {              // two 16-token groups per load
                    float v[16];
                    const uint32_t ga = s_col + 32 * GG + lanes_of(blk);
                    tmem_ld_16x256b_x4(ga, v);
                    uint32_t w[2][8];
#pragma unroll
                    for (int h4 = 0; h4 < 4; ++h4) {          // repetition n = 4GG + h4
                        const int n = 4 * GG + h4, G = h4 >> 1, h2 = h4 & 1;
#pragma unroll
                        for (int rr = 0; rr < 2; ++rr) {      // row g or g + 8
                            const int k = 2 * blk + rr;
                            // packed f32x2 arithmetic on the column pair
                            const float2 e = __ffma2_rn(
                                make_float2(v[4 * h4 + 2 * rr], v[4 * h4 + 2 * rr + 1]), ks[n],
                                make_float2(neg_m[k], neg_m[k]));
                            float e0 = e.x, e1 = e.y;
                            if (masked_tile) {
                                const int c = kv0 + 8 * n;
                                if (c > rlim[k]) e0 = -INFINITY;
                                if (c + 1 > rlim[k]) e1 = -INFINITY;
                            }
                            const float2 pp = make_float2(fast_exp2(e0), fast_exp2(e1));
                            l_run[k] = __fadd2_rn(l_run[k], pp);
                            const float2 pv = __fmul2_rn(pp, vs[n]);
                            const __half2 hh = __floats2half2_rn(pv.x, pv.y);
                            const float2 lo = minus_f16x2_from_f32x2(hh, pv);
                            const __half2 ll = __floats2half2_rn(lo.x, lo.y);
                            w[G][2 * h2 + rr] = *reinterpret_cast<const uint32_t*>(&hh);
                            w[G][4 + 2 * h2 + rr] = *reinterpret_cast<const uint32_t*>(&ll);
                        }
                    }
                    tmem_st_16x128b_x4(ga, w[0]);
                    tmem_st_16x128b_x4(ga + 16, w[1]);
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(S.bar(B_P_FULL + sb));
        }
        // ---- epilogue: O / l for live rows, l summed over the quad and both halves
        const bool ran = j == ntiles;
        float l_sum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (ran) {
            const int lj = ntiles - 1;
            bad |= !warp_wait_abortable(S.bar(B_PV_BUF + lj % NSP), (lj / NSP) & 1, abort_flag);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                l_sum[k] = l_run[k].x + l_run[k].y;
                l_sum[k] += __shfl_xor_sync(kFull, l_sum[k], 1);
                l_sum[k] += __shfl_xor_sync(kFull, l_sum[k], 2);
            }
            if (qq == 0) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    red[((ntiles & 1) * 2 + half) * BM + (warp & 3) * 32 + 16 * (k >> 1) + gq + 8 * (k & 1)] =
                        l_sum[k];
            }
        }
        // every softmax thread reaches this barrier exactly once
        const bool failed = bar_any(1, kSoftmaxThreads, bad || !ran);
        if (!failed) {
            tc_fence_after();
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
                float o[32];
                tmem_ld_16x256b_x8(*S.tmem_slot() + TM_O + c0 + lanes_of(blk), o);
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int k = 2 * blk + rr;
                    const int rw = (warp & 3) * 32 + 16 * blk + gq + 8 * rr;
                    const float l = l_sum[k] + red[((ntiles & 1) * 2 + (half ^ 1)) * BM + rw];
                    bool row_live;
                    float* op = out_row(a, rw, row_live) + c0 + 2 * qq;
                    const float inv = (row_live && l > 0.0f) ? __fdiv_rn(1.0f, l) : 0.0f;
                    if (row_live) {
#pragma unroll
                        for (int n = 0; n < 8; ++n)
                            *reinterpret_cast<float2*>(op + 8 * n) =
                                make_float2(o[4 * n + 2 * rr] * inv, o[4 * n + 2 * rr + 1] * inv);
                    }
                }
            }
        } else if (lane == 0) {
            flag_error(a.err, EC_DEVERR_TIMEOUT);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS) : "memory");
    }
}

}  // namespace

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t st) {
    static std::atomic<unsigned long long> done_contig{0}, done_paged{0};
    cudaError_t e = a.pages.table
        ? ensure_smem_limit(reinterpret_cast<const void*>(prefill_kernel<true>), SMEM, done_paged)
        : ensure_smem_limit(reinterpret_cast<const void*>(prefill_kernel<false>), SMEM, done_contig);
    if (e != cudaSuccess) return e;
    CUtensorMap mk, mv;
    if ((e = make_code_map(&mk, a.keys, a.num_kv_heads, a.total_slots, BN)) != cudaSuccess) return e;
    if ((e = make_code_map(&mv, a.values, a.num_kv_heads, a.total_slots, BN)) != cudaSuccess) return e;
    const int nqb = (a.n_new + BM - 1) / BM;
    const long long blocks = (long long)a.num_seqs * a.num_heads * nqb;
    if (blocks == 0) return cudaSuccess;
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    if (a.pages.table)
        prefill_kernel<true><<<(unsigned)blocks, kThreads, SMEM, st>>>(mk, mv, a);
    else
        prefill_kernel<false><<<(unsigned)blocks, kThreads, SMEM, st>>>(mk, mv, a);
    return cudaGetLastError();
}

}  // namespace ec
