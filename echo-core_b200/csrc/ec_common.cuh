// ec_common.cuh -- shared device helpers for the sm_100a INT8 KV-cache kernels.
//
// Every wait on an mbarrier is bounded by a clock64 budget (about one second
// at B200 clocks).  A wait that runs out records EC_DEVERR_TIMEOUT in the
// error word and reports failure, so that the caller can stop issuing work
// and return instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "ec_internal.h"
#include "ec_kv.h"

namespace ec {

constexpr long long kWaitBudgetCycles = 2000000000LL;  // ~1 s at 1.9-2 GHz

// Library-owned error word per device, used when the caller supplies none.
extern __device__ int32_t g_error_word;

__device__ __forceinline__ void flag_error(int32_t* err, int32_t code) {
    atomicCAS(err ? err : &g_error_word, 0, code);
}

// Programmatic dependent launch.  A kernel launched by launch_pdl may become
// resident while the previous kernel on its stream is still running.  Every
// thread calls pdl_wait() before its first global memory access (read or
// write) and before any exit, so the kernel sees all of the predecessor's
// writes and never completes ahead of it; pdl_trigger() then lets the next
// kernel's CTAs be scheduled.  Both are no-ops in a kernel launched without
// the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Paged KV layout (PageMap in ec_internal.h).  With a page table, token t of
// sequence s lives in slot table[s * max_pages + (t >> shift)] << shift |
// (t & (page - 1)); without one, in slot seq_offset[s] + t (per-sequence
// contiguous slabs).  False for a page id outside the pool or a t past the
// table row: the caller flags the table and skips the access.
__device__ __forceinline__ bool page_slot(const PageMap& pm, int s, int32_t off, int t,
                                          uint64_t total_slots, int64_t& out) {
    if (!pm.table) {
        out = (int64_t)off + t;
        return true;
    }
    const int pg = t >> pm.shift;
    if (t < 0 || pg >= pm.max_pages) return false;
    const int32_t id = pm.table[(size_t)s * pm.max_pages + pg];
    const uint64_t base = (uint64_t)(int64_t)id << pm.shift;
    if (id < 0 || base + ((uint64_t)1 << pm.shift) > total_slots) return false;
    out = (int64_t)base + (t & ((1 << pm.shift) - 1));
    return true;
}

// Bounds of a table entry: within its slab (contiguous) or its page row.
__device__ __forceinline__ bool page_entry_ok(const PageMap& pm, int32_t off, int32_t cap,
                                              int32_t len, uint64_t total_slots) {
    if (cap < 0 || len < 0 || len > cap) return false;
    if (pm.table) return (int64_t)cap <= ((int64_t)pm.max_pages << pm.shift);
    return off >= 0 && (uint64_t)off + (uint64_t)cap <= total_slots;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or about `hint_ns` nanoseconds pass, instead of spinning
// and taking issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitBudgetCycles) return false;
    }
    return true;
}

// 1-D bulk copy global -> this CTA's shared memory, completion counted on
// `bar` in bytes.  dst, src and bytes must be multiples of 16.  Plain (not
// multicast) form.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Same with an L2 eviction-priority hint (streamed data read exactly once).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// int8x4 -> 4 x fp32, exact: bias each byte to unsigned, splice it under the
// exponent of 2^23 with a byte permute, subtract 2^23 + 128.
struct F4 {
    float x, y, z, w;
};
__device__ __forceinline__ uint32_t bias_bytes(uint32_t w) { return w ^ 0x80808080u; }
__device__ __forceinline__ float byte_as_float(uint32_t biased, uint32_t sel) {
    return __uint_as_float(__byte_perm(biased, 0x4B000000u, sel));
}
constexpr float kByteMagic = 8388736.0f;  // 2^23 + 128

__device__ __forceinline__ void i8x4_to_f2x2(uint32_t w, float2& lo, float2& hi) {
    const uint32_t b = bias_bytes(w);
    lo = make_float2(byte_as_float(b, 0x7540u), byte_as_float(b, 0x7541u));
    hi = make_float2(byte_as_float(b, 0x7542u), byte_as_float(b, 0x7543u));
    const float2 m = make_float2(-kByteMagic, -kByteMagic);
    lo = __fadd2_rn(lo, m);
    hi = __fadd2_rn(hi, m);
}

}  // namespace ec
