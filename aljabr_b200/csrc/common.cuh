// Shared device helpers for the Blackwell (sm_100a) quantized-decode kernels:
// mbarrier / bulk-copy PTX wrappers, bounded waits with a device fault word,
// packed f32x2 arithmetic, and the scalar decoders of the GGUF / NF4 formats.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "aljabr_blackwell_internal.h"

namespace alj {

// ---------------------------------------------------------------- fault word
// Set (never cleared on the device) when a bounded wait gives up; read and
// cleared by the host through aljabr_blackwell_device_status().
extern __device__ unsigned int g_fault_word;

// Upper bound for any spin on an mbarrier: ~2 s at 2 GHz.  A wait that runs
// out records ALJ_FAULT_TIMEOUT and the CTA stops early instead of hanging.
constexpr long long kSpinLimitCycles = 4000000000LL;

__device__ __forceinline__ void record_fault(unsigned int code) { atomicOr(&g_fault_word, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps in the barrier unit
// until the phase completes (or ~0.5 ms pass) instead of spinning, so a
// waiting warp does not take issue slots from the warps sharing its scheduler.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(500000u)
        : "memory");
    return ok != 0;
}
// Bounded wait: returns false (and records the fault) if the phase never flips.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (clock64() - t0 > kSpinLimitCycles) {
            record_fault(ALJ_FAULT_TIMEOUT);
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------- bulk copy
// Untiled TMA copy global -> shared, completion counted on `bar` in bytes.
// Both addresses must be 16-byte aligned and `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------- cross-GPU flags
// Release / acquire at system scope for the tensor-parallel exchange: a rank
// writes its output rows into every peer's buffer (NVLink peer mappings),
// fences, and publishes a monotonically increasing flag value on each peer.
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait until flags[0..n) all reach `target` (wrap-safe).  Returns
// false and records ALJ_FAULT_TIMEOUT if a peer never publishes.
// If an earlier wait has already timed out (a peer is gone), return at once:
// the rest of a token's exchanges then fail fast instead of each spending
// the full limit.
__device__ __forceinline__ bool fault_timeout_recorded() {
    return (*static_cast<volatile unsigned int*>(&g_fault_word) & ALJ_FAULT_TIMEOUT) != 0u;
}
__device__ __forceinline__ bool wait_flags_sys(const unsigned int* flags, int n, unsigned int target) {
    const long long t0 = clock64();
    for (int r = 0; r < n; ++r) {
        while (static_cast<int>(ld_acquire_sys(flags + r) - target) < 0) {
            if (fault_timeout_recorded()) return false;
            if (clock64() - t0 > kSpinLimitCycles) {
                record_fault(ALJ_FAULT_TIMEOUT);
                return false;
            }
        }
    }
    return true;
}
// Generic-proxy writes observed above become visible to this thread's later
// TMA (async-proxy) reads.
// Fetch a TMA descriptor (a kernel parameter) ahead of its first use.
__device__ __forceinline__ void prefetch_tensormap(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// L2 prefetch of this CTA's 1/grid share of [base, base + bytes) -- the part
// the same CTA index of the next launch reads first (rows are contiguous and
// dealt out in order) -- capped at `limit` bytes (128 KB by default),
// strictly inside the range.
__device__ __forceinline__ void prefetch_share(const uint8_t* base, size_t bytes, size_t limit = size_t(128) << 10) {
    const size_t share = bytes / gridDim.x;
    const uintptr_t b0 = reinterpret_cast<uintptr_t>(base);
    uintptr_t a = (b0 + share * blockIdx.x + 15) & ~uintptr_t(15);
    const size_t cap = share < limit ? share : limit;
    const uintptr_t lim = b0 + share * blockIdx.x + cap;
    const uintptr_t end = (lim < b0 + bytes ? lim : b0 + bytes) & ~uintptr_t(15);
    for (; a + 16 <= end; a += 16384) {
        const uintptr_t left = end - a;
        const uint32_t n = static_cast<uint32_t>(left < 16384 ? left : 16384) & ~15u;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
    }
}

// Programmatic dependent launch: wait for the producer grid's writes, and let
// the next grid in the stream begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Named barrier among a subset of warps (id 0 is __syncthreads).
// Arrive on a named barrier without waiting (the waiting side uses named_bar).
__device__ __forceinline__ void named_bar_arrive(int id, int threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_bar(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- f32x2
// Packed two-lane fp32 arithmetic (sm_100a): one instruction, two results,
// each rounded exactly as the scalar instruction would.
struct f2 {
    unsigned long long v;
};
__device__ __forceinline__ f2 mk2u(uint32_t a, uint32_t b) {
    return f2{(static_cast<unsigned long long>(b) << 32) | a};
}
__device__ __forceinline__ f2 mk2(float a, float b) { return mk2u(__float_as_uint(a), __float_as_uint(b)); }
__device__ __forceinline__ float lo(f2 a) { return __uint_as_float(static_cast<uint32_t>(a.v)); }
__device__ __forceinline__ float hi(f2 a) { return __uint_as_float(static_cast<uint32_t>(a.v >> 32)); }
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r.v) : "l"(a.v), "l"(b.v), "l"(c.v));
    return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}

// ---------------------------------------------------------------- decoders
// fp16 -> fp32 exactly as RT/GgufQuantTables.f16ToF32 (every NaN becomes the
// canonical Float.NaN pattern 0x7FC00000; all other values are exact).
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
    if (e == 31 && m != 0) return __uint_as_float(0x7FC00000u);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
}

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t mask, uint32_t c) {
    // (a & mask) ^ c in one LOP3
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(mask), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t c) {
    // (a & mask) | c in one LOP3
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(c));
    return r;
}

// NF4 codebook (engine/safetensor/.../DequantizationKernel.java:23-28).
__device__ __forceinline__ float nf4_value(int v) {
    constexpr float t[16] = {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
                             -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
                             0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
                             0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};
    return t[v & 15];
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace alj
