// Batch-1 GGUF K-quant dequantise-and-matvec (y = W x) for Q4_K and Q6_K,
// the 256-value super-block formats the reference's raw rows serve with
// GgufQ4RawDot.dotRowQ4K and GgufQ6RawDot.dotRowQ6K
// (engine/gguf/aljabr-gguf-core/.../runtime/GgufQ4RawDot.java:38-141,
// GgufQ6RawDot.java:33-133,403-513; block layouts in GgufQuantFormats.java:51-53
// and GgufKQuantLayout.java:37-66).
//
// Q4_K (144 B): fp16 d, fp16 dmin, 12 bytes of packed 6-bit (scale, min)
// pairs for 8 sub-blocks of 32, 128 bytes of nibbles; value 64j + t is the
// low (t < 32) or high nibble of byte 32j + t % 32, times d*scale, minus
// dmin*min of sub-block 2j + (t >= 32).
// Q6_K (210 B): ql[128], qh[64], int8 scales[16], fp16 d at byte 208; in
// half h, value 32k + i is nibble (k >> 1) of ql[64h + 32(k & 1) + i] with
// bits 2k..2k+1 of qh[32h + i] above it, minus 32, times
// d*scales[8h + 2k + i/16].
//
// A CTA serves kKRows consecutive rows; its 8 warps split the super-blocks
// (warp w takes blocks w, w + 8, ...) and meet in shared memory at the end,
// summed in fixed order.  A warp walks its blocks for all kKRows rows in
// step, its 32 lanes spread over one block, so codes and x are read with
// consecutive lanes on consecutive addresses, and x (with its sub-block sums)
// is loaded once for all the rows:
//   * Q4_K: lane l takes code word l (bytes 4l..4l+3 of the 128): values
//     64j + t..t+3 (low nibbles) and 64j + 32 + t..t+3 (high nibbles) with
//     j = l / 8, t = 4l % 32; the 16-byte block header (d, dmin, scales) is
//     one broadcast load per row;
//   * Q6_K blocks are only 2-byte aligned (210 B): lane l takes ql 16-bit
//     words l (half 0) and 32 + l (half 1) and the matching qh words, i.e.
//     the values at byte position p = 2l, 2l+1 of each 64-byte ql half.
// A code becomes a float by OR-ing it into the mantissa of 2^23 and
// subtracting (exact, full rate, unlike an int-to-float conversion); the
// multiply-adds run on packed f32x2 pairs.  The row bytes are read once
// (HBM-bound by design).
#include "common.cuh"

namespace alj {
namespace {

constexpr int kKWarps = 8;
constexpr int kKRows = 4;     // rows a warp walks in step
constexpr int kKGroups = 1;   // row groups per CTA

__device__ __forceinline__ uint32_t byte_of(const uint4& v, int i) {
    const uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
    return (w >> (8 * (i & 3))) & 0xFFu;
}
// 6-bit scale and min of Q4_K sub-block `i` (header bytes 4..15 hold the packed pairs)
__device__ __forceinline__ void q4k_scale_min(const uint4& hd, int i, float& sc, float& mn) {
    uint32_t s, m;
    if (i < 4) {
        s = byte_of(hd, 4 + i) & 63u;
        m = byte_of(hd, 8 + i) & 63u;
    } else {
        const uint32_t top = byte_of(hd, 8 + i);
        s = (top & 0x0Fu) | ((byte_of(hd, i) >> 6) << 4);
        m = (top >> 4) | ((byte_of(hd, 4 + i) >> 6) << 4);
    }
    sc = static_cast<float>(s);
    mn = static_cast<float>(m);
}
// four 4-bit fields of w at bits sh, sh+8, sh+16, sh+24 as floats (exact), packed in pairs
__device__ __forceinline__ void nibbles4(uint32_t w, int sh, f2& p01, f2& p23) {
    const uint32_t v = w >> sh;
    p01 = mk2u(0x4B000000u | (v & 15u), 0x4B000000u | ((v >> 8) & 15u));
    p23 = mk2u(0x4B000000u | ((v >> 16) & 15u), 0x4B000000u | ((v >> 24) & 15u));
    const f2 off = mk2(-8388608.0f, -8388608.0f);
    p01 = add2(p01, off);
    p23 = add2(p23, off);
}

// L2 prefetch of the 16-byte-aligned inside of [base, base + bytes), in
// 16 KB bulk requests: the CTA's rows are one contiguous range, and one
// thread puts all of it in flight at once, so the warps' own loads find it
// in L2 instead of each paying the HBM round trip in turn.
__device__ __forceinline__ void prefetch_rows_l2(const uint8_t* base, size_t bytes) {
    uintptr_t a = (reinterpret_cast<uintptr_t>(base) + 15) & ~uintptr_t(15);
    const uintptr_t end = (reinterpret_cast<uintptr_t>(base) + bytes) & ~uintptr_t(15);
    for (; a + 16 <= end; a += 16384) {
        const uintptr_t left = end - a;
        const uint32_t n = static_cast<uint32_t>(left < 16384 ? left : 16384) & ~15u;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
    }
}

struct KRows {
    const uint8_t* w;
    const float* x;
    float* y;
    const float* bias;
    const float* residual;
    int K, N;
};

// Warp sums of the rows' partials, then the 8 warps' sums in fixed order.
__device__ __forceinline__ void store_rows(const KRows& p, int row0, float (&acc)[kKGroups][kKRows], int warp,
                                           int lane) {
    constexpr int R = kKGroups * kKRows;
    __shared__ float red[kKWarps][R];
#pragma unroll
    for (int g = 0; g < kKGroups; ++g)
#pragma unroll
        for (int r = 0; r < kKRows; ++r) {
            const float v = warp_sum(acc[g][r]);
            if (lane == 0) red[warp][g * kKRows + r] = v;
        }
    __syncthreads();
    if (warp == 0 && lane < R && row0 + lane < p.N) {
        float out = 0.0f;
#pragma unroll
        for (int w = 0; w < kKWarps; ++w) out += red[w][lane];
        if (p.bias) out += p.bias[row0 + lane];
        if (p.residual) out = p.residual[row0 + lane] + out;
        p.y[row0 + lane] = out;
    }
}

__global__ void __launch_bounds__(kKWarps * 32, 3) q4k_matvec_kernel(const KRows p) {
    pdl_launch_dependents();
    pdl_wait();   // x may come from the previous kernel
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kKGroups * kKRows;
    const int nb = p.K / 256;
    const size_t row_bytes = static_cast<size_t>(nb) * 144;
    if (threadIdx.x == 0) prefetch_rows_l2(p.w + row0 * row_bytes, min(kKGroups * kKRows, p.N - row0) * row_bytes);
    const int j = lane >> 3, t = (lane * 4) & 31;
    float acc[kKGroups][kKRows];
#pragma unroll
    for (int g = 0; g < kKGroups; ++g)
#pragma unroll
        for (int r = 0; r < kKRows; ++r) acc[g][r] = 0.0f;
#pragma unroll 2
    for (int b = warp; b < nb; b += kKWarps) {
        const float4 xl = __ldg(reinterpret_cast<const float4*>(p.x + b * 256 + 64 * j + t));
        const float4 xh = __ldg(reinterpret_cast<const float4*>(p.x + b * 256 + 64 * j + 32 + t));
        const f2 xl01 = mk2(xl.x, xl.y), xl23 = mk2(xl.z, xl.w), xh01 = mk2(xh.x, xh.y), xh23 = mk2(xh.z, xh.w);
        const float sl = (xl.x + xl.y) + (xl.z + xl.w), sh = (xh.x + xh.y) + (xh.z + xh.w);
#pragma unroll
        for (int gr = 0; gr < kKGroups * kKRows; ++gr) {
            const int rr = min(row0 + gr, p.N - 1);
            const uint8_t* blk = p.w + rr * row_bytes + static_cast<size_t>(b) * 144;
            const uint4 hd = __ldg(reinterpret_cast<const uint4*>(blk));
            const uint32_t q = __ldg(reinterpret_cast<const uint32_t*>(blk + 16) + lane);
            float s1, m1, s2, m2;
            q4k_scale_min(hd, 2 * j, s1, m1);
            q4k_scale_min(hd, 2 * j + 1, s2, m2);
            const float d = f16_bits_to_f32(hd.x & 0xFFFFu), dmin = f16_bits_to_f32(hd.x >> 16);
            f2 a01, a23, b01, b23;
            nibbles4(q, 0, a01, a23);
            nibbles4(q, 4, b01, b23);
            const f2 dl = fma2(a23, xl23, mul2(a01, xl01));
            const f2 dh = fma2(b23, xh23, mul2(b01, xh01));
            float a = acc[gr / kKRows][gr % kKRows];
            a = fmaf(d * s1, lo(dl) + hi(dl), a);
            a = fmaf(d * s2, lo(dh) + hi(dh), a);
            a = fmaf(-dmin * m1, sl, a);
            a = fmaf(-dmin * m2, sh, a);
            acc[gr / kKRows][gr % kKRows] = a;
        }
    }
    store_rows(p, row0, acc, warp, lane);
}

__global__ void __launch_bounds__(kKWarps * 32, 3) q6k_matvec_kernel(const KRows p) {
    pdl_launch_dependents();
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kKGroups * kKRows;
    const int nb = p.K / 256;
    const size_t row_bytes = static_cast<size_t>(nb) * 210;
    if (threadIdx.x == 0) prefetch_rows_l2(p.w + row0 * row_bytes, min(kKGroups * kKRows, p.N - row0) * row_bytes);
    // byte position p = 2 lane + e of a 64-byte ql half: quarter k0 = p / 32
    // (low nibble) or 2 + k0 (high nibble), value index i0 + e = p % 32
    const int k0 = lane >> 4, i0 = (lane * 2) & 31, g = i0 >> 4;
    float acc[kKGroups][kKRows];
#pragma unroll
    for (int g = 0; g < kKGroups; ++g)
#pragma unroll
        for (int r = 0; r < kKRows; ++r) acc[g][r] = 0.0f;
#pragma unroll 2
    for (int b = warp; b < nb; b += kKWarps) {
        // x pairs of this lane's 8 values: [half h][low / high nibble]
        f2 xv[2][2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float2 x0 = __ldg(reinterpret_cast<const float2*>(p.x + b * 256 + 128 * h + 32 * k0 + i0));
            const float2 x1 = __ldg(reinterpret_cast<const float2*>(p.x + b * 256 + 128 * h + 32 * (2 + k0) + i0));
            xv[h][0] = mk2(x0.x, x0.y);
            xv[h][1] = mk2(x1.x, x1.y);
        }
#pragma unroll
        for (int gr = 0; gr < kKGroups * kKRows; ++gr) {
            const int rr = min(row0 + gr, p.N - 1);
            const uint8_t* blk = p.w + rr * row_bytes + static_cast<size_t>(b) * 210;
            const unsigned short* w16 = reinterpret_cast<const unsigned short*>(blk);
            const float d = f16_bits_to_f32(__ldg(w16 + 104));
            float a = acc[gr / kKRows][gr % kKRows];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t ql = __ldg(w16 + 32 * h + lane);                 // bytes p, p+1 of half h
                const uint32_t qh = __ldg(w16 + 64 + 16 * h + (lane & 15));     // qh bytes i0, i0+1 of half h
                const uint32_t hl = (qh >> (2 * k0)) & 0x0303u, hh = (qh >> (2 * (2 + k0))) & 0x0303u;
                // low nibbles | two high bits, minus 32 (as 2^23 + q - (2^23 + 32))
                const f2 vl = add2(mk2u(0x4B000000u | (ql & 15u) | ((hl & 3u) << 4),
                                        0x4B000000u | ((ql >> 8) & 15u) | ((hl >> 8) << 4)),
                                   mk2(-8388640.0f, -8388640.0f));
                const f2 vh = add2(mk2u(0x4B000000u | ((ql >> 4) & 15u) | ((hh & 3u) << 4),
                                        0x4B000000u | ((ql >> 12) & 15u) | ((hh >> 8) << 4)),
                                   mk2(-8388640.0f, -8388640.0f));
                const f2 pl = mul2(vl, xv[h][0]), ph = mul2(vh, xv[h][1]);
                const float sc_l = static_cast<float>(static_cast<signed char>(__ldg(blk + 192 + 8 * h + 2 * k0 + g)));
                const float sc_h = static_cast<float>(static_cast<signed char>(__ldg(blk + 192 + 8 * h + 2 * (2 + k0) + g)));
                a = fmaf(d * sc_l, lo(pl) + hi(pl), a);
                a = fmaf(d * sc_h, lo(ph) + hi(ph), a);
            }
            acc[gr / kKRows][gr % kKRows] = a;
        }
    }
    store_rows(p, row0, acc, warp, lane);
}

}  // namespace

bool matvec_k_supported(int fmt, int K) { return (fmt == FMT_Q4_K || fmt == FMT_Q6_K) && K > 0 && K % 256 == 0; }

cudaError_t launch_matvec_k(int fmt, const MatvecParams& mp, cudaStream_t stream, bool pdl) {
    if (!matvec_k_supported(fmt, mp.K)) return cudaErrorNotSupported;
    if (mp.epilogue != EPI_STORE || mp.norm_out || mp.norm_defer || mp.in_parts || mp.tpl.tp > 1)
        return cudaErrorNotSupported;
    if (reinterpret_cast<uintptr_t>(mp.x) & 15) return cudaErrorNotSupported;
    for (int s = 0; s < mp.nseg; ++s) {
        const MatvecSegment& sg = mp.seg[s];
        if (sg.rows <= 0) continue;
        // Q4_K reads 16-byte header / code vectors, Q6_K 2-byte words
        if (reinterpret_cast<uintptr_t>(sg.w) & (fmt == FMT_Q4_K ? 15 : 1)) return cudaErrorNotSupported;
        KRows p{sg.w, mp.x, sg.y, sg.bias, sg.residual, mp.K, sg.rows};
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((sg.rows + kKGroups * kKRows - 1) / (kKGroups * kKRows));
        cfg.blockDim = dim3(kKWarps * 32);
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = pdl ? 1 : 0;
        const cudaError_t e = cudaLaunchKernelEx(&cfg, fmt == FMT_Q4_K ? q4k_matvec_kernel : q6k_matvec_kernel, p);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace alj
