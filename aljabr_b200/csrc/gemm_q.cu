// Batched GGUF Q4_0 / Q8_0 dequantise-and-GEMM on the 5th-generation tensor
// cores (tcgen05, sm_100a): Y[m][n] = sum_k X[m][k] * W[n][k] for a batch of
// M >= 2 tokens with fp32 activations -- the prefill projections that the
// reference runs per token through dispatchMatVecBatch
// (engine/gguf/aljabr-gguf-java/.../javabackend/GgufExecutionDispatcher.java:
// 57-72, the Metal seam's aljabr_metal_matvec_tb_batch / _tb_triple_batch),
// whose fp32 arithmetic is d * (q - 8) * x summed per row.
//
// Arithmetic.  A Q4_0 / Q8_0 weight is v = d q with d an fp16 block scale (one
// per 32 elements) and q an integer (|q| <= 8, or <= 128).  The block scale
// changes every 32 columns, faster than a TMEM accumulator could be drained
// and rescaled, so it is folded into the A operand:
//   * A: v' = d' q, d' = d 2^s with one exponent s per matrix (chosen at
//     packing so that max |v'| <= 2^15), split as hi = fp16(v'), lo =
//     fp16(v' - hi) (HMUL2, then HFMA2 for the exact residual): v' has at
//     most 19 significant bits, so hi + lo holds it exactly unless lo falls
//     below fp16's normal range;
//   * B: x' = x 2^f per token (max |x'| in [2^14, 2^15)), split the same way
//     into fp16 hi / lo planes by gemm_q_x_prep_kernel;
//   * token tiles of up to 64: the hi and lo activation tiles lie back to
//     back in shared memory, so one B operand of N = 2 MT tokens covers both
//     and two tcgen05.mma per 16-column k-step (A_hi and A_lo against it) form
//     all four products, the accumulator's two halves holding the x_hi and
//     x_lo sums (a small MMA costs about the same issue time whatever its N,
//     so two wide ones beat three narrow ones);
//   * 128-token tiles: three tcgen05.mma per k-step -- A_hi B_hi, A_hi B_lo,
//     A_lo B_hi (the A_lo B_lo term is below 2^-22 relative) -- into one
//     accumulator of MT columns;
//   * the accumulator covers one 64-column stage: the epilogue drains it
//     after every stage into fp32 registers (round-to-nearest adds) and the
//     next stage starts a fresh one.  The tensor core's fp32 accumulation
//     truncates: over a whole 4096-column row its error reached ~5e-6 of the
//     row's scale (over 1e-3 of the smallest outputs), and over 256-column
//     units it still reached 2e-3 where a row's partial sums are large
//     against its result (constant weights against a periodic input); 12
//     adds per chain keep it at the level of fp32 summation.  The output is
//     scaled by 2^-(f + s) at the end.
// The products are exact in the tensor core; what rounds is the fp32
// accumulation and the dropped lo x lo term (~2^-22 relative per product).
//
// Weight layout.  Packed once per matrix (gemm_q_pack_kernel; the C-ABI's
// host-buffer batch entry points cache the packed copy per registered
// matrix, as the reference caches prepared Q4_0 rows):
//   header  256 B: int s, the matrix exponent, and the scratch word of the
//           max |d| reduction (uint bits; >= Inf bits means a non-finite d);
//   codes   per 128-row tile and 256-column unit, 1 (Q4_0) or 2 (Q8_0)
//           blocks of 128 rows x 128 B (16 KB, TMA box with 128-byte
//           swizzle).  Q4_0: byte i holds elements 2i (high nibble) and
//           2i + 1 (low nibble) of the unit, as codes 0..15; Q8_0: the int8
//           codes in element order, columns 0-127 then 128-255;
//   scales  per tile and unit, 128 rows x 8 fp16 d' (the unit's 8 blocks).
// Rows past the matrix are zero.  A unit's codes and scales land in one ring
// slot; pieces of 128 B per row, as the row-major GGUF layout would give,
// streamed at a fraction of the HBM rate in the NF4 GEMM.
//
// Warp roles (one CTA per SM, all 512 TMEM columns: 4 A stages x 64 columns,
// then the accumulator buffers of CH x MT columns, one per stage in flight):
//   warps 0-3      dequant: thread r owns weight row r = TMEM lane r; per
//                  64-column stage it reads its 32 (Q4_0) or 64 (Q8_0) code
//                  bytes and 2 block scales, forms the 32 fp16 (hi, hi) and 32
//                  (lo, lo) column pairs and stores them into the stage's
//                  TMEM columns with two tcgen05.st;
//   warps 4..      epilogue (1 or 2 warpgroups): after every stage warp w
//                  reads TMEM lanes 32 (w % 4) .. +31, a token half each, and
//                  adds the stage's accumulators into its registers; at the
//                  end of a tile piece it writes y (or the piece's partial,
//                  for a tile split between CTAs);
//   next warp      weight stream: one TMA copy (two for Q8_0) of a unit's
//                  codes and one of its scales per ring slot;
//   next warp      activation stream: the x hi and lo tiles of each stage
//                  (box 64 x MT, 128-byte swizzle) into one slot;
//   last warp      TMEM allocation and the MMA issue (one thread).
// The schedule (stream-K over 256-column units, split tiles summed in K
// order after a grid barrier) and every bounded wait are those of
// tc_gemm.cuh.
#include "tc_gemm.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

namespace alj {
namespace {

using namespace tcg;

constexpr int kHeaderBytes = 256;
constexpr int kCodeBlock = kRows * 128;             // 16 KB: 128 rows x 128 B
constexpr int kScaleBytes = kRows * 16;             // 2 KB: 128 rows x 8 fp16
constexpr int kACols = 64;                          // TMEM columns per A stage: 32 hi pairs, 32 lo pairs
constexpr int kARing = 4;
constexpr int kDCol0 = kARing * kACols;             // first accumulator column
constexpr int kMaxSeg = 3;
constexpr int kMaxCodesRing = 4;
constexpr int kMaxXRing = 8;
constexpr int kMaxDBufs = 8;

__host__ __device__ constexpr int code_blocks(int fmt) { return fmt == FMT_Q8_0 ? 2 : 1; }
__host__ __device__ constexpr int block_bytes(int fmt) { return fmt == FMT_Q8_0 ? 34 : 18; }
__host__ __device__ constexpr int slot_bytes(int fmt) { return code_blocks(fmt) * kCodeBlock + kScaleBytes; }
// Exponent so that max |d'| * max |q| <= 2^15: 2^12 for Q4_0 (|q| <= 8), 2^8 for Q8_0.
__host__ __device__ constexpr int scale_target(int fmt) { return fmt == FMT_Q8_0 ? 8 : 12; }

struct alignas(64) QSeg {
    CUtensorMap codes;      // uint8 [tiles * units * blocks * 128][128], box {128, 128}, 128 B swizzle
    CUtensorMap scales;     // fp16 [tiles * units * 128][8], box {8, 128}
    const int* exp;         // the packed header's matrix exponent s
    float* y;               // y[m * ldy + n]
    int rows;
    int ldy;
    int tile0;              // first row tile of the segment
};

struct alignas(64) QParams {
    QSeg seg[kMaxSeg];
    CUtensorMap xhi, xlo;   // fp16 [M][K] planes of x' = x 2^f, box {64, MT}, 128 B swizzle
    const int* tokexp;      // [M]
    float* partials;        // [2 * grid][MT][128]
    unsigned int* gbar;     // grid barrier flags, cleared by gemm_q_x_prep_kernel
    int nseg, M, K;
    int row_tiles, tok_tiles, tiles, units_per_tile;
    long long units;
    int grid, codes_ring, x_ring, dbufs;
    int nsplit;
    unsigned short split_tile[kMaxSplit], split_off[kMaxSplit], split_n[kMaxSplit];
    unsigned short piece_slot[kMaxPieces];
    __device__ int exp_of(int s) const { return __ldg(seg[s].exp); }
};

// ------------------------------------------------------------------ packing
// max |d| over the matrix into header word 1 (uint bits of a non-negative
// float order like the floats; NaN and Inf order above every finite value).
__global__ void gemm_q_scale_max_kernel(unsigned int* __restrict__ maxbits, const uint8_t* __restrict__ w,
                                        long long nblocks, int bbytes) {
    unsigned int m = 0u;
    for (long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; b < nblocks;
         b += static_cast<long long>(gridDim.x) * blockDim.x) {
        const uint8_t* p = w + b * bbytes;
        const uint32_t h = static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
        const uint32_t f = __float_as_uint(fabsf(f16_bits_to_f32(h)));
        m = f > m ? f : m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned int v = __shfl_xor_sync(0xffffffffu, m, o);
        m = v > m ? v : m;
    }
    if ((threadIdx.x & 31) == 0 && m) atomicMax(maxbits, m);
}

// The matrix exponent s from max |d|: 0 when the max is zero or not finite.
__device__ __forceinline__ int matrix_exponent(unsigned int maxbits, int fmt) {
    if (maxbits == 0u || maxbits >= 0x7F800000u) return 0;
    int e;
    frexpf(__uint_as_float(maxbits), &e);         // max = m 2^e, m in [0.5, 1)
    const int s = scale_target(fmt) - e;
    return s < -100 ? -100 : (s > 100 ? 100 : s);
}

// One thread per (row tile, unit, row, block of the unit): the block's codes
// in the packed order and its scale d 2^s.
__global__ void gemm_q_pack_kernel(int fmt, uint8_t* __restrict__ packed, const uint8_t* __restrict__ w, int rows,
                                   int K, int row_tiles, int units) {
    int* header = reinterpret_cast<int*>(packed);
    const int s = matrix_exponent(reinterpret_cast<const unsigned int*>(header)[1], fmt);
    if (blockIdx.x == 0 && threadIdx.x == 0) header[0] = s;
    const float sc = ldexpf(1.0f, s);
    const int cb = code_blocks(fmt);
    const int bb = block_bytes(fmt);
    uint8_t* codes = packed + kHeaderBytes;
    __half* scales = reinterpret_cast<__half*>(codes + static_cast<size_t>(row_tiles) * units * cb * kCodeBlock);
    const size_t total = static_cast<size_t>(row_tiles) * units * kRows * 8;
    const size_t row_bytes = static_cast<size_t>(K / 32) * bb;
    for (size_t q = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < total;
         q += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const int j = static_cast<int>(q & 7);                       // block within the unit
        const int rr = static_cast<int>((q >> 3) & (kRows - 1));
        const size_t tu = q >> 10;                                   // rt * units + u
        const int u = static_cast<int>(tu % units);
        const int row = static_cast<int>(tu / units) * kRows + rr;
        alignas(16) uint8_t out[32];
        float d = 0.0f;
        if (row < rows) {
            const uint8_t* blk = w + static_cast<size_t>(row) * row_bytes + static_cast<size_t>(u * 8 + j) * bb;
            d = f16_bits_to_f32(static_cast<uint32_t>(blk[0]) | (static_cast<uint32_t>(blk[1]) << 8));
            if (fmt == FMT_Q4_0) {
                // element p of the block: low nibble of byte p (p < 16), else high nibble of byte p - 16
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                    const int p0 = 2 * k, p1 = 2 * k + 1;
                    const int n0 = p0 < 16 ? (blk[2 + p0] & 15) : (blk[2 + p0 - 16] >> 4);
                    const int n1 = p1 < 16 ? (blk[2 + p1] & 15) : (blk[2 + p1 - 16] >> 4);
                    out[k] = static_cast<uint8_t>((n0 << 4) | n1);
                }
            } else {
#pragma unroll
                for (int k = 0; k < 32; ++k) out[k] = blk[2 + k];
            }
        } else {
#pragma unroll
            for (int k = 0; k < 32; ++k) out[k] = 0;
        }
        const size_t unit_base = tu * cb * kCodeBlock;
        if (fmt == FMT_Q4_0) {
            // 16 bytes: the block's 32 elements are bytes 16 j .. 16 j + 15 of the row
            uint8_t* dst = codes + unit_base + static_cast<size_t>(rr) * 128 + j * 16;
            reinterpret_cast<uint4*>(dst)[0] = *reinterpret_cast<const uint4*>(out);
        } else {
            // 32 bytes: half j / 4 (columns 0-127 or 128-255), bytes 32 (j % 4) .. +31
            uint8_t* dst = codes + unit_base + static_cast<size_t>(j / 4) * kCodeBlock + static_cast<size_t>(rr) * 128 +
                           (j % 4) * 32;
            reinterpret_cast<uint4*>(dst)[0] = *reinterpret_cast<const uint4*>(out);
            reinterpret_cast<uint4*>(dst)[1] = *reinterpret_cast<const uint4*>(out + 16);
        }
        scales[(tu * kRows + rr) * 8 + j] = __float2half_rn(d * sc);
    }
}

// ------------------------------------------------------------------ activations
constexpr int kPrepThreads = 1024;
constexpr int kPrepVecs = 8;                // float4 a thread keeps in registers: K <= 32768

__device__ __forceinline__ uint2 split_f16x4(float4 v, float sc, uint2& lo) {
    const float a[4] = {v.x * sc, v.y * sc, v.z * sc, v.w * sc};
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half hh = __float2half_rn(a[j]);
        h[j] = __half_as_ushort(hh);
        l[j] = __half_as_ushort(__float2half_rn(a[j] - __half2float(hh)));
    }
    lo = make_uint2(l[0] | (l[1] << 16), l[2] | (l[3] << 16));
    return make_uint2(h[0] | (h[1] << 16), h[2] | (h[3] << 16));
}

// fp32 activations -> fp16 planes hi / lo of x' = x 2^f per token, f = 15 - e
// with max |x| = m 2^e, m in [0.5, 1): max |x'| in [2^14, 2^15).  One block
// per token, a row of K <= 32768 read once and kept in registers.  Block 0
// also clears the GEMM's grid-barrier flags.  Each block lets the dependent
// GEMM launch as soon as it is resident.
__global__ void __launch_bounds__(kPrepThreads) gemm_q_x_prep_kernel(const float* __restrict__ x, int K,
                                                                     __half* __restrict__ xh, __half* __restrict__ xl,
                                                                     int* __restrict__ tokexp,
                                                                     unsigned int* __restrict__ flags, int nflags) {
    pdl_launch_dependents();
    const int m = blockIdx.x;
    if (m == 0)
        for (int i = threadIdx.x; i < nflags; i += blockDim.x) flags[i] = 0u;
    const float4* row = reinterpret_cast<const float4*>(x + static_cast<size_t>(m) * K);
    const int n4 = K / 4;
    const int nt = blockDim.x;
    float4 v[kPrepVecs];
    float mx = 0.0f;
#pragma unroll
    for (int k = 0; k < kPrepVecs; ++k) {
        const int i = threadIdx.x + k * nt;
        v[k] = i < n4 ? __ldg(row + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
    }
    __shared__ float red[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        float r = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) r = fmaxf(r, __shfl_xor_sync(0xffffffffu, r, o));
        if (threadIdx.x == 0) red[0] = r;
    }
    __syncthreads();
    mx = red[0];
    int f = 0;
    if (mx > 0.0f && mx <= 3.4028234663852886e38f) {
        int e;
        frexpf(mx, &e);
        f = 15 - e;
        f = f < -100 ? -100 : (f > 100 ? 100 : f);
    }
    if (threadIdx.x == 0) tokexp[m] = f;
    const float sc = ldexpf(1.0f, f);
    uint2* oh = reinterpret_cast<uint2*>(xh + static_cast<size_t>(m) * K);
    uint2* ol = reinterpret_cast<uint2*>(xl + static_cast<size_t>(m) * K);
#pragma unroll
    for (int k = 0; k < kPrepVecs; ++k) {
        const int i = threadIdx.x + k * nt;
        if (i < n4) {
            uint2 l;
            oh[i] = split_f16x4(v[k], sc, l);
            ol[i] = l;
        }
    }
}

// ------------------------------------------------------------------ kernel
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
// (hi, lo) of d' q for an fp16 pair of exact integers q: hi rounds the
// product, the fused residual q d' - hi is exact (at most 8 significant bits).
__device__ __forceinline__ void split_pair(uint32_t q, uint32_t dd, uint32_t& hi, uint32_t& lo) {
    hi = hmul2(q, dd);
    lo = hfma2(q, dd, hi ^ 0x80008000u);
}

// One stage: 4 k-steps x (A_hi B_hi, A_hi B_lo, A_lo B_hi) = 12 MMAs, each
// into the other accumulator than the one before (d1 == d0: one chain), then
// one commit onto `bar`.  `accum` = 0 starts a fresh accumulator: the first
// MMA into d0 overwrites it, and the first into d1 too unless d1 is d0.
// Token tiles <= 64: one stage as 4 k-steps x (A_hi, A_lo) x [x_hi | x_lo]
// (N = 2 MT) = 8 MMAs into one accumulator, then one commit onto `bar`; the
// first MMA overwrites the accumulator.
__device__ __forceinline__ void q_stage_mma_wide(uint32_t d, uint32_t ah, uint64_t b, uint32_t idesc, uint64_t* bar) {
    const uint32_t al = ah + kACols / 2;
    asm volatile(
        "{\n .reg .pred p0, p1;\n"
        " setp.ne.b32 p0, %0, %0;\n"
        " setp.eq.b32 p1, %0, %0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %9, %13, p0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %9, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %10, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], %10, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %11, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %11, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %12, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], %12, %13, p1;\n"
        " tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%14];\n"
        "}\n" ::"r"(d),
        "r"(ah), "r"(ah + 8), "r"(ah + 16), "r"(ah + 24), "r"(al), "r"(al + 8), "r"(al + 16), "r"(al + 24),
        "l"(b), "l"(b + 2), "l"(b + 4), "l"(b + 6), "r"(idesc), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void q_stage_mma(uint32_t d0, uint32_t d1, uint32_t ah, uint64_t bh, uint64_t bl,
                                            uint32_t idesc, uint32_t accum, uint64_t* bar) {
    const uint32_t al = ah + kACols / 2;
    const uint32_t accum1 = d1 == d0 ? 1u : accum;
    asm volatile(
        "{\n .reg .pred p0, p1, p2;\n"
        " setp.ne.b32 p0, %19, 0;\n"
        " setp.eq.b32 p1, %19, %19;\n"
        " setp.ne.b32 p2, %21, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %10, %18, p0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%1], [%2], %14, %18, p2;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], %10, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%1], [%3], %11, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %15, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%1], [%7], %11, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %12, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%1], [%4], %16, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], %12, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%1], [%5], %13, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %17, %18, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%1], [%9], %13, %18, p1;\n"
        " tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%20];\n"
        "}\n" ::"r"(d0),
        "r"(d1), "r"(ah), "r"(ah + 8), "r"(ah + 16), "r"(ah + 24), "r"(al), "r"(al + 8), "r"(al + 16), "r"(al + 24),
        "l"(bh), "l"(bh + 2), "l"(bh + 4), "l"(bh + 6), "l"(bl), "l"(bl + 2), "l"(bl + 4), "l"(bl + 6), "r"(idesc),
        "r"(accum), "r"(smem_u32(bar)), "r"(accum1)
        : "memory");
}

// The 32 hi and 32 lo column pairs of one 64-column stage of row r.
//   Q4_0: packed byte b of word j holds stage elements 8j + 2b (high nibble)
//         and 8j + 2b + 1 (low nibble); PRMT puts the two nibbles in the
//         low bytes of the two halves, LOP3 masks them and ORs in fp16 1024,
//         and 1024 + c - 1032 = c - 8 exactly;
//   Q8_0: bytes biased by 128 become the low mantissa byte of fp16 1024 + u
//         (PRMT with 0x64), and 1024 + u - 1152 = q exactly.
template <int FMT>
__device__ __forceinline__ void dequant_stage(uint32_t slot, int r, int st, uint32_t dd0, uint32_t dd1,
                                              uint32_t (&hi)[32], uint32_t (&lo)[32]) {
    const uint32_t swz = static_cast<uint32_t>(r & 7);
    if constexpr (FMT == FMT_Q4_0) {
        const uint32_t crow = slot + r * 128;
        const uint4 w0 = lds128(crow + ((static_cast<uint32_t>(2 * st) ^ swz) << 4));
        const uint4 w1 = lds128(crow + ((static_cast<uint32_t>(2 * st + 1) ^ swz) << 4));
        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t ws = words[j] >> 4;
            const uint32_t dd = j < 4 ? dd0 : dd1;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint32_t t = prmt(ws, words[j], static_cast<uint32_t>(b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12)));
                const uint32_t u = lop3_and_or(t, 0x000F000Fu, 0x64006400u);
                split_pair(hsub2(u, 0x64086408u), dd, hi[4 * j + b], lo[4 * j + b]);
            }
        }
    } else {
        const uint32_t crow = slot + static_cast<uint32_t>(st >> 1) * kCodeBlock + r * 128;
        const uint32_t c0 = static_cast<uint32_t>((st & 1) * 4);
        uint32_t words[16];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint4 w = lds128(crow + (((c0 + k) ^ swz) << 4));
            words[4 * k] = w.x;
            words[4 * k + 1] = w.y;
            words[4 * k + 2] = w.z;
            words[4 * k + 3] = w.w;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t wx = words[j] ^ 0x80808080u;
            const uint32_t dd = j < 8 ? dd0 : dd1;
            split_pair(hsub2(prmt(wx, 0x6464u, 0x4140u), 0x64806480u), dd, hi[2 * j], lo[2 * j]);
            split_pair(hsub2(prmt(wx, 0x6464u, 0x4342u), 0x64806480u), dd, hi[2 * j + 1], lo[2 * j + 1]);
        }
    }
}

template <int FMT, int MT, int EW>
__global__ void __launch_bounds__(32 * (7 + 4 * EW), 1) q_tc_gemm_kernel(const __grid_constant__ QParams p) {
    constexpr int NT = MT / EW;                 // tokens per epilogue thread
    constexpr bool WIDE = MT <= 64;             // one B operand of 2 MT tokens (x hi | x lo)
    constexpr int CH = WIDE ? 2 : 1;            // accumulator width in MT columns
    constexpr int kEpiWarp0 = 4;
    constexpr int kProdWarp = 4 + 4 * EW;       // codes + scales stream
    constexpr int kXWarp = kProdWarp + 1;       // activation tiles
    constexpr int kMmaWarp = kProdWarp + 2;     // TMEM allocation and MMA issue
    constexpr int CB = code_blocks(FMT);
    constexpr int SB = slot_bytes(FMT);
    constexpr int kXPlane = MT * 128;
    constexpr int kXBytes = 2 * kXPlane;        // hi then lo tile
    constexpr uint32_t kIdesc = idesc_f16(WIDE ? 2 * MT : MT);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int CQ = p.codes_ring;
    constexpr int SA = kARing;
    const int SX = p.x_ring;
    const int NB = p.dbufs;
    uint8_t* codes_ring = smem;
    uint8_t* x_ring = codes_ring + static_cast<size_t>(CQ) * SB;
    uint64_t* bars = reinterpret_cast<uint64_t*>(x_ring + static_cast<size_t>(SX) * kXBytes);
    uint64_t* codes_full = bars;
    uint64_t* codes_empty = codes_full + kMaxCodesRing;
    uint64_t* a_full = codes_empty + kMaxCodesRing;
    uint64_t* x_full = a_full + kARing;
    uint64_t* sdone = x_full + kMaxXRing;
    uint64_t* d_empty = sdone + kSDone;
    uint64_t* done_bar = d_empty + kMaxDBufs;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(done_bar + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1) + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxCodesRing; ++i) {
            mbar_init(&codes_full[i], 1);
            mbar_init(&codes_empty[i], 4);
        }
        for (int i = 0; i < kARing; ++i) mbar_init(&a_full[i], 4);
        for (int i = 0; i < kMaxXRing; ++i) mbar_init(&x_full[i], 1);
        for (int i = 0; i < kSDone; ++i) mbar_init(&sdone[i], 1);
        for (int i = 0; i < kMaxDBufs; ++i) mbar_init(&d_empty[i], 4 * EW);
        mbar_init(done_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

    const long long u0 = unit_begin(p, blockIdx.x);
    const long long u1 = unit_begin(p, blockIdx.x + 1);
    const int t_first = static_cast<int>(u0 / p.units_per_tile);
    const int t_last = static_cast<int>((u1 - 1) / p.units_per_tile);

    if (warp < 4) {
        // ---------------------------------------------------------- dequant
        const int r = threadIdx.x;              // tile row = TMEM lane
        const uint32_t ta_row = tmem_base + (static_cast<uint32_t>(32 * warp) << 16);
        Cursor cc{0, 0u}, ac{0, 0u}, rel{0, 0u};
        int si = 0;
        bool ok = u1 > u0;
        for (int t = t_first; ok && t <= t_last; ++t) {
            const Piece pc = make_piece(p, t, u0, u1);
            for (int c = pc.c0; ok && c < pc.c1; ++c) {
                if (!warp_wait(&codes_full[cc.slot], cc.phase, abort_flag)) { ok = false; break; }
                const uint32_t slot = smem_u32(codes_ring + static_cast<size_t>(cc.slot) * SB);
                const uint4 dq = lds128(slot + CB * kCodeBlock + r * 16);   // the unit's 8 block scales
                const uint32_t dw[4] = {dq.x, dq.y, dq.z, dq.w};
                for (int st = 0; st < kUnitStages; ++st, ++si) {
                    if (si >= SA) {   // the MMAs of stage si - SA have released this A slot
                        if (!warp_wait(&sdone[rel.slot], rel.phase, abort_flag)) { ok = false; break; }
                        rel.next(kSDone);
                    }
                    tc_fence_after();
                    uint32_t hi[32], lo[32];
                    dequant_stage<FMT>(slot, r, st, prmt(dw[st], 0u, 0x1010u), prmt(dw[st], 0u, 0x3232u), hi, lo);
                    tmem_st32(ta_row + ac.slot * kACols, hi);
                    tmem_st32(ta_row + ac.slot * kACols + kACols / 2, lo);
                    tmem_wait_st();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[ac.slot]);
                    ac.next(SA);
                }
                __syncwarp();
                if (ok && lane == 0) mbar_arrive(&codes_empty[cc.slot]);
                cc.next(CQ);
            }
        }
    } else if (warp < kProdWarp) {
        // ---------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int eh = (warp - kEpiWarp0) >> 2;
        const int r = 32 * q + lane;
        const uint32_t tq = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
        pdl_wait();       // token exponents (read at write-out)
        // The MMA thread is at most NB stages ahead (it waits for d_empty), so
        // a stage's sdone slot is not reused before this wait (NB < kSDone).
        Cursor dc{0, 0u}, sdc{0, 0u};
        bool ok = u1 > u0;
        for (int t = t_first; ok && t <= t_last; ++t) {
            const Piece pc = make_piece(p, t, u0, u1);
            const QSeg& sg = p.seg[pc.seg];
            float acc[NT];
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[j] = 0.0f;
            for (int i = 0; i < (pc.c1 - pc.c0) * kUnitStages; ++i) {
                if (!warp_wait(&sdone[sdc.slot], sdc.phase, abort_flag)) { ok = false; break; }
                sdc.next(kSDone);
                tc_fence_after();
                const uint32_t ta = tq + static_cast<uint32_t>(kDCol0 + dc.slot * CH * MT + eh * NT);
#pragma unroll
                for (int h = 0; h < NT / 16; ++h) {
                    uint32_t v[16];
                    tmem_ld16(ta + 16 * h, v);
                    if constexpr (CH == 2) {
                        uint32_t w[16];
                        tmem_ld16(ta + MT + 16 * h, w);
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            acc[16 * h + j] += __uint_as_float(v[j]) + __uint_as_float(w[j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) acc[16 * h + j] += __uint_as_float(v[j]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&d_empty[dc.slot]);
                dc.next(NB);
            }
            if (!ok) break;
            // ---- write-out: a whole tile goes to y; a piece of a split tile
            // to its partial slot (summed after the grid barrier).
            const int n = pc.row0 + r;
            const int m0 = pc.tok0 * MT + eh * NT;
            const int cf = cta_of(p, static_cast<long long>(t) * p.units_per_tile);
            const int cl = cta_of(p, static_cast<long long>(t + 1) * p.units_per_tile - 1);
            if (cf != cl) {
                float* part = p.partials + static_cast<size_t>(slot_of(p, blockIdx.x, t)) * (MT * kRows);
#pragma unroll
                for (int j = 0; j < NT; ++j) part[(eh * NT + j) * kRows + r] = acc[j];
            } else if (n < sg.rows) {
                const int e = __ldg(sg.exp);
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const int m = m0 + j;
                    if (m < p.M) sg.y[static_cast<size_t>(m) * sg.ldy + n] = acc[j] * out_scale(__ldg(p.tokexp + m), e);
                }
            }
        }
    } else if (warp == kProdWarp) {
        // ---------------------------------------------------------- codes + scales stream
        if (lane == 0) {
            Cursor cc{0, 0u};
            bool ok = u1 > u0;
            for (int t = t_first; ok && t <= t_last; ++t) {
                const Piece pc = make_piece(p, t, u0, u1);
                const QSeg& sg = p.seg[pc.seg];
                const int rt = pc.row0 / kRows;
                for (int c = pc.c0; ok && c < pc.c1; ++c) {
                    if (!wait_bar(&codes_empty[cc.slot], cc.phase ^ 1u, abort_flag)) { ok = false; break; }
                    mbar_arrive_expect_tx(&codes_full[cc.slot], SB);
                    const uint32_t dst = smem_u32(codes_ring + static_cast<size_t>(cc.slot) * SB);
                    const int g = rt * p.units_per_tile + c;
#pragma unroll
                    for (int b = 0; b < CB; ++b)
                        tma_load_2d(dst + b * kCodeBlock, &sg.codes, 0, (g * CB + b) * kRows, &codes_full[cc.slot]);
                    tma_load_2d(dst + CB * kCodeBlock, &sg.scales, 0, g * kRows, &codes_full[cc.slot]);
                    cc.next(CQ);
                }
            }
        }
    } else if (warp == kXWarp) {
        // ---------------------------------------------------------- activation tiles
        if (lane == 0) {
            pdl_wait();   // x planes and token exponents come from gemm_q_x_prep_kernel
            Cursor xc{0, 0u}, rel{0, 0u};
            int xi = 0;
            bool ok = u1 > u0;
            for (int t = t_first; ok && t <= t_last; ++t) {
                const Piece pc = make_piece(p, t, u0, u1);
                for (int c = pc.c0; ok && c < pc.c1; ++c) {
                    for (int st = 0; st < kUnitStages; ++st, ++xi) {
                        if (xi >= SX) {   // the MMAs of stage xi - SX have released this slot
                            if (!wait_bar(&sdone[rel.slot], rel.phase, abort_flag)) { ok = false; break; }
                            rel.next(kSDone);
                        }
                        mbar_arrive_expect_tx(&x_full[xc.slot], kXBytes);
                        const uint32_t dst = smem_u32(x_ring + static_cast<size_t>(xc.slot) * kXBytes);
                        const int kx = c * kUnitK + st * kStageK;
                        tma_load_2d(dst, &p.xhi, kx, pc.tok0 * MT, &x_full[xc.slot]);
                        tma_load_2d(dst + kXPlane, &p.xlo, kx, pc.tok0 * MT, &x_full[xc.slot]);
                        xc.next(SX);
                    }
                }
            }
        }
    } else {
        // ---------------------------------------------------------- MMA issue
        if (lane == 0) {
            Cursor dc{0, 0u}, xc{0, 0u}, ac{0, 0u}, sd{0, 0u};
            bool ok = u1 > u0;
            for (int t = t_first; ok && t <= t_last; ++t) {
                const Piece pc = make_piece(p, t, u0, u1);
                for (int i = 0; i < (pc.c1 - pc.c0) * kUnitStages; ++i) {
                    if (!wait_bar(&d_empty[dc.slot], dc.phase ^ 1u, abort_flag) ||
                        !wait_bar(&x_full[xc.slot], xc.phase, abort_flag) ||
                        !wait_bar(&a_full[ac.slot], ac.phase, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d0 = tmem_base + static_cast<uint32_t>(kDCol0 + dc.slot * CH * MT);
                    const uint32_t ah = tmem_base + static_cast<uint32_t>(ac.slot * kACols);
                    const uint32_t xs = smem_u32(x_ring + static_cast<size_t>(xc.slot) * kXBytes);
                    // a fresh accumulator per stage; sdone reports it complete
                    if constexpr (WIDE)
                        q_stage_mma_wide(d0, ah, sdesc(xs), kIdesc, &sdone[sd.slot]);
                    else
                        q_stage_mma(d0, d0, ah, sdesc(xs), sdesc(xs + kXPlane), kIdesc, 0u, &sdone[sd.slot]);
                    xc.next(SX);
                    ac.next(SA);
                    sd.next(kSDone);
                    dc.next(NB);
                }
            }
            // Every MMA issued has completed before TMEM is released.
            tc_commit(done_bar);
            mbar_wait(done_bar, 0);
        }
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == kMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512) : "memory");
    }
    if (p.nsplit == 0) return;
    finish_split_tiles(p, MT, abort_flag);
}

// ------------------------------------------------------------------ host
struct QWs {
    size_t xh, xl, tokexp, gbar, partials, total;
};
QWs q_ws_layout(int M, int K, int grid) {
    const int MT = token_tile_for(M);
    QWs w;
    w.xh = 0;
    w.xl = align_up(w.xh + static_cast<size_t>(M) * K * 2, 256);
    w.tokexp = align_up(w.xl + static_cast<size_t>(M) * K * 2, 256);
    w.gbar = align_up(w.tokexp + static_cast<size_t>(M) * 4, 256);
    w.partials = align_up(w.gbar + static_cast<size_t>(kMaxSplit) * 4, 256);
    w.total = align_up(w.partials + static_cast<size_t>(2) * grid * MT * kRows * 4, 256);
    return w;
}

// Ring depths in shared memory: 4 codes slots if 4 activation slots still
// fit, else 3 and 3, else 2 (Q8_0 with wide token tiles).  The launch always
// asks for the whole 227 KB, so that one CTA -- the one TMEM owner -- runs
// per SM.
struct QRings {
    int codes, x;
};
QRings q_rings(int fmt, int MT) {
    const size_t fixed = 1024 + 1024;           // alignment slack, barriers
    const size_t sb = slot_bytes(fmt);
    const size_t xb = static_cast<size_t>(2) * MT * 128;
    auto x_for = [&](int codes) {
        const size_t used = fixed + codes * sb;
        return used < static_cast<size_t>(kSmemMax) ? static_cast<int>(std::min<size_t>(kMaxXRing, (kSmemMax - used) / xb))
                                                     : 0;
    };
    if (x_for(4) >= 4) return QRings{4, x_for(4)};
    if (x_for(3) >= 3) return QRings{3, x_for(3)};
    return QRings{2, x_for(2)};
}

size_t q_packed_codes_bytes(int fmt, int rows, int K) {
    return static_cast<size_t>((rows + kRows - 1) / kRows) * (K / kUnitK) * code_blocks(fmt) * kCodeBlock;
}

template <int FMT, int MT, int EW>
cudaError_t q_launch_mt(const QParams& p, size_t smem, cudaStream_t stream) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(q_tc_gemm_kernel<FMT, MT, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemMax);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    // Cooperative when split tiles need the grid barrier (all CTAs resident:
    // one per SM by shared memory, grid <= SM count); programmatic dependent
    // launch on the activation prep just before it.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(32 * (7 + 4 * EW));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.nsplit > 0 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, q_tc_gemm_kernel<FMT, MT, EW>, p);
}

template <int FMT>
cudaError_t q_launch_fmt(int MT, const QParams& p, size_t smem, cudaStream_t stream) {
    switch (MT) {
        case 16: return q_launch_mt<FMT, 16, 1>(p, smem, stream);
        case 32: return q_launch_mt<FMT, 32, 1>(p, smem, stream);
        case 64: return q_launch_mt<FMT, 64, 2>(p, smem, stream);
        default: return q_launch_mt<FMT, 128, 2>(p, smem, stream);
    }
}

}  // namespace

bool gemm_q_supported(int fmt, int M, int K) {
    return (fmt == FMT_Q4_0 || fmt == FMT_Q8_0) && M >= 1 && M <= (1 << 20) && K > 0 && K % kUnitK == 0 &&
           K <= 32768 && tensor_map_encoder() != nullptr;
}

size_t gemm_q_packed_bytes(int fmt, int rows, int K) {
    return kHeaderBytes + q_packed_codes_bytes(fmt, rows, K) +
           static_cast<size_t>((rows + kRows - 1) / kRows) * (K / kUnitK) * kScaleBytes;
}

cudaError_t launch_gemm_q_pack(int fmt, void* packed, const void* w, int rows, int K, cudaStream_t stream) {
    if (rows < 1 || !gemm_q_supported(fmt, 2, K)) return cudaErrorNotSupported;
    if (reinterpret_cast<uintptr_t>(packed) & 255) return cudaErrorInvalidValue;
    uint8_t* pk = static_cast<uint8_t*>(packed);
    cudaError_t e = cudaMemsetAsync(pk, 0, kHeaderBytes, stream);
    if (e != cudaSuccess) return e;
    const int sms = sm_count_for_current_device();
    const long long nblocks = static_cast<long long>(rows) * (K / 32);
    gemm_q_scale_max_kernel<<<2 * sms, 256, 0, stream>>>(reinterpret_cast<unsigned int*>(pk) + 1,
                                                         static_cast<const uint8_t*>(w), nblocks, block_bytes(fmt));
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int row_tiles = (rows + kRows - 1) / kRows;
    gemm_q_pack_kernel<<<4 * sms, 256, 0, stream>>>(fmt, pk, static_cast<const uint8_t*>(w), rows, K, row_tiles,
                                                    K / kUnitK);
    return cudaGetLastError();
}

int gemm_q_tiles(int M, int nseg, const int* rows) {
    int rt = 0;
    for (int s = 0; s < nseg; ++s) rt += (rows[s] + kRows - 1) / kRows;
    const int MT = token_tile_for(M);
    return rt * ((M + MT - 1) / MT);
}

size_t gemm_q_workspace_bytes(int M, int K) { return q_ws_layout(M, K, kMaxSplit).total; }

cudaError_t launch_gemm_q(const GemmQArgs& a, cudaStream_t stream) {
    if (a.nseg < 1 || a.nseg > kMaxSeg || !gemm_q_supported(a.fmt, a.M, a.K)) return cudaErrorNotSupported;
    const int MT = token_tile_for(a.M);
    const int CB = code_blocks(a.fmt);
    QParams p;
    memset(&p, 0, sizeof p);
    p.nseg = a.nseg;
    p.M = a.M;
    p.K = a.K;
    int rt = 0;
    const int units = a.K / kUnitK;
    for (int s = 0; s < a.nseg; ++s) {
        QSeg& g = p.seg[s];
        if (a.rows[s] <= 0 || !a.y[s] || a.ldy[s] < a.rows[s] || (reinterpret_cast<uintptr_t>(a.packed[s]) & 255))
            return cudaErrorInvalidValue;
        const int tiles_s = (a.rows[s] + kRows - 1) / kRows;
        const uint8_t* pk = static_cast<const uint8_t*>(a.packed[s]);
        const uint8_t* pc = pk + kHeaderBytes;
        const uint8_t* ps = pc + q_packed_codes_bytes(a.fmt, a.rows[s], a.K);
        if (!encode_2d(&g.codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, pc, 128,
                       static_cast<uint64_t>(tiles_s) * units * CB * kRows, 128, kRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !encode_2d(&g.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ps, 8, static_cast<uint64_t>(tiles_s) * units * kRows,
                       8, kRows, CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
        g.exp = reinterpret_cast<const int*>(pk);
        g.y = a.y[s];
        g.rows = a.rows[s];
        g.ldy = a.ldy[s];
        g.tile0 = rt;
        rt += tiles_s;
    }
    p.row_tiles = rt;
    p.tok_tiles = (a.M + MT - 1) / MT;
    p.tiles = rt * p.tok_tiles;
    p.units_per_tile = units;
    if (!plan_stream_k(p, sm_count_for_current_device())) return cudaErrorNotSupported;
    const QWs w = q_ws_layout(a.M, a.K, p.grid);
    if (!a.workspace || a.workspace_bytes < w.total || (reinterpret_cast<uintptr_t>(a.workspace) & 255))
        return cudaErrorInvalidValue;
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    __half* xh = reinterpret_cast<__half*>(ws + w.xh);
    __half* xl = reinterpret_cast<__half*>(ws + w.xl);
    p.tokexp = reinterpret_cast<const int*>(ws + w.tokexp);
    p.gbar = reinterpret_cast<unsigned int*>(ws + w.gbar);
    p.partials = reinterpret_cast<float*>(ws + w.partials);
    if (!encode_2d(&p.xhi, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, a.K, a.M, kStageK, MT, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_2d(&p.xlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xl, a.K, a.M, kStageK, MT, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const QRings rg = q_rings(a.fmt, MT);
    if (rg.x < 2) return cudaErrorNotSupported;
    p.codes_ring = rg.codes;
    p.x_ring = rg.x;
    p.dbufs = std::min(kMaxDBufs, (512 - kDCol0) / ((MT <= 64 ? 2 : 1) * MT));

    const int prep_threads = std::min(kPrepThreads, std::max(128, (a.K / 4 / kPrepVecs + 31) / 32 * 32));
    gemm_q_x_prep_kernel<<<a.M, prep_threads, 0, stream>>>(a.x, a.K, xh, xl, reinterpret_cast<int*>(ws + w.tokexp),
                                                           p.gbar, p.grid);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    return a.fmt == FMT_Q4_0 ? q_launch_fmt<FMT_Q4_0>(MT, p, kSmemMax, stream)
                             : q_launch_fmt<FMT_Q8_0>(MT, p, kSmemMax, stream);
}

}  // namespace alj
