// Batch-1 dequantise-and-matvec kernels (y = W x) for GGUF Q4_0 / Q8_0 and
// NF4 weights on B200 (sm_100a), plus the bit-exact dequantisation kernels.
//
// Design (HBM-bound streaming; two CTAs per SM so that, under programmatic
// dependent launch, the next matvec's weight copies start while the
// previous one finishes):
//   * rows are handed out in units of 4; each CTA owns a contiguous,
//     balanced range of units and walks it in tiles (32 rows NF4, 16 rows
//     GGUF) x K-chunks;
//   * one producer thread streams each tile's chunk into shared memory with
//     2-D TMA tensor copies (one 4-row box per copy, cp.async.bulk.tensor)
//     completing on an mbarrier, through a multi-stage ring of empty/full
//     barrier pairs; boxes land densely, row after row;
//   * 8 consumer warps each own every 8th row of the tile; inside a warp the
//     lanes split the chunk's columns, and each lane loads its slice of x
//     straight from global memory into registers once per chunk and reuses
//     it for all its rows -- shared memory carries only weights;
//   * per-row partial sums stay in the lane until the tile's last chunk and
//     are then reduced with 5 shuffles: no cross-warp reduction;
//   * 4-bit / 8-bit GGUF codes become exact floats with one LOP3 each (the
//     code placed in the mantissa of 2^23) and one packed f32x2 add per two
//     codes; products accumulate with packed f32x2 FMA;
//   * NF4 bytes index a 256-entry table of value pairs (T[hi], T[lo]) with 16
//     copies in shared memory (entry b, copy c at 8 * (16 b + c)); an LDS.64
//     is served per half-warp, so lane l reading copy l % 16 is
//     conflict-free, and one load yields both weights of a byte;
//   * block scales (fp16 d for GGUF, fp32 absmax for NF4) are applied once
//     per block to the block's partial sum.
// Epilogues: plain store with optional bias / residual; SwiGLU over a
// gate/up segment pair (both rows of a pair land in the same warp); and an
// optional RMSNorm of the finished output vector, written by the last CTA
// to finish (fixed-order reduction of per-CTA partials, deterministic).
// Shapes the TMA path cannot stage (K not a multiple of 256, segment rows
// not a multiple of 4, unaligned pointers, other NF4 groups) run a plain
// one-warp-per-row kernel instead.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

namespace alj {

__device__ unsigned int g_fault_word = 0;

namespace {

__device__ const float kNf4Table[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

__device__ __forceinline__ float nf4_at(int code) { return kNf4Table[code & 15]; }

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kUnitRows = 4;                      // rows per TMA box
constexpr int kMaxStages = 8;
constexpr int kCtaSmemBudget = 115712;            // two CTAs per SM (228 KB minus 1 KB each)
constexpr int kLutBytes = 256 * 16 * 8;           // NF4 byte-pair table, 16 copies

template <int FMT>
struct Fmt;
template <>
struct Fmt<FMT_Q4_0> {
    static constexpr int kChunkElems = 2048;     // 64 blocks: 2 per lane
    static constexpr int kChunkBytes = 1152;     // per row
    static constexpr int kLaneF4 = 16;           // x float4s per lane
    static constexpr int kBoxInner = 144;        // in UINT64 elements
    static constexpr int kElemBytes = 8;
    static constexpr int kTileRows = 16;
    static size_t row_bytes(int K) { return static_cast<size_t>(K) / 32 * 18; }
};
template <>
struct Fmt<FMT_Q8_0> {
    static constexpr int kChunkElems = 1024;     // 32 blocks: 1 per lane
    static constexpr int kChunkBytes = 1088;
    static constexpr int kLaneF4 = 8;
    static constexpr int kBoxInner = 136;
    static constexpr int kElemBytes = 8;
    static constexpr int kTileRows = 16;
    static size_t row_bytes(int K) { return static_cast<size_t>(K) / 32 * 34; }
};
template <>
struct Fmt<FMT_NF4> {
    static constexpr int kChunkElems = 1024;     // 32 codes (16 bytes) per lane
    static constexpr int kChunkBytes = 512;
    static constexpr int kLaneF4 = 8;
    static constexpr int kBoxInner = 128;        // in UINT32 elements
    static constexpr int kElemBytes = 4;
    static constexpr int kTileRows = 32;
    static size_t row_bytes(int K) { return static_cast<size_t>(K) / 2; }
};

struct alignas(64) TmaSegment {
    CUtensorMap codes;    // 2-D: [rows][row bytes], box = 4 rows x one chunk
    CUtensorMap absmax;   // NF4: [rows][K/group] fp32, box = 4 rows x chunk/group
    const float* bias;
    const float* residual;
    float* y;
    int rows;
    int row0;             // first global row of this segment
};

struct alignas(64) TmaParams {
    TmaSegment seg[3];
    int nseg;
    int K;
    int total_rows;
    int epilogue;
    const float* x;
    float* norm_out;
    const float* norm_w;
    float norm_eps;
    float* norm_partials;
    unsigned int* norm_counter;
};

// Exact magic constants: float(0x4B000000 | (c << s)) = 2^23 + c * 2^s.
constexpr uint32_t kMagic = 0x4B000000u;
constexpr float kTwo23 = 8388608.0f;

__device__ __forceinline__ float2 lds_f2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// ---- per-format row dots over one chunk (this lane's columns) -------------
// Q4_0 block with natural-order x (xb[i] = x[4i..4i+3], xb[4+i] =
// x[16+4i..]): byte j holds element j (low nibble) and j+16 (high nibble).
// Low nibbles of bytes (j, j+1) sit at bits (0, 8) of a code word and pair
// with (x_j, x_{j+1}); high nibbles at bits (4, 12) pair with (x_{j+16},
// x_{j+17}).  Scales per lane of the packed pair: lo (1, 256), hi (16, 4096).
__device__ __forceinline__ float q4_0_block(uint32_t dbits, const uint32_t (&c)[4], const float4* xb) {
    const f2 klo = mk2(-(kTwo23 + 8.0f), -(kTwo23 + 2048.0f));
    const f2 khi = mk2(-(kTwo23 + 128.0f), -(kTwo23 + 32768.0f));
    f2 alo = mk2(0.0f, 0.0f), ahi = mk2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 xl = xb[i], xh = xb[4 + i];
        const uint32_t w = c[i], w2 = w >> 16;
        const f2 l0 = add2(mk2u((w & 0xFu) | kMagic, (w & 0xF00u) | kMagic), klo);       // elements 4i, 4i+1
        const f2 h0 = add2(mk2u((w & 0xF0u) | kMagic, (w & 0xF000u) | kMagic), khi);     // 4i+16, 4i+17
        const f2 l1 = add2(mk2u((w2 & 0xFu) | kMagic, (w2 & 0xF00u) | kMagic), klo);     // 4i+2, 4i+3
        const f2 h1 = add2(mk2u((w2 & 0xF0u) | kMagic, (w2 & 0xF000u) | kMagic), khi);   // 4i+18, 4i+19
        alo = fma2(l0, mk2(xl.x, xl.y), alo);
        ahi = fma2(h0, mk2(xh.x, xh.y), ahi);
        alo = fma2(l1, mk2(xl.z, xl.w), alo);
        ahi = fma2(h1, mk2(xh.z, xh.w), ahi);
    }
    // alo = (s1, 256 s1'), ahi = (16 s, 4096 s'): fold to 16x units, then 1x
    const f2 t = fma2(alo, mk2(16.0f, 1.0f / 16.0f), mk2(hi(ahi) * (1.0f / 256.0f), lo(ahi)));
    const float bs = (lo(t) + hi(t)) * 0.0625f;
    return __half2float(__ushort_as_half(static_cast<unsigned short>(dbits))) * bs;
}

// Block bb (0 or 1) of this lane's two: block 0's fp16 d is word-aligned and
// its codes 2 bytes off, block 1 the reverse (words 4..8 of the 36 bytes).
__device__ __forceinline__ float q4_0_half(uint32_t row_addr, int lane, int bb, const float4* x) {
    const uint32_t a = row_addr + lane * 36 + bb * 16;
    uint32_t W[5];
#pragma unroll
    for (int k = 0; k < 5; ++k) W[k] = lds_u32(a + 4 * k);
    uint32_t c[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) c[i] = bb ? W[1 + i] : __funnelshift_r(W[i], W[i + 1], 16);
    return q4_0_block(bb ? (W[0] >> 16) : (W[0] & 0xFFFFu), c, x);
}

// Q8_0: this lane's block (34 B at 34*lane).  Even lanes start word-aligned
// (d low half, codes 2 bytes off), odd lanes 2 bytes in (d high half, codes
// aligned); a clamped funnel shift of 16 or 32 bits serves both.
__device__ __forceinline__ float q8_0_row(uint32_t row_addr, int lane, const float4* x) {
    uint32_t W[9];
    const uint32_t a = row_addr + ((lane * 34) & ~3);
#pragma unroll
    for (int k = 0; k < 9; ++k) W[k] = lds_u32(a + 4 * k);
    const uint32_t odd = lane & 1;
    const uint32_t dbits = __funnelshift_rc(W[0], W[1], 16 * odd) & 0xFFFFu;
    const uint32_t sh = 16 + 16 * odd;
    const f2 kq = mk2(-(kTwo23 + 128.0f), -(kTwo23 + 32768.0f));
    f2 A = mk2(0.0f, 0.0f), B = mk2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t w = __funnelshift_rc(W[i], W[i + 1], sh), w2 = w >> 16;
        const float4 xv = x[i];
        // signed byte b -> 2^23 + (b + 128): xor bit 7 into the magic
        const f2 p = add2(mk2u((w & 0xFFu) ^ 0x4B000080u, (w & 0xFF00u) ^ 0x4B008000u), kq);    // (b0, 256 b1)
        const f2 q = add2(mk2u((w2 & 0xFFu) ^ 0x4B000080u, (w2 & 0xFF00u) ^ 0x4B008000u), kq);  // (b2, 256 b3)
        if (i & 1) {
            B = fma2(p, mk2(xv.x, xv.y), B);
            B = fma2(q, mk2(xv.z, xv.w), B);
        } else {
            A = fma2(p, mk2(xv.x, xv.y), A);
            A = fma2(q, mk2(xv.z, xv.w), A);
        }
    }
    const f2 t = add2(A, B);
    return __half2float(__ushort_as_half(static_cast<unsigned short>(dbits))) * fmaf(hi(t), 1.0f / 256.0f, lo(t));
}

// NF4: this lane's 16 code bytes (32 weights, inside one absmax group) at
// 16*lane.  lut_lane = shared address of copy (lane % 16) of entry 0.
__device__ __forceinline__ float nf4_row(uint32_t row_addr, float am, uint32_t lane_off, uint32_t lut_lane,
                                         const float4* x) {
    uint32_t w[4];
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
                 : "r"(row_addr + lane_off));
    f2 A = mk2(0.0f, 0.0f), B = mk2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        // byte b of word k -> weights 8k+2b (high nibble), 8k+2b+1 (low nibble);
        // entry of byte v: lut_lane + 128 v
        const float2 t0 = lds_f2(lut_lane + (__byte_perm(w[k], 0, 0x4440) << 7));
        const float2 t1 = lds_f2(lut_lane + (__byte_perm(w[k], 0, 0x4441) << 7));
        const float2 t2 = lds_f2(lut_lane + (__byte_perm(w[k], 0, 0x4442) << 7));
        const float2 t3 = lds_f2(lut_lane + (__byte_perm(w[k], 0, 0x4443) << 7));
        const float4 x0 = x[2 * k], x1 = x[2 * k + 1];
        A = fma2(mk2(t0.x, t0.y), mk2(x0.x, x0.y), A);
        B = fma2(mk2(t1.x, t1.y), mk2(x0.z, x0.w), B);
        A = fma2(mk2(t2.x, t2.y), mk2(x1.x, x1.y), A);
        B = fma2(mk2(t3.x, t3.y), mk2(x1.z, x1.w), B);
    }
    const f2 t = add2(A, B);
    return am * (lo(t) + hi(t));
}

__device__ __forceinline__ void locate_row(const TmaParams& p, int row, int& seg, int& lrow) {
    seg = 0;
    if (p.nseg > 1 && row >= p.seg[1].row0) seg = 1;
    if (p.nseg > 2 && row >= p.seg[2].row0) seg = 2;
    lrow = row - p.seg[seg].row0;
}

template <int FMT, int GROUP>
constexpr int stage_bytes() {
    return ((Fmt<FMT>::kTileRows * Fmt<FMT>::kChunkBytes +
             (FMT == FMT_NF4 ? Fmt<FMT>::kTileRows * (1024 / GROUP) * 4 : 0)) + 1023) & ~1023;
}

template <int FMT, int GROUP>
__global__ void __launch_bounds__(kThreads, 2) matvec_tma_kernel(const __grid_constant__ TmaParams p, int stages) {
    using F = Fmt<FMT>;
    constexpr int T = F::kTileRows;
    constexpr int R = T / kConsumerWarps;                    // rows per warp per tile
    constexpr int kStage = stage_bytes<FMT, GROUP>();
    constexpr int kAbsPerRow = 1024 / GROUP;                 // NF4 absmax floats per row-chunk
    constexpr int kCodeTile = T * F::kChunkBytes;            // codes region of a stage
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    pdl_launch_dependents();

    const int K = p.K;
    const int nchunks = (K + F::kChunkElems - 1) / F::kChunkElems;
    const bool pair = p.epilogue == EPI_SWIGLU_PAIR;
    const int unit_rows_per_tile = pair ? T / 2 : T;         // logical rows per tile
    const int tile_units = unit_rows_per_tile / kUnitRows;

    const uint32_t base = smem_u32(smem_raw);
    const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
    uint8_t* sp = smem_raw + pad;
    uint8_t* stage0 = sp;
    sp += static_cast<size_t>(stages) * kStage;
    float2* lut = reinterpret_cast<float2*>(sp);
    if (FMT == FMT_NF4) sp += kLutBytes;
    float* red = reinterpret_cast<float*>(sp);
    sp += 64;
    uint64_t* full = reinterpret_cast<uint64_t*>(sp);
    uint64_t* empty = full + kMaxStages;
    volatile int* flags = reinterpret_cast<volatile int*>(empty + kMaxStages);   // [0] abort, [1] last CTA

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = p.total_rows / kUnitRows;
    const int u_begin = static_cast<int>(static_cast<long long>(units) * blockIdx.x / gridDim.x);
    const int u_end = static_cast<int>(static_cast<long long>(units) * (blockIdx.x + 1) / gridDim.x);
    const int ntiles = (u_end - u_begin + tile_units - 1) / tile_units;
    const int items = ntiles * nchunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        flags[0] = 0;
        flags[1] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        // Weights never depend on the previous kernel, so the copies start
        // before griddepcontrol.wait.
        if (lane == 0) {
            for (int it = 0; it < items; ++it) {
                const int t = it / nchunks, c = it - t * nchunks;
                const int s = it % stages;
                const uint32_t round = static_cast<uint32_t>(it / stages);
                const int tu0 = u_begin + t * tile_units;
                const int nunits = min(tile_units, u_end - tu0);
                if (flags[0] || !mbar_wait(&empty[s], (round & 1u) ^ 1u)) {
                    flags[0] = 1;
                    break;
                }
                const uint32_t per_box = kUnitRows * (F::kChunkBytes + (FMT == FMT_NF4 ? kAbsPerRow * 4 : 0));
                mbar_arrive_expect_tx(&full[s], per_box * nunits * (pair ? 2 : 1));
                uint8_t* st = stage0 + static_cast<size_t>(s) * kStage;
                for (int u = 0; u < nunits; ++u) {
                    const int lrow_g = (tu0 + u) * kUnitRows;
                    for (int half = 0; half < (pair ? 2 : 1); ++half) {
                        int seg, lrow;
                        if (pair) {
                            seg = half;
                            lrow = lrow_g;
                        } else {
                            locate_row(p, lrow_g, seg, lrow);
                        }
                        const int srow = u * kUnitRows + half * (T / 2);
                        tma_load_2d(smem_u32(st + srow * F::kChunkBytes), &p.seg[seg].codes, c * F::kBoxInner, lrow,
                                    &full[s]);
                        if (FMT == FMT_NF4)
                            tma_load_2d(smem_u32(st + kCodeTile + srow * kAbsPerRow * 4), &p.seg[seg].absmax,
                                        c * kAbsPerRow, lrow, &full[s]);
                    }
                }
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        if (FMT == FMT_NF4) {
            for (int i = threadIdx.x; i < 256 * 16; i += kConsumerThreads) {
                const int b = i >> 4;
                lut[i] = make_float2(nf4_at(b >> 4), nf4_at(b & 15));
            }
            named_bar(1, kConsumerThreads);
        }
        const uint32_t lut_lane = smem_u32(lut) + (lane & 15) * 8;
        pdl_wait();   // x (and residual) come from the previous kernel
        float acc[R];
#pragma unroll
        for (int k = 0; k < R; ++k) acc[k] = 0.0f;
        float sq = 0.0f;   // this warp's share of sum(y^2) for the optional norm
        for (int it = 0; it < items; ++it) {
            const int t = it / nchunks, c = it - t * nchunks;
            const int s = it % stages;
            const uint32_t round = static_cast<uint32_t>(it / stages);
            const int tu0 = u_begin + t * tile_units;
            const int valid = min(tile_units, u_end - tu0) * kUnitRows;   // valid rows per tile half
            // this lane's slice of x for chunk c: 32 floats (one Q4_0 block at a time)
            const int e0 = c * F::kChunkElems + lane * (F::kLaneF4 * 4);
            float4 xr[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                xr[j] = (e0 + 4 * j < K) ? __ldg(reinterpret_cast<const float4*>(p.x + e0) + j)
                                         : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            const bool ok = (flags[0] == 0) && mbar_wait(&full[s], round & 1u);
            if (!ok) flags[0] = 1;
            if (ok) {
                const uint32_t st = smem_u32(stage0 + static_cast<size_t>(s) * kStage);
                const float* am = reinterpret_cast<const float*>(stage0 + static_cast<size_t>(s) * kStage + kCodeTile);
#pragma unroll
                for (int bb = 0; bb < (FMT == FMT_Q4_0 ? 2 : 1); ++bb) {
                    if (bb == 1) {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            xr[j] = (e0 + 32 + 4 * j < K)
                                        ? __ldg(reinterpret_cast<const float4*>(p.x + e0 + 32) + j)
                                        : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    }
#pragma unroll
                    for (int k = 0; k < R; ++k) {
                        const int r = warp + kConsumerWarps * k;
                        const int rl = pair ? (r % (T / 2)) : r;
                        if (rl < valid) {
                            if (FMT == FMT_Q4_0) {
                                acc[k] += q4_0_half(st + r * F::kChunkBytes, lane, bb, xr);
                            } else if (FMT == FMT_Q8_0) {
                                acc[k] += q8_0_row(st + r * F::kChunkBytes, lane, xr);
                            } else {
                                acc[k] += nf4_row(st + r * F::kChunkBytes, am[r * kAbsPerRow + (lane * 32) / GROUP],
                                                  lane * 16, lut_lane, xr);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (c == nchunks - 1) {
                float v[R];
#pragma unroll
                for (int k = 0; k < R; ++k) {
                    const int r = warp + kConsumerWarps * k;
                    const int rl = pair ? (r % (T / 2)) : r;
                    v[k] = rl < valid ? warp_sum(acc[k]) : 0.0f;
                    acc[k] = 0.0f;
                }
                if (lane == 0 && flags[0] == 0) {
                    if (pair) {
#pragma unroll
                        for (int k = 0; k < R / 2; ++k) {
                            const int r = warp + kConsumerWarps * k;
                            if (r < valid) {
                                const float g = v[k], u = v[k + R / 2];
                                p.seg[0].y[tu0 * kUnitRows + r] = g / (1.0f + expf(-g)) * u;
                            }
                        }
                    } else {
#pragma unroll
                        for (int k = 0; k < R; ++k) {
                            const int r = warp + kConsumerWarps * k;
                            if (r < valid) {
                                int seg, lrow;
                                locate_row(p, tu0 * kUnitRows + r, seg, lrow);
                                const TmaSegment& sg = p.seg[seg];
                                float out = v[k];
                                if (sg.bias) out += sg.bias[lrow];
                                if (sg.residual) out = sg.residual[lrow] + out;
                                sg.y[lrow] = out;
                                sq = fmaf(out, out, sq);
                            }
                        }
                    }
                }
            }
        }
        if (p.norm_out) {
            // Deterministic RMSNorm of the whole output: per-CTA partials in
            // fixed order, finished by the last CTA to arrive.
            __threadfence();
            if (lane == 0) red[warp] = sq;
            named_bar(1, kConsumerThreads);
            if (threadIdx.x == 0) {
                float cta = 0.0f;
                for (int w = 0; w < kConsumerWarps; ++w) cta += red[w];
                p.norm_partials[blockIdx.x] = cta;
                __threadfence();
                const unsigned int prev = atomicAdd(p.norm_counter, 1u);
                flags[1] = prev == gridDim.x - 1;
            }
            named_bar(1, kConsumerThreads);
            if (flags[1]) {
                __threadfence();
                if (threadIdx.x == 0) {
                    float tot = 0.0f;
                    for (unsigned int b = 0; b < gridDim.x; ++b) tot += __ldcg(p.norm_partials + b);
                    red[8] = 1.0f / sqrtf(tot / static_cast<float>(p.total_rows) + p.norm_eps);
                    *p.norm_counter = 0u;
                }
                named_bar(1, kConsumerThreads);
                const float scale = red[8];
                const float* y = p.seg[0].y;
                for (int i = threadIdx.x; i < p.total_rows; i += kConsumerThreads)
                    p.norm_out[i] = __ldcg(y + i) * scale * p.norm_w[i];
            }
        }
    }
}

// ---- generic fallback: one warp per row, any K that the format allows -----
struct RowLoc {
    int seg;
    int row;
};
__device__ __forceinline__ RowLoc locate(const MatvecParams& p, int r) {
    RowLoc l{0, r};
    if (p.nseg > 1 && l.row >= p.seg[0].rows) {
        l.row -= p.seg[0].rows;
        l.seg = 1;
        if (p.nseg > 2 && l.row >= p.seg[1].rows) {
            l.row -= p.seg[1].rows;
            l.seg = 2;
        }
    }
    return l;
}

template <int FMT>
__global__ void matvec_generic_kernel(const MatvecParams p) {
    pdl_launch_dependents();
    pdl_wait();
    const int warps = blockDim.x >> 5;
    const int r = blockIdx.x * warps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= p.total_rows) return;
    const RowLoc l = locate(p, r);
    const MatvecSegment& sg = p.seg[l.seg];
    const int K = p.K;
    float acc = 0.0f;
    if (FMT == FMT_Q4_0 || FMT == FMT_Q8_0) {
        const int bb = FMT == FMT_Q4_0 ? 18 : 34;
        const uint8_t* row = sg.w + static_cast<size_t>(l.row) * (K / 32) * bb;
        for (int b = lane; b < K / 32; b += 32) {
            const uint8_t* blk = row + static_cast<size_t>(b) * bb;
            const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
            float s = 0.0f;
            if (FMT == FMT_Q4_0) {
                for (int j = 0; j < 16; ++j) {
                    const int q = blk[2 + j];
                    s = fmaf(static_cast<float>((q & 15) - 8), p.x[b * 32 + j], s);
                    s = fmaf(static_cast<float>((q >> 4) - 8), p.x[b * 32 + 16 + j], s);
                }
            } else {
                for (int j = 0; j < 32; ++j)
                    s = fmaf(static_cast<float>(static_cast<int8_t>(blk[2 + j])), p.x[b * 32 + j], s);
            }
            acc = fmaf(d, s, acc);
        }
    } else {
        // flat NF4 indexing exactly as DequantizationKernel: element e of the
        // [N][K] tensor is nibble (e & 1 ? low : high) of byte e >> 1, and
        // uses absmax[(e >> 1) * 2 / group].
        const long long base = static_cast<long long>(l.row) * K;
        for (int k = lane; k < K; k += 32) {
            const long long e = base + k;
            const int byte = sg.w[e >> 1];
            const int code = (e & 1) ? (byte & 15) : (byte >> 4);
            acc = fmaf(nf4_at(code) * sg.absmax[((e >> 1) * 2) / p.group], p.x[k], acc);
        }
    }
    acc = warp_sum(acc);
    if (lane == 0) {
        if (sg.bias) acc += sg.bias[l.row];
        if (sg.residual) acc = sg.residual[l.row] + acc;
        sg.y[l.row] = acc;
    }
}

// ---- dequantisation (bit-exact with the reference) -------------------------
__global__ void dequant_nf4_kernel(float* dst, const uint8_t* src, const float* scales, long long numel, int group) {
    // DequantizationKernel.java:84-102: byte i -> elements 2i (high nibble)
    // and 2i+1 (low nibble), both scaled by scales[(2i) / group].
    const long long nbytes = (numel + 1) / 2;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < nbytes;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int b = src[i];
        const float s = scales[(i * 2) / group];
        dst[2 * i] = __fmul_rn(nf4_at(b >> 4), s);
        if (2 * i + 1 < numel) dst[2 * i + 1] = __fmul_rn(nf4_at(b & 15), s);
    }
}

__global__ void dequant_q4_0_kernel(float* dst, const uint8_t* blocks, long long nblocks) {
    // GgufBlockDequantizer.java:33-37,403-415: ((q & 15) - 8) * d + 0.0f for
    // element j, ((q >> 4) - 8) * d + 0.0f for element j + 16.
    for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < nblocks * 16;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long b = t >> 4;
        const int j = static_cast<int>(t & 15);
        const uint8_t* blk = blocks + b * 18;
        const float d = f16_bits_to_f32(blk[0] | (blk[1] << 8));
        const int q = blk[2 + j];
        dst[b * 32 + j] = __fadd_rn(__fmul_rn(static_cast<float>((q & 15) - 8), d), 0.0f);
        dst[b * 32 + 16 + j] = __fadd_rn(__fmul_rn(static_cast<float>((q >> 4) - 8), d), 0.0f);
    }
}

__global__ void dequant_q8_0_kernel(float* dst, const uint8_t* blocks, long long nblocks) {
    // GgufBlockDequantizer.java:256-265: signedByte * d.
    for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < nblocks * 32;
         t += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long b = t >> 5;
        const int j = static_cast<int>(t & 31);
        const uint8_t* blk = blocks + b * 34;
        const float d = f16_bits_to_f32(blk[0] | (blk[1] << 8));
        dst[t] = __fmul_rn(static_cast<float>(static_cast<int8_t>(blk[2 + j])), d);
    }
}

// ---- host side -----------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        cudaGetLastError();
    });
    return fn;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, size_t row_bytes,
               int rows, int box_inner) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {row_bytes / elem_bytes, static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(kUnitRows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t fixed_smem(int fmt) { return 1024 + (fmt == FMT_NF4 ? kLutBytes : 0) + 64 + 2 * kMaxStages * 8 + 64; }

int stage_size(int fmt, int group) {
    switch (fmt) {
        case FMT_Q4_0: return stage_bytes<FMT_Q4_0, 32>();
        case FMT_Q8_0: return stage_bytes<FMT_Q8_0, 32>();
        default: return group == 64 ? stage_bytes<FMT_NF4, 64>() : stage_bytes<FMT_NF4, 128>();
    }
}

int stages_for(int fmt, int group) {
    const long long avail = kCtaSmemBudget - static_cast<long long>(fixed_smem(fmt));
    const long long s = avail / stage_size(fmt, group);
    return static_cast<int>(std::min<long long>(s, kMaxStages));
}

template <int FMT, int GROUP>
cudaError_t launch_tma(const MatvecParams& mp, cudaStream_t stream, bool pdl) {
    using F = Fmt<FMT>;
    TmaParams p;
    memset(&p, 0, sizeof p);
    p.nseg = mp.nseg;
    p.K = mp.K;
    p.total_rows = mp.total_rows;
    p.epilogue = mp.epilogue;
    p.x = mp.x;
    p.norm_out = mp.norm_out;
    p.norm_w = mp.norm_w;
    p.norm_eps = mp.norm_eps;
    p.norm_partials = mp.norm_partials;
    p.norm_counter = mp.norm_counter;
    const CUtensorMapDataType dt = F::kElemBytes == 8 ? CU_TENSOR_MAP_DATA_TYPE_UINT64 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    int row0 = 0;
    for (int s = 0; s < mp.nseg; ++s) {
        const MatvecSegment& sg = mp.seg[s];
        TmaSegment& ts = p.seg[s];
        if (!encode_2d(&ts.codes, dt, F::kElemBytes, sg.w, F::row_bytes(mp.K), sg.rows, F::kBoxInner))
            return cudaErrorInvalidValue;
        if (FMT == FMT_NF4 && !encode_2d(&ts.absmax, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, sg.absmax,
                                         static_cast<size_t>(mp.K) / GROUP * 4, sg.rows, 1024 / GROUP))
            return cudaErrorInvalidValue;
        ts.bias = sg.bias;
        ts.residual = sg.residual;
        ts.y = sg.y;
        ts.rows = sg.rows;
        ts.row0 = row0;
        row0 += sg.rows;
    }
    const int stages = stages_for(FMT, GROUP);
    const size_t smem = fixed_smem(FMT) + static_cast<size_t>(stages) * stage_bytes<FMT, GROUP>();
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(matvec_tma_kernel<FMT, GROUP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kCtaSmemBudget);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    const int grid = std::max(1, std::min(matvec_max_ctas(), mp.total_rows / kUnitRows));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, matvec_tma_kernel<FMT, GROUP>, p, stages);
}

template <int FMT>
cudaError_t launch_generic(const MatvecParams& p, cudaStream_t stream, bool pdl) {
    const int warps = 8;
    const int grid = (p.total_rows + warps - 1) / warps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(warps * 32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, matvec_generic_kernel<FMT>, p);
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return encode_fn(); }

int matvec_max_ctas() { return 2 * sm_count_for_current_device(); }

bool matvec_tma_supported(int fmt, int K, int group) {
    if (K <= 0 || K % 256 != 0) return false;
    if (fmt == FMT_NF4 && !(group == 64 || (group == 128 && K % 512 == 0))) return false;
    if (stages_for(fmt, fmt == FMT_NF4 ? group : 32) < 2) return false;
    return encode_fn() != nullptr;
}

cudaError_t launch_matvec(int fmt, const MatvecParams& p, cudaStream_t stream, bool pdl) {
    if (p.total_rows <= 0) return cudaSuccess;
    if ((fmt == FMT_Q4_K || fmt == FMT_Q6_K) && matvec_imma_supported(fmt, p.K)) {   // K a multiple of 2048
        const cudaError_t e = launch_matvec_imma(fmt, p, stream, pdl);
        if (e != cudaErrorNotSupported) return e;
    }
    if (fmt == FMT_Q4_K || fmt == FMT_Q6_K) return launch_matvec_k(fmt, p, stream, pdl);
    if (p.norm_defer || p.in_parts) {   // the NF4 table and integer tensor-core kernels split the RMSNorm
        if (fmt == FMT_NF4)
            return matvec_lut_supported(fmt, p.K, p.group) ? launch_matvec_lut(fmt, p, stream, pdl)
                                                           : cudaErrorNotSupported;
        return matvec_imma_supported(fmt, p.K) ? launch_matvec_imma(fmt, p, stream, pdl) : cudaErrorNotSupported;
    }
    if (matvec_imma_supported(fmt, p.K)) {
        const cudaError_t e = launch_matvec_imma(fmt, p, stream, pdl);
        if (e != cudaErrorNotSupported) return e;
    }
    if (matvec_mma_supported(fmt, p.K)) {
        const cudaError_t e = launch_matvec_mma(fmt, p, stream, pdl);
        if (e != cudaErrorNotSupported) return e;
    }
    if (matvec_lut_supported(fmt, p.K, p.group)) {
        const cudaError_t e = launch_matvec_lut(fmt, p, stream, pdl);
        if (e != cudaErrorNotSupported) return e;
    }
    // TMA tensor boxes need 16-byte aligned bases and whole 4-row units per
    // segment; x is read as float4.
    bool ok = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    for (int s = 0; s < p.nseg; ++s) {
        ok = ok && (reinterpret_cast<uintptr_t>(p.seg[s].w) & 15) == 0 && p.seg[s].rows % kUnitRows == 0;
        if (fmt == FMT_NF4) ok = ok && (reinterpret_cast<uintptr_t>(p.seg[s].absmax) & 15) == 0;
    }
    if (p.epilogue == EPI_SWIGLU_PAIR) ok = ok && p.nseg == 2 && p.seg[0].rows == p.seg[1].rows &&
                                              p.total_rows == p.seg[0].rows;
    if (p.norm_out) ok = ok && p.nseg == 1 && p.norm_partials && p.norm_counter && p.norm_w;
    if (ok && matvec_tma_supported(fmt, p.K, p.group)) {
        switch (fmt) {
            case FMT_Q4_0: return launch_tma<FMT_Q4_0, 32>(p, stream, pdl);
            case FMT_Q8_0: return launch_tma<FMT_Q8_0, 32>(p, stream, pdl);
            case FMT_NF4:
                return p.group == 64 ? launch_tma<FMT_NF4, 64>(p, stream, pdl)
                                     : launch_tma<FMT_NF4, 128>(p, stream, pdl);
        }
        return cudaErrorInvalidValue;
    }
    if (p.epilogue != EPI_STORE || p.norm_out) return cudaErrorNotSupported;
    switch (fmt) {
        case FMT_Q4_0: return launch_generic<FMT_Q4_0>(p, stream, pdl);
        case FMT_Q8_0: return launch_generic<FMT_Q8_0>(p, stream, pdl);
        case FMT_NF4: return launch_generic<FMT_NF4>(p, stream, pdl);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_dequant(int fmt, float* dst, const uint8_t* src, const float* absmax, int64_t numel, int group,
                           cudaStream_t stream) {
    if (numel <= 0) return cudaSuccess;
    const int sms = sm_count_for_current_device();
    const int threads = 256;
    long long work = fmt == FMT_NF4 ? (numel + 1) / 2 : fmt == FMT_Q4_0 ? numel / 32 * 16 : numel;
    const int grid =
        static_cast<int>(std::max<long long>(1, std::min<long long>((work + threads - 1) / threads, sms * 16LL)));
    switch (fmt) {
        case FMT_NF4: dequant_nf4_kernel<<<grid, threads, 0, stream>>>(dst, src, absmax, numel, group); break;
        case FMT_Q4_0: dequant_q4_0_kernel<<<grid, threads, 0, stream>>>(dst, src, numel / 32); break;
        case FMT_Q8_0: dequant_q8_0_kernel<<<grid, threads, 0, stream>>>(dst, src, numel / 32); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace alj
