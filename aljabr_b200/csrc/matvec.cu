// Batch-1 dequantise-and-matvec kernels (y = W x) for GGUF Q4_0 / Q8_0 and
// NF4 weights on B200 (sm_100a), plus the bit-exact dequantisation kernels.
//
// Design (HBM-bound streaming, one persistent CTA per SM):
//   * rows are handed out in units of 4; each CTA owns a contiguous,
//     balanced range of units and walks it in tiles of 32 rows x K-chunks;
//   * one producer thread streams each tile's chunk into shared memory with
//     2-D TMA tensor copies (one 4-row box per copy, cp.async.bulk.tensor),
//     completing on an mbarrier, through a multi-stage ring of empty/full
//     barrier pairs; the boxes land densely, row after row;
//   * 16 consumer warps each own 2 rows of the tile; inside a warp the lanes
//     split the chunk's columns, and each lane keeps its column slice of x in
//     registers for both rows, so shared memory carries only the weights;
//     per-row partial sums stay in the lane until the tile's last chunk and
//     are then reduced with 5 shuffles -- no cross-warp reduction;
//   * 4-bit / 8-bit GGUF codes become exact floats with one LOP3 each (the
//     code placed in the mantissa of 2^23) and one packed f32x2 add per two
//     codes; products accumulate with packed f32x2 FMA;
//   * NF4 bytes index a 256-entry table of value pairs (T[hi], T[lo]),
//     replicated per lane in shared memory (entry b of lane l at
//     8 * (32 b + l)): one conflict-free LDS.64 yields both weights of a byte
//     as an f32x2 operand;
//   * block scales (fp16 d for GGUF, fp32 absmax for NF4) are applied once
//     per block to the block's partial sum.
// Shapes the TMA path cannot stage (K not a multiple of 256, segment rows
// not a multiple of 4, unaligned pointers, other NF4 groups) run a plain
// one-warp-per-row kernel instead.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
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

constexpr int kConsumerWarps = 16;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kUnitRows = 4;                      // rows per TMA box
constexpr int kTileUnits = 8;
constexpr int kTileRows = kUnitRows * kTileUnits; // 32 = 16 warps x 2 rows
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;                // 227 KB opt-in per CTA on sm_100
constexpr int kLutBytes = 256 * 32 * 8;           // NF4 byte-pair table, per lane

template <int FMT>
struct Fmt;
template <>
struct Fmt<FMT_Q4_0> {
    static constexpr int kChunkElems = 2048;     // 64 blocks: 2 per lane
    static constexpr int kChunkBytes = 1152;     // per row
    static constexpr int kLaneF4 = 16;           // x float4s per lane
    static constexpr int kBoxInner = 144;        // in UINT64 elements
    static constexpr int kElemBytes = 8;
    static size_t row_bytes(int K) { return static_cast<size_t>(K) / 32 * 18; }
};
template <>
struct Fmt<FMT_Q8_0> {
    static constexpr int kChunkElems = 1024;     // 32 blocks: 1 per lane
    static constexpr int kChunkBytes = 1088;
    static constexpr int kLaneF4 = 8;
    static constexpr int kBoxInner = 136;
    static constexpr int kElemBytes = 8;
    static size_t row_bytes(int K) { return static_cast<size_t>(K) / 32 * 34; }
};
template <>
struct Fmt<FMT_NF4> {
    static constexpr int kChunkElems = 1024;     // 32 codes (16 bytes) per lane
    static constexpr int kChunkBytes = 512;
    static constexpr int kLaneF4 = 8;
    static constexpr int kBoxInner = 128;        // in UINT32 elements
    static constexpr int kElemBytes = 4;
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
    int prologue;
    float norm_eps;
    const float* x;
    const float* norm_w;
    const float* gate;
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
// Q4_0: this lane's two blocks (36 B at 36*lane: word-aligned, conflict-free
// since 9 is odd).  Block A's fp16 d is word-aligned and its codes 2 bytes
// off; block B the reverse.  x holds per block eight float4s in the order
// (x_j, x_{j+16}, x_{j+1}, x_{j+17}), (x_{j+2}, x_{j+18}, x_{j+3}, x_{j+19}),
// j = 4i, matching ggml's nibble order (low nibble of byte j = element j,
// high nibble = element j + 16).
__device__ __forceinline__ float q4_0_block(uint32_t dbits, const uint32_t (&c)[4], const float4* xb) {
    const f2 k01 = mk2(-(kTwo23 + 8.0f), -(kTwo23 + 128.0f));
    const f2 k23 = mk2(-(kTwo23 + 2048.0f), -(kTwo23 + 32768.0f));
    const f2 fold = mk2(1.0f / 256.0f, 1.0f / 256.0f);   // a23's 256x / 4096x units onto a01's 1x / 16x
    f2 a01 = mk2(0.0f, 0.0f), a23 = mk2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 xa = xb[2 * i], xc = xb[2 * i + 1];
        const uint32_t w = c[i], w2 = w >> 16;
        const f2 p0 = add2(mk2u((w & 0xFu) | kMagic, (w & 0xF0u) | kMagic), k01);
        const f2 p1 = add2(mk2u((w & 0xF00u) | kMagic, (w & 0xF000u) | kMagic), k23);
        const f2 p2 = add2(mk2u((w2 & 0xFu) | kMagic, (w2 & 0xF0u) | kMagic), k01);
        const f2 p3 = add2(mk2u((w2 & 0xF00u) | kMagic, (w2 & 0xF000u) | kMagic), k23);
        a01 = fma2(p0, mk2(xa.x, xa.y), a01);
        a23 = fma2(p1, mk2(xa.z, xa.w), a23);
        a01 = fma2(p2, mk2(xc.x, xc.y), a01);
        a23 = fma2(p3, mk2(xc.z, xc.w), a23);
    }
    const f2 t = fma2(a23, fold, a01);
    const float bs = fmaf(hi(t), 0.0625f, lo(t));
    return __half2float(__ushort_as_half(static_cast<unsigned short>(dbits))) * bs;
}

__device__ __forceinline__ float q4_0_row(uint32_t row_addr, int lane, const float4* x) {
    uint32_t W[9];
    const uint32_t a = row_addr + lane * 36;
#pragma unroll
    for (int k = 0; k < 9; ++k) W[k] = lds_u32(a + 4 * k);
    uint32_t cA[4], cB[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        cA[i] = __funnelshift_r(W[i], W[i + 1], 16);
        cB[i] = W[5 + i];
    }
    return q4_0_block(W[0] & 0xFFFFu, cA, x) + q4_0_block(W[4] >> 16, cB, x + 8);
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
// 16*lane.  lut_lane = shared address of this lane's column of the table.
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
        // __byte_perm(w, 0, 0x44b4) moves byte b to bits 8..15 = 256 * byte
        const float2 t0 = lds_f2(lut_lane + __byte_perm(w[k], 0, 0x4404));
        const float2 t1 = lds_f2(lut_lane + __byte_perm(w[k], 0, 0x4414));
        const float2 t2 = lds_f2(lut_lane + __byte_perm(w[k], 0, 0x4424));
        const float2 t3 = lds_f2(lut_lane + __byte_perm(w[k], 0, 0x4434));
        const float4 x0 = x[2 * k], x1 = x[2 * k + 1];
        A = fma2(mk2(t0.x, t0.y), mk2(x0.x, x0.y), A);
        B = fma2(mk2(t1.x, t1.y), mk2(x0.z, x0.w), B);
        A = fma2(mk2(t2.x, t2.y), mk2(x1.x, x1.y), A);
        B = fma2(mk2(t3.x, t3.y), mk2(x1.z, x1.w), B);
    }
    const f2 t = add2(A, B);
    return am * (lo(t) + hi(t));
}

// ---- x staging --------------------------------------------------------------
// Destination layout: per chunk, per lane float4 slot j, per lane:
// xs4[(chunk * kLaneF4 + j) * 32 + lane], so that a warp's load of slot j is
// 32 consecutive float4s (conflict-free).  Elements past K are zero.
template <int FMT>
__device__ __forceinline__ int x_source(int q, int comp) {
    using F = Fmt<FMT>;
    constexpr int per_chunk = F::kLaneF4 * 32;
    const int chunk = q / per_chunk;
    const int rem = q - chunk * per_chunk;
    const int j = rem >> 5, ln = rem & 31;
    if (FMT == FMT_Q4_0) {
        const int bb = j >> 3, f = j & 7;
        const int base = chunk * F::kChunkElems + (ln * 2 + bb) * 32 + 4 * (f >> 1) + 2 * (f & 1);
        return base + (comp >> 1) + 16 * (comp & 1);   // (x_j, x_{j+16}, x_{j+1}, x_{j+17})
    }
    return chunk * F::kChunkElems + ln * 32 + 4 * j + comp;
}

template <int FMT>
__device__ void stage_x(const TmaParams& p, float4* xs4, float* red, int Kp) {
    const int tid = threadIdx.x;
    const int K = p.K;
    float scale = 1.0f;
    if (p.prologue == PRO_RMSNORM) {
        float ss = 0.0f;
        for (int i = tid * 4; i < K; i += kConsumerThreads * 4) {
            const float4 v = *reinterpret_cast<const float4*>(p.x + i);
            ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
        }
        ss = warp_sum(ss);
        if ((tid & 31) == 0) red[tid >> 5] = ss;
        named_bar(1, kConsumerThreads);
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
        scale = 1.0f / sqrtf(tot / static_cast<float>(K) + p.norm_eps);
    }
    for (int q = tid; q < Kp / 4; q += kConsumerThreads) {
        float v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int e = x_source<FMT>(q, c);
            float a = 0.0f;
            if (e < K) {
                a = p.x[e];
                if (p.prologue == PRO_RMSNORM) {
                    a = a * scale * p.norm_w[e];
                } else if (p.prologue == PRO_SWIGLU) {
                    const float g = p.gate[e];
                    a = g / (1.0f + expf(-g)) * a;
                }
            }
            v[c] = a;
        }
        xs4[q] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

__device__ __forceinline__ void locate_row(const TmaParams& p, int row, int& seg, int& lrow) {
    seg = 0;
    if (p.nseg > 1 && row >= p.seg[1].row0) seg = 1;
    if (p.nseg > 2 && row >= p.seg[2].row0) seg = 2;
    lrow = row - p.seg[seg].row0;
}

template <int FMT, int GROUP>
constexpr int stage_bytes() {
    return ((kTileRows * Fmt<FMT>::kChunkBytes + (FMT == FMT_NF4 ? kTileRows * (1024 / GROUP) * 4 : 0)) + 1023) &
           ~1023;
}

template <int FMT, int GROUP>
__global__ void __launch_bounds__(kThreads, 1) matvec_tma_kernel(const __grid_constant__ TmaParams p, int stages) {
    using F = Fmt<FMT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    pdl_launch_dependents();

    const int K = p.K;
    const int nchunks = (K + F::kChunkElems - 1) / F::kChunkElems;
    const int Kp = nchunks * F::kChunkElems;
    constexpr int kStage = stage_bytes<FMT, GROUP>();
    constexpr int kAbsPerRow = 1024 / GROUP;                 // NF4 absmax floats per row-chunk
    constexpr int kCodeTile = kTileRows * F::kChunkBytes;    // codes region of a stage

    const uint32_t base = smem_u32(smem_raw);
    const uint32_t pad = (1024u - (base & 1023u)) & 1023u;
    uint8_t* sp = smem_raw + pad;
    uint8_t* stage0 = sp;
    sp += static_cast<size_t>(stages) * kStage;
    float4* xs4 = reinterpret_cast<float4*>(sp);
    sp += static_cast<size_t>(Kp) * 4;
    uint32_t lut_lane = 0;
    if (FMT == FMT_NF4) {
        float2* lut = reinterpret_cast<float2*>(sp);
        for (int i = threadIdx.x; i < 256 * 32; i += kThreads) {
            const int b = i >> 5;
            lut[i] = make_float2(nf4_at(b >> 4), nf4_at(b & 15));
        }
        lut_lane = smem_u32(lut) + (threadIdx.x & 31) * 8;
        sp += kLutBytes;
    }
    float* red = reinterpret_cast<float*>(sp);
    sp += kConsumerWarps * 4;
    uint64_t* full = reinterpret_cast<uint64_t*>(sp);
    uint64_t* empty = full + kMaxStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMaxStages);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = p.total_rows / kUnitRows;
    const int u_begin = static_cast<int>(static_cast<long long>(units) * blockIdx.x / gridDim.x);
    const int u_end = static_cast<int>(static_cast<long long>(units) * (blockIdx.x + 1) / gridDim.x);
    const int ntiles = (u_end - u_begin + kTileUnits - 1) / kTileUnits;
    const int items = ntiles * nchunks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            for (int it = 0; it < items; ++it) {
                const int t = it / nchunks, c = it - t * nchunks;
                const int s = it % stages;
                const uint32_t round = static_cast<uint32_t>(it / stages);
                const int tu0 = u_begin + t * kTileUnits;
                const int nunits = min(kTileUnits, u_end - tu0);
                if (*abort_flag || !mbar_wait(&empty[s], (round & 1u) ^ 1u)) {
                    *abort_flag = 1;
                    break;
                }
                const uint32_t per_unit = kUnitRows * (F::kChunkBytes + (FMT == FMT_NF4 ? kAbsPerRow * 4 : 0));
                mbar_arrive_expect_tx(&full[s], per_unit * nunits);
                uint8_t* st = stage0 + static_cast<size_t>(s) * kStage;
                for (int u = 0; u < nunits; ++u) {
                    int seg, lrow;
                    locate_row(p, (tu0 + u) * kUnitRows, seg, lrow);
                    tma_load_2d(smem_u32(st + u * kUnitRows * F::kChunkBytes), &p.seg[seg].codes, c * F::kBoxInner,
                                lrow, &full[s]);
                    if (FMT == FMT_NF4)
                        tma_load_2d(smem_u32(st + kCodeTile + u * kUnitRows * kAbsPerRow * 4), &p.seg[seg].absmax,
                                    c * kAbsPerRow, lrow, &full[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        pdl_wait();
        stage_x<FMT>(p, xs4, red, Kp);
        named_bar(1, kConsumerThreads);
        float acc0 = 0.0f, acc1 = 0.0f;
        const int r0 = warp, r1 = warp + kConsumerWarps;
        for (int it = 0; it < items; ++it) {
            const int t = it / nchunks, c = it - t * nchunks;
            const int s = it % stages;
            const uint32_t round = static_cast<uint32_t>(it / stages);
            const int tu0 = u_begin + t * kTileUnits;
            const int trows = min(kTileUnits, u_end - tu0) * kUnitRows;
            const bool ok = (*abort_flag == 0) && mbar_wait(&full[s], round & 1u);
            if (!ok) *abort_flag = 1;
            if (ok && r0 < trows) {
                float4 xr[F::kLaneF4];
#pragma unroll
                for (int j = 0; j < F::kLaneF4; ++j) xr[j] = xs4[(c * F::kLaneF4 + j) * 32 + lane];
                const uint32_t st = smem_u32(stage0 + static_cast<size_t>(s) * kStage);
                if (FMT == FMT_Q4_0) {
                    acc0 += q4_0_row(st + r0 * F::kChunkBytes, lane, xr);
                    if (r1 < trows) acc1 += q4_0_row(st + r1 * F::kChunkBytes, lane, xr);
                } else if (FMT == FMT_Q8_0) {
                    acc0 += q8_0_row(st + r0 * F::kChunkBytes, lane, xr);
                    if (r1 < trows) acc1 += q8_0_row(st + r1 * F::kChunkBytes, lane, xr);
                } else {
                    const float* am =
                        reinterpret_cast<const float*>(stage0 + static_cast<size_t>(s) * kStage + kCodeTile);
                    const int g = (lane * 32) / GROUP;
                    acc0 += nf4_row(st + r0 * F::kChunkBytes, am[r0 * kAbsPerRow + g], lane * 16, lut_lane, xr);
                    if (r1 < trows)
                        acc1 += nf4_row(st + r1 * F::kChunkBytes, am[r1 * kAbsPerRow + g], lane * 16, lut_lane, xr);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (c == nchunks - 1) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int r = h ? r1 : r0;
                    if (r < trows) {
                        const float v = warp_sum(h ? acc1 : acc0);
                        if (lane == 0 && *abort_flag == 0) {
                            int seg, lrow;
                            locate_row(p, tu0 * kUnitRows + r, seg, lrow);
                            const TmaSegment& sg = p.seg[seg];
                            float out = v;
                            if (sg.bias) out += sg.bias[lrow];
                            if (sg.residual) out = sg.residual[lrow] + out;
                            sg.y[lrow] = out;
                        }
                    }
                }
                acc0 = acc1 = 0.0f;
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

size_t fixed_smem(int fmt, int K) {
    const int chunk = fmt == FMT_Q4_0 ? Fmt<FMT_Q4_0>::kChunkElems : 1024;
    const size_t Kp = (static_cast<size_t>(K) + chunk - 1) / chunk * chunk;
    return 1024 + Kp * 4 + (fmt == FMT_NF4 ? kLutBytes : 0) + kConsumerWarps * 4 + 2 * kMaxStages * 8 + 64;
}

int stage_size(int fmt, int group) {
    switch (fmt) {
        case FMT_Q4_0: return stage_bytes<FMT_Q4_0, 32>();
        case FMT_Q8_0: return stage_bytes<FMT_Q8_0, 32>();
        default: return group == 64 ? stage_bytes<FMT_NF4, 64>() : stage_bytes<FMT_NF4, 128>();
    }
}

int stages_for(int fmt, int K, int group) {
    const long long avail = kSmemLimit - static_cast<long long>(fixed_smem(fmt, K));
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
    p.prologue = mp.prologue;
    p.norm_eps = mp.norm_eps;
    p.x = mp.x;
    p.norm_w = mp.norm_w;
    p.gate = mp.gate;
    const CUtensorMapDataType dt = F::kElemBytes == 8 ? CU_TENSOR_MAP_DATA_TYPE_UINT64 : CU_TENSOR_MAP_DATA_TYPE_UINT32;
    int row0 = 0;
    for (int s = 0; s < mp.nseg; ++s) {
        const MatvecSegment& sg = mp.seg[s];
        TmaSegment& ts = p.seg[s];
        if (!encode_2d(&ts.codes, dt, F::kElemBytes, sg.w, F::row_bytes(mp.K), sg.rows, F::kBoxInner))
            return cudaErrorInvalidValue;
        if (FMT == FMT_NF4 &&
            !encode_2d(&ts.absmax, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, sg.absmax,
                       static_cast<size_t>(mp.K) / GROUP * 4, sg.rows, 1024 / GROUP))
            return cudaErrorInvalidValue;
        ts.bias = sg.bias;
        ts.residual = sg.residual;
        ts.y = sg.y;
        ts.rows = sg.rows;
        ts.row0 = row0;
        row0 += sg.rows;
    }
    const int stages = stages_for(FMT, mp.K, GROUP);
    const size_t smem = fixed_smem(FMT, mp.K) + static_cast<size_t>(stages) * stage_bytes<FMT, GROUP>();
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(matvec_tma_kernel<FMT, GROUP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    const int sms = sm_count_for_current_device();
    const int grid = std::max(1, std::min(sms, mp.total_rows / kUnitRows));
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

bool matvec_tma_supported(int fmt, int K, int group) {
    if (K <= 0 || K % 256 != 0) return false;
    if (fmt == FMT_NF4 && !(group == 64 || (group == 128 && K % 512 == 0))) return false;
    if (stages_for(fmt, K, fmt == FMT_NF4 ? group : 32) < 2) return false;
    return encode_fn() != nullptr;
}

cudaError_t launch_matvec(int fmt, const MatvecParams& p, cudaStream_t stream, bool pdl) {
    if (p.total_rows <= 0) return cudaSuccess;
    // TMA tensor boxes need 16-byte aligned bases and whole 4-row units per
    // segment; the x prologue reads float4.
    bool ok = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    for (int s = 0; s < p.nseg; ++s) {
        ok = ok && (reinterpret_cast<uintptr_t>(p.seg[s].w) & 15) == 0 && p.seg[s].rows % kUnitRows == 0;
        if (fmt == FMT_NF4) ok = ok && (reinterpret_cast<uintptr_t>(p.seg[s].absmax) & 15) == 0;
    }
    if (p.prologue == PRO_RMSNORM) ok = ok && (reinterpret_cast<uintptr_t>(p.norm_w) & 15) == 0;
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
    if (p.prologue != PRO_NONE) return cudaErrorNotSupported;
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
