// Batch-1 dequantise-and-matvec kernels (y = W x) for GGUF Q4_0 / Q8_0 and
// NF4 weights on B200 (sm_100a), plus the bit-exact dequantisation kernels.
//
// Design (HBM-bound streaming, one persistent CTA per SM):
//   * each CTA owns a contiguous range of output rows (balanced to +-1 row)
//     and walks it in tiles of up to 32 rows x K-chunks;
//   * a producer warp streams every row's chunk into shared memory with
//     untiled TMA bulk copies (cp.async.bulk) completing on an mbarrier,
//     through a multi-stage ring (empty/full barrier pairs);
//   * 8 consumer warps split the chunk's columns; inside a warp, lane = row,
//     so the activation x is a shared-memory broadcast and each lane keeps
//     its own row's partial sum -- no shuffle reduction on the hot path;
//   * 4-bit / 8-bit codes become exact floats with one LOP3 each (the code
//     placed in the mantissa of 2^23 = 0x4B000000) and one packed f32x2 add
//     per two codes; products accumulate with packed f32x2 FMA;
//   * NF4 codes index a 16-entry codebook replicated once per lane in
//     shared memory (entry v of lane l at word 32 v + l: conflict-free);
//   * per-block scales (fp16 d for GGUF, fp32 absmax for NF4) are applied
//     once per block to the block's partial sum.
// Shapes the TMA path cannot stage (K not a multiple of 256, odd NF4 group
// layouts) run a plain one-warp-per-row kernel instead.
#include "common.cuh"

#include <algorithm>

namespace alj {

__device__ unsigned int g_fault_word = 0;

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kTileRows = 32;
constexpr int kMaxStages = 8;
constexpr int kSmemLimit = 232448;   // 227 KB opt-in per CTA on sm_100

template <int FMT>
struct Layout;
template <>
struct Layout<FMT_Q4_0> {
    static constexpr int kWarpElems = 256;                          // 8 blocks of 32
    static constexpr int kChunkElems = kWarpElems * kConsumerWarps; // 2048
    static constexpr int kSlot = 1168;                              // 1152 B codes, 73 x 16
    static constexpr int code_bytes(int elems) { return elems / 32 * 18; }
};
template <>
struct Layout<FMT_Q8_0> {
    static constexpr int kWarpElems = 256;
    static constexpr int kChunkElems = kWarpElems * kConsumerWarps;
    static constexpr int kSlot = 2192;                              // 2176 B codes, 137 x 16
    static constexpr int code_bytes(int elems) { return elems / 32 * 34; }
};
template <>
struct Layout<FMT_NF4> {
    static constexpr int kWarpElems = 128;
    static constexpr int kChunkElems = kWarpElems * kConsumerWarps; // 1024
    static constexpr int kSlot = 592;                               // 512 B codes + 64 B absmax, 37 x 16
    static constexpr int kAbsmaxOff = 512;
    static constexpr int code_bytes(int elems) { return elems / 2; }
};

// Exact magic constants: float(0x4B000000 | (c << s)) = 2^23 + c * 2^s.
constexpr uint32_t kMagic = 0x4B000000u;
constexpr float kTwo23 = 8388608.0f;

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// ---- Q4_0: 8 consecutive blocks (144 B = 9 x 16 B) of one row -------------
// Block u starts at byte 18u; for even u its fp16 d is word-aligned and its
// codes sit 2 bytes off word alignment, for odd u the reverse.  x is stored
// pair-permuted per block: xs[2j] = x_j, xs[2j+1] = x_{j+16}, matching the
// ggml nibble order (low nibble of byte j = element j, high = element j+16).
__device__ __forceinline__ float q4_0_group(const uint8_t* src, const float* xg) {
    uint32_t W[36];
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        uint4 v = s4[i];
        W[4 * i] = v.x; W[4 * i + 1] = v.y; W[4 * i + 2] = v.z; W[4 * i + 3] = v.w;
    }
    const f2 k01 = mk2(-(kTwo23 + 8.0f), -(kTwo23 + 128.0f));
    const f2 k23 = mk2(-(kTwo23 + 2048.0f), -(kTwo23 + 32768.0f));
    // a23 holds 256x / 4096x partials; scaled by 1/256 they line up with a01's 1x / 16x units
    const f2 fold = mk2(1.0f / 256.0f, 1.0f / 256.0f);
    float acc = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        uint32_t dbits, c[4];
        if ((u & 1) == 0) {
            const int a = 9 * u / 2;
            dbits = W[a] & 0xFFFFu;
#pragma unroll
            for (int i = 0; i < 4; ++i) c[i] = __funnelshift_r(W[a + i], W[a + i + 1], 16);
        } else {
            const int a = (9 * u - 1) / 2;
            dbits = W[a] >> 16;
#pragma unroll
            for (int i = 0; i < 4; ++i) c[i] = W[a + 1 + i];
        }
        const float4* xb = reinterpret_cast<const float4*>(xg + 32 * u);
        f2 a01 = mk2(0.0f, 0.0f), a23 = mk2(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 xa = xb[2 * i], xc = xb[2 * i + 1];
            const uint32_t w = c[i], w2 = w >> 16;
            const f2 p0 = add2(mk2u((w & 0xFu) | kMagic, (w & 0xF0u) | kMagic), k01);      // (q-8, 16(q-8))
            const f2 p1 = add2(mk2u((w & 0xF00u) | kMagic, (w & 0xF000u) | kMagic), k23);  // (256(q-8), 4096(q-8))
            const f2 p2 = add2(mk2u((w2 & 0xFu) | kMagic, (w2 & 0xF0u) | kMagic), k01);
            const f2 p3 = add2(mk2u((w2 & 0xF00u) | kMagic, (w2 & 0xF000u) | kMagic), k23);
            a01 = fma2(p0, mk2(xa.x, xa.y), a01);
            a23 = fma2(p1, mk2(xa.z, xa.w), a23);
            a01 = fma2(p2, mk2(xc.x, xc.y), a01);
            a23 = fma2(p3, mk2(xc.z, xc.w), a23);
        }
        const f2 t = fma2(a23, fold, a01);               // (1x sums, 16x sums)
        const float bs = fmaf(hi(t), 0.0625f, lo(t));
        acc = fmaf(__half2float(__ushort_as_half(static_cast<unsigned short>(dbits))), bs, acc);
    }
    return acc;
}

// ---- Q8_0: 8 consecutive blocks (272 B = 17 x 16 B) of one row -------------
__device__ __forceinline__ float q8_0_group(const uint8_t* src, const float* xg) {
    uint32_t W[68];
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 17; ++i) {
        uint4 v = s4[i];
        W[4 * i] = v.x; W[4 * i + 1] = v.y; W[4 * i + 2] = v.z; W[4 * i + 3] = v.w;
    }
    const f2 kq = mk2(-(kTwo23 + 128.0f), -(kTwo23 + 32768.0f));
    float acc = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        uint32_t dbits, c[8];
        if ((u & 1) == 0) {
            const int a = 17 * u / 2;
            dbits = W[a] & 0xFFFFu;
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = __funnelshift_r(W[a + i], W[a + i + 1], 16);
        } else {
            const int a = (17 * u - 1) / 2;
            dbits = W[a] >> 16;
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i] = W[a + 1 + i];
        }
        const float4* xb = reinterpret_cast<const float4*>(xg + 32 * u);
        f2 A = mk2(0.0f, 0.0f), B = mk2(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 xv = xb[i];
            const uint32_t w = c[i], w2 = w >> 16;
            // signed byte b -> 2^23 + (b + 128) via xor of bit 7 into the magic
            const f2 p = add2(mk2u((w & 0xFFu) ^ 0x4B000080u, (w & 0xFF00u) ^ 0x4B008000u), kq);   // (b0, 256 b1)
            const f2 q = add2(mk2u((w2 & 0xFFu) ^ 0x4B000080u, (w2 & 0xFF00u) ^ 0x4B008000u), kq); // (b2, 256 b3)
            if (i & 1) {
                B = fma2(p, mk2(xv.x, xv.y), B);
                B = fma2(q, mk2(xv.z, xv.w), B);
            } else {
                A = fma2(p, mk2(xv.x, xv.y), A);
                A = fma2(q, mk2(xv.z, xv.w), A);
            }
        }
        const f2 t = add2(A, B);
        const float bs = fmaf(hi(t), 1.0f / 256.0f, lo(t));
        acc = fmaf(__half2float(__ushort_as_half(static_cast<unsigned short>(dbits))), bs, acc);
    }
    return acc;
}

// ---- NF4: 128 consecutive elements (64 B codes) of one row ----------------
// Byte b of a 32-bit code word holds element 2b in its high nibble and
// element 2b+1 in its low nibble.  lut_lane = shared address of this
// lane's column of the replicated codebook (bits 7..10 clear).
template <int GROUP>
__device__ __forceinline__ float nf4_group(const uint8_t* src, const float* absmax_s, const float* xg,
                                           uint32_t lut_lane) {
    uint32_t W[16];
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint4 v = s4[i];
        W[4 * i] = v.x; W[4 * i + 1] = v.y; W[4 * i + 2] = v.z; W[4 * i + 3] = v.w;
    }
    constexpr int kGroups = 128 / GROUP;
    constexpr int kWordsPerGroup = GROUP / 8;
    float acc = 0.0f;
#pragma unroll
    for (int g = 0; g < kGroups; ++g) {
        f2 A = mk2(0.0f, 0.0f), B = mk2(0.0f, 0.0f);
#pragma unroll
        for (int k = g * kWordsPerGroup; k < (g + 1) * kWordsPerGroup; ++k) {
            const uint32_t w = W[k];
            const float4 x0 = reinterpret_cast<const float4*>(xg)[2 * k];
            const float4 x1 = reinterpret_cast<const float4*>(xg)[2 * k + 1];
            const float t0h = lds_f32(((w << 3) & 0x780u) | lut_lane);
            const float t0l = lds_f32(((w << 7) & 0x780u) | lut_lane);
            const float t1h = lds_f32(((w >> 5) & 0x780u) | lut_lane);
            const float t1l = lds_f32(((w >> 1) & 0x780u) | lut_lane);
            const float t2h = lds_f32(((w >> 13) & 0x780u) | lut_lane);
            const float t2l = lds_f32(((w >> 9) & 0x780u) | lut_lane);
            const float t3h = lds_f32(((w >> 21) & 0x780u) | lut_lane);
            const float t3l = lds_f32(((w >> 17) & 0x780u) | lut_lane);
            A = fma2(mk2(t0h, t0l), mk2(x0.x, x0.y), A);
            B = fma2(mk2(t1h, t1l), mk2(x0.z, x0.w), B);
            A = fma2(mk2(t2h, t2l), mk2(x1.x, x1.y), A);
            B = fma2(mk2(t3h, t3l), mk2(x1.z, x1.w), B);
        }
        const f2 t = add2(A, B);
        acc = fmaf(absmax_s[g], lo(t) + hi(t), acc);
    }
    return acc;
}

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

// Load x into shared memory (layout per format), applying the fused prologue.
template <int FMT>
__device__ void load_x(const MatvecParams& p, float* xs, float* red) {
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
        named_bar(1, kConsumerThreads);   // red is reused below by the tile reductions
    }
    for (int i = tid * 4; i < K; i += kConsumerThreads * 4) {
        float4 v = *reinterpret_cast<const float4*>(p.x + i);
        if (p.prologue == PRO_RMSNORM) {
            const float4 w = *reinterpret_cast<const float4*>(p.norm_w + i);
            v.x = v.x * scale * w.x; v.y = v.y * scale * w.y; v.z = v.z * scale * w.z; v.w = v.w * scale * w.w;
        } else if (p.prologue == PRO_SWIGLU) {
            const float4 g = *reinterpret_cast<const float4*>(p.gate + i);
            v.x = g.x / (1.0f + expf(-g.x)) * v.x; v.y = g.y / (1.0f + expf(-g.y)) * v.y;
            v.z = g.z / (1.0f + expf(-g.z)) * v.z; v.w = g.w / (1.0f + expf(-g.w)) * v.w;
        }
        if (FMT == FMT_Q4_0) {
            const int b = i & ~31, j = i & 31;   // 4 consecutive elements stay in one half-block
            const int base = b + (j < 16 ? 2 * j : 2 * (j - 16) + 1);
            xs[base] = v.x; xs[base + 2] = v.y; xs[base + 4] = v.z; xs[base + 6] = v.w;
        } else {
            *reinterpret_cast<float4*>(xs + i) = v;
        }
    }
}

template <int FMT, int GROUP>
__global__ void __launch_bounds__(kThreads, 1) matvec_tma_kernel(const MatvecParams p, int stages) {
    using L = Layout<FMT>;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    pdl_launch_dependents();

    const int K = p.K;
    uint8_t* sp = smem_raw;
    uint32_t lut_lane = 0;
    if (FMT == FMT_NF4) {
        const uint32_t pad = (2048u - (smem_u32(sp) & 2047u)) & 2047u;
        float* lut = reinterpret_cast<float*>(sp + pad);
        for (int i = threadIdx.x; i < 512; i += kThreads) lut[i] = nf4_value(i >> 5);
        lut_lane = smem_u32(lut) + (threadIdx.x & 31) * 4;
        sp += pad + 2048;
    }
    float* xs = reinterpret_cast<float*>(sp);
    sp += static_cast<size_t>(K) * 4;
    float* red = reinterpret_cast<float*>(sp);
    sp += 2 * kConsumerThreads * 4;
    uint64_t* full = reinterpret_cast<uint64_t*>(sp);
    uint64_t* empty = full + kMaxStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kMaxStages);
    sp += 2 * kMaxStages * 8 + 128;
    uint8_t* stage0 = sp;
    const int stage_bytes = kTileRows * L::kSlot;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int N = p.total_rows;
    const int r_begin = static_cast<int>(static_cast<long long>(N) * blockIdx.x / gridDim.x);
    const int r_end = static_cast<int>(static_cast<long long>(N) * (blockIdx.x + 1) / gridDim.x);
    const int rows = r_end - r_begin;
    const int ntiles = (rows + kTileRows - 1) / kTileRows;
    const int nchunks = (K + L::kChunkElems - 1) / L::kChunkElems;
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
        for (int it = 0; it < items; ++it) {
            const int t = it / nchunks, c = it - t * nchunks;
            const int s = it % stages;
            const uint32_t round = static_cast<uint32_t>(it / stages);
            const int t0 = r_begin + rows * t / ntiles, t1 = r_begin + rows * (t + 1) / ntiles;
            const int trows = t1 - t0;
            const int e0 = c * L::kChunkElems;
            const int ce = min(L::kChunkElems, K - e0);
            const uint32_t cbytes = L::code_bytes(ce);
            const uint32_t abytes = (FMT == FMT_NF4) ? static_cast<uint32_t>(ce / GROUP) * 4u : 0u;
            int ok = 1;
            if (lane == 0) {
                ok = (*abort_flag == 0) && mbar_wait(&empty[s], (round & 1u) ^ 1u);
                if (!ok) *abort_flag = 1;
                else mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(trows) * (cbytes + abytes));
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            if (lane < trows) {
                const RowLoc l = locate(p, t0 + lane);
                const MatvecSegment& sg = p.seg[l.seg];
                uint8_t* dst = stage0 + s * stage_bytes + lane * L::kSlot;
                const uint8_t* src = sg.w + static_cast<size_t>(l.row) * L::code_bytes(K) + L::code_bytes(e0);
                bulk_g2s(dst, src, cbytes, &full[s]);
                if (FMT == FMT_NF4) {
                    const float* asrc = sg.absmax + static_cast<size_t>(l.row) * (K / GROUP) + e0 / GROUP;
                    bulk_g2s(dst + Layout<FMT_NF4>::kAbsmaxOff, asrc, abytes, &full[s]);
                }
            }
        }
    } else {
        // ------------------------------------------------------------ consumers
        pdl_wait();
        load_x<FMT>(p, xs, red);
        named_bar(1, kConsumerThreads);
        float acc = 0.0f;
        for (int it = 0; it < items; ++it) {
            const int t = it / nchunks, c = it - t * nchunks;
            const int s = it % stages;
            const uint32_t round = static_cast<uint32_t>(it / stages);
            const int e0 = c * L::kChunkElems;
            const int ce = min(L::kChunkElems, K - e0);
            bool ok = (*abort_flag == 0) && mbar_wait(&full[s], round & 1u);
            if (!ok) *abort_flag = 1;
            const int we = warp * L::kWarpElems;
            if (ok && we < ce) {
                const uint8_t* slot = stage0 + s * stage_bytes + lane * L::kSlot;
                if (FMT == FMT_Q4_0) {
                    acc += q4_0_group(slot + we / 32 * 18, xs + e0 + we);
                } else if (FMT == FMT_Q8_0) {
                    acc += q8_0_group(slot + we / 32 * 34, xs + e0 + we);
                } else {
                    acc += nf4_group<GROUP>(slot + we / 2,
                                            reinterpret_cast<const float*>(slot + Layout<FMT_NF4>::kAbsmaxOff) +
                                                we / GROUP,
                                            xs + e0 + we, lut_lane);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (c == nchunks - 1) {
                float* rb = red + (t & 1) * kConsumerThreads;
                rb[warp * 32 + lane] = acc;
                acc = 0.0f;
                named_bar(1, kConsumerThreads);
                const int t0 = r_begin + rows * t / ntiles, t1 = r_begin + rows * (t + 1) / ntiles;
                if (warp == 0 && lane < t1 - t0 && *abort_flag == 0) {
                    float sum = 0.0f;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; ++w) sum += rb[w * 32 + lane];
                    const RowLoc l = locate(p, t0 + lane);
                    const MatvecSegment& sg = p.seg[l.seg];
                    if (sg.bias) sum += sg.bias[l.row];
                    if (sg.residual) sum = sg.residual[l.row] + sum;
                    sg.y[l.row] = sum;
                }
            }
        }
    }
}

// ---- generic fallback: one warp per row, any K that the format allows -----
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
                for (int j = 0; j < 32; ++j) s = fmaf(static_cast<float>(static_cast<int8_t>(blk[2 + j])), p.x[b * 32 + j], s);
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
            acc = fmaf(nf4_value(code) * sg.absmax[((e >> 1) * 2) / p.group], p.x[k], acc);
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
        dst[2 * i] = __fmul_rn(nf4_value(b >> 4), s);
        if (2 * i + 1 < numel) dst[2 * i + 1] = __fmul_rn(nf4_value(b & 15), s);
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

template <typename Kern>
cudaError_t launch_ex(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                      const MatvecParams& p, int stages) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, p, stages);
}

size_t fixed_smem(int fmt, int K) {
    size_t b = static_cast<size_t>(K) * 4 + 2 * kConsumerThreads * 4 + 2 * kMaxStages * 8 + 128;
    if (fmt == FMT_NF4) b += 4096;
    return b + 128;   // alignment slack
}
int slot_bytes(int fmt) {
    return fmt == FMT_Q4_0 ? Layout<FMT_Q4_0>::kSlot : fmt == FMT_Q8_0 ? Layout<FMT_Q8_0>::kSlot : Layout<FMT_NF4>::kSlot;
}
int stages_for(int fmt, int K) {
    const long long avail = kSmemLimit - static_cast<long long>(fixed_smem(fmt, K));
    const long long s = avail / (static_cast<long long>(kTileRows) * slot_bytes(fmt));
    return static_cast<int>(std::min<long long>(s, kMaxStages));
}

template <int FMT, int GROUP>
cudaError_t launch_tma(const MatvecParams& p, cudaStream_t stream, bool pdl) {
    static bool configured[64] = {};
    const int stages = stages_for(FMT, p.K);
    const size_t smem = fixed_smem(FMT, p.K) + static_cast<size_t>(stages) * kTileRows * slot_bytes(FMT);
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(matvec_tma_kernel<FMT, GROUP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemLimit);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    const int sms = sm_count_for_current_device();
    const int grid = std::max(1, std::min(sms, p.total_rows));
    return launch_ex(matvec_tma_kernel<FMT, GROUP>, dim3(grid), dim3(kThreads), smem, stream, pdl, p, stages);
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
    if (stages_for(fmt, K) < 2) return false;
    if (fmt == FMT_NF4) return group == 64 || (group == 128 && K % 1024 == 0);
    return true;
}

cudaError_t launch_matvec(int fmt, const MatvecParams& p, cudaStream_t stream, bool pdl) {
    if (p.total_rows <= 0) return cudaSuccess;
    // TMA bulk copies need 16-byte aligned sources; the x prologue reads float4.
    bool aligned = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    for (int s = 0; s < p.nseg; ++s) {
        aligned = aligned && (reinterpret_cast<uintptr_t>(p.seg[s].w) & 15) == 0;
        if (fmt == FMT_NF4) aligned = aligned && (reinterpret_cast<uintptr_t>(p.seg[s].absmax) & 15) == 0;
    }
    if (aligned && matvec_tma_supported(fmt, p.K, p.group)) {
        switch (fmt) {
            case FMT_Q4_0: return launch_tma<FMT_Q4_0, 32>(p, stream, pdl);
            case FMT_Q8_0: return launch_tma<FMT_Q8_0, 32>(p, stream, pdl);
            case FMT_NF4:
                return p.group == 64 ? launch_tma<FMT_NF4, 64>(p, stream, pdl) : launch_tma<FMT_NF4, 128>(p, stream, pdl);
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
    const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((work + threads - 1) / threads, sms * 16LL)));
    switch (fmt) {
        case FMT_NF4: dequant_nf4_kernel<<<grid, threads, 0, stream>>>(dst, src, absmax, numel, group); break;
        case FMT_Q4_0: dequant_q4_0_kernel<<<grid, threads, 0, stream>>>(dst, src, numel / 32); break;
        case FMT_Q8_0: dequant_q8_0_kernel<<<grid, threads, 0, stream>>>(dst, src, numel / 32); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace alj
