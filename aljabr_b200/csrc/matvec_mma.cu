// Batch-1 GGUF Q4_0 and Q8_0 dequantise-and-matvec (y = W x) on the tensor
// cores of B200 (sm_100a), for K a multiple of 2048.
//
// Why tensor cores for a matvec: the kernel is HBM-bound only if the SM can
// decode 40 Q4_0 weights per cycle (6.5 TB/s / 148 SMs / 0.5625 B per
// weight).  On the CUDA cores that costs ~2.5 instructions per weight; here a
// 4-bit code becomes an fp16 operand with ONE LOP3 per two codes, and the
// multiply-add moves to mma.sync.m16n8k16 (f16 x f16 -> f32), ~1.7
// instructions per weight in all.
//
// Data flow per CTA (one CTA per SM, 16 consumer warps, 1 producer warp, 1
// epilogue warp):
//   * rows are dealt out in balanced units of 4 and walked in slabs of 16
//     rows (two 8-row halves; a slab never straddles a weight segment) x
//     chunks of 2048 columns (1152 bytes of Q4_0 per row);
//   * the producer streams each slab-chunk with 3-D TMA tensor copies
//     ({16 x 8 B, 9 column groups of 128 B, 8 or 4 rows}, 9 KB / 4.5 KB per
//     copy) with 128-byte swizzle: row r's 128-byte column group lands with
//     its 16-byte granules XOR-permuted by (9 r + group) mod 8, which makes
//     the fragment loads below bank-conflict free;
//   * warp w owns "span" w of every chunk: the four blocks {b, b+2, b+4, b+6}
//     with b = 8 (w / 2) + (w % 2) (same parity, so the 2-byte misalignment
//     of even blocks is warp-uniform); lane (g, t) decodes block t of rows g
//     and g + 8 straight into the A fragments of 8 MMAs;
//   * codes enter the MMA as fp16 subnormals: for Q4_0, (w & 0x000F000F) is
//     the pair (c0, c2) * 2^-24 and (w & 0x00F000F0) is (16 c1', 16 c3') *
//     2^-24; for Q8_0, PRMT(w ^ 0x80808080, 0, 0x4140) is (b0 + 128, b1 +
//     128) * 2^-24 -- exact, one instruction per two codes;
//   * x is staged once per CTA into shared memory as the B fragments, per
//     32-element block: x' = x 2^-E (E from the block's max |x|, so
//     |x'| < 2^11 for Q4_0, 2^10 for Q8_0), hi = rint(x') and lo = (x' - hi)
//     on a 2^-11 grid, both
//     exact in fp16.  B column 2t carries block t's hi, 2t + 1 its lo, so one
//     MMA keeps the four blocks of a span apart and D(row, 2t) + D(row, 2t+1)
//     is block t's dot product; every partial sum is an exact multiple of a
//     power of two below 2^24, so the tensor core's accumulation rounds
//     nothing.  What is not exact is the split itself: x keeps 22 bits
//     relative to its block's largest |x| (hi on the integer grid, lo on the
//     2^-11 grid), so an element far below its block maximum loses low bits;
//     the other roundings are the fp32 sums over blocks;
//   * the code offset (-8 for Q4_0, -128 for the biased Q8_0 bytes) enters as
//     the accumulator's initial value -off sum(hi) 2^-24 (hi column) and
//     -off sum(lo) 2^-24 (lo column);
//   * the block scale d (fp16, decoded from the fetched words) and 2^(E+24)
//     are applied once per block in fp32;
//   * per-warp row partials go through a shared-memory ring to the epilogue
//     warp, which sums the 16 warps in fixed order (deterministic), applies
//     bias / residual / SwiGLU and stores; consumers never wait on a CTA
//     barrier.
// Every mbarrier wait is bounded (ALJ_FAULT_TIMEOUT in the device fault word).
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>

namespace alj {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();   // matvec.cu

namespace {

constexpr int kCW = 16;                        // consumer warps
constexpr int kProducerWarp = kCW;
constexpr int kEpilogueWarp = kCW + 1;
constexpr int kThreads = (kCW + 2) * 32;
constexpr int kUnit = 4;                       // rows per balancing unit
constexpr int kChunkElems = 2048;              // 16 spans of 128 columns
constexpr int kMaxStages = 8;

// Per-format geometry.  Both formats store 32-element blocks (fp16 d first),
// so a chunk of 2048 columns is 64 blocks and an odd number of 128-byte
// column groups per row (9 for Q4_0, 17 for Q8_0): row r's groups then get
// pairwise different swizzle keys (9 r + g or 17 r + g mod 8).
template <int FMT>
struct MmaFmt;
template <>
struct MmaFmt<FMT_Q4_0> {
    static constexpr int kBlockBytes = 18;
    static constexpr int kWords = 5;           // 32-bit words a lane fetches per block row
    static constexpr float kOffset = 8.0f;     // code c stands for c - 8
    static constexpr int kXBits = 11;          // |x'| < 2^11: 32 products c * hi (c < 16) stay below 2^20
};
template <>
struct MmaFmt<FMT_Q8_0> {
    static constexpr int kBlockBytes = 34;
    static constexpr int kWords = 9;
    static constexpr float kOffset = 128.0f;   // int8 b enters as the unsigned b + 128
    static constexpr int kXBits = 10;          // |x'| < 2^10: 32 products (b + 128) * hi stay below 2^23
};
template <int FMT>
struct MmaGeom {
    static constexpr int kChunkBytes = 64 * MmaFmt<FMT>::kBlockBytes;   // 1152 | 2176
    static constexpr int kGroups = kChunkBytes / 128;                   // 9 | 17
    static constexpr int kBoxBytes = 8 * kChunkBytes;                   // one 8-row half slab
    static constexpr int kStageBytes = 2 * kBoxBytes;
};

// Block element (0..31) that B slot `pos` (0..3) of k-step j carries.  The
// A side: code word i of a block is (b0 b1 b2 b3) = bytes at code index
// byte_idx(par, i, .); even blocks start 2 bytes into a word (the word holds
// d), odd blocks start on a word.
//   Q4_0: word i feeds k-steps 2i (low nibbles) and 2i + 1 (high nibbles,
//         elements + 16); slots (0, 1) = bytes (b0, b2), (2, 3) = (b1, b3).
//   Q8_0: word j feeds k-step j; slots (0, 1) = (b0, b1), (2, 3) = (b2, b3).
__host__ __device__ constexpr int q4_byte_idx(int par, int i, int q) {
    return par ? (i == 0 ? 12 + q : 4 * (i - 1) + q) : (i == 0 ? (q < 2 ? q : 12 + q) : 2 + 4 * (i - 1) + q);
}
__host__ __device__ constexpr int q8_byte_idx(int par, int i, int q) {
    return par ? (i == 0 ? 28 + q : 4 * (i - 1) + q) : (i == 0 ? (q < 2 ? q : 28 + q) : 4 * i - 2 + q);
}
template <int FMT>
__host__ __device__ constexpr int slot_elem(int par, int j, int pos) {
    return FMT == FMT_Q4_0
               ? q4_byte_idx(par, j >> 1, pos == 0 ? 0 : pos == 1 ? 2 : pos == 2 ? 1 : 3) + 16 * (j & 1)
               : q8_byte_idx(par, j, pos);
}
constexpr int kRecBytes = 128;                 // B fragments of a (span, k-step pair): 8 lane slots of 16 B
constexpr int kSpanBytes = 4 * kRecBytes;
constexpr int kBlockInfoBytes = 16;            // per 32-element block: -off_hi, -off_lo, 2^(E+24), 0
constexpr int kRing = 4;                       // slab partial buffers
constexpr int kSmemMax = 232448;               // 227 KB opt-in per CTA
constexpr float kTwoM24 = 5.9604644775390625e-8f;

struct alignas(64) MmaSegment {
    CUtensorMap map8;                          // box {16, 9, 8}
    CUtensorMap map4;                          // box {16, 9, 4}
    const float* bias;
    const float* residual;
    float* y;
    int rows;
    int row0;
};

struct alignas(64) MmaParams {
    MmaSegment seg[3];
    int nseg;
    int K;
    int total_rows;                            // EPI_SWIGLU_PAIR: rows of one segment
    int pair;
    const float* x;
    float* norm_out;
    const float* norm_w;
    float norm_eps;
    float* norm_partials;
    unsigned int* norm_counter;
    const uint8_t* prefetch;
    size_t prefetch_bytes;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t land(uint32_t w, uint32_t m) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xC0;" : "=r"(r) : "r"(w), "r"(m), "r"(0u));
    return r;
}

// Slabs of a CTA's unit range, split at segment boundaries (pair mode: both
// segments advance together over the logical rows).
// norm_out = y * scale * norm_w over the whole output, by the last CTA's
// consumer warps and epilogue warp (participant index 0 .. 16 * 32 + 31).
template <typename P>
__device__ __forceinline__ void norm_pass(const P& p, float scale, int idx) {
    const float* y = p.seg[0].y;
    for (int i = idx; i < p.total_rows; i += kCW * 32 + 32) p.norm_out[i] = __ldcg(y + i) * scale * p.norm_w[i];
}

struct SlabWalk {
    int u, u_end;
    __device__ __forceinline__ bool next(const MmaParams& p, int& seg, int& su, int& nunits) {
        if (u >= u_end) return false;
        seg = 0;
        int seg_end = p.total_rows / kUnit;
        if (!p.pair) {
            if (p.nseg > 1 && u * kUnit >= p.seg[1].row0) seg = 1;
            if (p.nseg > 2 && u * kUnit >= p.seg[2].row0) seg = 2;
            seg_end = (p.seg[seg].row0 + p.seg[seg].rows) / kUnit;
        }
        su = u;
        nunits = min(p.pair ? 2 : 4, min(u_end, seg_end) - u);
        u += nunits;
        return true;
    }
};

template <int FMT>
__global__ void __launch_bounds__(kThreads, 1) quant_mma_kernel(const __grid_constant__ MmaParams p, int stages) {
    using G = MmaGeom<FMT>;
    using F = MmaFmt<FMT>;
    constexpr int kChunkBytes = G::kChunkBytes;
    constexpr int kGroups = G::kGroups;
    constexpr int kBoxBytes = G::kBoxBytes;
    constexpr int kStageBytes = G::kStageBytes;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    pdl_launch_dependents();
    const int K = p.K;
    const int nchunks = K / kChunkElems;
    const int nspans = nchunks * 16;
    const uint32_t base = smem_u32(smem_raw);
    uint8_t* sp = smem_raw + ((1024u - (base & 1023u)) & 1023u);
    uint8_t* stage0 = sp;
    sp += static_cast<size_t>(stages) * kStageBytes;
    uint8_t* xfrag = sp;
    sp += static_cast<size_t>(nspans) * kSpanBytes;
    float4* binfo = reinterpret_cast<float4*>(sp);
    sp += static_cast<size_t>(nspans) * 4 * kBlockInfoBytes;
    float* red = reinterpret_cast<float*>(sp);           // [kRing][kCW][16]
    sp += kRing * kCW * 16 * 4;
    float* misc = reinterpret_cast<float*>(sp);          // [0] norm scale, [1] last-CTA flag, [12..15] zeros
    sp += 16 * 4;
    uint64_t* full = reinterpret_cast<uint64_t*>(sp);
    uint64_t* empty = full + kMaxStages;
    uint64_t* rfull = empty + kMaxStages;
    uint64_t* rempty = rfull + kRing;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lrows = p.total_rows;
    const int units = lrows / kUnit;
    const int u_begin = static_cast<int>(static_cast<long long>(units) * blockIdx.x / gridDim.x);
    const int u_end = static_cast<int>(static_cast<long long>(units) * (blockIdx.x + 1) / gridDim.x);

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        for (int b = 0; b < kRing; ++b) {
            mbar_init(&rfull[b], kCW);
            mbar_init(&rempty[b], 1);
        }
        fence_mbar_init();
        *reinterpret_cast<float4*>(misc + 12) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    __syncthreads();

    if (warp == kProducerWarp) {
        // Weights never depend on the previous kernel: copies start before
        // griddepcontrol.wait.
        if (lane == 0) {
            SlabWalk walk{u_begin, u_end};
            int seg, su, nunits, s = 0;
            uint32_t ph = 0;
            bool alive = true;
            while (alive && walk.next(p, seg, su, nunits)) {
                const int halves = p.pair ? 2 : 1;
                for (int c = 0; c < nchunks; ++c) {
                    if (!mbar_wait(&empty[s], ph ^ 1u)) {
                        alive = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(halves * nunits * kUnit * kChunkBytes));
                    const uint32_t st = smem_u32(stage0) + s * kStageBytes;
                    if (p.pair) {
                        const CUtensorMap* mg = nunits == 2 ? &p.seg[0].map8 : &p.seg[0].map4;
                        const CUtensorMap* mu = nunits == 2 ? &p.seg[1].map8 : &p.seg[1].map4;
                        tma_load_3d(st, mg, 0, c * kGroups, su * kUnit, &full[s]);
                        tma_load_3d(st + kBoxBytes, mu, 0, c * kGroups, su * kUnit, &full[s]);
                    } else {
                        const MmaSegment& sg = p.seg[seg];
                        const int r0 = su * kUnit - sg.row0;
                        tma_load_3d(st, nunits >= 2 ? &sg.map8 : &sg.map4, 0, c * kGroups, r0, &full[s]);
                        if (nunits > 2)
                            tma_load_3d(st + kBoxBytes, nunits == 4 ? &sg.map8 : &sg.map4, 0, c * kGroups, r0 + 8,
                                        &full[s]);
                    }
                    if (++s == stages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (alive && p.prefetch) prefetch_share(p.prefetch, p.prefetch_bytes);
        }
        return;
    }

    if (warp == kEpilogueWarp) {
        // Fixed-order sum of the 16 warps' partials per slab, then the epilogue.
        pdl_wait();
        SlabWalk walk{u_begin, u_end};
        int seg, su, nunits, sl = 0;
        float sq = 0.0f;
        while (walk.next(p, seg, su, nunits)) {
            const int b = sl % kRing;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&rfull[b], (sl / kRing) & 1));
            if (ok && lane < 16) {
                float acc = 0.0f;
#pragma unroll
                for (int w = 0; w < kCW; ++w) acc += red[(b * kCW + w) * 16 + lane];
                if (p.pair) {
                    // lanes 0..7 hold gate rows, 8..15 the matching up rows
                    const float up = __shfl_down_sync(0x0000ffffu, acc, 8, 16);
                    if (lane < nunits * kUnit) {
                        const float out = acc / (1.0f + expf(-acc)) * up;
                        p.seg[0].y[su * kUnit + lane] = out;
                        sq = fmaf(out, out, sq);
                    }
                } else if (lane < nunits * kUnit) {
                    const MmaSegment& sg = p.seg[seg];
                    const int lrow = su * kUnit + lane - sg.row0;
                    float out = acc;
                    if (sg.bias) out += sg.bias[lrow];
                    if (sg.residual) out = sg.residual[lrow] + out;
                    sg.y[lrow] = out;
                    sq = fmaf(out, out, sq);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rempty[b]);
            ++sl;
        }
        if (p.norm_out) {
            // Deterministic RMSNorm of the whole output: per-CTA partials in
            // fixed order; the last CTA to arrive computes the scale, and all of
            // its consumer warps plus this warp write norm_out.
            __threadfence();   // this lane's y stores before the arrival below
            const float cta = warp_sum(sq);
            if (lane == 0) {
                p.norm_partials[blockIdx.x] = cta;
                __threadfence();
                const unsigned int prev = atomicAdd(p.norm_counter, 1u);
                misc[1] = prev == gridDim.x - 1 ? 1.0f : 0.0f;
            }
            __syncwarp();
            if (misc[1] != 0.0f) {
                __threadfence();
                float part = 0.0f;
                for (unsigned int b = lane; b < gridDim.x; b += 32) part += __ldcg(p.norm_partials + b);
                const float tot = warp_sum(part);
                if (lane == 0) {
                    misc[0] = 1.0f / sqrtf(tot / static_cast<float>(lrows) + p.norm_eps);
                    *p.norm_counter = 0u;
                }
            }
            named_bar(2, kCW * 32 + 32);
            if (misc[1] != 0.0f) norm_pass(p, misc[0], kCW * 32 + lane);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    pdl_wait();   // x comes from the previous kernel
    const int par = warp & 1;              // parity of this warp's blocks
    const int blk = 8 * (warp >> 1) + par; // first block of this warp's span within a chunk
    {
        // Stage the B fragments of this warp's spans (read by no other warp).
        // Lane (t, j) = (lane / 8, lane % 8) converts the 4 elements of block
        // blk + 2t that B slots 0..3 of k-step j carry.
        const int st_t = lane >> 3, st_j = lane & 7;
        const int hs = FMT == FMT_Q4_0 ? (st_j & 1) : 0;   // Q4_0 high nibbles enter the MMA as 16 c
        int e[4];
#pragma unroll
        for (int pos = 0; pos < 4; ++pos) e[pos] = slot_elem<FMT>(par, st_j, pos);
        // x reads of up to kXBatch chunks go out together: one L2 round trip
        // per batch instead of one per chunk (every CTA reads all of x, so
        // these lines are contended)
        constexpr int kXBatch = 8;
        for (int c0 = 0; c0 < nchunks; c0 += kXBatch) {
            float vb[kXBatch][4];
#pragma unroll
            for (int cb = 0; cb < kXBatch; ++cb) {
                const float* xb = p.x + static_cast<size_t>((c0 + cb) * 64 + blk + 2 * st_t) * 32;
#pragma unroll
                for (int pos = 0; pos < 4; ++pos) vb[cb][pos] = c0 + cb < nchunks ? __ldg(xb + e[pos]) : 0.0f;
            }
#pragma unroll
            for (int cb = 0; cb < kXBatch; ++cb) {
            const int c = c0 + cb;
            if (c >= nchunks) break;
            const int bg = c * 64 + blk + 2 * st_t;
            float v[4];
#pragma unroll
            for (int pos = 0; pos < 4; ++pos) v[pos] = vb[cb][pos];
            float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            int E = 0;
            if (mx > 0.0f && mx < INFINITY) E = min(90, max(-90, ilogbf(mx) - (F::kXBits - 1)));
            const float xs = __int_as_float((127 - E) << 23);
            float hv[4], lv[4], shi = 0.0f, slo = 0.0f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float xq = v[q] * xs;
                hv[q] = rintf(xq);
                lv[q] = rintf((xq - hv[q]) * 2048.0f) * (1.0f / 2048.0f);
                shi += hv[q];
                slo += lv[q];
            }
            shi += __shfl_xor_sync(0xffffffffu, shi, 1);
            shi += __shfl_xor_sync(0xffffffffu, shi, 2);
            shi += __shfl_xor_sync(0xffffffffu, shi, 4);
            slo += __shfl_xor_sync(0xffffffffu, slo, 1);
            slo += __shfl_xor_sync(0xffffffffu, slo, 2);
            slo += __shfl_xor_sync(0xffffffffu, slo, 4);
            const float hsc = hs ? 0.0625f : 1.0f;
            uint32_t hw[2], lw[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const __half2 h = __floats2half2_rn(hv[2 * u] * hsc, hv[2 * u + 1] * hsc);
                const __half2 l = __floats2half2_rn(lv[2 * u] * hsc, lv[2 * u + 1] * hsc);
                hw[u] = *reinterpret_cast<const uint32_t*>(&h);
                lw[u] = *reinterpret_cast<const uint32_t*>(&l);
            }
            // k-steps 2i and 2i + 1 share a 16-byte lane slot: k-step j at 8 (j & 1)
            uint8_t* rec = xfrag + static_cast<size_t>(c * 16 + warp) * kSpanBytes + (st_j >> 1) * kRecBytes;
            *reinterpret_cast<uint2*>(rec + 32 * st_t + 8 * (st_j & 1)) = make_uint2(hw[0], hw[1]);
            *reinterpret_cast<uint2*>(rec + 32 * st_t + 16 + 8 * (st_j & 1)) = make_uint2(lw[0], lw[1]);
            if (st_j == 0)
                binfo[bg] = make_float4(-F::kOffset * shi * kTwoM24, -F::kOffset * slo * kTwoM24,
                                        __int_as_float((127 + E + 24) << 23), 0.0f);
            }
        }
        __syncwarp();
    }

    const int g = lane >> 2, t = lane & 3;
    const uint32_t bact = (g >> 1) == t ? 1u : 0u;       // lanes whose B column belongs to their quad
    const uint32_t boff = 16u * (2 * t + (g & 1));
    const uint32_t sel_d = par ? 0x4432u : 0x4410u;      // fp16 d: low half (even block) or high half (odd)
    const uint32_t sel_c0 = par ? 0x7654u : 0x5432u;     // first code word: W[last] (odd) or W0.hi:W[last].lo
    const int myblk = blk + 2 * t;
    constexpr int kW = F::kWords;
    uint32_t aoff[kW];                                   // swizzled offsets of this lane's words in row g
    {
        const uint32_t boffs = (static_cast<uint32_t>(F::kBlockBytes) * myblk) & ~3u;
#pragma unroll
        for (int k = 0; k < kW; ++k) {
            const uint32_t o = boffs + 4 * k;
            const uint32_t segidx = g * kGroups + (o >> 7);
            aoff[k] = segidx * 128 + ((((o >> 4) & 7) ^ (segidx & 7)) << 4) + (o & 15);
        }
    }
    const uint32_t stage_s = smem_u32(stage0);
    const uint32_t brec0 = smem_u32(xfrag) + warp * kSpanBytes + boff;
    const uint32_t binfo0 = smem_u32(binfo) + myblk * kBlockInfoBytes;
    // lanes whose B slots stay zero read them from a 16-byte zero slot (a
    // broadcast load) instead of zero-filling registers and predicating
    const uint32_t zero16 = smem_u32(misc + 12);

    SlabWalk walk{u_begin, u_end};
    int seg, su, nunits, s = 0, sl = 0;
    uint32_t ph = 0;
    while (walk.next(p, seg, su, nunits)) {
        float y0 = 0.0f, y1 = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
            // warp-uniform: the MMAs below need all 32 lanes
            if (__all_sync(0xffffffffu, mbar_wait(&full[s], ph))) {
                const uint32_t st = stage_s + s * kStageBytes;
                uint32_t W0[kW], W1[kW];
#pragma unroll
                for (int k = 0; k < kW; ++k) {
                    W0[k] = lds32(st + aoff[k]);
                    W1[k] = lds32(st + kBoxBytes + aoff[k]);
                }
                const uint4 bi = lds128(binfo0 + c * (64 * kBlockInfoBytes));
                const uint32_t rb = brec0 + c * (16 * kSpanBytes);
                uint4 B[4];
#pragma unroll
                for (int jp = 0; jp < 4; ++jp) B[jp] = lds128(bact ? rb + jp * kRecBytes : zero16);
                const float scale = __uint_as_float(bi.z);
                const float d0 = __half2float(__ushort_as_half(static_cast<unsigned short>(__byte_perm(W0[0], 0u, sel_d)))) * scale;
                const float d1 = __half2float(__ushort_as_half(static_cast<unsigned short>(__byte_perm(W1[0], 0u, sel_d)))) * scale;
                float d[4] = {__uint_as_float(bi.x), __uint_as_float(bi.y), __uint_as_float(bi.x), __uint_as_float(bi.y)};
                if constexpr (FMT == FMT_Q4_0) {
                    uint32_t cw0[4], cw1[4];
                    cw0[0] = __byte_perm(W0[0], W0[4], sel_c0);
                    cw1[0] = __byte_perm(W1[0], W1[4], sel_c0);
#pragma unroll
                    for (int i = 1; i < 4; ++i) {
                        cw0[i] = W0[i];
                        cw1[i] = W1[i];
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t s0 = cw0[i] >> 8, s1 = cw1[i] >> 8;
                        // k-step 2i: low nibbles of bytes (0,2) | (1,3); k-step 2i+1: high nibbles
                        mma16816(d, land(cw0[i], 0x000F000Fu), land(cw1[i], 0x000F000Fu), land(s0, 0x000F000Fu),
                                 land(s1, 0x000F000Fu), B[i].x, B[i].y);
                        mma16816(d, land(cw0[i], 0x00F000F0u), land(cw1[i], 0x00F000F0u), land(s0, 0x00F000F0u),
                                 land(s1, 0x00F000F0u), B[i].z, B[i].w);
                    }
                } else {
                    // int8 b -> (b ^ 0x80) = b + 128 as an fp16 subnormal, two per PRMT
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t c0 = (j == 0 ? __byte_perm(W0[0], W0[8], sel_c0) : W0[j]) ^ 0x80808080u;
                        const uint32_t c1 = (j == 0 ? __byte_perm(W1[0], W1[8], sel_c0) : W1[j]) ^ 0x80808080u;
                        const uint4& Bq = B[j >> 1];
                        mma16816(d, __byte_perm(c0, 0u, 0x4140u), __byte_perm(c1, 0u, 0x4140u),
                                 __byte_perm(c0, 0u, 0x4342u), __byte_perm(c1, 0u, 0x4342u),
                                 (j & 1) ? Bq.z : Bq.x, (j & 1) ? Bq.w : Bq.y);
                    }
                }
                y0 = fmaf(d0, d[0] + d[1], y0);
                y1 = fmaf(d1, d[2] + d[3], y1);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == stages) {
                s = 0;
                ph ^= 1u;
            }
        }
        y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
        y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
        y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
        y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
        const int b = sl % kRing;
        mbar_wait(&rempty[b], ((sl / kRing) & 1) ^ 1u);
        if (t == 0) {
            red[(b * kCW + warp) * 16 + g] = y0;
            red[(b * kCW + warp) * 16 + g + 8] = y1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfull[b]);
        ++sl;
    }
    if (p.norm_out) {
        named_bar(2, kCW * 32 + 32);
        if (misc[1] != 0.0f) norm_pass(p, misc[0], threadIdx.x);
    }
}

template <int FMT>
bool encode_maps(MmaSegment& ms, const void* w, int K, int rows) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    const size_t row_bytes = static_cast<size_t>(K) / 32 * MmaFmt<FMT>::kBlockBytes;
    const cuuint64_t dims[3] = {16, row_bytes / 128, static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[2] = {128, row_bytes};
    const cuuint32_t es[3] = {1, 1, 1};
    for (int v = 0; v < 2; ++v) {
        const cuuint32_t box[3] = {16, static_cast<cuuint32_t>(MmaGeom<FMT>::kGroups), v == 0 ? 8u : 4u};
        if (fn(v == 0 ? &ms.map8 : &ms.map4, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<void*>(w), dims, strides,
               box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    }
    return true;
}

int stage_bytes_of(int fmt) { return fmt == FMT_Q4_0 ? MmaGeom<FMT_Q4_0>::kStageBytes : MmaGeom<FMT_Q8_0>::kStageBytes; }

size_t fixed_smem(int K) {
    const size_t nspans = static_cast<size_t>(K / kChunkElems) * 16;
    return 1024 + nspans * (kSpanBytes + 4 * kBlockInfoBytes) + kRing * kCW * 16 * 4 + 16 * 4 +
           (2 * kMaxStages + 2 * kRing) * 8;
}

}  // namespace

bool matvec_mma_supported(int fmt, int K) {
    if ((fmt != FMT_Q4_0 && fmt != FMT_Q8_0) || K <= 0 || K % kChunkElems != 0) return false;
    if (static_cast<long long>(fixed_smem(K)) + 2LL * stage_bytes_of(fmt) > kSmemMax) return false;
    return tensor_map_encoder() != nullptr;
}

cudaError_t launch_matvec_mma(int fmt, const MatvecParams& mp, cudaStream_t stream, bool pdl) {
    if (!matvec_mma_supported(fmt, mp.K)) return cudaErrorNotSupported;
    const bool pair = mp.epilogue == EPI_SWIGLU_PAIR;
    if (pair && (mp.nseg != 2 || mp.seg[0].rows != mp.seg[1].rows || mp.total_rows != mp.seg[0].rows))
        return cudaErrorNotSupported;
    if (mp.norm_out && (mp.nseg != 1 && !pair)) return cudaErrorNotSupported;
    for (int s = 0; s < mp.nseg; ++s)
        if (mp.seg[s].rows % kUnit != 0 || (reinterpret_cast<uintptr_t>(mp.seg[s].w) & 15) != 0)
            return cudaErrorNotSupported;
    MmaParams p;
    memset(&p, 0, sizeof p);
    p.nseg = mp.nseg;
    p.K = mp.K;
    p.total_rows = mp.total_rows;
    p.pair = pair ? 1 : 0;
    p.x = mp.x;
    p.norm_out = mp.norm_out;
    p.norm_w = mp.norm_w;
    p.norm_eps = mp.norm_eps;
    p.norm_partials = mp.norm_partials;
    p.norm_counter = mp.norm_counter;
    p.prefetch = static_cast<const uint8_t*>(mp.prefetch);
    p.prefetch_bytes = mp.prefetch_bytes;
    int row0 = 0;
    for (int s = 0; s < mp.nseg; ++s) {
        MmaSegment& ms = p.seg[s];
        const bool ok = fmt == FMT_Q4_0 ? encode_maps<FMT_Q4_0>(ms, mp.seg[s].w, mp.K, mp.seg[s].rows)
                                        : encode_maps<FMT_Q8_0>(ms, mp.seg[s].w, mp.K, mp.seg[s].rows);
        if (!ok) return cudaErrorInvalidValue;
        ms.bias = mp.seg[s].bias;
        ms.residual = mp.seg[s].residual;
        ms.y = mp.seg[s].y;
        ms.rows = mp.seg[s].rows;
        ms.row0 = pair ? 0 : row0;
        row0 += mp.seg[s].rows;
    }
    const size_t fixed = fixed_smem(mp.K);
    const int sb = stage_bytes_of(fmt);
    const int stages = static_cast<int>(std::min<size_t>(kMaxStages, (kSmemMax - fixed) / sb));
    const size_t smem = fixed + static_cast<size_t>(stages) * sb;
    auto kern = fmt == FMT_Q4_0 ? quant_mma_kernel<FMT_Q4_0> : quant_mma_kernel<FMT_Q8_0>;
    static bool configured[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    bool& done = configured[fmt == FMT_Q4_0 ? 0 : 1][dev & 63];
    if (!done) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        done = true;
    }
    const int units = mp.total_rows / kUnit;
    const int grid = std::max(1, std::min(sm_count_for_current_device(), units));
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
    return cudaLaunchKernelEx(&cfg, kern, p, stages);
}

}  // namespace alj
