// Batched NF4 dequantise-and-GEMM on the 5th-generation tensor cores (tcgen05,
// sm_100a): Y[m][n] = sum_k X[m][k] * W[n][k] for a batch of M >= 2 tokens
// (prefill, batched decode), the weights in the NF4 layout of the batch-1 path
// (two codes per byte, high nibble first, one fp32 absmax per `group` = 64 or
// 128 consecutive elements of a row).  This is AccelOps.linear for M > 1
// (engine/safetensor/.../tensor/AccelOps.java:453-456: cblas_sgemm NoTrans x
// Trans on the dequantised fp32 weight), with the activations in bf16.
//
// Arithmetic.  The reference multiplies fp32 weights T[c] * s by fp32
// activations.  Rounding either operand to one 16-bit float costs ~1e-3
// relative per output, over the 1e-3 element-wise bound, so:
//   * A operand (weights): the codebook value only, T[c] = Th[c] + Tl[c] with
//     Th = fp16(T), Tl = fp16(T - Th) (|T - Th - Tl| <= 2^-22 |T|).  Two
//     tcgen05.mma per k-step (A = the Th columns, then the Tl columns, same B).
//   * B operand (activations): x' = x * 2^f per token, f chosen so that
//     max|x'| lies in [2^14, 2^15) -- exact, since a bf16 value has 8
//     significant bits and fp16 11 (gemm_x_prep_kernel).
//   * The absmax is not folded into the operands: each NF4 group gets its own
//     TMEM accumulator D_g = sum_{k in g} T[c_k] x'_k, and the epilogue warps
//     accumulate acc += s_g * D_g in fp32 on the CUDA cores, then scale by
//     2^-f.  So the scale enters exactly as in the reference (one fp32
//     product per group instead of per element) and no per-row exponent or
//     weight preparation is needed.
//
// Weight layout.  The GEMM reads NF4 weights packed once (gemm_nf4_pack_
// kernel, at weight registration, like the reference's prepared Q4_0 cache):
// for each 128-row tile and each 256-column unit, the 128 rows x 128 code
// bytes are one contiguous 16 KB block, and for each 16-group slot the 128
// rows x 16 absmax one contiguous 8 KB block (rows past the matrix are zero).
// A tile's codes in the original row-major layout are 128-byte pieces 2 KB
// to 14 KB apart, and streamed that way DRAM served one 16 KB copy per ~4 us
// per SM (about 0.5 TB/s in all).
//
// Tiles and schedule.  A tile is 128 weight rows (the MMA's M, TMEM lanes) x
// MT tokens (the MMA's N: 16, 32, 64 or 128; more tokens use several token
// tiles).  A unit is one tile x 256 columns of K.  Units are dealt out to one
// CTA per SM in equal contiguous ranges ("stream-K").  A piece of a tile whose
// K range is split between CTAs is written as an fp32 partial; after a grid
// barrier (cooperative launch, bounded wait) every CTA sums a share of the
// split tiles' outputs over their pieces in K order (deterministic).  One CTA
// summing a whole tile's ~18 partials was latency bound at ~15 us.
//
// Warp roles (one CTA per SM, up to 227 KB shared memory, all 512 TMEM
// columns: 4 A stages x 64 columns, then the accumulators):
//   warps 0-3      dequant: thread r owns weight row r of the tile = TMEM
//                  lane r; per stage (64 columns) it reads its 32 code bytes,
//                  looks up the (Th, Tl) pairs of each byte's two codes in a
//                  64 KB table (32 bank-private copies: one PRMT + one 8-byte
//                  load per byte) and stores the 32 Th pairs and 32 Tl pairs
//                  into the stage's TMEM columns with two tcgen05.st.  The A
//                  operand never touches shared memory, whose bandwidth a
//                  shared-memory A tile (written, then read by the MMA) used
//                  up at about a third of the HBM rate;
//   warps 4..      epilogue (1 or 2 warpgroups): warp w reads TMEM lanes
//                  32 (w % 4) .. +31 = its 32 rows, a token half each;
//   next warp      weight stream: TMA copies of the codes (box 128 B x 128
//                  rows = 4 stages) and the absmax (box 16 groups x 128 rows);
//   next warp      activation stream: TMA copies of the fp16 activations
//                  (box 64 x MT, 128-byte swizzle) into their own deeper ring,
//                  so neither stream waits on the other's consumers;
//   last warp      TMEM allocation and the MMA issue (one thread):
//                  tcgen05.mma with A from TMEM and B from shared memory.
// Every mbarrier wait is bounded; the first wait that runs out sets a shared
// abort flag, records ALJ_FAULT_TIMEOUT, and every role leaves its loop; the
// MMA thread waits (bounded) for its last commit before TMEM is released.
#include "tc_gemm.cuh"

#include <algorithm>
#include <cstring>

namespace alj {
namespace {

using namespace tcg;

constexpr int kAbsCols = 16;                // absmax groups per absmax copy
constexpr int kMaxCodesRing = 4;
constexpr int kAbsRing = 2;
constexpr int kTableBytes = 256 * 32 * 8;   // 64 KB
constexpr int kCodesBytes = kRows * 128;    // 16 KB
constexpr int kAbsBytes = kRows * kAbsCols * 4;   // 8 KB
constexpr int kACols = 64;                  // TMEM columns per A stage: 32 of Th pairs, 32 of Tl pairs
constexpr int kARing = 4;                   // A stages in TMEM (columns 0 .. 255)
constexpr int kDCol0 = kARing * kACols;     // first TMEM column of the accumulators
constexpr int kMaxSeg = 3;
constexpr int kMaxARing = 4;                // dequantised A stages
constexpr int kMaxXRing = 16;               // activation stages
constexpr int kMaxDBufs = 8;
// One tcgen05.commit per stage, onto sdone[stage % kSDone]: the A slot, the
// activation slot and (at a group's last stage) the accumulator of that stage
// are all released by it.  Each waiter lags the MMA by fewer than kSDone
// stages (A ring 4, activation ring <= 16, accumulators <= 8 groups), so a
// slot's parity cannot alias.  (A commit costs the issuing thread a few
// hundred cycles; three per stage paced the whole pipeline.)

struct alignas(64) GemmSeg {
    CUtensorMap codes;     // packed codes: uint8 [tiles * units * 128][128], box {128, 128}, 128 B swizzle
    CUtensorMap absmax;    // packed absmax: fp32 [tiles * slots * 128][16], box {16, 128}, 64 B swizzle
    float* y;              // y[m * ldy + n]
    int rows;
    int ldy;
    int tile0;             // first row tile of the segment
};

struct alignas(64) GemmParams {
    GemmSeg seg[kMaxSeg];
    CUtensorMap xmap;      // fp16 [M][K], box {64, MT}, 128 B swizzle
    const int* tokexp;     // [M]: x' = x * 2^tokexp
    float* partials;       // [2 * grid][MT][128]
    unsigned int* gbar;    // grid barrier: one flag per CTA, cleared by gemm_x_prep_kernel
    int nseg, M, K, group;
    int row_tiles, tok_tiles, tiles, units_per_tile, abs_slots;
    long long units;
    int grid, codes_ring, x_ring, dbufs;
    int nsplit;                                 // tiles whose K range is split between CTAs
    unsigned short split_tile[kMaxSplit], split_off[kMaxSplit], split_n[kMaxSplit];
    unsigned short piece_slot[kMaxPieces];      // partial slots of the split tiles' pieces, in K order
    __device__ int exp_of(int) const { return 0; }   // outputs scale by the token exponent alone
};

// ------------------------------------------------------------------ PTX
// One stage: 4 k-steps x (Th, Tl) = 8 MMAs, then one commit onto `bar`
// (arrives when they and every earlier MMA of this thread have completed).
// The Th products accumulate in dh and the Tl products in dl: two independent
// chains of 4, so consecutive MMAs do not wait on each other's accumulator
// (with dl == dh it is one chain of 8).  `accum` = 0 starts a new group (the
// first MMA of each chain overwrites it).
__device__ __forceinline__ void tc_stage_mma(uint32_t dh, uint32_t dl, uint32_t ah, uint64_t b, uint32_t idesc,
                                             uint32_t accum, uint64_t* bar) {
    const uint32_t al = ah + kACols / 2;
    const uint32_t accum_l = (dl == dh) ? 1u : accum;
    asm volatile(
        "{\n .reg .pred p0, p1, p2;\n"
        " setp.ne.b32 p0, %12, 0;\n"
        " setp.ne.b32 p2, %17, 0;\n"
        " setp.eq.b32 p1, %12, %12;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %9, %13, p0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%16], [%5], %9, %13, p2;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %10, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%16], [%6], %10, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %11, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%16], [%7], %11, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %14, %13, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%16], [%8], %14, %13, p1;\n"
        " tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%15];\n"
        "}\n" ::"r"(dh),
        "r"(ah), "r"(ah + 8), "r"(ah + 16), "r"(ah + 24), "r"(al), "r"(al + 8), "r"(al + 16), "r"(al + 24),
        "l"(b), "l"(b + 2), "l"(b + 4), "r"(accum), "r"(idesc), "l"(b + 6), "r"(smem_u32(bar)), "r"(dl),
        "r"(accum_l)
        : "memory");
}

// ------------------------------------------------------------------ kernel
// MMA-issuing warps (round-robin over NF4 groups): the tensor pipe takes a
// 128-row MMA every ~64 cycles whatever N is, and one thread's issue path
// (waits, address set-up, 8 MMAs, commit) does not keep it busy.
__host__ __device__ constexpr int issuers_for(int EW) { return EW == 1 ? 4 : 2; }

template <int MT, int EW>
__global__ void __launch_bounds__(32 * (6 + issuers_for(EW) + 4 * EW), 1)
    nf4_tc_gemm_kernel(const __grid_constant__ GemmParams p) {
    constexpr int kIssuers = issuers_for(EW);
    constexpr int NT = MT / EW;                 // tokens per epilogue thread
    constexpr int CH = MT <= 16 ? 2 : 1;        // accumulator chains per group (Th, Tl); more TMEM per group
                                                // leaves fewer accumulator buffers for wider token tiles
    constexpr int kEpiWarp0 = 4;
    constexpr int kProdWarp = 4 + 4 * EW;       // codes + absmax stream
    constexpr int kXWarp = kProdWarp + 1;       // activation tiles
    constexpr int kMmaWarp = kProdWarp + 2;     // first issuer; also allocates TMEM
    constexpr int kXBytes = MT * 128;
    constexpr uint32_t kIdesc = idesc_f16(MT);

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int CQ = p.codes_ring;
    constexpr int SA = kARing;
    const int SX = p.x_ring;
    const int NB = p.dbufs;
    uint8_t* table = smem;
    uint8_t* codes_ring = table + kTableBytes;
    uint8_t* abs_ring = codes_ring + static_cast<size_t>(CQ) * kCodesBytes;
    uint8_t* x_ring = abs_ring + kAbsRing * kAbsBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(x_ring + static_cast<size_t>(SX) * kXBytes);
    uint64_t* codes_full = bars;
    uint64_t* codes_empty = codes_full + kMaxCodesRing;
    uint64_t* abs_full = codes_empty + kMaxCodesRing;
    uint64_t* abs_empty = abs_full + kAbsRing;
    uint64_t* a_full = abs_empty + kAbsRing;
    uint64_t* x_full = a_full + kMaxARing;
    uint64_t* sdone = x_full + kMaxXRing;
    uint64_t* d_empty = sdone + kSDone;
    uint64_t* done_bar = d_empty + kMaxDBufs;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(done_bar + 1);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1) + 1;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // Byte -> (Th pair, Tl pair) table: entry b, copy l at 256 b + 8 l.  The
    // 16 (Th, Tl) code pairs go to a scratch word array first (in the
    // activation ring, not yet in use), then every thread writes two copies
    // per 16-byte store.
    uint32_t* pairs = reinterpret_cast<uint32_t*>(x_ring);
    if (threadIdx.x < 16) {
        const float t = nf4_value(threadIdx.x);
        const __half h = __float2half_rn(t);
        const __half l = __float2half_rn(t - __half2float(h));
        pairs[threadIdx.x] = static_cast<uint32_t>(__half_as_ushort(h)) |
                             (static_cast<uint32_t>(__half_as_ushort(l)) << 16);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 256 * 16; e += blockDim.x) {
        const int b = e >> 4;
        const uint32_t p0 = pairs[b >> 4], p1 = pairs[b & 15];
        const uint32_t hx = (p0 & 0xFFFFu) | (p1 << 16);
        const uint32_t lx = (p0 >> 16) | (p1 & 0xFFFF0000u);
        reinterpret_cast<uint4*>(table)[e] = make_uint4(hx, lx, hx, lx);
    }
    if (threadIdx.x == 0) {
        for (int i = 0; i < kMaxCodesRing; ++i) {
            mbar_init(&codes_full[i], 1);
            mbar_init(&codes_empty[i], 4);
        }
        for (int i = 0; i < kAbsRing; ++i) {
            mbar_init(&abs_full[i], 1);
            mbar_init(&abs_empty[i], 4 * EW);
        }
        for (int i = 0; i < kMaxARing; ++i) mbar_init(&a_full[i], 4);
        for (int i = 0; i < kMaxXRing; ++i) mbar_init(&x_full[i], 1);
        for (int i = 0; i < kSDone; ++i) mbar_init(&sdone[i], 1);
        for (int i = 0; i < kMaxDBufs; ++i) {
            mbar_init(&d_empty[i], 4 * EW);
        }
        mbar_init(done_bar, kIssuers);
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
    const int gpu = p.group / kStageK;          // stages per group (1 or 2)

    if (warp < 4) {
        // ---------------------------------------------------------- dequant
        const int r = threadIdx.x;              // tile row = TMEM lane
        const uint32_t lane8 = static_cast<uint32_t>(lane) * 8u;
        const uint32_t tab = smem_u32(table);
        const uint32_t swz = static_cast<uint32_t>(r & 7);
        const uint32_t ta_row = tmem_base + (static_cast<uint32_t>(32 * warp) << 16);   // lanes of this warp
        Cursor cc{0, 0u}, ac{0, 0u}, rel{0, 0u};
        int si = 0;
        bool ok = u1 > u0;
        for (int t = t_first; ok && t <= t_last; ++t) {
            const Piece pc = make_piece(p, t, u0, u1);
            for (int c = pc.c0; ok && c < pc.c1; ++c) {
                if (!warp_wait(&codes_full[cc.slot], cc.phase, abort_flag)) { ok = false; break; }
                const uint32_t crow = smem_u32(codes_ring + static_cast<size_t>(cc.slot) * kCodesBytes) + r * 128;
                for (int st = 0; st < kUnitStages; ++st, ++si) {
                    if (si >= SA) {   // the MMAs of stage si - SA have released this A slot
                        if (!warp_wait(&sdone[rel.slot], rel.phase, abort_flag)) { ok = false; break; }
                        rel.next(kSDone);
                    }
                    tc_fence_after();
                    const uint4 w0 = lds128(crow + ((static_cast<uint32_t>(2 * st) ^ swz) << 4));
                    const uint4 w1 = lds128(crow + ((static_cast<uint32_t>(2 * st + 1) ^ swz) << 4));
                    const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    uint32_t hi[32], lo[32];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const uint2 e = lds64(tab + prmt(words[j], lane8, 0x5504u | (b << 4)));
                            hi[4 * j + b] = e.x;
                            lo[4 * j + b] = e.y;
                        }
                    }
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
        Cursor abc{0, 0u}, dc{0, 0u}, sdc{gpu - 1, 0u};
        bool ok = u1 > u0;
        float acc[NT];
        for (int t = t_first; ok && t <= t_last; ++t) {
            const Piece pc = make_piece(p, t, u0, u1);
            const GemmSeg& sg = p.seg[pc.seg];
#pragma unroll
            for (int j = 0; j < NT; ++j) acc[j] = 0.0f;
            int as = -1;
            for (int c = pc.c0; ok && c < pc.c1; ++c) {
                const int col0 = c * (kUnitK / p.group);
                if (c == pc.c0 || (col0 & (kAbsCols - 1)) == 0) {
                    if (as >= 0) {
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&abs_empty[as]);
                    }
                    as = abc.slot;
                    if (!warp_wait(&abs_full[as], abc.phase, abort_flag)) { ok = false; as = -1; break; }
                    abc.next(kAbsRing);
                }
                const uint32_t arow = smem_u32(abs_ring + as * kAbsBytes) + r * 64;
                const uint32_t aswz = static_cast<uint32_t>((r >> 1) & 3);
                for (int gi = 0; gi < kUnitK / p.group; ++gi) {
                    if (!warp_wait(&sdone[sdc.slot], sdc.phase, abort_flag)) { ok = false; break; }
                    tc_fence_after();
                    const int col = (col0 + gi) & (kAbsCols - 1);
                    const float s = lds_f32(arow + (((static_cast<uint32_t>(col >> 2) ^ aswz) << 4) | ((col & 3) << 2)));
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
                                acc[16 * h + j] =
                                    fmaf(s, __uint_as_float(v[j]) + __uint_as_float(w[j]), acc[16 * h + j]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j)
                                acc[16 * h + j] = fmaf(s, __uint_as_float(v[j]), acc[16 * h + j]);
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&d_empty[dc.slot]);
                    dc.next(NB);
                    for (int k = 0; k < gpu; ++k) sdc.next(kSDone);
                }
            }
            if (as >= 0) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&abs_empty[as]);
            }
            if (!ok) break;
            // ---- write-out: a whole tile goes to y; a piece of a split tile
            // to its partial slot (summed after the grid barrier below).
            const int n = pc.row0 + r;
            const int m0 = pc.tok0 * MT + eh * NT;
            const int cf = cta_of(p, static_cast<long long>(t) * p.units_per_tile);
            const int cl = cta_of(p, static_cast<long long>(t + 1) * p.units_per_tile - 1);
            if (cf != cl) {
                float* part = p.partials + static_cast<size_t>(slot_of(p, blockIdx.x, t)) * (MT * kRows);
#pragma unroll
                for (int j = 0; j < NT; ++j) part[(eh * NT + j) * kRows + r] = acc[j];
            } else if (n < sg.rows) {
#pragma unroll
                for (int j = 0; j < NT; ++j) {
                    const int m = m0 + j;
                    if (m < p.M) {
                        const int f = __ldg(p.tokexp + m);
                        sg.y[static_cast<size_t>(m) * sg.ldy + n] = acc[j] * __int_as_float((127 - f) << 23);
                    }
                }
            }
        }
    } else if (warp == kProdWarp) {
        // ---------------------------------------------------------- codes + absmax stream
        if (lane == 0) {
            Cursor cc{0, 0u}, abc{0, 0u};
            bool ok = u1 > u0;
            for (int t = t_first; ok && t <= t_last; ++t) {
                const Piece pc = make_piece(p, t, u0, u1);
                const GemmSeg& sg = p.seg[pc.seg];
                const int rt = pc.row0 / kRows;
                for (int c = pc.c0; ok && c < pc.c1; ++c) {
                    const int col0 = c * (kUnitK / p.group);
                    if (c == pc.c0 || (col0 & (kAbsCols - 1)) == 0) {
                        if (!wait_bar(&abs_empty[abc.slot], abc.phase ^ 1u, abort_flag)) { ok = false; break; }
                        mbar_arrive_expect_tx(&abs_full[abc.slot], kAbsBytes);
                        tma_load_2d(smem_u32(abs_ring + abc.slot * kAbsBytes), &sg.absmax, 0,
                                    (rt * p.abs_slots + col0 / kAbsCols) * kRows, &abs_full[abc.slot]);
                        abc.next(kAbsRing);
                    }
                    if (!wait_bar(&codes_empty[cc.slot], cc.phase ^ 1u, abort_flag)) { ok = false; break; }
                    mbar_arrive_expect_tx(&codes_full[cc.slot], kCodesBytes);
                    tma_load_2d(smem_u32(codes_ring + static_cast<size_t>(cc.slot) * kCodesBytes), &sg.codes, 0,
                                (rt * p.units_per_tile + c) * kRows, &codes_full[cc.slot]);
                    cc.next(CQ);
                }
            }
        }
    } else if (warp == kXWarp) {
        // ---------------------------------------------------------- activation tiles
        if (lane == 0) {
            pdl_wait();   // fp16 activations and token exponents come from gemm_x_prep_kernel
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
                        tma_load_2d(smem_u32(x_ring + static_cast<size_t>(xc.slot) * kXBytes), &p.xmap,
                                    c * kUnitK + st * kStageK, pc.tok0 * MT, &x_full[xc.slot]);
                        xc.next(SX);
                    }
                }
            }
        }
    } else {
        // ---------------------------------------------------------- MMA issue
        // Issuer k takes the NF4 groups whose CTA-local index is k mod
        // kIssuers; it walks every stage to keep its ring cursors in step.
        const int issuer = warp - kMmaWarp;
        if (lane == 0) {
            Cursor dc{0, 0u}, xc{0, 0u}, ac{0, 0u}, sd{0, 0u};
            int g = 0, grp = 0;
            bool ok = u1 > u0;
            for (int t = t_first; ok && t <= t_last; ++t) {
                const Piece pc = make_piece(p, t, u0, u1);
                const int nst = (pc.c1 - pc.c0) * kUnitStages;
                for (int i = 0; i < nst; ++i) {
                    if (grp == issuer) {
                        if (g == 0 && !wait_bar(&d_empty[dc.slot], dc.phase ^ 1u, abort_flag)) { ok = false; break; }
                        if (!wait_bar(&x_full[xc.slot], xc.phase, abort_flag) ||
                            !wait_bar(&a_full[ac.slot], ac.phase, abort_flag)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t ah = tmem_base + static_cast<uint32_t>(ac.slot * kACols);
                        const uint64_t bx = sdesc(smem_u32(x_ring + static_cast<size_t>(xc.slot) * kXBytes));
                        const uint32_t d = tmem_base + static_cast<uint32_t>(kDCol0 + dc.slot * CH * MT);
                        tc_stage_mma(d, d + (CH - 1) * MT, ah, bx, kIdesc, g > 0 ? 1u : 0u, &sdone[sd.slot]);
                    }
                    xc.next(SX);
                    ac.next(SA);
                    sd.next(kSDone);
                    if (++g == gpu) {
                        g = 0;
                        dc.next(NB);
                        if (++grp == kIssuers) grp = 0;
                    }
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

constexpr int kPrepThreads = 1024;
constexpr int kPrepVecs = 4;                // uint4 (8 bf16) a thread keeps in registers: K <= 32768

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint4 to_f16x8(uint4 v, float sc) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half lo = __float2half_rn(bf16_lo(w[j]) * sc);
        const __half hi = __float2half_rn(bf16_hi(w[j]) * sc);
        o[j] = static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// bf16 activations -> fp16 x * 2^f (per token row), f = 15 - e with
// max|x| = m * 2^e, m in [0.5, 1): max|x'| in [2^14, 2^15).  One block per
// token, sized so that a row of K <= 32768 is read once and kept in registers
// (4 x 8 values a thread).  Block 0 also clears the GEMM's grid-barrier flags.  Each block
// lets the dependent GEMM launch as soon as it is resident.
__global__ void __launch_bounds__(kPrepThreads) gemm_x_prep_kernel(const __nv_bfloat16* __restrict__ x, int K,
                                                                   __half* __restrict__ xh, int* __restrict__ tokexp,
                                                                   unsigned int* __restrict__ flags, int nflags) {
    pdl_launch_dependents();
    const int m = blockIdx.x;
    if (m == 0)
        for (int i = threadIdx.x; i < nflags; i += blockDim.x) flags[i] = 0u;
    const uint4* row = reinterpret_cast<const uint4*>(x + static_cast<size_t>(m) * K);
    const int n8 = K / 8;
    const int nt = blockDim.x;
    const bool in_regs = n8 <= kPrepVecs * nt;
    uint4 v[kPrepVecs];
    float mx = 0.0f;
    if (in_regs) {
#pragma unroll
        for (int k = 0; k < kPrepVecs; ++k) {
            const int i = threadIdx.x + k * nt;
            v[k] = i < n8 ? __ldg(row + i) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int k = 0; k < kPrepVecs; ++k) {
            const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) mx = fmaxf(mx, fmaxf(fabsf(bf16_lo(w[j])), fabsf(bf16_hi(w[j]))));
        }
    } else {
        for (int i = threadIdx.x; i < n8; i += blockDim.x) {
            const uint4 u = __ldg(row + i);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) mx = fmaxf(mx, fmaxf(fabsf(bf16_lo(w[j])), fabsf(bf16_hi(w[j]))));
        }
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
    const float sc = __int_as_float((127 + f) << 23);    // 2^f, |f| <= 100
    uint4* out = reinterpret_cast<uint4*>(xh + static_cast<size_t>(m) * K);
    if (in_regs) {
#pragma unroll
        for (int k = 0; k < kPrepVecs; ++k) {
            const int i = threadIdx.x + k * nt;
            if (i < n8) out[i] = to_f16x8(v[k], sc);
        }
    } else {
        for (int i = threadIdx.x; i < n8; i += blockDim.x) out[i] = to_f16x8(__ldg(row + i), sc);
    }
}

// One-time repack of an NF4 matrix [rows][K] (codes, absmax in the original
// layout) into the GEMM's tile-contiguous layout (see the file comment).
__global__ void gemm_nf4_pack_kernel(uint8_t* __restrict__ pcodes, float* __restrict__ pabs,
                                     const uint8_t* __restrict__ codes, const float* __restrict__ absmax, int rows,
                                     int K, int group, int row_tiles, int units, int slots) {
    const size_t nchunks = static_cast<size_t>(row_tiles) * units * kRows * 8;     // 16-byte pieces
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t q = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < nchunks; q += stride) {
        const int j = static_cast<int>(q & 7);
        const int rr = static_cast<int>((q >> 3) & (kRows - 1));
        const size_t tu = q >> 10;                      // rt * units + u
        const int u = static_cast<int>(tu % units);
        const int row = static_cast<int>(tu / units) * kRows + rr;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (row < rows)
            v = __ldg(reinterpret_cast<const uint4*>(codes + static_cast<size_t>(row) * (K / 2) + u * 128 + j * 16));
        reinterpret_cast<uint4*>(pcodes)[q] = v;
    }
    const int ncols = K / group;
    const size_t nabs = static_cast<size_t>(row_tiles) * slots * kRows * kAbsCols;
    for (size_t f = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; f < nabs; f += stride) {
        const int c = static_cast<int>(f & (kAbsCols - 1));
        const int rr = static_cast<int>((f >> 4) & (kRows - 1));
        const size_t ts = f >> 11;                      // rt * slots + s
        const int col = static_cast<int>(ts % slots) * kAbsCols + c;
        const int row = static_cast<int>(ts / slots) * kRows + rr;
        pabs[f] = (row < rows && col < ncols) ? __ldg(absmax + static_cast<size_t>(row) * ncols + col) : 0.0f;
    }
}

// ------------------------------------------------------------------ host
struct WsLayout {
    size_t xh, tokexp, gbar, partials, total;
};
WsLayout ws_layout(int M, int K, int tiles, int grid) {
    const int MT = token_tile_for(M);
    WsLayout w;
    w.xh = 0;
    w.tokexp = align_up(w.xh + static_cast<size_t>(M) * K * 2, 256);
    w.gbar = align_up(w.tokexp + static_cast<size_t>(M) * 4, 256);
    w.partials = align_up(w.gbar + static_cast<size_t>(kMaxSplit) * 4, 256);
    w.total = align_up(w.partials + static_cast<size_t>(2) * grid * MT * kRows * 4, 256);
    return w;
}

// Ring depths in shared memory: 4 codes units and as deep an activation ring
// (up to 16 stages) as fits.  The dequantised A stages live in TMEM.
struct Rings {
    int codes, x;
    size_t smem;
};
Rings rings_for(int MT) {
    const size_t fixed = 1024 + kTableBytes + kAbsRing * kAbsBytes + 1024;
    const size_t xb = static_cast<size_t>(MT) * 128;
    Rings r{kMaxCodesRing, 0, 0};
    const size_t used = fixed + static_cast<size_t>(r.codes) * kCodesBytes;
    r.x = static_cast<int>(std::min<size_t>(kMaxXRing, (kSmemMax - used) / xb));
    r.smem = used + r.x * xb;
    return r;
}

template <int MT, int EW>
cudaError_t launch_mt(const GemmParams& p, size_t smem, cudaStream_t stream) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(nf4_tc_gemm_kernel<MT, EW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemMax);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    // Cooperative when split tiles need the grid barrier (all CTAs resident:
    // one per SM by shared memory, grid <= SM count).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(32 * (6 + issuers_for(EW) + 4 * EW));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    // Programmatic dependent launch on the activation prep just before it:
    // set-up, the table, TMEM and the weight stream overlap it; the roles that
    // read its output wait with griddepcontrol.wait.
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.nsplit > 0 ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, nf4_tc_gemm_kernel<MT, EW>, p);
}

}  // namespace

bool gemm_nf4_supported(int M, int K, int group) {
    return M >= 1 && K > 0 && K % kUnitK == 0 && (group == 64 || group == 128) && tensor_map_encoder() != nullptr;
}

namespace {
int abs_slots_of(int K, int group) { return (K / group + kAbsCols - 1) / kAbsCols; }
size_t packed_codes_bytes(int rows, int K) {
    return static_cast<size_t>((rows + kRows - 1) / kRows) * (K / kUnitK) * kCodesBytes;
}
}  // namespace

size_t gemm_nf4_packed_bytes(int rows, int K, int group) {
    return packed_codes_bytes(rows, K) + static_cast<size_t>((rows + kRows - 1) / kRows) * abs_slots_of(K, group) * kAbsBytes;
}

cudaError_t launch_gemm_nf4_pack(void* packed, const void* codes, const void* absmax, int rows, int K, int group,
                                 cudaStream_t stream) {
    if (rows < 1 || !gemm_nf4_supported(1, K, group)) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(packed) & 255) || (reinterpret_cast<uintptr_t>(codes) & 15) || (K / 2) % 16)
        return cudaErrorInvalidValue;
    uint8_t* pc = static_cast<uint8_t*>(packed);
    float* pa = reinterpret_cast<float*>(pc + packed_codes_bytes(rows, K));
    const int row_tiles = (rows + kRows - 1) / kRows;
    gemm_nf4_pack_kernel<<<2 * sm_count_for_current_device(), 256, 0, stream>>>(
        pc, pa, static_cast<const uint8_t*>(codes), static_cast<const float*>(absmax), rows, K, group, row_tiles,
        K / kUnitK, abs_slots_of(K, group));
    return cudaGetLastError();
}

size_t gemm_nf4_workspace_bytes(int M, int K, int total_tiles, int grid) {
    return ws_layout(M, K, total_tiles, grid).total;
}

int gemm_nf4_tiles(int M, int nseg, const int* rows) {
    int rt = 0;
    for (int s = 0; s < nseg; ++s) rt += (rows[s] + kRows - 1) / kRows;
    const int MT = token_tile_for(M);
    return rt * ((M + MT - 1) / MT);
}

cudaError_t launch_gemm_nf4(const GemmNf4Args& a, cudaStream_t stream) {
    if (a.nseg < 1 || a.nseg > kMaxSeg || !gemm_nf4_supported(a.M, a.K, a.group)) return cudaErrorNotSupported;
    const int MT = token_tile_for(a.M);
    GemmParams p;
    memset(&p, 0, sizeof p);
    p.nseg = a.nseg;
    p.M = a.M;
    p.K = a.K;
    p.group = a.group;
    int rt = 0;
    p.abs_slots = abs_slots_of(a.K, a.group);
    for (int s = 0; s < a.nseg; ++s) {
        GemmSeg& g = p.seg[s];
        if (a.rows[s] <= 0 || (reinterpret_cast<uintptr_t>(a.packed[s]) & 255)) return cudaErrorInvalidValue;
        const int tiles_s = (a.rows[s] + kRows - 1) / kRows;
        const uint8_t* pc = static_cast<const uint8_t*>(a.packed[s]);
        const void* pa = pc + packed_codes_bytes(a.rows[s], a.K);
        if (!encode_2d(&g.codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, pc, 128,
                    static_cast<uint64_t>(tiles_s) * (a.K / kUnitK) * kRows, 128, kRows, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !encode_2d(&g.absmax, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, pa, kAbsCols,
                    static_cast<uint64_t>(tiles_s) * p.abs_slots * kRows, kAbsCols, kRows, CU_TENSOR_MAP_SWIZZLE_64B))
            return cudaErrorInvalidValue;
        g.y = a.y[s];
        g.rows = a.rows[s];
        g.ldy = a.ldy[s];
        g.tile0 = rt;
        rt += (a.rows[s] + kRows - 1) / kRows;
    }
    p.row_tiles = rt;
    p.tok_tiles = (a.M + MT - 1) / MT;
    p.tiles = rt * p.tok_tiles;
    p.units_per_tile = a.K / kUnitK;
    if (!plan_stream_k(p, sm_count_for_current_device())) return cudaErrorNotSupported;
    const WsLayout w = ws_layout(a.M, a.K, p.tiles, p.grid);
    if (!a.workspace || a.workspace_bytes < w.total || (reinterpret_cast<uintptr_t>(a.workspace) & 255))
        return cudaErrorInvalidValue;
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    __half* xh = reinterpret_cast<__half*>(ws + w.xh);
    p.tokexp = reinterpret_cast<const int*>(ws + w.tokexp);
    p.gbar = reinterpret_cast<unsigned int*>(ws + w.gbar);
    p.partials = reinterpret_cast<float*>(ws + w.partials);
    if (!encode_2d(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, a.K, a.M, kStageK, MT, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const Rings rg = rings_for(MT);
    if (rg.x < 2) return cudaErrorNotSupported;
    p.codes_ring = rg.codes;
    p.x_ring = rg.x;
    p.dbufs = std::min(kMaxDBufs, (512 - kDCol0) / (MT <= 16 ? 2 * MT : MT));

    const int prep_threads = std::min(kPrepThreads, std::max(128, (a.K / 8 / kPrepVecs + 31) / 32 * 32));
    gemm_x_prep_kernel<<<a.M, prep_threads, 0, stream>>>(static_cast<const __nv_bfloat16*>(a.x), a.K, xh,
                                               reinterpret_cast<int*>(ws + w.tokexp), p.gbar, p.grid);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t smem = rg.smem;
    switch (MT) {
        case 16: return launch_mt<16, 1>(p, smem, stream);
        case 32: return launch_mt<32, 1>(p, smem, stream);
        case 64: return launch_mt<64, 2>(p, smem, stream);
        default: return launch_mt<128, 2>(p, smem, stream);
    }
}

}  // namespace alj
