// Pieces shared by the batched dequantise-and-GEMM kernels on tcgen05
// (gemm_nf4.cu for NF4, gemm_q.cu for GGUF Q4_0 / Q8_0): PTX wrappers for
// TMA, TMEM and the MMA, bounded ring waits, and the stream-K schedule with
// its deterministic split-tile reduction.
//
// Schedule.  A tile is kRows weight rows x MT tokens; a unit is one tile x
// kUnitK columns of K.  Units are dealt out to one CTA per SM in equal
// contiguous ranges; a tile whose K range is split between CTAs is written
// as fp32 partials (one slot per CTA piece), and after a grid barrier every
// CTA sums a share of the split tiles over their pieces in K order.
//
// A params type P used with these templates provides: seg[] (with tile0,
// rows, ldy, y), exp_of(seg) (outputs are scaled by 2^-(tokexp + exp_of)),
// nseg, units, grid, units_per_tile, tok_tiles, M, tokexp, partials, gbar,
// nsplit, split_tile / split_off / split_n / piece_slot.
#pragma once

#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

namespace alj {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();   // matvec.cu

namespace tcg {

constexpr int kRows = 128;                  // weight rows per tile (the MMA's M, TMEM lanes)
constexpr int kStageK = 64;                 // K per A stage (64 fp16 = one 128-byte swizzle row)
constexpr int kUnitK = 256;                 // K per stream-K unit
constexpr int kUnitStages = kUnitK / kStageK;
constexpr int kMaxSplit = 160;              // >= grid: each CTA boundary splits at most one tile
constexpr int kMaxPieces = 320;             // >= split tiles + grid
constexpr int kSmemMax = 232448;            // 227 KB opt-in per CTA
// One tcgen05.commit per stage, onto sdone[stage % kSDone]; every waiter lags
// the MMA by fewer than kSDone stages, so a slot's parity cannot alias.
constexpr int kSDone = 32;

// ------------------------------------------------------------------ PTX
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B,
// 8-row groups 1024 B apart (SBO), LBO 16 B (unused for swizzled K-major),
// descriptor version 1, base offset 0 (tiles are 1024-byte aligned).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}
// Instruction descriptor, kind::f16: D f32, A/B f16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kRows >> 4) << 24);
}

// 32 lanes x 32 columns of 32 bit to TMEM (this warp's lane quarter).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Arrive once on `bar` when every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 16 columns of 32 bit from TMEM; the wait is tied to the outputs
// so no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

// ------------------------------------------------------------------ waits
// Bounded wait that also gives up as soon as another role has (abort flag).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > kSpinLimitCycles) {
            record_fault(ALJ_FAULT_TIMEOUT);
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void st_release_gpu(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The same wait by every lane of a warp, with one verdict for all of them.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    return __all_sync(0xffffffffu, wait_bar(bar, parity, abort_flag));
}

// Position in a ring of mbarriers: the slot and the parity of the phase its
// next waiter expects, advanced once per use (no division on the issue path).
struct Cursor {
    int slot;
    uint32_t phase;
    __device__ __forceinline__ void next(int n) {
        if (++slot == n) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

// ------------------------------------------------------------------ schedule
template <class P>
__device__ __forceinline__ long long unit_begin(const P& p, int c) {
    return static_cast<long long>(c) * p.units / p.grid;
}
// CTA whose unit range holds unit u.
template <class P>
__device__ __forceinline__ int cta_of(const P& p, long long u) {
    int c = static_cast<int>(u * p.grid / p.units);
    while (c + 1 < p.grid && unit_begin(p, c + 1) <= u) ++c;
    while (c > 0 && unit_begin(p, c) > u) --c;
    return c;
}
// Partial slot of CTA c's piece of tile t (a CTA has at most two split pieces:
// its first and its last tile).
template <class P>
__device__ __forceinline__ int slot_of(const P& p, int c, int t) {
    return 2 * c + (t == static_cast<int>(unit_begin(p, c) / p.units_per_tile) ? 0 : 1);
}

struct Piece {
    int t, seg, row0, tok0, c0, c1;   // tile, segment, first row in segment, token tile, unit range in tile
};
template <class P>
__device__ __forceinline__ Piece make_piece(const P& p, int t, long long u0, long long u1) {
    Piece pc;
    pc.t = t;
    const long long tb = static_cast<long long>(t) * p.units_per_tile;
    pc.c0 = static_cast<int>((u0 > tb ? u0 : tb) - tb);
    const long long te = tb + p.units_per_tile;
    pc.c1 = static_cast<int>((u1 < te ? u1 : te) - tb);
    const int rt = t / p.tok_tiles;
    pc.tok0 = (t % p.tok_tiles);
    int s = 0;
    while (s + 1 < p.nseg && rt >= p.seg[s + 1].tile0) ++s;
    pc.seg = s;
    pc.row0 = (rt - p.seg[s].tile0) * kRows;
    return pc;
}

// 2^-(f + e) as a float, for the output scale of token exponent f and
// segment exponent e (|f + e| stays well inside the normal range).
__device__ __forceinline__ float out_scale(int f, int e) { return __int_as_float((127 - f - e) << 23); }

// Sum the split tiles' partials (pieces in K order) into y, a share per thread
// of the whole grid.  Work item = 4 consecutive rows of one token of one
// split tile (a float4 of every piece's partial).  Q items per iteration and
// all their loads (B pieces at a time) in flight before the in-order sums, so
// a thread waits one L2 round trip per batch, not one per piece.
template <class P, int Q, int B>
__device__ __forceinline__ void reduce_items(const P& p, int MT) {
    const int vpt = MT * kRows / 4;
    const long long total = static_cast<long long>(p.nsplit) * vpt;
    const long long nthr = static_cast<long long>(gridDim.x) * blockDim.x;
    const float4* part4 = reinterpret_cast<const float4*>(p.partials);
    for (long long e0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e0 < total; e0 += Q * nthr) {
        int np[Q], off[Q], within[Q], item[Q];
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const long long e = e0 + q * nthr;
            const bool live = e < total;
            item[q] = live ? static_cast<int>(e / vpt) : -1;
            within[q] = live ? static_cast<int>(e - static_cast<long long>(item[q]) * vpt) : 0;
            np[q] = live ? p.split_n[item[q]] : 0;
            off[q] = live ? p.split_off[item[q]] : 0;
        }
        float4 acc[Q];
        int npm = 0;
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            npm = np[q] > npm ? np[q] : npm;
        }
        for (int k0 = 0; k0 < npm; k0 += B) {
            float4 a[Q][B];
#pragma unroll
            for (int q = 0; q < Q; ++q)
#pragma unroll
                for (int k = 0; k < B; ++k)
                    a[q][k] = k0 + k < np[q]
                                  ? __ldcg(part4 + static_cast<size_t>(p.piece_slot[off[q] + k0 + k]) * vpt + within[q])
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int q = 0; q < Q; ++q)
#pragma unroll
                for (int k = 0; k < B; ++k) {
                    acc[q].x += a[q][k].x;
                    acc[q].y += a[q][k].y;
                    acc[q].z += a[q][k].z;
                    acc[q].w += a[q][k].w;
                }
        }
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            if (item[q] < 0) continue;
            const int m = within[q] * 4 / kRows;            // token within the tile
            const int rr = within[q] * 4 - m * kRows;       // first of the 4 rows
            const Piece pc = make_piece(p, p.split_tile[item[q]], 0, p.units);
            const auto& sg = p.seg[pc.seg];
            const int tok = pc.tok0 * MT + m;
            if (tok >= p.M) continue;
            const float sc = out_scale(__ldg(p.tokexp + tok), p.exp_of(pc.seg));
            float* yr = sg.y + static_cast<size_t>(tok) * sg.ldy + pc.row0 + rr;
            const float v[4] = {acc[q].x, acc[q].y, acc[q].z, acc[q].w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (pc.row0 + rr + j < sg.rows) yr[j] = v[j] * sc;
        }
    }
}

// Sum the split tiles' partials into y, a share per thread of the whole grid.
// Out of line, so that its registers do not add to the pipeline roles'.
template <class P>
__device__ __noinline__ void reduce_split_tiles(const P& p, int MT) {
    const long long items = static_cast<long long>(p.nsplit) * (MT * kRows / 4);
    if (items <= static_cast<long long>(gridDim.x) * blockDim.x)
        reduce_items<P, 1, 16>(p, MT);       // few items, many pieces each (small matrices)
    else
        reduce_items<P, 2, 8>(p, MT);
}

// Split tiles: every CTA sums a share of their outputs over the pieces in K
// order (deterministic), after a grid barrier.  The launch is cooperative, so
// all CTAs are resident; the wait is bounded.  The barrier has no contended
// atomic: each CTA publishes its own flag (cleared to 0 by the activation
// prep kernel, hence the griddepcontrol.wait), then thread j polls CTA j's.
template <class P>
__device__ __forceinline__ void finish_split_tiles(const P& p, int MT, volatile int* abort_flag) {
    pdl_wait();
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        st_release_gpu(p.gbar + blockIdx.x, 1u);
    }
    if (threadIdx.x < gridDim.x) {
        const long long t0 = clock64();
        while (ld_acquire_gpu(p.gbar + threadIdx.x) == 0u) {
            if (clock64() - t0 > kSpinLimitCycles) {
                record_fault(ALJ_FAULT_TIMEOUT);
                *abort_flag = 1;
                break;
            }
        }
    }
    __syncthreads();
    if (*abort_flag) return;
    reduce_split_tiles(p, MT);
}

// ------------------------------------------------------------------ host
inline int token_tile_for(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                      uint64_t outer, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {inner * esize};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t es[2] = {1, 1};
    return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Grid size, and the tiles whose K range is split between CTAs with the
// partial slots of their pieces (summed after the grid barrier).  p.tiles,
// p.units_per_tile must be set.  False when the split tables overflow.
template <class P>
inline bool plan_stream_k(P& p, int sms) {
    p.units = static_cast<long long>(p.tiles) * p.units_per_tile;
    p.grid = static_cast<int>(std::min<long long>(std::min(sms, kMaxSplit), p.units));
    auto ub = [&](int c) { return static_cast<long long>(c) * p.units / p.grid; };
    auto cta_of_h = [&](long long u) {
        int c = static_cast<int>(u * p.grid / p.units);
        while (c + 1 < p.grid && ub(c + 1) <= u) ++c;
        while (c > 0 && ub(c) > u) --c;
        return c;
    };
    p.nsplit = 0;
    int npieces = 0;
    for (int t = 0; t < p.tiles; ++t) {
        const int cf = cta_of_h(static_cast<long long>(t) * p.units_per_tile);
        const int cl = cta_of_h(static_cast<long long>(t + 1) * p.units_per_tile - 1);
        if (cf == cl) continue;
        if (p.nsplit >= kMaxSplit || t > 65535 || npieces + (cl - cf + 1) > kMaxPieces) return false;
        p.split_tile[p.nsplit] = static_cast<unsigned short>(t);
        p.split_off[p.nsplit] = static_cast<unsigned short>(npieces);
        p.split_n[p.nsplit] = static_cast<unsigned short>(cl - cf + 1);
        for (int c = cf; c <= cl; ++c)   // slot of CTA c's piece of t: 2c, +1 unless t is c's first tile
            p.piece_slot[npieces++] = static_cast<unsigned short>(2 * c + (t == ub(c) / p.units_per_tile ? 0 : 1));
        ++p.nsplit;
    }
    return true;
}

}  // namespace tcg
}  // namespace alj
