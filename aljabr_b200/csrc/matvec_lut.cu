// Batch-1 NF4 dequantise-and-matvec (y = W x, bitsandbytes layout: two codes
// per byte, high nibble first, one fp32 absmax per `group` elements) on B200
// (sm_100a), for K a multiple of 2048 and group 64 or 128.
//
// NF4 values are 16 arbitrary constants, so a code cannot become a tensor-core
// operand with bit tricks; the work stays on the CUDA cores and is shaped so
// that each weight costs ~1.8 instructions:
//   * a 32 KB table in shared memory maps a code byte b to the float pair
//     (T[b >> 4], T[b & 15]), 16 copies (entry b, copy c at 128 b + 8 c): lane
//     l reads copy l % 16, so the 8-byte loads of a half warp (the unit in
//     which 8-byte shared loads are served) hit 16 distinct bank pairs
//     whatever the bytes are; a PRMT and a shift build the address
//     (b << 7 | 8 (l % 16)) from the code word.  The 32 KB the table does not
//     take (against one copy per lane) hold a fourth TMA stage;
//   * one packed f32x2 FMA per byte multiplies the pair with (x[2i], x[2i+1]);
//   * rows are dealt out in balanced units of 4 and walked in slabs of up to
//     32 rows (pair mode: 16 gate + 16 up rows) x chunks of 2048 columns; a
//     producer warp streams each slab-chunk with 2-D TMA boxes of 8 or 4 rows
//     (codes: 1024 B per row; absmax: 2048 / group floats per row) plus the
//     chunk of x as a 2-D box {32 floats, 64} with 128-byte swizzle, so the
//     16-byte x loads below are bank-conflict free;
//   * warp w covers column quarter w % 4 (512 columns, 16 per lane) of the
//     slab rows r with r % 4 == w / 4: x (16 floats per lane) is loaded once
//     per chunk and reused for up to 8 rows, each lane applies the absmax of
//     its 16 columns once per row;
//   * per-lane row partials are reduced across the warp with a butterfly at
//     the end of the slab, and the epilogue warp sums the four column quarters
//     in fixed order (deterministic), applying bias / residual / SwiGLU and
//     the optional last-CTA RMSNorm, as the tensor-core Q4_0 kernel does.
// Every mbarrier wait is bounded (ALJ_FAULT_TIMEOUT in the device fault word).
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>

namespace alj {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();   // matvec.cu

namespace {

constexpr int kCW = 16;
constexpr int kConsumers = kCW * 32;
constexpr int kProducerWarp = kCW;
constexpr int kEpilogueWarp = kCW + 1;
constexpr int kThreads = (kCW + 2) * 32;
constexpr int kUnit = 4;
constexpr int kSlabRows = 32;
constexpr int kChunkElems = 2048;
constexpr int kCodeRowBytes = kChunkElems / 2;             // 1024
constexpr int kXBytes = kChunkElems * 4;                   // 8 KB
constexpr int kLutCopies = 16;                             // one per lane of a half warp
constexpr int kLutBytes = 256 * kLutCopies * 8;            // 32 KB
constexpr int kMaxStages = 4;
constexpr int kRing = 4;
constexpr int kSmemMax = 232448;

__constant__ float kNf4[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

struct alignas(64) LutSegment {
    CUtensorMap codes8, codes4;     // box {128 x 8 B, 8 | 4 rows}
    CUtensorMap abs8, abs4;         // box {2048 / group floats, 8 | 4 rows}
    const float* bias;
    const float* residual;
    float* y;
    int rows;
    int row0;
};

struct alignas(64) LutParams {
    LutSegment seg[3];
    CUtensorMap xmap;               // x as [K / 32][32] floats, box {32, 64}, 128-byte swizzle
    int nseg;
    int K;
    int group;
    int total_rows;
    int pair;
    float* norm_out;
    const float* norm_w;
    float norm_eps;
    float* norm_partials;
    unsigned int* norm_counter;
    int norm_defer;
    const float* in_parts;
    int in_nparts;
    int in_rows;
    float in_eps;
    const uint8_t* prefetch;
    size_t prefetch_bytes;
    TpLink tpl;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint2 lds64u(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ f2 lds_pair(uint32_t a) {
    unsigned long long v;
    asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(a));
    return f2{v};
}
// Two packed f32x2 operands from 16 bytes of shared memory.
__device__ __forceinline__ void lds_pairs2(uint32_t a, f2& p0, f2& p1) {
    asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(p0.v), "=l"(p1.v) : "r"(a));
}
__device__ __forceinline__ f2 mul2f(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r.v) : "l"(a.v), "l"(b.v));
    return r;
}
__device__ __forceinline__ float lds32f(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}

// norm_out = y * scale * norm_w over the whole output, by the last CTA's
// consumer warps and epilogue warp (participant index 0 .. 16 * 32 + 31).
template <typename P>
__device__ __forceinline__ void norm_pass(const P& p, float scale, int idx) {
    const float* y = p.seg[0].y;
    for (int i = idx; i < p.total_rows; i += kCW * 32 + 32) p.norm_out[i] = __ldcg(y + i) * scale * p.norm_w[i];
}

// Row geometry of a launch, read from the parameters once at kernel start
// (independent loads, one round trip) instead of by each walk step.
struct SlabGeom {
    int total_rows, pair, nseg;
    int row0[3], rows[3];
};
__device__ __forceinline__ SlabGeom slab_geom(const LutParams& p) {
    SlabGeom g;
    g.total_rows = p.total_rows;
    g.pair = p.pair;
    g.nseg = p.nseg;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        g.row0[i] = p.seg[i].row0;
        g.rows[i] = p.seg[i].rows;
    }
    return g;
}

struct SlabWalk {
    int u, u_end;
    __device__ __forceinline__ bool next(const SlabGeom& p, int& seg, int& su, int& nunits) {
        if (u >= u_end) return false;
        seg = 0;
        int seg_end = p.total_rows / kUnit;
        if (!p.pair) {
            if (p.nseg > 1 && u * kUnit >= p.row0[1]) seg = 1;
            if (p.nseg > 2 && u * kUnit >= p.row0[2]) seg = 2;
            seg_end = (p.row0[seg] + p.rows[seg]) / kUnit;
        }
        su = u;
        nunits = min(p.pair ? kSlabRows / (2 * kUnit) : kSlabRows / kUnit, min(u_end, seg_end) - u);
        u += nunits;
        return true;
    }
};

struct StageLayout {
    int abs_row_bytes;   // 4 * 2048 / group
    int abs_off;         // codes: 32 rows x 1024 B
    int x_off;           // 1024-aligned
    int bytes;
};
__host__ __device__ inline StageLayout stage_layout(int group) {
    StageLayout L;
    L.abs_row_bytes = 4 * (kChunkElems / group);
    L.abs_off = kSlabRows * kCodeRowBytes;
    L.x_off = (L.abs_off + kSlabRows * L.abs_row_bytes + 1023) & ~1023;
    L.bytes = L.x_off + kXBytes;
    return L;
}

// The boxes of `nunits` 4-row units starting at segment row r0, into slab
// rows [srow, srow + 4 nunits), one per lane: lane 2b takes the code box of
// units 2b, 2b + 1 (8 rows, or 4 for a last single unit), lane 2b + 1 its
// absmax box.  Lanes past the slab's boxes issue nothing.
__device__ __forceinline__ void load_rows_lane(int lane, const LutSegment& sg, int r0, int nunits, int srow,
                                               int chunk, uint32_t st, const StageLayout& L, int abs_elems,
                                               uint64_t* bar) {
    const int u = 2 * (lane >> 1);
    if (u >= nunits) return;
    const bool eight = nunits - u >= 2;
    const int rr = srow + u * kUnit;
    if ((lane & 1) == 0)
        tma_load_2d(st + rr * kCodeRowBytes, eight ? &sg.codes8 : &sg.codes4, chunk * (kCodeRowBytes / 8),
                    r0 + u * kUnit, bar);
    else
        tma_load_2d(st + L.abs_off + rr * L.abs_row_bytes, eight ? &sg.abs8 : &sg.abs4, chunk * abs_elems,
                    r0 + u * kUnit, bar);
}

template <int GROUP>
__global__ void __launch_bounds__(kThreads, 1) nf4_lut_kernel(const __grid_constant__ LutParams p, int stages) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    // x's descriptor on its way (the weight boxes go out first thing below)
    if (threadIdx.x == (kProducerWarp << 5)) prefetch_tensormap(&p.xmap);
    pdl_launch_dependents();
    const SlabGeom geo = slab_geom(p);
    const int K = p.K;
    const int nchunks = K / kChunkElems;
    const StageLayout L = stage_layout(GROUP);
    constexpr int kAbsElems = kChunkElems / GROUP;
    // [0, 32 KB) table | stages (1024-aligned) | ring | misc | barriers
    const uint32_t lut_s = smem_u32(smem_raw);
    const uint32_t base = lut_s + kLutBytes;
    const uint32_t stage_s = (base + 1023u) & ~1023u;
    uint8_t* after = smem_raw + (stage_s - lut_s) + static_cast<size_t>(stages) * L.bytes;
    float* red = reinterpret_cast<float*>(after);      // [kRing][kCW][8]
    float* misc = red + kRing * kCW * 8;
    uint64_t* full = reinterpret_cast<uint64_t*>(misc + 16);
    uint64_t* empty = full + kMaxStages;
    uint64_t* rfull = empty + kMaxStages;
    uint64_t* rempty = rfull + kRing;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = geo.total_rows / kUnit;
    // units <= 2^15 (rows <= 131072), so 32-bit products suffice
    const int u_begin = static_cast<int>(static_cast<unsigned int>(units) * blockIdx.x / gridDim.x);
    const int u_end = static_cast<int>(static_cast<unsigned int>(units) * (blockIdx.x + 1) / gridDim.x);

    // The producer warp initialises the barriers and goes straight on to its
    // first copies; the other warps wait on named barrier 3 (all threads)
    // before they touch a barrier.
    if (warp == kProducerWarp) {
        if (lane == 0) {
            for (int s = 0; s < stages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], kCW);
            }
            for (int b = 0; b < kRing; ++b) {
                mbar_init(&rfull[b], kCW);
                mbar_init(&rempty[b], 1);
            }
            fence_mbar_init();
        }
        __syncwarp();
        named_bar_arrive(3, kThreads);
    } else {
        named_bar(3, kThreads);
    }

    if (warp == kProducerWarp) {
        // The whole warp walks the slabs; lane 0 waits and arms, the box
        // copies of a stage go out one per lane.  The first `stages` fills
        // use fresh slots (no wait).
        SlabWalk walk{u_begin, u_end};
        int seg, su, nunits, s = 0, issued = 0;
        uint32_t ph = 0;
        bool alive = true;
        bool x_waited = false;
        while (alive && walk.next(geo, seg, su, nunits)) {
            const int rows = nunits * kUnit * (p.pair ? 2 : 1);
            for (int c = 0; c < nchunks; ++c) {
                if (issued >= stages) {
                    int ok = 1;
                    if (lane == 0) ok = mbar_wait(&empty[s], ph ^ 1u) ? 1 : 0;
                    if (!__shfl_sync(0xffffffffu, ok, 0)) {
                        alive = false;
                        break;
                    }
                }
                const uint32_t st = stage_s + s * L.bytes;
                if (lane == 0)
                    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(rows * (kCodeRowBytes + L.abs_row_bytes) + kXBytes));
                __syncwarp();
                if (p.pair) {
                    if (lane < 8)
                        load_rows_lane(lane, p.seg[0], su * kUnit, nunits, 0, c, st, L, kAbsElems, &full[s]);
                    else if (lane < 16)
                        load_rows_lane(lane - 8, p.seg[1], su * kUnit, nunits, kSlabRows / 2, c, st, L, kAbsElems,
                                       &full[s]);
                } else if (lane < 8) {
                    load_rows_lane(lane, p.seg[seg], su * kUnit - p.seg[seg].row0, nunits, 0, c, st, L, kAbsElems,
                                   &full[s]);
                }
                if (lane == 0) {
                    // x comes from the previous kernel: its first copy waits for it.
                    if (!x_waited) {
                        pdl_wait();
                        // tensor parallel: x is gathered from every rank's push
                        if (p.tpl.tp > 1 && p.tpl.wait_flags) {
                            wait_flags_sys(p.tpl.wait_flags, p.tpl.tp,
                                           static_cast<unsigned int>(*p.tpl.seq * p.tpl.wait_mul + p.tpl.wait_add));
                            fence_proxy_async_global();
                        }
                    }
                    tma_load_2d(st + L.x_off, &p.xmap, 0, c * (kChunkElems / 32), &full[s]);
                }
                x_waited = true;
                ++issued;
                if (++s == stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        if (lane == 0 && alive && p.prefetch) prefetch_share(p.prefetch, p.prefetch_bytes);
        return;
    }

    if (warp == kEpilogueWarp) {
        pdl_wait();
        // deferred RMSNorm of x: its scale from the producer's partials (fixed order)
        float in_s = 1.0f;
        if (p.in_parts) {
            float part = 0.0f;
            for (int b = lane; b < p.in_nparts; b += 32) part += __ldcg(p.in_parts + b);
            in_s = 1.0f / sqrtf(warp_sum(part) / static_cast<float>(p.in_rows) + p.in_eps);
        }
        SlabWalk walk{u_begin, u_end};
        int seg, su, nunits, sl = 0;
        float sq = 0.0f;
        while (walk.next(geo, seg, su, nunits)) {
            const int b = sl % kRing;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&rfull[b], (sl / kRing) & 1));
            if (ok) {
                // slab row r: row group r % 4, slot r / 4; the four column quarters in order
                const int i = lane & 3, j = lane >> 2;
                float acc = 0.0f;
#pragma unroll
                for (int q = 0; q < 4; ++q) acc += red[(b * kCW + 4 * i + q) * 8 + j];
                acc *= in_s;
                if (p.pair) {
                    const float up = __shfl_down_sync(0xffffffffu, acc, 16);
                    if (lane < nunits * kUnit) {
                        const float out = acc / (1.0f + expf(-acc)) * up;
                        if (p.tpl.tp > 1) {
                            for (int r = 0; r < p.tpl.tp; ++r) p.tpl.push_y[r][su * kUnit + lane] = out;
                        } else {
                            p.seg[0].y[su * kUnit + lane] = out;
                        }
                        sq = fmaf(out, out, sq);
                    }
                } else if (lane < nunits * kUnit) {
                    const LutSegment& sg = p.seg[seg];
                    const int lrow = su * kUnit + lane - sg.row0;
                    float out = acc;
                    if (sg.bias) out += sg.bias[lrow];
                    if (sg.residual) out = sg.residual[lrow] + out;
                    if (p.tpl.tp > 1) {
                        for (int r = 0; r < p.tpl.tp; ++r) p.tpl.push_y[r][lrow] = out;
                    } else {
                        sg.y[lrow] = out;
                    }
                    if (p.norm_defer) p.norm_out[lrow] = out * p.norm_w[lrow];
                    sq = fmaf(out, out, sq);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rempty[b]);
            ++sl;
        }
        if (p.tpl.tp > 1) {
            // Publish this rank's slice: the last CTA to finish writes the
            // rank's sum of squares (fixed order over the CTAs) and the flag
            // value on every rank, after a system-scope fence that covers
            // every CTA's peer stores.
            __threadfence_system();
            const float cta = warp_sum(sq);
            if (lane == 0) {
                p.norm_partials[blockIdx.x] = cta;
                __threadfence_system();
                const unsigned int prev = atomicAdd(p.tpl.counter, 1u);
                misc[1] = prev == gridDim.x - 1 ? 1.0f : 0.0f;
            }
            __syncwarp();
            if (misc[1] != 0.0f) {
                __threadfence_system();
                float part = 0.0f;
                for (unsigned int b = lane; b < gridDim.x; b += 32) part += __ldcg(p.norm_partials + b);
                const float tot = warp_sum(part);
                if (lane < p.tpl.tp && p.tpl.push_part[lane]) *p.tpl.push_part[lane] = tot;
                __threadfence_system();
                if (lane < p.tpl.tp)
                    st_release_sys(p.tpl.push_flag[lane],
                                   static_cast<unsigned int>(*p.tpl.seq * p.tpl.push_mul + p.tpl.push_add));
                if (lane == 0) *p.tpl.counter = 0u;
            }
        }
        if (p.norm_out && p.norm_defer) {
            // the consuming launch sums the partials and applies the scale
            const float cta = warp_sum(sq);
            if (lane == 0) p.norm_partials[blockIdx.x] = cta;
        } else if (p.norm_out) {
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
                    misc[0] = 1.0f / sqrtf(tot / static_cast<float>(p.total_rows) + p.norm_eps);
                    *p.norm_counter = 0u;
                }
            }
            named_bar(2, kCW * 32 + 32);
            if (misc[1] != 0.0f) norm_pass(p, misc[0], kCW * 32 + lane);
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    {
        // Byte-pair table, 16 copies: entry b, copy c at 128 b + 8 c.
        float2* lut = reinterpret_cast<float2*>(smem_raw);
        // lane l holds T[l % 16]; the pair of entry b comes from two shuffles
        const float tl = kNf4[lane & 15];
        for (int e = threadIdx.x; e < 256 * kLutCopies; e += kConsumers) {
            const int b = e >> 4;
            lut[e] = make_float2(__shfl_sync(0xffffffffu, tl, b >> 4), __shfl_sync(0xffffffffu, tl, b & 15));
        }
        named_bar(1, kConsumers);
    }
    const int q = warp & 3;                 // column quarter: columns [512 q, 512 q + 512) of a chunk
    const int rg = warp >> 2;               // rows rg, rg + 4, ... of the slab
    // table address (b << 7 | (lane % 16) << 3) = PRMT(b << 8 | (lane % 16) << 4) >> 1
    const uint32_t lane16 = static_cast<uint32_t>(lane & 15) * 16u;
    const uint32_t code_off = q * 256 + lane * 8;                           // this lane's 8 code bytes
    const uint32_t abs_off = L.abs_off + ((q * 512 + lane * 16) / GROUP) * 4;
    uint32_t xoff[4];                                                       // swizzled x granules
    {
        const uint32_t xrow = q * 16 + (lane >> 1);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t gran = (lane & 1) * 4 + k;
            xoff[k] = L.x_off + xrow * 128 + ((gran ^ (xrow & 7)) << 4);
        }
    }

    constexpr int kAbsRowBytes = 4 * (kChunkElems / GROUP);
    SlabWalk walk{u_begin, u_end};
    int seg, su, nunits, s = 0, sl = 0;
    uint32_t ph = 0;
    while (walk.next(geo, seg, su, nunits)) {
        // slab rows with data: pair mode holds gate rows [0, 4n) and up rows [16, 16 + 4n)
        const int valid = nunits * kUnit;
        const bool all_live = p.pair ? rg + 12 < valid : rg + 28 < valid;   // warp-uniform
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
        for (int c = 0; c < nchunks; ++c) {
            if (__all_sync(0xffffffffu, mbar_wait(&full[s], ph))) {
                const uint32_t st = stage_s + s * L.bytes;
                // x of this lane's 16 columns as 8 packed pairs, loaded once for all rows
                f2 xp[8];
#pragma unroll
                for (int k = 0; k < 4; ++k) lds_pairs2(st + xoff[k], xp[2 * k], xp[2 * k + 1]);
                const uint32_t code_base = st + rg * kCodeRowBytes + code_off;      // row rg; row rg + 4j at + 4096 j
                const uint32_t abs_base = st + abs_off + rg * kAbsRowBytes;
                // one row: 8 code bytes -> 8 table pairs -> 8 packed multiply-adds
                auto row_dot = [&](uint2 w, float am, float a) {
                    f2 t[8];
#pragma unroll
                    for (int m = 0; m < 8; ++m) {
                        const uint32_t word = m < 4 ? w.x : w.y;
                        t[m] = lds_pair(lut_s + (__byte_perm(word, lane16, 0x5504u | (static_cast<uint32_t>(m & 3) << 4)) >> 1));
                    }
                    f2 A = mul2f(t[0], xp[0]), B = mul2f(t[1], xp[1]);
#pragma unroll
                    for (int m = 2; m < 8; m += 2) {
                        A = fma2(t[m], xp[m], A);
                        B = fma2(t[m + 1], xp[m + 1], B);
                    }
                    const f2 t2 = add2(A, B);
                    return fmaf(am, lo(t2) + hi(t2), a);
                };
                if (all_live) {
                    // the next row's code word is read before this row's table loads
                    uint2 w = lds64u(code_base);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint2 wj = w;
                        if (j < 7) w = lds64u(code_base + (j + 1) * 4 * kCodeRowBytes);
                        const float am = lds32f(abs_base + j * 4 * kAbsRowBytes);
                        acc[j] = row_dot(wj, am, acc[j]);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const int r = rg + 4 * j;
                        if (p.pair ? ((r & 15) < valid) : (r < valid))
                            acc[j] = row_dot(lds64u(code_base + j * 4 * kCodeRowBytes),
                                             lds32f(abs_base + j * 4 * kAbsRowBytes), acc[j]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == stages) {
                s = 0;
                ph ^= 1u;
            }
        }
        // Butterfly: after it, lane j (j < 8) holds slot j's sum over the warp.
#pragma unroll
        for (int j = 0; j < 4; ++j) {   // xor 16: lanes < 16 keep slots 0..3, others 4..7
            const float mine = lane < 16 ? acc[j] : acc[j + 4];
            const float other = lane < 16 ? acc[j + 4] : acc[j];
            acc[j] = mine + __shfl_xor_sync(0xffffffffu, other, 16);
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {   // xor 8
            const bool up = (lane & 8) != 0;
            const float mine = up ? acc[j + 2] : acc[j];
            const float other = up ? acc[j] : acc[j + 2];
            acc[j] = mine + __shfl_xor_sync(0xffffffffu, other, 8);
        }
        {                               // xor 4
            const bool up = (lane & 4) != 0;
            const float mine = up ? acc[1] : acc[0];
            const float other = up ? acc[0] : acc[1];
            acc[0] = mine + __shfl_xor_sync(0xffffffffu, other, 4);
        }
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 2);
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], 1);
        // lane L now holds slot (L>>4)*4 + ((L>>3)&1)*2 + ((L>>2)&1); lanes 4m hold distinct slots
        const int b = sl % kRing;
        mbar_wait(&rempty[b], ((sl / kRing) & 1) ^ 1u);
        if ((lane & 3) == 0) {
            const int slot = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
            red[(b * kCW + warp) * 8 + slot] = acc[0];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfull[b]);
        ++sl;
    }
    if (p.norm_out && !p.norm_defer) {
        named_bar(2, kCW * 32 + 32);
        if (misc[1] != 0.0f) norm_pass(p, misc[0], threadIdx.x);
    }
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, cuuint64_t inner, cuuint64_t rows,
               cuuint64_t row_bytes, cuuint32_t box_inner, cuuint32_t box_rows, CUtensorMapSwizzle swz) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t smem_bytes(int group, int stages) {
    return kLutBytes + 1024 + static_cast<size_t>(stages) * stage_layout(group).bytes + kRing * kCW * 8 * 4 + 16 * 4 +
           (2 * kMaxStages + 2 * kRing) * 8;
}

}  // namespace

int matvec_lut_grid(int total_rows) {
    return std::max(1, std::min(sm_count_for_current_device(), total_rows / kUnit));
}

bool matvec_lut_supported(int fmt, int K, int group) {
    if (fmt != FMT_NF4 || K <= 0 || K % kChunkElems != 0 || (group != 64 && group != 128)) return false;
    return tensor_map_encoder() != nullptr && smem_bytes(group, 2) <= static_cast<size_t>(kSmemMax);
}

cudaError_t launch_matvec_lut(int fmt, const MatvecParams& mp, cudaStream_t stream, bool pdl) {
    if (!matvec_lut_supported(fmt, mp.K, mp.group)) return cudaErrorNotSupported;
    const bool pair = mp.epilogue == EPI_SWIGLU_PAIR;
    if (pair && (mp.nseg != 2 || mp.seg[0].rows != mp.seg[1].rows || mp.total_rows != mp.seg[0].rows))
        return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(mp.x) & 15) != 0) return cudaErrorNotSupported;
    for (int s = 0; s < mp.nseg; ++s)
        if (mp.seg[s].rows % kUnit != 0 || (reinterpret_cast<uintptr_t>(mp.seg[s].w) & 15) != 0 ||
            (reinterpret_cast<uintptr_t>(mp.seg[s].absmax) & 15) != 0)
            return cudaErrorNotSupported;
    LutParams p;
    memset(&p, 0, sizeof p);
    p.nseg = mp.nseg;
    p.K = mp.K;
    p.group = mp.group;
    p.total_rows = mp.total_rows;
    p.pair = pair ? 1 : 0;
    p.norm_out = mp.norm_out;
    p.norm_w = mp.norm_w;
    p.norm_eps = mp.norm_eps;
    p.norm_partials = mp.norm_partials;
    p.norm_counter = mp.norm_counter;
    p.norm_defer = mp.norm_defer;
    p.in_parts = mp.in_parts;
    p.in_nparts = mp.in_nparts;
    p.in_rows = mp.in_rows;
    p.in_eps = mp.in_eps;
    if ((p.norm_defer && (!p.norm_out || !p.norm_w || !p.norm_partials || mp.nseg != 1)) ||
        (p.in_parts && (p.in_nparts <= 0 || p.in_rows <= 0)))
        return cudaErrorInvalidValue;
    p.prefetch = static_cast<const uint8_t*>(mp.prefetch);
    p.prefetch_bytes = mp.prefetch_bytes;
    p.tpl = mp.tpl;
    if (p.tpl.tp > 1 && (p.tpl.tp > kMaxTp || !p.tpl.counter || !p.tpl.seq || !p.norm_partials || mp.nseg > 2 ||
                         (mp.nseg == 2 && !pair) || p.norm_out))
        return cudaErrorInvalidValue;
    const cuuint32_t abs_elems = static_cast<cuuint32_t>(kChunkElems / mp.group);
    int row0 = 0;
    for (int s = 0; s < mp.nseg; ++s) {
        LutSegment& ls = p.seg[s];
        const MatvecSegment& sg = mp.seg[s];
        const cuuint64_t rows = static_cast<cuuint64_t>(sg.rows);
        const cuuint64_t row_bytes = static_cast<cuuint64_t>(mp.K) / 2;
        const cuuint64_t abs_row = static_cast<cuuint64_t>(mp.K / mp.group);
        if (!encode_2d(&ls.codes8, CU_TENSOR_MAP_DATA_TYPE_UINT64, sg.w, row_bytes / 8, rows, row_bytes, 128, 8,
                       CU_TENSOR_MAP_SWIZZLE_NONE) ||
            !encode_2d(&ls.codes4, CU_TENSOR_MAP_DATA_TYPE_UINT64, sg.w, row_bytes / 8, rows, row_bytes, 128, 4,
                       CU_TENSOR_MAP_SWIZZLE_NONE) ||
            !encode_2d(&ls.abs8, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, sg.absmax, abs_row, rows, abs_row * 4, abs_elems, 8,
                       CU_TENSOR_MAP_SWIZZLE_NONE) ||
            !encode_2d(&ls.abs4, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, sg.absmax, abs_row, rows, abs_row * 4, abs_elems, 4,
                       CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
        ls.bias = sg.bias;
        ls.residual = sg.residual;
        ls.y = sg.y;
        ls.rows = sg.rows;
        ls.row0 = pair ? 0 : row0;
        row0 += sg.rows;
    }
    if (!encode_2d(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, mp.x, 32, static_cast<cuuint64_t>(mp.K / 32), 128, 32, 64,
                   CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    int stages = kMaxStages;
    while (stages > 2 && smem_bytes(mp.group, stages) > static_cast<size_t>(kSmemMax)) --stages;
    const size_t smem = smem_bytes(mp.group, stages);
    auto kern = mp.group == 64 ? nf4_lut_kernel<64> : nf4_lut_kernel<128>;
    static bool configured[2][64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    bool& done = configured[mp.group == 64 ? 0 : 1][dev & 63];
    if (!done) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        done = true;
    }
    const int grid = matvec_lut_grid(mp.total_rows);
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
