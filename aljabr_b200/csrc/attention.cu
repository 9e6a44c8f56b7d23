// Grouped-query decode attention for one token over a KV cache (fp32 or
// bf16), as GgufDecodeAttentionExecution.execute computes it
// (engine/gguf/aljabr-gguf-java/.../GgufDecodeAttentionExecution.java:70-106):
// for each query head h, kv head h / (Hq / Hkv), scores = (q . k_p) * scale
// over positions [start, seq), softmax, output = sum_p softmax_p * v_p.
//
// Fast path (head_dim 64/128/256, group size <= 8): split-K flash decoding.
//   grid = (kv_heads, splits); each CTA streams its slice of positions of
//   one kv head once and serves all G = Hq/Hkv query heads that share it.
//   Inside a warp, lane l owns head-dim slice [l*E, l*E+E) (E = D/32), so a
//   K or V row is one coalesced warp load.  A warp takes P = 32/G positions
//   per step: each lane forms P*G partial dots, one 31-shuffle
//   reduce-scatter leaves lane j with the full score of (position j/G,
//   head j%G), the online-softmax statistics are reduced over the lanes of
//   each head, and the probabilities are broadcast back for the V update.
//   Partial (max, sum, unnormalised output) per split go to scratch and a
//   combine kernel merges them with the usual log-sum-exp rescaling.
// Other shapes run a plain three-pass kernel (one CTA per query head).
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

namespace alj {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();   // matvec.cu

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kAttnWarps = 4;

template <int KVT>
__device__ __forceinline__ void load_row(const void* base, long long off, int E, float* dst);

// E elements starting at element offset `off` (E in {2,4,8}).
template <>
__device__ __forceinline__ void load_row<ALJ_KV_BF16>(const void* base, long long off, int E, float* dst) {
    const uint16_t* p = static_cast<const uint16_t*>(base) + off;
    if (E == 2) {
        const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
        dst[0] = __uint_as_float(u << 16); dst[1] = __uint_as_float(u & 0xFFFF0000u);
    } else if (E == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        dst[0] = __uint_as_float(u.x << 16); dst[1] = __uint_as_float(u.x & 0xFFFF0000u);
        dst[2] = __uint_as_float(u.y << 16); dst[3] = __uint_as_float(u.y & 0xFFFF0000u);
    } else {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        dst[0] = __uint_as_float(u.x << 16); dst[1] = __uint_as_float(u.x & 0xFFFF0000u);
        dst[2] = __uint_as_float(u.y << 16); dst[3] = __uint_as_float(u.y & 0xFFFF0000u);
        dst[4] = __uint_as_float(u.z << 16); dst[5] = __uint_as_float(u.z & 0xFFFF0000u);
        dst[6] = __uint_as_float(u.w << 16); dst[7] = __uint_as_float(u.w & 0xFFFF0000u);
    }
}
template <>
__device__ __forceinline__ void load_row<ALJ_KV_F32>(const void* base, long long off, int E, float* dst) {
    const float* p = static_cast<const float*>(base) + off;
    if (E == 2) {
        const float2 v = *reinterpret_cast<const float2*>(p);
        dst[0] = v.x; dst[1] = v.y;
    } else {
        for (int i = 0; i < E; i += 4) {
            const float4 v = *reinterpret_cast<const float4*>(p + i);
            dst[i] = v.x; dst[i + 1] = v.y; dst[i + 2] = v.z; dst[i + 3] = v.w;
        }
    }
}

// Reduce-scatter of 32 values across the warp: afterwards v[0] of lane j
// holds the warp-wide sum of everyone's v[j].
__device__ __forceinline__ void reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
    for (int h = 16; h >= 1; h >>= 1) {
        const bool upper = (lane & h) != 0;
#pragma unroll
        for (int i = 0; i < h; ++i) {
            const float send = upper ? v[i] : v[i + h];
            const float keep = upper ? v[i + h] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, h);
        }
    }
}

// Merge the per-warp softmax state of one CTA -- running max (natural-log
// units), running sum and unnormalised output, in shared memory as
// [warp][head slot] with `gs` slots per warp -- and store the split's
// partials, or the normalised output when there is a single split.
template <int D>
__device__ __forceinline__ void merge_warps_store(const AttnParams& p, const float* s_ml, const float* s_o, int gs, int G,
                                                  int kvh, int split) {
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx - g * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_ml[(w * gs + g) * 2]);
        float L = 0.0f, acc = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            const float mw = s_ml[(w * gs + g) * 2];
            const float f = mw == -INFINITY ? 0.0f : exp2f((mw - M) * kLog2e);
            L = fmaf(s_ml[(w * gs + g) * 2 + 1], f, L);
            acc = fmaf(s_o[(w * gs + g) * D + d], f, acc);
        }
        const int qh = kvh * G + g;
        if (p.splits == 1) {
            p.out[qh * D + d] = L > 0.0f ? acc / L : 0.0f;
        } else {
            p.part_o[(static_cast<long long>(qh) * p.splits + split) * D + d] = acc;
            if (d == 0) {
                p.part_ml[(static_cast<long long>(qh) * p.splits + split) * 2] = M;
                p.part_ml[(static_cast<long long>(qh) * p.splits + split) * 2 + 1] = L;
            }
        }
    }
}

template <int KVT, int E, int G>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(const AttnParams p) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int D = 32 * E;
    constexpr int P = 32 / G;           // positions per warp step
    const int kvh = blockIdx.x;
    const int split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int seq_len = p.dev_pos ? *p.dev_pos + 1 : p.seq_len;
    const int active = seq_len - p.start_pos;
    const int c0 = p.start_pos + static_cast<int>(static_cast<long long>(active) * split / p.splits);
    const int c1 = p.start_pos + static_cast<int>(static_cast<long long>(active) * (split + 1) / p.splits);

    float q[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < E; ++e) q[g][e] = p.q[(kvh * G + g) * D + lane * E + e];

    // lane j's statistics describe head (j % G); every lane of a head holds the same values
    float m = -INFINITY, l = 0.0f;
    float o[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < E; ++e) o[g][e] = 0.0f;

    const long long head_off = static_cast<long long>(kvh) * p.head_stride + lane * E;
    for (int p0 = c0 + warp * P; p0 < c1; p0 += kAttnWarps * P) {
        float kr[P][E], vr[P][E];
#pragma unroll
        for (int i = 0; i < P; ++i) {
            const int pos = min(p0 + i, c1 - 1);
            const long long off = static_cast<long long>(pos) * p.stride + head_off;
            load_row<KVT>(p.k, off, E, kr[i]);
            load_row<KVT>(p.v, off, E, vr[i]);
        }
        float s[32];
#pragma unroll
        for (int i = 0; i < P; ++i)
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float a = 0.0f;
#pragma unroll
                for (int e = 0; e < E; ++e) a = fmaf(q[g][e], kr[i][e], a);
                s[i * G + g] = a;
            }
        reduce_scatter32(s, lane);
        // lane j: position p0 + j / G, head j % G
        const bool valid = p0 + lane / G < c1;
        float sc = valid ? s[0] * p.scale : -INFINITY;
        float mx = sc;
#pragma unroll
        for (int o2 = G; o2 < 32; o2 <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
        const float m_new = fmaxf(m, mx);
        const float alpha = exp2f((m - m_new) * kLog2e);
        const float pr = valid ? exp2f((sc - m_new) * kLog2e) : 0.0f;
        float ps = pr;
#pragma unroll
        for (int o2 = G; o2 < 32; o2 <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o2);
        l = l * alpha + ps;
        m = m_new;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float ag = __shfl_sync(0xffffffffu, alpha, g);
#pragma unroll
            for (int e = 0; e < E; ++e) o[g][e] *= ag;
        }
#pragma unroll
        for (int i = 0; i < P; ++i)
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float w = __shfl_sync(0xffffffffu, pr, i * G + g);
#pragma unroll
                for (int e = 0; e < E; ++e) o[g][e] = fmaf(w, vr[i][e], o[g][e]);
            }
    }

    // merge the warps of this CTA through shared memory
    __shared__ float s_ml[kAttnWarps][G][2];
    __shared__ float s_o[kAttnWarps][G][D];
    if (lane < G) {
        s_ml[warp][lane][0] = m;
        s_ml[warp][lane][1] = l;
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < E; ++e) s_o[warp][g][lane * E + e] = o[g][e];
    __syncthreads();
    merge_warps_store<D>(p, &s_ml[0][0][0], &s_o[0][0][0], G, G, kvh, split);
}

// ---------------------------------------------------------------- tensor-core split kernel
// bf16 caches with head_dim 64 or 128 and up to 8 query heads per kv head.
// The shuffle formulation above spends ~15 warp instructions per (position,
// head) pair, which leaves it issue-bound well below the HBM rate; here both
// products run on mma.sync.m16n8k16 (bf16 operands, f32 accumulation):
//   * the split's K/V rows arrive by TMA as 32-row boxes of 64-element
//     halves (128-byte swizzle, so the ldmatrix reads below are free of bank
//     conflicts), each box completing on its own mbarrier;
//   * fp32 accuracy from bf16 operands: the query (times scale * log2 e) and
//     the probabilities are each split into three bf16 parts x = h + m + l
//     (|x - h - m - l| <= 2^-26 |x|) while K and V are exact in bf16.  With
//     G <= 4 heads the three parts share one A operand (rows [0, G) = h,
//     [G, 2G) = m, [8, 8 + G) = l), and a shuffle joins the m rows to the
//     others; with 5..8 heads two MMAs run per step, [h ; m] and [l ; 0];
//   * scores: B = 8 cached positions of K straight from shared memory; the
//     accumulator of a lane holds its head's score for two positions;
//   * a warp owns every W-th 16-position chunk of the split and keeps all
//     its scores in registers; the warps agree on each head's CTA-wide
//     maximum once, so their partial sums add without rescaling; the score
//     accumulator layout is the A-operand layout of the next product;
//   * output: B = V rows through ldmatrix.trans, accumulated over the warp's
//     chunks in 64 (head_dim 128) registers;
//   * the warps' sums add in shared memory into the split's partial; then
//     either the splits of a kv head form one thread-block cluster and merge
//     over distributed shared memory, or the last CTA of a kv head (a
//     per-head arrival counter) merges them from global memory -- no second
//     kernel either way.
constexpr int kMaxSplits = 256;
constexpr int kBoxRows = 32;     // positions per TMA box and per staging barrier
constexpr int kMaxBoxes = 6;     // at most 192 positions per split
constexpr int kChunkRows = 16;
constexpr int kMmaSmemMax = 2 * kMaxBoxes * kBoxRows * 128 * 2 + 1024;   // K + V at head_dim 128, + alignment
// The cluster variant: the splits of one kv head form one thread-block
// cluster (up to 16 CTAs, one SM each) and merge over distributed shared
// memory -- no partials in global memory, no arrival counter.
constexpr int kClusterMax = 16;
constexpr int kClusterBoxes = 13;   // at most 416 positions per split
constexpr int kClusterWarps = 8;
constexpr int kPartFloats = 1536;   // pushed partials: [splits][items / splits] float4 + [splits][8] (max, sum)
constexpr int kClusterSmemMax = 2 * kClusterBoxes * kBoxRows * 128 * 2 + kPartFloats * 4 + 1024;

struct KvMaps {
    CUtensorMap k;      // bf16 cache viewed as [rows][kv_heads][head_dim / 64][64]
    CUtensorMap v;
};
struct AttnMmaParams {  // host side: what one launch of the kernel takes
    KvMaps maps;
    AttnParams a;
    int cap_rows;       // staged rows per split: a multiple of kBoxRows, >= the longest split
    int merge_smem;     // the split merge copies the partial outputs into shared memory
};

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t a, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a)
                 : "memory");
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// Distributed shared memory: this CTA's shared address `a` in cluster CTA
// `rank`, and stores there.
__device__ __forceinline__ uint32_t cluster_map(uint32_t a, int rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f2(uint32_t a, float2 v) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(v.x), "f"(v.y) : "memory");
}
__device__ __forceinline__ void st_cluster_f4(uint32_t a, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
// The value, held in a register from here on: the compiler otherwise reads
// kernel parameters again where they are used, and a late read of the
// parameter bank can miss its cache.
__device__ __forceinline__ int pin_reg(int v) {
    asm volatile("" : "+r"(v));
    return v;
}
template <typename T>
__device__ __forceinline__ T* pin_reg(T* v) {
    asm volatile("" : "+l"(v));
    return v;
}
// Split cluster barrier without ordering: arrive early, wait before the
// first access to another CTA's shared memory (all CTAs have started then).
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// Every thread of every CTA of the cluster: stores before it are visible to
// loads after it anywhere in the cluster (a hardware barrier, no spin).
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t bf16x2_bits(__nv_bfloat162 v) { return *reinterpret_cast<const uint32_t*>(&v); }
// Three-part bf16 split of (x0, x1): pairs packed as MMA operands (x0 low).
struct Split3 {
    uint32_t h, m, l;
};
__device__ __forceinline__ Split3 split3(float x0, float x1) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float r0 = x0 - __low2float(h), r1 = x1 - __high2float(h);
    const __nv_bfloat162 m = __floats2bfloat162_rn(r0, r1);
    const __nv_bfloat162 l = __floats2bfloat162_rn(r0 - __low2float(m), r1 - __high2float(m));
    return {bf16x2_bits(h), bf16x2_bits(m), bf16x2_bits(l)};
}
// Byte offset of (row, element d) in a staged region of 32-row boxes, each
// [head-dim half][32 rows][128 B], written by TMA with the 128-byte swizzle
// (16-byte unit ^= row % 8).
template <int NH>
__device__ __forceinline__ uint32_t swz(int row, int d) {
    return static_cast<uint32_t>((((row >> 5) * NH + (d >> 6)) * 32 + (row & 31)) * 128 +
                                 ((((d >> 3) & 7) ^ (row & 7)) << 4));
}

// A operands of one k16 step from the lane's (x0, x1) at k = kq + {0,1} and
// (x2, x3) at k = kq + 8 + {0,1}, for the lane's row r = lane / 4.
// PACK (G <= 4): r < G carries head r's h (row r) and l (row r + 8);
// G <= r < 2G carries head r - G's m (row r).  Otherwise a0 = [h ; m] and
// a1 = [l ; 0] with r < G the head.  `role`: 0 = h/l rows, 1 = m rows,
// 2 = no head.
template <bool PACK>
__device__ __forceinline__ void a_operands(float x0, float x1, float x2, float x3, int role, uint32_t (&a0)[4],
                                           uint32_t (&a1)[4]) {
    const Split3 lo = split3(x0, x1), hi = split3(x2, x3);
    if (PACK) {
        a0[0] = role == 0 ? lo.h : role == 1 ? lo.m : 0u;
        a0[1] = role == 0 ? lo.l : 0u;
        a0[2] = role == 0 ? hi.h : role == 1 ? hi.m : 0u;
        a0[3] = role == 0 ? hi.l : 0u;
    } else {
        const bool on = role == 0;
        a0[0] = on ? lo.h : 0u;
        a0[1] = on ? lo.m : 0u;
        a0[2] = on ? hi.h : 0u;
        a0[3] = on ? hi.m : 0u;
        a1[0] = on ? lo.l : 0u;
        a1[1] = 0u;
        a1[2] = on ? hi.l : 0u;
        a1[3] = 0u;
    }
}

// The last CTA of kv head `kvh`: merge the splits of its G query heads
// (partials in natural-log units) and write the output, or push it to every
// tensor-parallel rank and publish when the last kv head is done.  Each
// thread owns float4 items (head, 4 outputs).  When the G heads' partial
// outputs fit in shared memory (`bulk`) they arrive by one bulk copy per
// head while the split weights are formed; otherwise each thread's first
// loads go out before the weights are formed and the rest in batches.
template <int D>
__device__ __forceinline__ void merge_splits(const AttnParams& p, int kvh, int G, bool bulk, float* sm, float* s_scale,
                                             uint64_t* bar) {
    constexpr int kBatch = 16;
    const int S = p.splits;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = G * D / 4;
    float* const s_w = bulk ? sm + static_cast<size_t>(G) * S * D : sm;
    float4 v[kBatch];
    if (bulk) {
        if (threadIdx.x == 0) {
            fence_proxy_async_global();   // other CTAs' generic stores, read by the async proxy
            mbar_arrive_expect_tx(bar, static_cast<uint32_t>(G * S * D * 4));
            for (int g = 0; g < G; ++g)
                bulk_g2s(sm + static_cast<size_t>(g) * S * D, p.part_o + static_cast<long long>(kvh * G + g) * S * D,
                         static_cast<uint32_t>(S * D * 4), bar);
        }
    } else {
        const int it = threadIdx.x, g = it / (D / 4), d = (it - g * (D / 4)) * 4;
        const float4* po = reinterpret_cast<const float4*>(p.part_o + static_cast<long long>(kvh * G + g) * S * D + d);
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
            v[u] = it < items && u < S ? __ldcg(po + u * (D / 4)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    // split weights: warp w forms those of heads w, w + 4, ...
    for (int g = warp; g < G; g += kAttnWarps) {
        const float2* ml = reinterpret_cast<const float2*>(p.part_ml + static_cast<long long>(kvh * G + g) * S * 2);
        float2 e[kMaxSplits / 32];
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < kMaxSplits / 32; ++k) {
            e[k] = lane + 32 * k < S ? __ldcg(ml + lane + 32 * k) : make_float2(-INFINITY, 0.0f);
            mx = fmaxf(mx, e[k].x);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float l = 0.0f;
#pragma unroll
        for (int k = 0; k < kMaxSplits / 32; ++k) {
            const float w = e[k].x == -INFINITY ? 0.0f : exp2f((e[k].x - mx) * kLog2e);
            if (lane + 32 * k < S) s_w[g * S + lane + 32 * k] = w;
            l = fmaf(e[k].y, w, l);
        }
        l = warp_sum(l);
        if (lane == 0) s_scale[g] = l > 0.0f ? 1.0f / l : 0.0f;
    }
    __syncthreads();
    if (bulk) mbar_wait(bar, 0);   // a timeout is recorded in the fault word
    for (int it = threadIdx.x; it < items; it += blockDim.x) {
        const int g = it / (D / 4), d = (it - g * (D / 4)) * 4;
        const int qh = kvh * G + g;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (bulk) {
            const float4* so = reinterpret_cast<const float4*>(sm + static_cast<size_t>(g) * S * D + d);
            for (int j0 = 0; j0 < S; j0 += 8) {   // 8 independent shared loads per step
                float4 x[8];
                float w[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const bool in = j0 + u < S;
                    x[u] = in ? so[(j0 + u) * (D / 4)] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    w[u] = in ? s_w[g * S + j0 + u] : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    acc.x = fmaf(x[u].x, w[u], acc.x);
                    acc.y = fmaf(x[u].y, w[u], acc.y);
                    acc.z = fmaf(x[u].z, w[u], acc.z);
                    acc.w = fmaf(x[u].w, w[u], acc.w);
                }
            }
        } else {
            const float4* po = reinterpret_cast<const float4*>(p.part_o + static_cast<long long>(qh) * S * D + d);
            for (int j0 = 0; j0 < S; j0 += kBatch) {
                if (it != static_cast<int>(threadIdx.x) || j0 > 0) {
#pragma unroll
                    for (int u = 0; u < kBatch; ++u)
                        v[u] = j0 + u < S ? __ldcg(po + (j0 + u) * (D / 4)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
#pragma unroll
                for (int u = 0; u < kBatch; ++u) {
                    const float w = j0 + u < S ? s_w[g * S + j0 + u] : 0.0f;
                    acc.x = fmaf(v[u].x, w, acc.x);
                    acc.y = fmaf(v[u].y, w, acc.y);
                    acc.z = fmaf(v[u].z, w, acc.z);
                    acc.w = fmaf(v[u].w, w, acc.w);
                }
            }
        }
        const float inv = s_scale[g];
        const float4 o = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        if (p.tpl.tp > 1) {
            for (int r = 0; r < p.tpl.tp; ++r) *reinterpret_cast<float4*>(p.tpl.push_y[r] + qh * D + d) = o;
        } else {
            *reinterpret_cast<float4*>(p.out + qh * D + d) = o;
        }
    }
    if (p.tpl.tp > 1) {
        // the last kv head publishes this rank's heads on every rank
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x == 0)
            s_scale[0] = atomicAdd(p.tpl.counter, 1u) == static_cast<unsigned int>(p.kv_heads - 1) ? 1.0f : 0.0f;
        __syncthreads();
        if (s_scale[0] != 0.0f) {
            __threadfence_system();
            if (static_cast<int>(threadIdx.x) < p.tpl.tp)
                st_release_sys(p.tpl.push_flag[threadIdx.x],
                               static_cast<unsigned int>(*p.tpl.seq * p.tpl.push_mul + p.tpl.push_add));
            if (threadIdx.x == 0) *p.tpl.counter = 0u;
        }
    }
}

// CL: the launch is a grid of clusters (1, splits, 1), one per kv head, and
// the splits merge over distributed shared memory; otherwise the last CTA of
// a kv head merges the partials from global memory.
//
// Staging: box b (32 positions) of K sits at sk + b * NH * 4096 as
// [head-dim half][32 rows][128 B] (one copy fetches both halves), V likewise
// at sv.  Every warp takes the scores of its own 16-row chunks; the CTA-wide
// running max of each head is agreed once (one barrier), so the warps'
// probability-weighted V sums and their sums of probabilities simply add.
template <int D, bool PACK, bool CL>
__global__ void __launch_bounds__((CL ? kClusterWarps : kAttnWarps) * 32)
    attn_mma_kernel(const __grid_constant__ KvMaps maps, const AttnParams p, const int cap, const int merge_smem) {
    constexpr int W = CL ? kClusterWarps : kAttnWarps;
    constexpr int MB = CL ? kClusterBoxes : kMaxBoxes;
    constexpr int MWC = (MB * kBoxRows / kChunkRows + W - 1) / W;   // 16-row chunks per warp
    constexpr int NH = D / 64;   // 128-byte halves of a row
    constexpr int KS = D / 16;   // k16 steps of q.k
    constexpr int NT = D / 8;    // n8 tiles of the output
    constexpr uint32_t kBoxBytes = NH * kBoxRows * 128;
    constexpr int kOStride = D + 8;   // per-warp sum rows, padded so that 4 head rows of a store hit distinct banks
    static_assert(MB <= 16, "one lane arms each box a warp issues");
    __shared__ uint64_t s_bar[MB + 1];   // K/V boxes, then the split merge's bulk copy
    __shared__ float s_wmax[W][8];       // per warp and head: running max (log2 units)
    __shared__ float s_wl[W][8];         // per warp and head: sum of probabilities
    __shared__ float s_scale[8];
    __shared__ unsigned int s_last;
    if (threadIdx.x == 0) {   // ahead of the previous kernel's completion
        prefetch_tensormap(&maps.k);
        prefetch_tensormap(&maps.v);
        for (int b = 0; b < MB + 1; ++b) mbar_init(&s_bar[b], 1);
        fence_mbar_init();
    }
    if constexpr (CL) cluster_arrive_relaxed();   // this CTA has started (waited on before any remote store)
    pdl_launch_dependents();
    pdl_wait();
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = pin_reg(p.q_heads / p.kv_heads);
    const int S = pin_reg(p.splits);
    float* const out = pin_reg(p.out);
    float* const part_o = CL ? nullptr : pin_reg(p.part_o);
    float* const part_ml = CL ? nullptr : pin_reg(p.part_ml);
    const int seq_len = p.dev_pos ? *p.dev_pos + 1 : p.seq_len;
    const int active = seq_len - p.start_pos;
    const int c0 = p.start_pos + static_cast<int>(static_cast<long long>(active) * split / S);
    const int c1 = p.start_pos + static_cast<int>(static_cast<long long>(active) * (split + 1) / S);
    int n = c1 - c0;
    if (n > cap) {   // a device position past the length the launch was sized for
        if (threadIdx.x == 0) record_fault(ALJ_FAULT_BOUNDS);
        n = cap;
    }

    extern __shared__ unsigned char smem_raw[];
    const uint32_t sk = (smem_u32(smem_raw) + 1023u) & ~1023u;
    const uint32_t sv = sk + static_cast<uint32_t>(cap) * D * 2;
    float* const stage_f = reinterpret_cast<float*>(smem_raw + (sk - smem_u32(smem_raw)));
    // the lane's row r = lane / 4 of the A / C fragments and its head; the
    // query loads go out ahead of the bulk traffic of the whole grid
    const int r = lane >> 2, kq = (lane & 3) * 2;
    const int role = r < G ? 0 : (PACK && r < 2 * G) ? 1 : 2;
    const int head = role == 0 ? r : role == 1 ? r - G : 0;
    const int partner = role == 0 ? lane + 4 * G : lane - 4 * G;   // PACK: the lane with the other part rows
    float qv[KS][4];
    {
        const float* qrow = p.q + static_cast<long long>(kvh * G + head) * D;
#pragma unroll
        for (int s = 0; s < KS; ++s) {
            qv[s][0] = qv[s][1] = qv[s][2] = qv[s][3] = 0.0f;
            if (role != 2) {
                qv[s][0] = qrow[16 * s + kq];
                qv[s][1] = qrow[16 * s + kq + 1];
                qv[s][2] = qrow[16 * s + 8 + kq];
                qv[s][3] = qrow[16 * s + 8 + kq + 1];
            }
        }
    }
    __syncthreads();   // barrier initialisation visible to every warp
    // The copies: box b goes out from warp 2 (b mod W/2), whose first chunk
    // it holds -- lane j arms its j-th box, then lanes j and 16 + j issue
    // that box's K and V copies.
    const int nboxes = (n + kBoxRows - 1) / kBoxRows;
    if ((warp & 1) == 0) {
        const int b = (lane & 15) * (W / 2) + (warp >> 1);
        if (lane < 16 && b < nboxes) mbar_arrive_expect_tx(&s_bar[b], 2u * kBoxBytes);
        __syncwarp();
        if (b < nboxes) {
            const uint32_t off = static_cast<uint32_t>(b) * kBoxBytes;
            if (lane < 16)
                tma_load_4d(sk + off, &maps.k, 0, c0 + b * kBoxRows, 0, kvh, &s_bar[b]);
            else
                tma_load_4d(sv + off, &maps.v, 0, c0 + b * kBoxRows, 0, kvh, &s_bar[b]);
        }
    }
    uint32_t qa[KS][4], qb[PACK ? 1 : KS][4];
    {
        const float qs = p.scale * kLog2e;
#pragma unroll
        for (int s = 0; s < KS; ++s)
            a_operands<PACK>(qv[s][0] * qs, qv[s][1] * qs, qv[s][2] * qs, qv[s][3] * qs, role, qa[s], qb[PACK ? 0 : s]);
    }

    // scores (log2 units) of this warp's chunks: sc[ci][t][j] is position
    // 16c + 8t + kq + j of chunk c = warp + W ci, for the lane's head
    const int nchunks = (n + kChunkRows - 1) / kChunkRows;
    float sc[MWC][2][2];
    float mx = -INFINITY;
#pragma unroll
    for (int ci = 0; ci < MWC; ++ci) {
        const int c = warp + ci * W;
        sc[ci][0][0] = sc[ci][0][1] = sc[ci][1][0] = sc[ci][1][1] = -INFINITY;
        if (c >= nchunks) continue;
        mbar_wait(&s_bar[c >> 1], 0);   // a timeout is recorded in the fault word
        float acc[2][4] = {};
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int row = kChunkRows * c + 8 * t + (lane & 7);
#pragma unroll
            for (int s2 = 0; s2 < KS / 2; ++s2) {
                uint32_t kb[4];
                ldsm_x4(sk + swz<NH>(row, 32 * s2 + 8 * (lane >> 3)), kb);
                mma_bf16(acc[t], qa[2 * s2], kb[0], kb[1]);
                mma_bf16(acc[t], qa[2 * s2 + 1], kb[2], kb[3]);
                if (!PACK) {
                    mma_bf16(acc[t], qb[2 * s2], kb[0], kb[1]);
                    mma_bf16(acc[t], qb[2 * s2 + 1], kb[2], kb[3]);
                }
            }
        }
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                float v = acc[t][j] + acc[t][j + 2];
                if (PACK) v += __shfl_sync(0xffffffffu, v, partner & 31);
                const int pos = kChunkRows * c + 8 * t + kq + j;
                sc[ci][t][j] = pos < n ? v : -INFINITY;
                mx = fmaxf(mx, sc[ci][t][j]);
            }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (role == 0 && (lane & 3) == 0) s_wmax[warp][r] = mx;
    __syncthreads();
    // the CTA-wide max of the lane's head
    mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; ++w) mx = fmaxf(mx, s_wmax[w][head]);

    // probabilities as A operands, split like the query
    uint32_t pa[MWC][4], pb[PACK ? 1 : MWC][4];
    float l = 0.0f;
#pragma unroll
    for (int ci = 0; ci < MWC; ++ci) {
        float e[2][2];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                e[t][j] = sc[ci][t][j] == -INFINITY ? 0.0f : exp2f(sc[ci][t][j] - mx);
                l += e[t][j];
            }
        a_operands<PACK>(e[0][0], e[0][1], e[1][0], e[1][1], role, pa[ci], pb[PACK ? 0 : ci]);
    }
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);

    float o[NT][4];
#pragma unroll
    for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
#pragma unroll
    for (int ci = 0; ci < MWC; ++ci) {
        const int c = warp + ci * W;
        if (c >= nchunks) break;
        if (c == nchunks - 1 && (n & (kChunkRows - 1))) {
            // rows past the split hold other positions (or unwritten cache):
            // zero them so that probability 0 never meets a NaN
            const int nz = kChunkRows * nchunks - n;
            for (int i = lane; i < nz * NH * 8; i += 32) {
                const int row = n + i / (NH * 8), h = (i / 8) % NH, u = i & 7;
                const uint32_t a = sv + static_cast<uint32_t>((((row >> 5) * NH + h) * kBoxRows + (row & 31)) * 128 + u * 16);
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
            }
            __syncwarp();
        }
        const int row = kChunkRows * c + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
        for (int u = 0; u < NT / 2; ++u) {
            uint32_t vb[4];
            ldsm_x4_trans(sv + swz<NH>(row, 16 * u + (lane >> 4) * 8), vb);
            mma_bf16(o[2 * u], pa[ci], vb[0], vb[1]);
            mma_bf16(o[2 * u + 1], pa[ci], vb[2], vb[3]);
            if (!PACK) {
                mma_bf16(o[2 * u], pb[ci], vb[0], vb[1]);
                mma_bf16(o[2 * u + 1], pb[ci], vb[2], vb[3]);
            }
        }
    }

    // per-warp sums to shared memory (the output part reuses the staging
    // buffer once every warp is done reading it), then their CTA sum
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            o[i][j] += o[i][j + 2];
            if (PACK) o[i][j] += __shfl_sync(0xffffffffu, o[i][j], partner & 31);
        }
    if (role == 0) {
        if ((lane & 3) == 0) s_wl[warp][r] = l;
#pragma unroll
        for (int i = 0; i < NT; ++i)
            *reinterpret_cast<float2*>(stage_f + (warp * 8 + r) * kOStride + 8 * i + kq) = make_float2(o[i][0], o[i][1]);
    }
    __syncthreads();
    const int items = G * D / 4;
    if constexpr (CL) {
        // Push: each item (head, 4 outputs) of this split goes to the shared
        // memory of the CTA that owns it (a 1 / splits share of the kv
        // head's items, in rank order), the (max, sum) of every head to every
        // CTA; one cluster barrier later each CTA merges its items locally.
        const int ipo = (items + S - 1) / S;   // items per owner
        float4* const recv = reinterpret_cast<float4*>(stage_f + max(cap * D, W * 8 * kOStride));   // [S][ipo]
        float2* const recv_ml = reinterpret_cast<float2*>(recv + S * ipo);                     // [S][8]
        cluster_wait();   // every CTA of the cluster has started
        for (int it = threadIdx.x; it < items; it += blockDim.x) {
            const int g = it / (D / 4), d = (it - g * (D / 4)) * 4;
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int w = 0; w < W; ++w) {
                const float4 x = *reinterpret_cast<const float4*>(stage_f + (w * 8 + g) * kOStride + d);
                acc.x += x.x;
                acc.y += x.y;
                acc.z += x.z;
                acc.w += x.w;
            }
            const int owner = it / ipo;
            st_cluster_f4(cluster_map(smem_u32(recv + split * ipo + (it - owner * ipo)), owner), acc);
        }
        if (static_cast<int>(threadIdx.x) < S * G) {
            const int g = threadIdx.x % G, dst = threadIdx.x / G;
            float M = -INFINITY, L = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) {
                M = fmaxf(M, s_wmax[w][g]);
                L += s_wl[w][g];
            }
            st_cluster_f2(cluster_map(smem_u32(recv_ml + split * 8 + g), dst), make_float2(M, L));
        }
        cluster_barrier();   // release / acquire: every pushed partial visible to its owner
        const int it = split * ipo + static_cast<int>(threadIdx.x);
        if (static_cast<int>(threadIdx.x) < ipo && it < items) {
            const int g = it / (D / 4), d = (it - g * (D / 4)) * 4;
            float Mx = -INFINITY;
            for (int j = 0; j < S; ++j) Mx = fmaxf(Mx, recv_ml[j * 8 + g].x);
            float L = 0.0f;
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int j = 0; j < S; ++j) {
                const float2 ml = recv_ml[j * 8 + g];
                const float w = ml.x == -INFINITY ? 0.0f : exp2f(ml.x - Mx);
                const float4 x = recv[j * ipo + threadIdx.x];
                L = fmaf(ml.y, w, L);
                acc.x = fmaf(x.x, w, acc.x);
                acc.y = fmaf(x.y, w, acc.y);
                acc.z = fmaf(x.z, w, acc.z);
                acc.w = fmaf(x.w, w, acc.w);
            }
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            *reinterpret_cast<float4*>(out + (kvh * G + g) * D + d) =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        }
    } else {
        for (int it = threadIdx.x; it < items; it += blockDim.x) {
            const int g = it / (D / 4), d = (it - g * (D / 4)) * 4;
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            float M = -INFINITY, L = 0.0f;
#pragma unroll
            for (int w = 0; w < W; ++w) {
                const float4 x = *reinterpret_cast<const float4*>(stage_f + (w * 8 + g) * kOStride + d);
                acc.x += x.x;
                acc.y += x.y;
                acc.z += x.z;
                acc.w += x.w;
                M = fmaxf(M, s_wmax[w][g]);
                L += s_wl[w][g];
            }
            const int qh = kvh * G + g;
            if (S == 1) {
                const float inv = L > 0.0f ? 1.0f / L : 0.0f;
                *reinterpret_cast<float4*>(out + qh * D + d) =
                    make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
            } else {
                *reinterpret_cast<float4*>(part_o + (static_cast<long long>(qh) * S + split) * D + d) = acc;
                if (d == 0)   // natural-log units for the merge
                    *reinterpret_cast<float2*>(part_ml + (static_cast<long long>(qh) * S + split) * 2) =
                        make_float2(M == -INFINITY ? -INFINITY : M * (1.0f / kLog2e), L);
            }
        }
        if (S == 1) return;

        // the last CTA of this kv head to finish merges the splits: the CTA
        // barrier orders every thread's partial stores before thread 0's
        // acquire-release arrival (release is cumulative), and the winner's
        // acquire orders the other CTAs' partials before its reads
        __syncthreads();
        if (threadIdx.x == 0) s_last = atom_add_acq_rel_gpu(&p.split_counter[kvh], 1u) == static_cast<unsigned int>(S - 1);
        __syncthreads();
        if (!s_last) return;
        merge_splits<D>(p, kvh, G, merge_smem != 0, stage_f, s_scale, &s_bar[MB]);
        if (threadIdx.x == 0) p.split_counter[kvh] = 0u;
    }
}

// Merge the splits of one query head: the per-split (max, sum) pairs are
// staged in shared memory and turned into weights once, then each thread
// sums its head-dim element over the splits with independent loads.

__global__ void __launch_bounds__(128) attn_combine_kernel(const AttnParams p) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float s_w[kMaxSplits];
    __shared__ float s_red[4];
    const int qh = blockIdx.x;
    const int D = p.head_dim;
    const int S = p.splits;
    const float* ml = p.part_ml + static_cast<long long>(qh) * S * 2;
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < S; j += blockDim.x) mx = fmaxf(mx, ml[2 * j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = mx;
    __syncthreads();
    const float M = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
    __syncthreads();
    float l = 0.0f;
    for (int j = threadIdx.x; j < S; j += blockDim.x) {
        const float mj = ml[2 * j];
        const float w = mj == -INFINITY ? 0.0f : exp2f((mj - M) * kLog2e);
        s_w[j] = w;
        l = fmaf(ml[2 * j + 1], w, l);
    }
    l = warp_sum(l);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = l;
    __syncthreads();
    const float inv = 1.0f / (s_red[0] + s_red[1] + s_red[2] + s_red[3]);
    const float* po = p.part_o + static_cast<long long>(qh) * S * D;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        int j = 0;
        for (; j + 4 <= S; j += 4) {
            a0 = fmaf(po[(j + 0) * D + d], s_w[j + 0], a0);
            a1 = fmaf(po[(j + 1) * D + d], s_w[j + 1], a1);
            a2 = fmaf(po[(j + 2) * D + d], s_w[j + 2], a2);
            a3 = fmaf(po[(j + 3) * D + d], s_w[j + 3], a3);
        }
        for (; j < S; ++j) a0 = fmaf(po[j * D + d], s_w[j], a0);
        const float o = ((a0 + a1) + (a2 + a3)) * inv;
        if (p.tpl.tp > 1) {
            for (int r = 0; r < p.tpl.tp; ++r) p.tpl.push_y[r][qh * D + d] = o;
        } else {
            p.out[qh * D + d] = o;
        }
    }
    if (p.tpl.tp > 1) {
        // the last CTA publishes this rank's heads on every rank
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x == 0) {
            const unsigned int prev = atomicAdd(p.tpl.counter, 1u);
            s_red[0] = prev == gridDim.x - 1 ? 1.0f : 0.0f;
        }
        __syncthreads();
        if (s_red[0] != 0.0f) {
            __threadfence_system();
            if (static_cast<int>(threadIdx.x) < p.tpl.tp)
                st_release_sys(p.tpl.push_flag[threadIdx.x],
                               static_cast<unsigned int>(*p.tpl.seq * p.tpl.push_mul + p.tpl.push_add));
            if (threadIdx.x == 0) *p.tpl.counter = 0u;
        }
    }
}

// Plain fallback for any head_dim / stride / group: one CTA per query head,
// scores in shared memory (positions <= kMaxFallbackPositions).
constexpr int kMaxFallbackPositions = 40960;

template <int KVT>
__device__ __forceinline__ float kv_at(const void* base, long long i) {
    if (KVT == ALJ_KV_BF16) return __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(base)[i]) << 16);
    return static_cast<const float*>(base)[i];
}

template <int KVT>
__global__ void attn_fallback_kernel(const AttnParams p) {
    pdl_launch_dependents();
    pdl_wait();
    extern __shared__ float sc[];
    __shared__ float red[32];
    const int h = blockIdx.x;
    const int G = p.q_heads / p.kv_heads;
    const int kvh = h / G;
    const int D = p.head_dim;
    const int n = p.seq_len - p.start_pos;
    const float* q = p.q + static_cast<long long>(h) * D;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const long long off = static_cast<long long>(p.start_pos + i) * p.stride + kvh * p.head_stride;
        float a = 0.0f;
        for (int d = 0; d < D; ++d) a = fmaf(q[d], kv_at<KVT>(p.k, off + d), a);
        sc[i] = a * p.scale;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, sc[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -INFINITY;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(sc[i] - mx);
        sc[i] = e;
        sum += e;
    }
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    sum = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) sum += red[w];
    const float inv = 1.0f / sum;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = 0.0f;
        for (int i = 0; i < n; ++i) {
            const long long off = static_cast<long long>(p.start_pos + i) * p.stride + kvh * p.head_stride + d;
            acc = fmaf(sc[i] * inv, kv_at<KVT>(p.v, off), acc);
        }
        p.out[static_cast<long long>(h) * D + d] = acc;
    }
}

template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                       const Args&... args) {
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
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Shared memory of the bulk split merge: the kv head's partial outputs and
// their weights.
size_t merge_bytes(const AttnParams& p) {
    const size_t gs = static_cast<size_t>(p.q_heads / p.kv_heads) * p.splits;
    return gs * p.head_dim * 4 + gs * 4;
}

// Tensor maps and staging rows for the tensor-core kernel; false when the
// cache type, shape or layout is outside it (the shuffle kernel runs then).
bool mma_params(const AttnParams& p, AttnMmaParams& mp, int max_boxes = kMaxBoxes) {
    if (p.kv_dtype != ALJ_KV_BF16 || !(p.head_dim == 64 || p.head_dim == 128)) return false;
    if (p.kv_heads <= 0 || p.q_heads % p.kv_heads || p.q_heads / p.kv_heads > 8) return false;
    const uintptr_t mis = reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v);
    if (mis % 16 || (static_cast<long long>(p.stride) * 2) % 16 || (p.head_stride * 2) % 16) return false;
    const int active = p.seq_len - p.start_pos;
    const int rows = (active + p.splits - 1) / p.splits;
    const int cap = (rows + kBoxRows - 1) / kBoxRows * kBoxRows;
    if (cap > max_boxes * kBoxRows) return false;
    if (p.splits > 1 && (!p.split_counter || reinterpret_cast<uintptr_t>(p.part_o) % 16 ||
                         reinterpret_cast<uintptr_t>(p.part_ml) % 8 || p.splits > kMaxSplits))
        return false;
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    // [64 elements][positions][head-dim halves][kv heads]: one box is both
    // halves of 32 positions of one kv head, staged half-major
    const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(p.seq_len), static_cast<cuuint64_t>(p.head_dim / 64),
                                static_cast<cuuint64_t>(p.kv_heads)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(p.stride) * 2, 128,
                                   static_cast<cuuint64_t>(p.head_stride) * 2};
    const cuuint32_t box[4] = {64, kBoxRows, static_cast<cuuint32_t>(p.head_dim / 64), 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    for (int t = 0; t < 2; ++t)
        if (fn(t == 0 ? &mp.maps.k : &mp.maps.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(t == 0 ? p.k : p.v),
               dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return false;
    mp.a = p;
    mp.cap_rows = cap;
    mp.merge_smem = p.splits > 1 && merge_bytes(p) + 1024 <= static_cast<size_t>(kMmaSmemMax);
    return true;
}

template <int D, bool PACK>
cudaError_t launch_mma(const AttnMmaParams& mp, dim3 grid, cudaStream_t stream, bool pdl) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(attn_mma_kernel<D, PACK, false>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kMmaSmemMax);
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    const size_t stage = 2ull * mp.cap_rows * D * 2;
    const size_t sums = static_cast<size_t>(kAttnWarps) * 8 * (D + 8) * 4;   // the per-warp sums reuse the staging
    const size_t smem = std::max(mp.merge_smem ? std::max(stage, merge_bytes(mp.a)) : stage, sums) + 1024;
    return launch_pdl(attn_mma_kernel<D, PACK, false>, grid, dim3(kAttnWarps * 32), smem, stream, pdl, mp.maps, mp.a,
                      mp.cap_rows, mp.merge_smem);
}

cudaError_t dispatch_mma(const AttnMmaParams& mp, dim3 grid, cudaStream_t stream, bool pdl) {
    const bool pack = mp.a.q_heads / mp.a.kv_heads <= 4;
    if (mp.a.head_dim == 64)
        return pack ? launch_mma<64, true>(mp, grid, stream, pdl) : launch_mma<64, false>(mp, grid, stream, pdl);
    return pack ? launch_mma<128, true>(mp, grid, stream, pdl) : launch_mma<128, false>(mp, grid, stream, pdl);
}

// Dynamic shared memory of the cluster variant: K + V staging (the per-warp
// state reuses it), one CTA's partials, alignment.
size_t cluster_smem(int cap, int D) {
    return static_cast<size_t>(std::max(cap * D, kClusterWarps * 8 * (D + 8)) + kPartFloats) * 4 + 1024;
}

// Clusters of `splits` CTAs the device holds at once with the largest
// staging (0 when it cannot run the cluster variant); asked once per device
// and split count.
template <int D, bool PACK>
int cluster_capacity(int splits) {
    static int known[64][kClusterMax + 1];
    static bool asked[64][kClusterMax + 1];
    int dev = 0;
    cudaGetDevice(&dev);
    dev &= 63;
    if (asked[dev][splits]) return known[dev][splits];
    asked[dev][splits] = true;
    auto kern = attn_mma_kernel<D, PACK, true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kClusterSmemMax) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, splits);
    cfg.blockDim = dim3(kClusterWarps * 32);
    cfg.dynamicSmemBytes = cluster_smem(kClusterBoxes * kBoxRows, D);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = splits;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    known[dev][splits] = n;
    return n;
}

template <int D, bool PACK>
cudaError_t launch_mma_cluster(const AttnMmaParams& mp, cudaStream_t stream, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(mp.a.kv_heads, mp.a.splits);
    cfg.blockDim = dim3(kClusterWarps * 32);
    cfg.dynamicSmemBytes = cluster_smem(mp.cap_rows, D);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = mp.a.splits;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, attn_mma_kernel<D, PACK, true>, mp.maps, mp.a, mp.cap_rows, 0);
}

// The cluster variant when it applies: single-rank output, a tensor-core
// shape, a split count (<= 16, >= 64 positions a split where the cache
// allows) whose clusters the device holds all at once, one per kv head, with
// every split within the staging -- and either enough CTAs to cover a good
// part of the SMs or no fewer splits than the global-merge launch would
// take.  Returns false (nothing launched) otherwise.
bool try_cluster(const AttnParams& p, cudaStream_t stream, bool pdl, cudaError_t* err) {
    if (p.tpl.tp > 1 || p.kv_dtype != ALJ_KV_BF16 || !(p.head_dim == 64 || p.head_dim == 128)) return false;
    if (p.kv_heads <= 0 || p.q_heads % p.kv_heads || p.q_heads / p.kv_heads > 8) return false;
    const int active = p.seq_len - p.start_pos;
    const bool pack = p.q_heads / p.kv_heads <= 4;
    int S = 0;
    for (int s = std::min(kClusterMax, std::max(2, (active + 63) / 64)); s >= 2; --s) {
        if ((active + s - 1) / s > kClusterBoxes * kBoxRows) break;   // fewer splits are only longer
        const int have = p.head_dim == 64 ? (pack ? cluster_capacity<64, true>(s) : cluster_capacity<64, false>(s))
                                          : (pack ? cluster_capacity<128, true>(s) : cluster_capacity<128, false>(s));
        if (have >= p.kv_heads) {
            S = s;
            break;
        }
    }
    if (S == 0 || (p.kv_heads * S < 64 && S < p.splits)) return false;
    AttnParams q = p;
    q.splits = S;
    AttnMmaParams mp{};
    if (!mma_params(q, mp, kClusterBoxes)) return false;
    mp.merge_smem = 0;
    if (q.head_dim == 64)
        *err = pack ? launch_mma_cluster<64, true>(mp, stream, pdl) : launch_mma_cluster<64, false>(mp, stream, pdl);
    else
        *err = pack ? launch_mma_cluster<128, true>(mp, stream, pdl) : launch_mma_cluster<128, false>(mp, stream, pdl);
    return true;
}

bool fast_path(const AttnParams& p) {
    const int G = p.q_heads / p.kv_heads;
    const int E = p.head_dim / 32;
    if (p.head_dim % 32 != 0 || !(E == 2 || E == 4 || E == 8)) return false;
    if (!(G == 1 || G == 2 || G == 4 || G == 8)) return false;
    if (G * E > 32) return false;                       // register budget of the per-lane output
    if ((32 / G) * E > 64) return false;                // and of the K/V rows held per step
    const int elem = p.kv_dtype == ALJ_KV_BF16 ? 2 : 4;
    const int vec = E * elem;                           // bytes per lane load
    const uintptr_t mis = (reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v));
    if (mis % (vec >= 16 ? 16 : vec)) return false;
    if ((static_cast<long long>(p.stride) * elem) % (vec >= 16 ? 16 : vec)) return false;
    if ((p.head_stride * elem) % (vec >= 16 ? 16 : vec)) return false;
    return true;
}

template <int KVT, int E>
cudaError_t dispatch_g(const AttnParams& p, dim3 grid, cudaStream_t stream, bool pdl) {
    switch (p.q_heads / p.kv_heads) {
        case 1: return launch_pdl(attn_split_kernel<KVT, E, 1>, grid, dim3(kAttnWarps * 32), 0, stream, pdl, p);
        case 2: return launch_pdl(attn_split_kernel<KVT, E, 2>, grid, dim3(kAttnWarps * 32), 0, stream, pdl, p);
        case 4: return launch_pdl(attn_split_kernel<KVT, E, 4>, grid, dim3(kAttnWarps * 32), 0, stream, pdl, p);
        case 8:
            if (E <= 4) return launch_pdl(attn_split_kernel<KVT, (E <= 4 ? E : 4), 8>, grid, dim3(kAttnWarps * 32), 0, stream, pdl, p);
            return cudaErrorNotSupported;
    }
    return cudaErrorNotSupported;
}

template <int KVT>
cudaError_t dispatch_e(const AttnParams& p, dim3 grid, cudaStream_t stream, bool pdl) {
    switch (p.head_dim / 32) {
        case 2: return dispatch_g<KVT, 2>(p, grid, stream, pdl);
        case 4: return dispatch_g<KVT, 4>(p, grid, stream, pdl);
        case 8: return dispatch_g<KVT, 8>(p, grid, stream, pdl);
    }
    return cudaErrorNotSupported;
}

}  // namespace

int attention_splits(int seq_len, int kv_heads, int sm_count) {
    // ~2 CTAs per SM in total and at least 64 positions per split; long
    // caches take more splits so that a split stays within the tensor-core
    // kernel's staging (kMaxBoxes * kBoxRows positions)
    const int want = std::max(1, (2 * sm_count + kv_heads - 1) / std::max(kv_heads, 1));
    const int cap = std::max(1, seq_len / 64);
    const int need = (seq_len + kMaxBoxes * kBoxRows - 1) / (kMaxBoxes * kBoxRows);
    return std::min(std::max(std::min(want, cap), need), kMaxSplits);
}

// [arrival counters: q_heads words, rounded to 16 bytes][partial outputs][partial (max, sum)]:
// the counters sit at a fixed place whatever the split count, so the zeros
// they return to after every launch stay zeros for the next shape.
static size_t counter_floats(int q_heads) { return (static_cast<size_t>(q_heads) + 3) / 4 * 4; }

size_t attention_scratch_floats(int q_heads, int head_dim, int splits) {
    return counter_floats(q_heads) + static_cast<size_t>(q_heads) * splits * (head_dim + 2);
}

void attention_bind_scratch(AttnParams& p, float* scratch) {
    p.split_counter = reinterpret_cast<unsigned int*>(scratch);
    p.part_o = scratch + counter_floats(p.q_heads);
    p.part_ml = p.part_o + static_cast<size_t>(p.q_heads) * p.splits * p.head_dim;
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl) {
    const int active = p.seq_len - p.start_pos;
    if (active <= 0) return cudaErrorInvalidValue;
    // the tensor-parallel push lives in the combine kernel
    AttnMmaParams mp{};
    const bool tc = mma_params(p, mp);
    const bool split_path = tc || fast_path(p);
    if (p.tpl.tp > 1 && (p.splits < 2 || p.tpl.tp > kMaxTp || !p.tpl.counter || !p.tpl.seq || !split_path))
        return cudaErrorInvalidValue;
    if (split_path) {
        cudaError_t ce = cudaSuccess;
        if (tc && try_cluster(p, stream, pdl, &ce)) return ce;
        dim3 grid(p.kv_heads, p.splits);
        if (tc) return dispatch_mma(mp, grid, stream, pdl);   // merges its splits itself
        cudaError_t e = p.kv_dtype == ALJ_KV_BF16 ? dispatch_e<ALJ_KV_BF16>(p, grid, stream, pdl)
                                                  : dispatch_e<ALJ_KV_F32>(p, grid, stream, pdl);
        if (e != cudaSuccess || p.splits == 1) return e;
        return launch_pdl(attn_combine_kernel, dim3(p.q_heads), dim3(128), 0, stream, pdl, p);
    }
    if (p.dev_pos || active > kMaxFallbackPositions) return cudaErrorNotSupported;
    const size_t smem = static_cast<size_t>(active) * sizeof(float);
    auto kern = p.kv_dtype == ALJ_KV_BF16 ? attn_fallback_kernel<ALJ_KV_BF16> : attn_fallback_kernel<ALJ_KV_F32>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(kern, dim3(p.q_heads), dim3(256), smem, stream, pdl, p);
}

}  // namespace alj
