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

#include <algorithm>

namespace alj {
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
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D, d = idx - g * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, s_ml[w][g][0]);
        float L = 0.0f, acc = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            const float mw = s_ml[w][g][0];
            const float f = mw == -INFINITY ? 0.0f : exp2f((mw - M) * kLog2e);
            L = fmaf(s_ml[w][g][1], f, L);
            acc = fmaf(s_o[w][g][d], f, acc);
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

// Merge the splits of one query head: the per-split (max, sum) pairs are
// staged in shared memory and turned into weights once, then each thread
// sums its head-dim element over the splits with independent loads.
constexpr int kMaxSplits = 256;

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

cudaError_t launch_pdl(void (*kernel)(AttnParams), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                       const AttnParams& p) {
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
    return cudaLaunchKernelEx(&cfg, kernel, p);
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
    // ~2 CTAs per SM in total, at least 64 positions per split
    const int want = std::max(1, (2 * sm_count + kv_heads - 1) / std::max(kv_heads, 1));
    const int cap = std::max(1, seq_len / 64);
    return std::min(std::min(want, cap), kMaxSplits);
}

size_t attention_scratch_floats(int q_heads, int head_dim, int splits) {
    return static_cast<size_t>(q_heads) * splits * (head_dim + 2);
}

cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl) {
    const int active = p.seq_len - p.start_pos;
    if (active <= 0) return cudaErrorInvalidValue;
    // the tensor-parallel push lives in the combine kernel
    if (p.tpl.tp > 1 && (p.splits < 2 || p.tpl.tp > kMaxTp || !p.tpl.counter || !p.tpl.seq || !fast_path(p)))
        return cudaErrorInvalidValue;
    if (fast_path(p)) {
        dim3 grid(p.kv_heads, p.splits);
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
