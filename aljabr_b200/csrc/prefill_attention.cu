// Prefill attention on B200 (sm_100a): T query tokens attend causally (or
// through a sliding window, or to all S keys) to fp32 K / V, GQA heads.
// Two reference contracts share this kernel:
//   * GgufPrefillAttentionExecution.execute's Java loop (engine/gguf/
//     aljabr-gguf-java/.../javabackend/GgufPrefillAttentionExecution.java:
//     44-82): q [t][Hq*D], k / v [t][kv_stride], token t sees positions
//     [t - window + 1, t] (window > 0) or [0, t];
//   * the FlashAttention-4 seam's CPU contract (backend/metal/aljabr-backend-
//     metal/.../binding/MetalFlashAttentionCpuFallback.java:46-104): q / out
//     [B][T][H][D], k / v [B][S][Hkv][D], causal key limit t + max(0, S - T),
//     optional tanh soft cap.
// Arithmetic is fp32 like the reference's (dots on the CUDA cores; the
// softmax is evaluated online, max-subtracted as in the reference).
//
// Layout per CTA: 64 query rows = the `group` q heads that share one KV head
// x 64 / group consecutive tokens, 8 warps x 8 rows.  K / V stream through
// shared memory in tiles of 32 positions:
//   * scores: lane s owns key s of the tile (its K row, padded by 4 floats so
//     the lanes' float4 reads hit distinct banks) and reads the warp's 8 query
//     rows as float4 broadcasts;
//   * online softmax per row (warp max / sum over the 32 lanes);
//   * P V: the tile's probabilities go through shared memory; lane l owns
//     head dimensions l, l + 32, ... of its rows' outputs.
// CTAs with the most keys (the last tokens, under a causal mask) start first.
#include "common.cuh"

#include <algorithm>

namespace alj {
namespace {

constexpr int kPWarps = 8;
constexpr int kPThreads = kPWarps * 32;
constexpr int kRPW = 8;                    // query rows per warp
constexpr int kPRows = kPWarps * kRPW;     // 64 query rows per CTA
constexpr int kTile = 32;                  // keys per tile: one per lane

struct PrefillParams {
    float* out;
    const float* q;
    const float* k;
    const float* v;
    long long q_tok, q_batch;      // floats between tokens / batches of q and out
    long long kv_pos, kv_batch;    // floats between positions / batches of k and v
    int T, S, Hq, Hkv, group, tq;  // tq: tokens per CTA
    int off;                       // causal limit: token t sees keys <= t + off
    int causal, window;
    float scale, softcap;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <int DPL>
__global__ void __launch_bounds__(kPThreads) prefill_attn_kernel(const PrefillParams p) {
    constexpr int D = DPL * 32;
    constexpr int D4 = D / 4;
    constexpr int KS = D + 4;                  // K tile row stride in floats
    extern __shared__ float4 smem4[];
    float* qs = reinterpret_cast<float*>(smem4);    // [kPRows][D]
    float* ks = qs + kPRows * D;                    // [kTile][KS]
    float* vs = ks + kTile * KS;                    // [kTile][D]
    float* ps = vs + kTile * D;                     // [kPWarps][kRPW][kTile]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.z, kvh = blockIdx.y;
    const int t0 = (gridDim.x - 1 - blockIdx.x) * p.tq;     // heavy (late) token tiles first
    const int ntok = min(p.tq, p.T - t0);
    const int nrows = ntok * p.group;
    const float* qb = p.q + b * p.q_batch;
    const float* kb = p.k + b * p.kv_batch + static_cast<long long>(kvh) * D;
    const float* vb = p.v + b * p.kv_batch + static_cast<long long>(kvh) * D;
    pdl_wait();

    // query rows: row i = (token t0 + i / group, head kvh * group + i % group)
    for (int e = threadIdx.x; e < kPRows * D4; e += kPThreads) {
        const int i = e / D4, c = e - (e / D4) * D4;
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < nrows) {
            const int t = t0 + i / p.group, h = kvh * p.group + i % p.group;
            val = __ldg(reinterpret_cast<const float4*>(qb + t * p.q_tok + static_cast<long long>(h) * D) + c);
        }
        smem4[e] = val;
    }

    // per-row key limits [lo, hi] and softmax state
    const int r0 = warp * kRPW;
    int lo[kRPW], hi[kRPW];
    float m[kRPW], l[kRPW], o[kRPW][DPL];
    int whi = -1, wlo = p.S;                   // the warp's key range
#pragma unroll
    for (int r = 0; r < kRPW; ++r) {
        const int i = r0 + r;
        if (i < nrows) {
            const int t = t0 + i / p.group;
            hi[r] = p.causal ? min(p.S - 1, t + p.off) : p.S - 1;
            lo[r] = p.window > 0 ? max(0, hi[r] - p.window + 1) : 0;
        } else {
            hi[r] = -1;
            lo[r] = 0;
        }
        whi = max(whi, hi[r]);
        if (hi[r] >= 0) wlo = min(wlo, lo[r]);
        m[r] = -INFINITY;
        l[r] = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) o[r][j] = 0.0f;
    }
    // the CTA's key range: its last token's limit, and the window of its first
    const int t_last = t0 + ntok - 1;
    const int kend = p.causal ? min(p.S - 1, t_last + p.off) : p.S - 1;
    const int hi0 = p.causal ? min(p.S - 1, t0 + p.off) : p.S - 1;
    const int kbeg = p.window > 0 ? max(0, hi0 - p.window + 1) : 0;

    for (int kt = kbeg / kTile * kTile; kt <= kend; kt += kTile) {
        __syncthreads();                       // the previous tile is consumed (and qs written)
        for (int e = threadIdx.x; e < kTile * D4; e += kPThreads) {
            const int s = e / D4, c = e - (e / D4) * D4;
            const int pos = kt + s;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (pos < p.S) {
                kv = __ldg(reinterpret_cast<const float4*>(kb + pos * p.kv_pos) + c);
                vv = __ldg(reinterpret_cast<const float4*>(vb + pos * p.kv_pos) + c);
            }
            reinterpret_cast<float4*>(ks + s * KS)[c] = kv;
            reinterpret_cast<float4*>(vs + s * D)[c] = vv;
        }
        __syncthreads();
        if (whi < kt || wlo > kt + kTile - 1) continue;   // no row of this warp sees the tile

        float sc[kRPW];
#pragma unroll
        for (int r = 0; r < kRPW; ++r) sc[r] = 0.0f;
        const float4* kr = reinterpret_cast<const float4*>(ks + lane * KS);
#pragma unroll 4
        for (int c = 0; c < D4; ++c) {
            const float4 kk = kr[c];
#pragma unroll
            for (int r = 0; r < kRPW; ++r) {
                const float4 qq = reinterpret_cast<const float4*>(qs + (r0 + r) * D)[c];
                sc[r] = fmaf(qq.x, kk.x, sc[r]);
                sc[r] = fmaf(qq.y, kk.y, sc[r]);
                sc[r] = fmaf(qq.z, kk.z, sc[r]);
                sc[r] = fmaf(qq.w, kk.w, sc[r]);
            }
        }
        const int pos = kt + lane;
        float* pw = ps + warp * kRPW * kTile;
#pragma unroll
        for (int r = 0; r < kRPW; ++r) {
            float s = sc[r] * p.scale;
            if (p.softcap > 0.0f) s = tanhf(s / p.softcap) * p.softcap;
            const bool valid = pos >= lo[r] && pos <= hi[r];
            s = valid ? s : -INFINITY;
            const float mn = fmaxf(m[r], warp_max(s));
            float pr = 0.0f;
            if (mn != -INFINITY) {
                const float corr = expf(m[r] - mn);          // 0 while m is still -inf
                pr = valid ? expf(s - mn) : 0.0f;
                l[r] = l[r] * corr + warp_sum(pr);
#pragma unroll
                for (int j = 0; j < DPL; ++j) o[r][j] *= corr;
                m[r] = mn;
            }
            pw[r * kTile + lane] = pr;
        }
        __syncwarp();
#pragma unroll 2
        for (int s = 0; s < kTile; s += 4) {
            float4 pp[kRPW];
#pragma unroll
            for (int r = 0; r < kRPW; ++r) pp[r] = *reinterpret_cast<const float4*>(pw + r * kTile + s);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
#pragma unroll
                for (int j = 0; j < DPL; ++j) {
                    const float vv = vs[(s + u) * D + lane + 32 * j];
#pragma unroll
                    for (int r = 0; r < kRPW; ++r) {
                        const float pu = u == 0 ? pp[r].x : u == 1 ? pp[r].y : u == 2 ? pp[r].z : pp[r].w;
                        o[r][j] = fmaf(pu, vv, o[r][j]);
                    }
                }
            }
        }
        __syncwarp();
    }

#pragma unroll
    for (int r = 0; r < kRPW; ++r) {
        const int i = r0 + r;
        if (i >= nrows) continue;
        const int t = t0 + i / p.group, h = kvh * p.group + i % p.group;
        float* orow = p.out + b * p.q_batch + t * p.q_tok + static_cast<long long>(h) * D;
        const float inv = 1.0f / l[r];
#pragma unroll
        for (int j = 0; j < DPL; ++j) orow[lane + 32 * j] = o[r][j] * inv;
    }
}

size_t prefill_smem(int D) { return static_cast<size_t>(kPRows * D + kTile * (D + 4) + kTile * D + kPRows * kTile) * 4; }

template <int DPL>
cudaError_t launch_dpl(const PrefillParams& p, int B, cudaStream_t stream) {
    const size_t smem = prefill_smem(DPL * 32);
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e =
            cudaFuncSetAttribute(prefill_attn_kernel<DPL>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        configured[dev & 63] = true;
    }
    const dim3 grid((p.T + p.tq - 1) / p.tq, p.Hkv, B);
    prefill_attn_kernel<DPL><<<grid, kPThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

bool prefill_attention_supported(int Hq, int Hkv, int D) {
    return D >= 32 && D <= 256 && D % 32 == 0 && Hkv >= 1 && Hq >= Hkv && Hq % Hkv == 0 && Hq / Hkv <= kPRows;
}

cudaError_t launch_prefill_attention(const PrefillArgs& a, cudaStream_t stream) {
    if (!prefill_attention_supported(a.Hq, a.Hkv, a.D) || a.B < 1 || a.T < 1 || a.S < 1) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) |
         reinterpret_cast<uintptr_t>(a.out)) & 15 || a.kv_stride % 4 != 0 || a.kv_stride < a.Hkv * a.D)
        return cudaErrorInvalidValue;
    PrefillParams p;
    p.out = a.out;
    p.q = a.q;
    p.k = a.k;
    p.v = a.v;
    p.q_tok = static_cast<long long>(a.Hq) * a.D;
    p.q_batch = p.q_tok * a.T;
    p.kv_pos = a.kv_stride;
    p.kv_batch = static_cast<long long>(a.kv_stride) * a.S;
    p.T = a.T;
    p.S = a.S;
    p.Hq = a.Hq;
    p.Hkv = a.Hkv;
    p.group = a.Hq / a.Hkv;
    p.tq = std::max(1, kPRows / p.group);
    p.off = a.causal_offset;
    p.causal = a.causal ? 1 : 0;
    p.window = a.window > 0 ? a.window : 0;
    p.scale = a.scale;
    p.softcap = a.soft_cap;
    switch (a.D / 32) {
        case 1: return launch_dpl<1>(p, a.B, stream);
        case 2: return launch_dpl<2>(p, a.B, stream);
        case 3: return launch_dpl<3>(p, a.B, stream);
        case 4: return launch_dpl<4>(p, a.B, stream);
        case 5: return launch_dpl<5>(p, a.B, stream);
        case 6: return launch_dpl<6>(p, a.B, stream);
        case 7: return launch_dpl<7>(p, a.B, stream);
        default: return launch_dpl<8>(p, a.B, stream);
    }
}

}  // namespace alj
