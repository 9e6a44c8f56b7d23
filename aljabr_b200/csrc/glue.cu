// Elementwise decode glue that the reference's FFM class binds next to the
// matvec and attention entry points (BlackwellBinding.java:574-583):
// RMSNorm and the SiLU-gated FFN product, with the arithmetic of the
// binding's own contract (BlackwellCpuFallback.java:50-79).
#include "common.cuh"

#include <algorithm>

namespace alj {
namespace {

constexpr int kNormThreads = 1024;

// One CTA: fixed-order tree sum of x^2 (deterministic), then
// out[i] = (x[i] / rms) * w[i] with rms = sqrt(sum / N + eps) -- fp32,
// IEEE division and square root as Java's float '/' and the float cast of
// Math.sqrt on a float argument give.
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(float* out, const float* x, const float* w, int n,
                                                               float eps) {
    __shared__ float red[kNormThreads / 32];
    __shared__ float s_rms;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += kNormThreads) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = red[threadIdx.x];
        v = warp_sum(v);
        if (threadIdx.x == 0) s_rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(v, static_cast<float>(n)), eps));
    }
    __syncthreads();
    const float rms = s_rms;
    for (int i = threadIdx.x; i < n; i += kNormThreads) out[i] = __fmul_rn(__fdiv_rn(x[i], rms), w[i]);
}

// out[i] = g / (1 + exp(-g)) * up[i]; aliasing of out with gate and/or up is
// allowed (each element is read before it is written by the same thread).
__global__ void silu_ffn_kernel(float* out, const float* gate, const float* up, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float g = gate[i];
        const float u = up[i];
        const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        out[i] = __fmul_rn(s, u);
    }
}

constexpr int kPullThreads = 256;
constexpr int kPullPerThread = 4;                           // float4 loads in flight per thread
constexpr int kPullCtaElems = kPullThreads * kPullPerThread;   // float4s per CTA round

// Pulls n floats from mapped pinned host memory into device memory.  The
// host-buffer entry points stage their inputs this way rather than with a
// copy-engine transfer, whose set-up costs more than the PCIe read itself
// at these sizes (KB to a few MB).  The kernel releases its dependent launch
// at once, so a consumer launched with programmatic dependent launch does
// its set-up and first weight copies while the reads are in flight (its
// griddepcontrol.wait still waits for this grid to finish).  dst and src
// are 16-byte aligned.
__global__ void __launch_bounds__(kPullThreads) host_pull_kernel(float* __restrict__ dst,
                                                                 const float* __restrict__ src, size_t n) {
    pdl_launch_dependents();
    const size_t n4 = n / 4;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (size_t base = static_cast<size_t>(blockIdx.x) * kPullCtaElems; base < n4;
         base += static_cast<size_t>(gridDim.x) * kPullCtaElems) {
        float4 v[kPullPerThread];
#pragma unroll
        for (int k = 0; k < kPullPerThread; ++k) {
            const size_t i = base + k * kPullThreads + threadIdx.x;
            if (i < n4) v[k] = s4[i];
        }
#pragma unroll
        for (int k = 0; k < kPullPerThread; ++k) {
            const size_t i = base + k * kPullThreads + threadIdx.x;
            if (i < n4) d4[i] = v[k];
        }
    }
    if (blockIdx.x == 0)
        for (size_t j = n4 * 4 + threadIdx.x; j < n; j += kPullThreads) dst[j] = src[j];
}

}  // namespace

cudaError_t launch_host_pull(float* dst, const float* src_mapped, size_t n, int sms, cudaStream_t stream) {
    if (n == 0) return cudaSuccess;
    const size_t rounds = (n / 4 + kPullCtaElems - 1) / kPullCtaElems;
    const int blocks = static_cast<int>(std::max<size_t>(1, std::min<size_t>(rounds, 2 * std::max(1, sms))));
    host_pull_kernel<<<blocks, kPullThreads, 0, stream>>>(dst, src_mapped, n);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(float* out, const float* x, const float* w, int n, float eps, cudaStream_t stream) {
    rmsnorm_kernel<<<1, kNormThreads, 0, stream>>>(out, x, w, n, eps);
    return cudaGetLastError();
}

cudaError_t launch_silu_ffn(float* out, const float* gate, const float* up, int n, int sms, cudaStream_t stream) {
    const int blocks = std::max(1, std::min(4 * sms, (n + 255) / 256));
    silu_ffn_kernel<<<blocks, 256, 0, stream>>>(out, gate, up, n);
    return cudaGetLastError();
}

}  // namespace alj
