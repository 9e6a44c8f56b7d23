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

}  // namespace

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
