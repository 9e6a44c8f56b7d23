// Decode attention for callers that cannot allocate device memory.
//
// Some hosts of this library run where no allocation may happen at call
// time: a JVM that hands over only pre-allocated device buffers through FFM,
// an embedding with a fixed memory budget reserved up front, or code that
// runs while a memory pool is locked.  The split-K attention needs a
// scratch area for the partial results of its splits, which the regular
// entry points obtain with cudaMalloc.  This file provides the same
// computation with that scratch in a fixed-size array compiled into the
// library: g_attn_scratch (kNoAllocScratchFloats floats = 4 MiB), which
// every GPU that loads the library keeps until the process exits.
//
// The array's name is a host-side stand-in in host code, not a device
// address; its device address is looked up with cudaGetSymbolAddress once
// per device, with that device current, on the entry point's first call on
// that device (so make that first call before any stream capture).  The
// entry point calls no cudaMalloc, cudaFree, stream or allocating library
// routine.  All calls share the array and it keeps the last call's
// contents.  Every split writes its whole slot before the merge reads it;
// the only words that must start at zero are the per-kv-head arrival
// counters at the head of the array, which each call clears on its stream
// (cudaMemsetAsync) before its kernel runs.  Calls whose kernels overlap on
// the GPU (on different streams, or from several threads) race on the array
// and must be ordered by the caller.
#include "common.cuh"

#include <mutex>

namespace alj {
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(1) << 20;
__device__ __align__(256) float g_attn_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

}  // namespace

int decode_fail(int code, const char* msg);

// Forget the looked-up device addresses (aljabr_blackwell_shutdown): after a
// device reset the array may sit at a new address, so the next call looks
// it up again.
void noalloc_forget_scratch() {
    std::lock_guard<std::mutex> g(g_scratch_mu);
    for (int d = 0; d < kMaxDevices; ++d) g_scratch_ptr[d] = nullptr;
}

}  // namespace alj

using namespace alj;

extern "C" int aljabr_blackwell_decode_attention_noalloc(float* out, const float* q, const void* k_cache,
                                                         const void* v_cache, int kv_dtype, int cache_head_stride,
                                                         int kv_heads, int q_heads, int head_dim, int seq_len,
                                                         int start_pos, float scale, void* stream) {
    if (!out || !q || !k_cache || !v_cache) return decode_fail(ALJ_ERR_BAD_ARG, "null pointer argument");
    if (kv_dtype != ALJ_KV_F32 && kv_dtype != ALJ_KV_BF16) return decode_fail(ALJ_ERR_UNSUPPORTED, "kv dtype");
    if (kv_heads <= 0 || head_dim <= 0 || q_heads <= 0 || q_heads % kv_heads)
        return decode_fail(ALJ_ERR_BAD_DIMS, "query heads must be a positive multiple of KV heads");
    if (cache_head_stride < kv_heads * head_dim) return decode_fail(ALJ_ERR_BAD_DIMS, "stride < kv_heads*head_dim");
    if (start_pos < 0 || start_pos >= seq_len) return decode_fail(ALJ_ERR_BAD_DIMS, "start outside [0, seq_len)");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return decode_fail(ALJ_ERR_NOT_INITIALIZED, "no current CUDA device");
    }
    float* scratch = nullptr;
    {
        std::lock_guard<std::mutex> g(g_scratch_mu);
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
            if (e != cudaSuccess || !p) {
                cudaGetLastError();
                return decode_fail(ALJ_ERR_CUDA, "cudaGetSymbolAddress(g_attn_scratch) failed");
            }
            g_scratch_ptr[dev] = static_cast<float*>(p);
        }
        scratch = g_scratch_ptr[dev];
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        return decode_fail(ALJ_ERR_CUDA, "querying the SM count failed");
    }
    AttnParams p = {};
    p.out = out;
    p.q = q;
    p.k = k_cache;
    p.v = v_cache;
    p.kv_dtype = kv_dtype;
    p.stride = cache_head_stride;
    p.head_stride = head_dim;
    p.kv_heads = kv_heads;
    p.q_heads = q_heads;
    p.head_dim = head_dim;
    p.seq_len = seq_len;
    p.start_pos = start_pos;
    p.scale = scale;
    p.splits = attention_splits(seq_len - start_pos, kv_heads, sms);
    if (p.splits > 1) {
        if (attention_scratch_floats(q_heads, head_dim, p.splits) > kNoAllocScratchFloats)
            return decode_fail(ALJ_ERR_BAD_DIMS,
                               "the split scratch (q_heads * splits * (head_dim + 2) floats and counters) exceeds the "
                               "1,048,576-float static scratch of "
                               "aljabr_blackwell_decode_attention_noalloc");
        attention_bind_scratch(p, scratch);
        if (cudaMemsetAsync(p.split_counter, 0, static_cast<size_t>(q_heads) * sizeof(unsigned int),
                            static_cast<cudaStream_t>(stream)) != cudaSuccess) {
            cudaGetLastError();
            return decode_fail(ALJ_ERR_CUDA, "clearing the split counters failed");
        }
    }
    const cudaError_t e = launch_attention(p, static_cast<cudaStream_t>(stream), false);
    if (e == cudaErrorNotSupported) return decode_fail(ALJ_ERR_UNSUPPORTED, "decode attention: shape not supported");
    if (e != cudaSuccess) return decode_fail(ALJ_ERR_CUDA, cudaGetErrorString(e));
    return ALJ_OK;
}
