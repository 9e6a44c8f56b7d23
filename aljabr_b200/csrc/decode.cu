// Full batch-1 decode step of a Llama-shaped model with NF4 linear weights,
// resident in HBM and replayed as one CUDA graph per token.  This is the
// device-resident counterpart of the reference's per-layer loop
// (engine/gguf/aljabr-gguf-java/.../GgufDecodePass.java:297-545) and of the
// Metal provider's registered-layer decode step (aljabr_metal_matvec_api.h:
// aljabr_metal_register_decode_layer / aljabr_metal_decode_step_token).
//
// Per layer (one GPU, NF4 weights): q/k/v triple matvec that scales its
// input by the deferred RMSNorm -> RoPE + KV store -> attention (one launch,
// split merge fused into its last CTAs) -> o-proj whose epilogue adds the
// residual and writes x, x * norm_w and one sum of squares per CTA (the
// RMSNorm scale is applied by the consumer) -> gate/up pair whose epilogue
// applies SwiGLU -> down-proj whose epilogue does as the o-proj's for the
// next layer.  Six launches per layer, chained with programmatic dependent
// launch inside one CUDA graph.  GGUF-typed weights run SwiGLU as a separate
// small launch; their residual + RMSNorm is deferred the same way when every
// matvec can carry it (typed_fusable), else it is a separate launch too.
// Projections of mixed types (Q4_K q / k with a Q6_K v) launch once per run
// of equal types.  Forming SiLU(gate) * up inside the down projection's x
// conversion instead of the SwiGLU launch measured slower (549 against 556
// tok/s for Q4_0 weights): the extra dependent load sits on that launch's
// critical path after its dependency wait, where the small launch overlaps
// the down projection's weight prologue.
//
// Tensor parallelism (2/4/8 GPUs, one process per GPU): every weight is
// row-sharded (the caller passes each rank's contiguous row block) and
// attention is local to the rank's heads.  Output slices are joined over
// NVLink by the kernels that produce them: at model creation the ranks map
// each other's exchange buffers (CUDA IPC, handles swapped through NCCL);
// the attention combine and the o / gate-up / down / lm_head epilogues store
// their rows into every rank's copy and publish a per-layer flag value with
// a system-scope release; the consuming kernel (or the RMSNorm join) waits
// for all ranks' flags with a bounded acquire spin.  When the projections
// cannot run the table kernel (K not a multiple of 2048) or the mapping
// fails on any rank, the slices are joined with ncclAllGather instead; both
// paths are captured in the per-token graph.  The NVLink path is opt-in
// (ALJ_TP_EXCHANGE=p2p): at Llama-3-8B shapes it measured 287 tok/s at TP 2
// against 326 for ncclAllGather, because each exchange adds a system-scope
// fence and a last-CTA publication to a launch whose fixed cost already
// dominates at 2048 rows per rank.
#include "common.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <array>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

namespace alj {
namespace {

// ------------------------------------------------------------------ NCCL
// NCCL is bound at run time, the first time a tensor-parallel model is
// created, so that loading this library never pins a libnccl.so.2 version
// into the process.  If the host process already loaded NCCL (for example
// through its ML framework), that copy is used; otherwise the system one.
struct NcclApi {
    bool tried = false, ok = false;
    ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
};
NcclApi g_nccl;
std::mutex g_nccl_mu;

bool nccl_load() {
    std::lock_guard<std::mutex> g(g_nccl_mu);
    if (g_nccl.tried) return g_nccl.ok;
    g_nccl.tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return false;
    g_nccl.getUniqueId = reinterpret_cast<decltype(g_nccl.getUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    g_nccl.commInitRank = reinterpret_cast<decltype(g_nccl.commInitRank)>(dlsym(h, "ncclCommInitRank"));
    g_nccl.allGather = reinterpret_cast<decltype(g_nccl.allGather)>(dlsym(h, "ncclAllGather"));
    g_nccl.commDestroy = reinterpret_cast<decltype(g_nccl.commDestroy)>(dlsym(h, "ncclCommDestroy"));
    g_nccl.ok = g_nccl.getUniqueId && g_nccl.commInitRank && g_nccl.allGather && g_nccl.commDestroy;
    return g_nccl.ok;
}

// ------------------------------------------------------------------ kernels
// Block-wide sum over a 1024-thread CTA (result in every thread).
__device__ __forceinline__ float block_sum_1024(float v, float* red) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < 32; ++w) t += red[w];
    __syncthreads();
    return t;
}

// io = {pos, token, argmax, -, argmax key (u64, io[4..5]), token counter (io[6],
// starts at 1; the tensor-parallel flag values derive from it)}.  First kernel of a step:
// x = dequantised embedding row of the token; xn = RMSNorm(x) * norm_w (the
// first layer's attention norm, GGUFVectorOps.rmsNorm); clears the argmax key.
// One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) embed_nf4_kernel(float* x, float* xn, const uint8_t* codes,
                                                         const float* absmax, int* io, int H, int group,
                                                         const float* norm_w, float eps) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const long long base = static_cast<long long>(io[1]) * H;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const long long e = base + i;
        const int b = codes[e >> 1];
        const int code = (e & 1) ? (b & 15) : (b >> 4);
        const float v = __fmul_rn(nf4_value(code), absmax[((e >> 1) * 2) / group]);
        x[i] = v;
        ss = fmaf(v, v, ss);
    }
    const float scale = 1.0f / sqrtf(block_sum_1024(ss, red) / static_cast<float>(H) + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) xn[i] = x[i] * scale * norm_w[i];
    if (threadIdx.x == 0) *reinterpret_cast<unsigned long long*>(io + 4) = 0ull;
}

// One value of a GGUF row, in the reference's dequantiser float order:
// Q4_0 / Q8_0 as GgufBlockDequantizer (q - 8) * d + 0.0f and q * d; Q4_K as
// GgufKBlockDequantizer.dequantizeQ4KBlock (:32-75), d1 = d * scale,
// m1 = dmin * min, d1 * q - m1; Q6_K as dequantizeQ6KBlock (:320-360),
// (d * scale) * (q - 32).  Bytes are read one at a time (rows of 18- and
// 210-byte blocks are only 2-byte aligned).
__device__ float gguf_value(int fmt, const uint8_t* row, int i) {
    auto f16 = [](const uint8_t* b) { return f16_bits_to_f32(static_cast<uint32_t>(b[0]) | (b[1] << 8)); };
    if (fmt == FMT_Q4_0 || fmt == FMT_Q8_0) {
        const int j = i & 31;
        const uint8_t* blk = row + (i >> 5) * (fmt == FMT_Q4_0 ? 18 : 34);
        const float d = f16(blk);
        if (fmt == FMT_Q8_0) return __fmul_rn(static_cast<float>(static_cast<signed char>(blk[2 + j])), d);
        const int byte = blk[2 + (j & 15)];
        const int q = j < 16 ? (byte & 15) : (byte >> 4);
        return __fadd_rn(__fmul_rn(static_cast<float>(q - 8), d), 0.0f);
    }
    const int e = i & 255;
    if (fmt == FMT_Q4_K) {
        const uint8_t* blk = row + (i >> 8) * 144;
        const int j = e >> 6, t = e & 63, sb = 2 * j + (t >= 32);
        const int byte = blk[16 + 32 * j + (t & 31)];
        const int q = t < 32 ? (byte & 15) : (byte >> 4);
        const uint8_t* sc = blk + 4;
        int s, mn;
        if (sb < 4) {
            s = sc[sb] & 63;
            mn = sc[sb + 4] & 63;
        } else {
            s = (sc[sb + 4] & 15) | ((sc[sb - 4] >> 6) << 4);
            mn = (sc[sb + 4] >> 4) | ((sc[sb] >> 6) << 4);
        }
        const float d1 = __fmul_rn(f16(blk), static_cast<float>(s));
        const float m1 = __fmul_rn(f16(blk + 2), static_cast<float>(mn));
        return __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
    }
    const uint8_t* blk = row + (i >> 8) * 210;   // Q6_K
    const int h = e >> 7, w = e & 127, k = w >> 5, ii = w & 31;
    const int lo = blk[64 * h + 32 * (k & 1) + ii];
    const int hb = blk[128 + 32 * h + ii];
    const int q = (((k >> 1) ? (lo >> 4) : (lo & 15)) | (((hb >> (2 * k)) & 3) << 4)) - 32;
    const float s = __fmul_rn(f16(blk + 208), static_cast<float>(static_cast<signed char>(blk[192 + 8 * h + 2 * k + ii / 16])));
    return __fmul_rn(s, static_cast<float>(q));
}

// embed_nf4_kernel for a GGUF-typed embedding table (row_bytes per token row).
__global__ void __launch_bounds__(1024) embed_gguf_kernel(float* x, float* xn, const uint8_t* table, int fmt,
                                                          long long row_bytes, int* io, int H, const float* norm_w,
                                                          float eps) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    const uint8_t* row = table + static_cast<long long>(io[1]) * row_bytes;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const float v = gguf_value(fmt, row, i);
        x[i] = v;
        ss = fmaf(v, v, ss);
    }
    const float scale = 1.0f / sqrtf(block_sum_1024(ss, red) / static_cast<float>(H) + eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x) xn[i] = x[i] * scale * norm_w[i];
    if (threadIdx.x == 0) *reinterpret_cast<unsigned long long*>(io + 4) = 0ull;
}

// h = SiLU(gate) * up (GGUFVectorOps.swiglu, the matvec epilogues' formula),
// in place over `up`, for projections whose kernel has no SwiGLU epilogue.
__global__ void swiglu_kernel(const float* gate, float* up, int n) {
    pdl_launch_dependents();
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float g = gate[i];
        up[i] = g / (1.0f + expf(-g)) * up[i];
    }
}

// Split-half RoPE (GGUFVectorOps.rope, GGUFVectorOps.java:383-440) on the
// rank's q and k heads, then the KV store at `pos`
// (GgufKvCacheWriteExecution.storeToken).  rope[pos * D/2 + i] holds
// (cos, sin) of the reference's angle, computed on the host once.
__global__ void rope_store_kernel(float* q, float* k, const float* v, void* kc, void* vc, const int* io,
                                  const float2* rope, int hq, int hkv, int D, int kv_dtype) {
    pdl_launch_dependents();
    pdl_wait();
    const int pos = io[0];
    const int half = D / 2;
    const int stride = hkv * D;
    const int pairs = (hq + hkv) * half;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < pairs; idx += gridDim.x * blockDim.x) {
        const int head = idx / half, i = idx - head * half;
        const float2 cs = rope[static_cast<long long>(pos) * half + i];
        const float c = cs.x, s = cs.y;
        float* b = head < hq ? q + head * D : k + (head - hq) * D;
        const float x0 = b[i], x1 = b[i + half];
        const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        b[i] = r0;
        b[i + half] = r1;
        if (head >= hq) {
            const long long off = static_cast<long long>(pos) * stride + (head - hq) * D + i;
            if (kv_dtype == ALJ_KV_BF16) {
                static_cast<__nv_bfloat16*>(kc)[off] = __float2bfloat16_rn(r0);
                static_cast<__nv_bfloat16*>(kc)[off + half] = __float2bfloat16_rn(r1);
            } else {
                static_cast<float*>(kc)[off] = r0;
                static_cast<float*>(kc)[off + half] = r1;
            }
        }
    }
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < stride; idx += gridDim.x * blockDim.x) {
        const long long off = static_cast<long long>(pos) * stride + idx;
        if (kv_dtype == ALJ_KV_BF16) static_cast<__nv_bfloat16*>(vc)[off] = __float2bfloat16_rn(v[idx]);
        else static_cast<float*>(vc)[off] = v[idx];
    }
}

// Tensor-parallel residual join: x += delta (the all-gathered slices), then
// xn = RMSNorm(x) * norm_w for the next matvec.  One CTA of 1024 threads.
__global__ void __launch_bounds__(1024) add_norm_kernel(float* x, const float* d, float* xn, const float* norm_w,
                                                        int n, float eps) {
    __shared__ float red[32];
    pdl_launch_dependents();
    pdl_wait();
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x[i] + d[i];
        x[i] = v;
        ss = fmaf(v, v, ss);
    }
    const float scale = 1.0f / sqrtf(block_sum_1024(ss, red) / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) xn[i] = x[i] * scale * norm_w[i];
}

// Tensor-parallel join after a row-sharded projection whose epilogue pushed
// this rank's rows of x (and its sum of squares) to every rank: wait until
// every rank's flag reaches (*seq) * mul + add, then xn = RMSNorm(x) * norm_w
// from the summed partials (fixed rank order).  One CTA of 1024 threads.
// Peer-written data is read through L2 (__ldcg) after the acquire.
__global__ void __launch_bounds__(1024) tp_norm_kernel(const float* x, float* xn, const float* norm_w, int n,
                                                       float eps, const float* part, const unsigned int* flags,
                                                       int tp, const int* seq, int mul, int add) {
    __shared__ float s_scale;
    pdl_launch_dependents();
    pdl_wait();
    const unsigned int target = static_cast<unsigned int>(*seq * mul + add);
    if (threadIdx.x == 0) {
        wait_flags_sys(flags, tp, target);
        float tot = 0.0f;
        for (int r = 0; r < tp; ++r) tot += __ldcg(part + r);
        s_scale = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    }
    __syncthreads();
    for (int r = 0; r < tp; ++r) (void)ld_acquire_sys(flags + r);
    const float scale = s_scale;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xn[i] = __ldcg(x + i) * scale * norm_w[i];
}

// Greedy hand-off inside the graph: the step's argmax becomes the next
// step's token, the position advances, and the token is logged at `pos`.
__global__ void advance_kernel(int* io, int* tokens, int max_ctx) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        const unsigned long long key = *reinterpret_cast<const unsigned long long*>(io + 4);
        // key 0: no finite logit was seen (all NaN); fall back to token 0
        const int idx = key ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key & 0xFFFFFFFFull)) : 0;
        const int pos = io[0];
        io[2] = idx;
        if (pos >= 0 && pos < max_ctx) tokens[pos] = idx;
        io[1] = idx;
        io[0] = pos + 1 < max_ctx ? pos + 1 : max_ctx - 1;
        io[6] = io[6] + 1;
    }
}

// Greedy sampling: index of the maximum logit, the first one on ties.  Each
// CTA reduces a slice and folds (order-preserving value bits, ~index) into
// one 64-bit atomicMax.
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
}

__global__ void argmax_kernel(const float* logits, int n, int* io, const unsigned int* flags, int tp) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned long long sk[32];
    if (flags) {   // tensor parallel: the logits slices are pushed by every rank
        if (threadIdx.x == 0) wait_flags_sys(flags, tp, static_cast<unsigned int>(io[6] + 1));
        __syncthreads();
        for (int r = 0; r < tp; ++r) (void)ld_acquire_sys(flags + r);
    }
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float v = __ldcg(logits + i);
        if (v == v) best = max(best, argmax_key(v, i));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) best = max(best, sk[w]);
        atomicMax(reinterpret_cast<unsigned long long*>(io + 4), best);
    }
}

template <typename... Args, typename... Actual>
cudaError_t launch_small(void (*kernel)(Args...), int grid, int block, cudaStream_t s, Actual... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Bytes of one row of `cols` values in a GGUF block format (NF4: packed codes).
long long gguf_row_bytes(int fmt, int cols) {
    switch (fmt) {
        case FMT_Q4_0: return cols / 32 * 18LL;
        case FMT_Q8_0: return cols / 32 * 34LL;
        case FMT_Q4_K: return cols / 256 * 144LL;
        case FMT_Q6_K: return cols / 256 * 210LL;
        default: return cols / 2;
    }
}

// ------------------------------------------------------------------ model
// One registered weight matrix: row-major ggml blocks of `fmt` (WeightFormat),
// or NF4 codes with their absmax scales.
struct Weight {
    const uint8_t* codes = nullptr;
    const float* absmax = nullptr;
    int fmt = FMT_NF4;
};

enum { W_Q = 0, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_COUNT };

struct DecodeModel {
    int device = 0;
    int layers, H, Hq, Hkv, D, F, V, max_ctx, group, kv_dtype;
    float eps, theta;
    int T = 1, rank = 0;
    int hq, hkv, f, h, v;              // this rank's shard sizes
    std::vector<std::array<Weight, W_COUNT>> w;
    std::vector<bool> layer_set;
    Weight embd, head;
    bool output_set = false;
    float* norms = nullptr;            // [layers][2][H] then [H]
    float2* rope = nullptr;            // [max_ctx][D/2] (cos, sin)
    void *kc = nullptr, *vc = nullptr; // [layers][max_ctx][hkv*D]
    float *x, *xn, *q, *k, *vv, *att_l, *att, *delta_l, *delta, *h_l, *hh, *logits_l, *logits, *scratch;
    float* norm_partials = nullptr;    // [matvec_max_ctas()] per-CTA sums of squares
    bool defer_norm = false;           // RMSNorm scale applied by the consuming matvec (one GPU)
    bool typed = false;                // some tensor is not NF4: SwiGLU (and maybe residual / norm) launched apart
    unsigned int* norm_counter = nullptr;
    float* act_base = nullptr;
    int* io = nullptr;                 // device {pos, token, argmax}
    int* tokens = nullptr;             // device [max_ctx]: greedy token emitted at each position
    int* host_io = nullptr;            // pinned
    float* host_logits = nullptr;      // pinned
    int splits = 1;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t exec = nullptr;
    int steps_run = 0;
    ncclComm_t comm = nullptr;
    // NVLink exchange (T > 1, p2p): one IPC-shared arena per rank holding the
    // replicated residual x, the gathered attention output, SwiGLU output and
    // logits, the per-rank sums of squares and the flags; peer_arena[r] is
    // rank r's arena mapped here (peer_arena[rank] == arena).
    bool p2p = false;
    uint8_t* arena = nullptr;
    uint8_t* peer_arena[kMaxTp] = {};
    size_t off_x = 0, off_att = 0, off_hh = 0, off_logits = 0, off_part_o = 0, off_part_d = 0, off_flags = 0,
           arena_bytes = 0;
    std::mutex mu;

    size_t kv_elem() const { return kv_dtype == ALJ_KV_BF16 ? 2 : 4; }
    size_t kv_layer_elems() const { return static_cast<size_t>(max_ctx) * hkv * D; }
};

std::mutex g_models_mu;
std::map<unsigned long long, std::unique_ptr<DecodeModel>> g_models;
unsigned long long g_next_handle = 1;

DecodeModel* find(unsigned long long h) {
    std::lock_guard<std::mutex> g(g_models_mu);
    auto it = g_models.find(h);
    return it == g_models.end() ? nullptr : it->second.get();
}

// One NF4 matvec launch over 1-3 row segments sharing x.
// With m.defer_norm (one GPU, every K on the NF4 table kernel), a launch
// given norm_out leaves x * norm_w and its per-CTA sums of squares, and
// `scaled_x` marks a launch whose x is such a vector: it applies the
// RMSNorm scale to its outputs from those partials.
cudaError_t matvec(const DecodeModel& m, const Weight* ws, float* const* ys, const int* rows, int n, const float* x,
                   int K, int epilogue, const float* residual, float* norm_out, const float* norm_w,
                   const TpLink* tpl = nullptr, bool scaled_x = false) {
    MatvecParams p = {};
    if (tpl) {
        p.tpl = *tpl;
        p.norm_partials = m.norm_partials;
    }
    p.nseg = n;
    p.K = K;
    p.group = m.group;
    p.x = x;
    p.epilogue = epilogue;
    for (int i = 0; i < n; ++i) {
        p.seg[i].w = ws[i].codes;
        p.seg[i].absmax = ws[i].absmax;
        p.seg[i].y = ys[i];
        p.seg[i].rows = rows[i];
        p.seg[i].residual = residual;
        p.total_rows += rows[i];
    }
    if (epilogue == EPI_SWIGLU_PAIR) p.total_rows = rows[0];
    if (norm_out) {
        p.norm_out = norm_out;
        p.norm_w = norm_w;
        p.norm_eps = m.eps;
        p.norm_partials = m.norm_partials;
        p.norm_counter = m.norm_counter;
        p.norm_defer = m.defer_norm ? 1 : 0;
    }
    if (scaled_x && m.defer_norm) {
        p.in_parts = m.norm_partials;
        // the producing o / down launch has H rows; the table and the integer
        // tensor-core kernels both launch min(SMs, rows / 4) CTAs, one partial each
        p.in_nparts = matvec_lut_grid(m.H);
        p.in_rows = m.H;
        p.in_eps = m.eps;
    }
    bool same = true;
    for (int i = 1; i < n; ++i) same = same && ws[i].fmt == ws[0].fmt;
    if (same) return launch_matvec(ws[0].fmt, p, m.stream, true);
    // q/k/v of mixed GGUF types (e.g. Q4_K q/k with a Q6_K v): one launch per
    // run of segments of one type
    if (epilogue != EPI_STORE || norm_out) return cudaErrorNotSupported;
    for (int i = 0; i < n;) {
        int j = i + 1;
        while (j < n && ws[j].fmt == ws[i].fmt) ++j;
        MatvecParams run = p;
        run.nseg = j - i;
        run.total_rows = 0;
        for (int s = i; s < j; ++s) {
            run.seg[s - i] = p.seg[s];
            run.total_rows += rows[s];
        }
        const cudaError_t e = launch_matvec(ws[i].fmt, run, m.stream, true);
        if (e != cudaSuccess) return e;
        i = j;
    }
    return cudaSuccess;
}

#define REC(expr)                                  \
    do {                                           \
        cudaError_t _e = (expr);                   \
        if (_e != cudaSuccess) return _e;          \
    } while (0)
#define RECN(expr)                                             \
    do {                                                       \
        if ((expr) != ncclSuccess) return cudaErrorUnknown;    \
    } while (0)

// Enqueue one full decode step on m.stream (eagerly or under capture).
// A GGUF-typed model defers its RMSNorms to the consuming launches (as the
// NF4 step does) when every matvec of the step can: NF4 tensors on the
// table kernel, the others on the integer tensor-core kernel (K a multiple
// of 2048, rows in 4s, 16-byte aligned weights).
bool typed_fusable(const DecodeModel& m) {
    if (m.T != 1) return false;
    auto ok = [&](const Weight& w, int K, int rows) {
        if (w.fmt == FMT_NF4) return matvec_lut_supported(FMT_NF4, K, m.group) && rows % 4 == 0;
        return matvec_imma_supported(w.fmt, K) && rows % 4 == 0 && (reinterpret_cast<uintptr_t>(w.codes) & 15) == 0;
    };
    const int D = m.D;
    for (int l = 0; l < m.layers; ++l) {
        const auto& w = m.w[l];
        if (!ok(w[W_Q], m.H, m.hq * D) || !ok(w[W_K], m.H, m.hkv * D) || !ok(w[W_V], m.H, m.hkv * D) ||
            !ok(w[W_O], m.Hq * D, m.h) || !ok(w[W_GATE], m.H, m.f) || !ok(w[W_UP], m.H, m.f) ||
            !ok(w[W_DOWN], m.F, m.h))
            return false;
    }
    return ok(m.head, m.H, m.v);
}

cudaError_t record_step(DecodeModel& m) {
    if (m.typed) m.defer_norm = typed_fusable(m);
    const int D = m.D;
    const int sms = sm_count_for_current_device();
    const float* out_norm = m.norms + static_cast<size_t>(m.layers) * 2 * m.H;
    if (m.embd.fmt == FMT_NF4)
        REC(launch_small(embed_nf4_kernel, 1, 1024, m.stream, m.x, m.xn, m.embd.codes, m.embd.absmax, m.io, m.H,
                         m.group, static_cast<const float*>(m.norms), m.eps));
    else
        REC(launch_small(embed_gguf_kernel, 1, 1024, m.stream, m.x, m.xn, m.embd.codes, m.embd.fmt,
                         gguf_row_bytes(m.embd.fmt, m.H), m.io, m.H, static_cast<const float*>(m.norms), m.eps));
    for (int l = 0; l < m.layers; ++l) {
        const auto& w = m.w[l];
        const float* ffn_norm = m.norms + static_cast<size_t>(l) * 2 * m.H + m.H;
        const float* next_norm = l + 1 < m.layers ? m.norms + static_cast<size_t>(l + 1) * 2 * m.H : out_norm;
        void* kc = static_cast<uint8_t*>(m.kc) + static_cast<size_t>(l) * m.kv_layer_elems() * m.kv_elem();
        void* vc = static_cast<uint8_t*>(m.vc) + static_cast<size_t>(l) * m.kv_layer_elems() * m.kv_elem();
        {   // q, k, v from the normed x (GgufDecodePass.java:305-309)
            const Weight ws[3] = {w[W_Q], w[W_K], w[W_V]};
            float* ys[3] = {m.q, m.k, m.vv};
            const int rows[3] = {m.hq * D, m.hkv * D, m.hkv * D};
            // layer 0's x comes normed from the embedding kernel
            REC(matvec(m, ws, ys, rows, 3, m.xn, m.H, EPI_STORE, nullptr, nullptr, nullptr, nullptr, l > 0));
        }
        // RoPE on q and k, KV store (GgufDecodePass.java:333-362)
        REC(launch_small(rope_store_kernel, std::max(1, ((m.hq + m.hkv) * D / 2 + 255) / 256), 256, m.stream, m.q,
                         m.k, static_cast<const float*>(m.vv), kc, vc, static_cast<const int*>(m.io),
                         static_cast<const float2*>(m.rope), m.hq, m.hkv, D, m.kv_dtype));
        {   // attention (GgufDecodePass.java:368-389)
            AttnParams a = {};
            a.out = m.T > 1 ? m.att_l : m.att;
            a.q = m.q;
            a.k = kc;
            a.v = vc;
            a.kv_dtype = m.kv_dtype;
            a.stride = m.hkv * D;
            a.head_stride = D;
            a.kv_heads = m.hkv;
            a.q_heads = m.hq;
            a.head_dim = D;
            a.seq_len = m.max_ctx;
            a.start_pos = 0;
            a.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
            a.splits = m.splits;
            attention_bind_scratch(a, m.scratch);
            a.dev_pos = m.io;
            REC(launch_attention(a, m.stream, true));
        }
        if (m.T > 1) RECN(g_nccl.allGather(m.att_l, m.att, static_cast<size_t>(m.hq) * D, ncclFloat, m.comm, m.stream));
        {   // o-proj + residual (GgufDecodePass.java:475-481), then the FFN norm (:485)
            const Weight ws[1] = {w[W_O]};
            const int rows[1] = {m.h};
            if (m.T > 1) {
                float* ys[1] = {m.delta_l};
                REC(matvec(m, ws, ys, rows, 1, m.att, m.Hq * D, EPI_STORE, nullptr, nullptr, nullptr));
                RECN(g_nccl.allGather(m.delta_l, m.delta, m.h, ncclFloat, m.comm, m.stream));
                REC(launch_small(add_norm_kernel, 1, 1024, m.stream, m.x, static_cast<const float*>(m.delta), m.xn,
                                 ffn_norm, m.H, m.eps));
            } else if (m.typed && !m.defer_norm) {
                float* ys[1] = {m.delta};
                REC(matvec(m, ws, ys, rows, 1, m.att, m.Hq * D, EPI_STORE, nullptr, nullptr, nullptr));
                REC(launch_small(add_norm_kernel, 1, 1024, m.stream, m.x, static_cast<const float*>(m.delta), m.xn,
                                 ffn_norm, m.H, m.eps));
            } else {
                float* ys[1] = {m.x};
                REC(matvec(m, ws, ys, rows, 1, m.att, m.Hq * D, EPI_STORE, m.x, m.xn, ffn_norm));
            }
        }
        {   // gate / up with the SwiGLU epilogue (GgufDecodePass.java:492-497)
            const Weight ws[2] = {w[W_GATE], w[W_UP]};
            const int rows[2] = {m.f, m.f};
            if (m.typed) {   // one GPU: gate -> h_l, up -> hh, then hh = SiLU(h_l) * hh
                float* ys[2] = {m.h_l, m.hh};
                REC(matvec(m, ws, ys, rows, 2, m.xn, m.H, EPI_STORE, nullptr, nullptr, nullptr, nullptr, true));
                REC(launch_small(swiglu_kernel, std::max(1, std::min(sms, (m.F + 255) / 256)), 256, m.stream,
                                 static_cast<const float*>(m.h_l), m.hh, m.F));
            } else {
                float* ys[2] = {m.T > 1 ? m.h_l : m.hh, nullptr};
                REC(matvec(m, ws, ys, rows, 2, m.xn, m.H, EPI_SWIGLU_PAIR, nullptr, nullptr, nullptr, nullptr, true));
            }
        }
        if (m.T > 1) RECN(g_nccl.allGather(m.h_l, m.hh, m.f, ncclFloat, m.comm, m.stream));
        {   // down-proj + residual (GgufDecodePass.java:504-511), then the next layer's norm
            const Weight ws[1] = {w[W_DOWN]};
            const int rows[1] = {m.h};
            if (m.T > 1) {
                float* ys[1] = {m.delta_l};
                REC(matvec(m, ws, ys, rows, 1, m.hh, m.F, EPI_STORE, nullptr, nullptr, nullptr));
                RECN(g_nccl.allGather(m.delta_l, m.delta, m.h, ncclFloat, m.comm, m.stream));
                REC(launch_small(add_norm_kernel, 1, 1024, m.stream, m.x, static_cast<const float*>(m.delta), m.xn,
                                 next_norm, m.H, m.eps));
            } else if (m.typed && !m.defer_norm) {
                float* ys[1] = {m.delta};
                REC(matvec(m, ws, ys, rows, 1, m.hh, m.F, EPI_STORE, nullptr, nullptr, nullptr));
                REC(launch_small(add_norm_kernel, 1, 1024, m.stream, m.x, static_cast<const float*>(m.delta), m.xn,
                                 next_norm, m.H, m.eps));
            } else {
                float* ys[1] = {m.x};
                REC(matvec(m, ws, ys, rows, 1, m.hh, m.F, EPI_STORE, m.x, m.xn, next_norm));
            }
        }
    }
    {   // logits from the output-normed x (GgufLogitsProcessor.compute)
        const Weight ws[1] = {m.head};
        float* ys[1] = {m.T > 1 ? m.logits_l : m.logits};
        const int rows[1] = {m.v};
        REC(matvec(m, ws, ys, rows, 1, m.xn, m.H, EPI_STORE, nullptr, nullptr, nullptr, nullptr, true));
    }
    if (m.T > 1) RECN(g_nccl.allGather(m.logits_l, m.logits, m.v, ncclFloat, m.comm, m.stream));
    REC(launch_small(argmax_kernel, std::max(1, std::min(sms, (m.V + 1023) / 1024)), 1024, m.stream,
                     static_cast<const float*>(m.logits), m.V, m.io, static_cast<const unsigned int*>(nullptr), 0));
    REC(launch_small(advance_kernel, 1, 32, m.stream, m.io, m.tokens, m.max_ctx));
    return cudaSuccess;
}

enum { FL_ATT = 0, FL_XO, FL_H, FL_XD, FL_LOGITS, FL_COUNT };

// One decode step with the NVLink exchange (T > 1, p2p): the same launches
// as the single-GPU step, where each row-sharded projection pushes its rows
// to every rank, and each consumer waits for the flags of the push it reads.
// Flag value of a per-layer exchange: token counter * layers + layer + 1.
cudaError_t record_step_p2p(DecodeModel& m) {
    const int D = m.D, T = m.T, L = m.layers, R = m.rank;
    const int sms = sm_count_for_current_device();
    const float* out_norm = m.norms + static_cast<size_t>(L) * 2 * m.H;
    auto peer = [&](int r, size_t off) { return reinterpret_cast<float*>(m.peer_arena[r] + off); };
    auto flag_at = [&](int r, int kind) {
        return reinterpret_cast<unsigned int*>(m.peer_arena[r] + m.off_flags) + kind * kMaxTp + R;
    };
    auto local_flags = [&](int kind) {
        return reinterpret_cast<const unsigned int*>(m.arena + m.off_flags) + kind * kMaxTp;
    };
    auto link = [&](size_t off, int row0, size_t part_off, int kind, int mul, int add) {
        TpLink t = {};
        t.tp = T;
        t.counter = m.norm_counter;
        t.seq = m.io + 6;
        t.push_mul = mul;
        t.push_add = add;
        for (int r = 0; r < T; ++r) {
            t.push_y[r] = peer(r, off) + row0;
            t.push_part[r] = part_off ? peer(r, part_off) + R : nullptr;
            t.push_flag[r] = flag_at(r, kind);
        }
        return t;
    };
    float* x = peer(R, m.off_x);
    float* att = peer(R, m.off_att);
    float* hh = peer(R, m.off_hh);
    REC(launch_small(embed_nf4_kernel, 1, 1024, m.stream, x, m.xn, m.embd.codes, m.embd.absmax, m.io, m.H, m.group,
                     static_cast<const float*>(m.norms), m.eps));
    for (int l = 0; l < L; ++l) {
        const auto& w = m.w[l];
        const float* ffn_norm = m.norms + static_cast<size_t>(l) * 2 * m.H + m.H;
        const float* next_norm = l + 1 < L ? m.norms + static_cast<size_t>(l + 1) * 2 * m.H : out_norm;
        void* kc = static_cast<uint8_t*>(m.kc) + static_cast<size_t>(l) * m.kv_layer_elems() * m.kv_elem();
        void* vc = static_cast<uint8_t*>(m.vc) + static_cast<size_t>(l) * m.kv_layer_elems() * m.kv_elem();
        {   // q, k, v of this rank's heads
            const Weight ws[3] = {w[W_Q], w[W_K], w[W_V]};
            float* ys[3] = {m.q, m.k, m.vv};
            const int rows[3] = {m.hq * D, m.hkv * D, m.hkv * D};
            REC(matvec(m, ws, ys, rows, 3, m.xn, m.H, EPI_STORE, nullptr, nullptr, nullptr));
        }
        REC(launch_small(rope_store_kernel, std::max(1, ((m.hq + m.hkv) * D / 2 + 255) / 256), 256, m.stream, m.q,
                         m.k, static_cast<const float*>(m.vv), kc, vc, static_cast<const int*>(m.io),
                         static_cast<const float2*>(m.rope), m.hq, m.hkv, D, m.kv_dtype));
        {   // attention of this rank's heads, pushed into every rank's att
            AttnParams a = {};
            a.out = att + R * m.hq * D;
            a.q = m.q;
            a.k = kc;
            a.v = vc;
            a.kv_dtype = m.kv_dtype;
            a.stride = m.hkv * D;
            a.head_stride = D;
            a.kv_heads = m.hkv;
            a.q_heads = m.hq;
            a.head_dim = D;
            a.seq_len = m.max_ctx;
            a.start_pos = 0;
            a.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
            a.splits = m.splits;
            attention_bind_scratch(a, m.scratch);
            a.dev_pos = m.io;
            a.tpl = link(m.off_att, R * m.hq * D, 0, FL_ATT, L, l + 1);
            REC(launch_attention(a, m.stream, true));
        }
        {   // o-proj: x rows += W_o att, pushed with this rank's sum of squares; then the FFN norm
            const Weight ws[1] = {w[W_O]};
            const int rows[1] = {m.h};
            float* ys[1] = {x + R * m.h};
            TpLink t = link(m.off_x, R * m.h, m.off_part_o, FL_XO, L, l + 1);
            t.wait_flags = local_flags(FL_ATT);
            t.wait_mul = L;
            t.wait_add = l + 1;
            REC(matvec(m, ws, ys, rows, 1, att, m.Hq * D, EPI_STORE, x + R * m.h, nullptr, nullptr, &t));
            REC(launch_small(tp_norm_kernel, 1, 1024, m.stream, static_cast<const float*>(x), m.xn, ffn_norm, m.H,
                             m.eps, static_cast<const float*>(peer(R, m.off_part_o)), local_flags(FL_XO), T,
                             static_cast<const int*>(m.io + 6), L, l + 1));
        }
        {   // gate / up with the SwiGLU epilogue, pushed into every rank's hh
            const Weight ws[2] = {w[W_GATE], w[W_UP]};
            float* ys[2] = {hh + R * m.f, nullptr};
            const int rows[2] = {m.f, m.f};
            TpLink t = link(m.off_hh, R * m.f, 0, FL_H, L, l + 1);
            REC(matvec(m, ws, ys, rows, 2, m.xn, m.H, EPI_SWIGLU_PAIR, nullptr, nullptr, nullptr, &t));
        }
        {   // down-proj: x rows += W_down hh, pushed; then the next norm
            const Weight ws[1] = {w[W_DOWN]};
            const int rows[1] = {m.h};
            float* ys[1] = {x + R * m.h};
            TpLink t = link(m.off_x, R * m.h, m.off_part_d, FL_XD, L, l + 1);
            t.wait_flags = local_flags(FL_H);
            t.wait_mul = L;
            t.wait_add = l + 1;
            REC(matvec(m, ws, ys, rows, 1, hh, m.F, EPI_STORE, x + R * m.h, nullptr, nullptr, &t));
            REC(launch_small(tp_norm_kernel, 1, 1024, m.stream, static_cast<const float*>(x), m.xn, next_norm, m.H,
                             m.eps, static_cast<const float*>(peer(R, m.off_part_d)), local_flags(FL_XD), T,
                             static_cast<const int*>(m.io + 6), L, l + 1));
        }
    }
    {   // logits of this rank's vocabulary rows, pushed into every rank's logits
        const Weight ws[1] = {m.head};
        float* ys[1] = {peer(R, m.off_logits) + R * m.v};
        const int rows[1] = {m.v};
        TpLink t = link(m.off_logits, R * m.v, 0, FL_LOGITS, 1, 1);
        REC(matvec(m, ws, ys, rows, 1, m.xn, m.H, EPI_STORE, nullptr, nullptr, nullptr, &t));
    }
    REC(launch_small(argmax_kernel, std::max(1, std::min(sms, (m.V + 1023) / 1024)), 1024, m.stream,
                     static_cast<const float*>(peer(R, m.off_logits)), m.V, m.io, local_flags(FL_LOGITS), T));
    REC(launch_small(advance_kernel, 1, 32, m.stream, m.io, m.tokens, m.max_ctx));
    return cudaSuccess;
}

// Enqueue n steps: the first ever step runs eagerly (NCCL connects there),
// later ones replay the captured graph.  No synchronisation.
cudaError_t enqueue_steps(DecodeModel& m, int n) {
    for (int i = 0; i < n; ++i) {
        cudaError_t e = cudaSuccess;
        if (m.steps_run == 0) {
            e = m.p2p ? record_step_p2p(m) : record_step(m);
        } else {
            if (!m.exec) {
                cudaGraph_t graph = nullptr;
                e = cudaStreamBeginCapture(m.stream, cudaStreamCaptureModeThreadLocal);
                if (e == cudaSuccess) {
                    cudaError_t rec = m.p2p ? record_step_p2p(m) : record_step(m);
                    e = cudaStreamEndCapture(m.stream, &graph);
                    if (rec != cudaSuccess) e = rec;
                }
                if (e == cudaSuccess) e = cudaGraphInstantiate(&m.exec, graph, 0);
                if (graph) cudaGraphDestroy(graph);
            }
            if (e == cudaSuccess) e = cudaGraphLaunch(m.exec, m.stream);
        }
        if (e != cudaSuccess) return e;
        m.steps_run++;
    }
    return cudaSuccess;
}

// Map every rank's exchange arena into this process (collective over the
// NCCL communicator: all ranks call it).  Returns true only if every rank
// allocated, exported and opened every arena; otherwise all ranks fall back
// to NCCL all-gathers.
bool setup_p2p(DecodeModel* m) {
    const int T = m->T, R = m->rank;
    auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
    size_t o = 0;
    m->off_x = o;      o = al(o + static_cast<size_t>(m->H) * 4);
    m->off_att = o;    o = al(o + static_cast<size_t>(m->Hq) * m->D * 4);
    m->off_hh = o;     o = al(o + static_cast<size_t>(m->F) * 4);
    m->off_logits = o; o = al(o + static_cast<size_t>(m->V) * 4);
    m->off_part_o = o; o = al(o + kMaxTp * 4);
    m->off_part_d = o; o = al(o + kMaxTp * 4);
    m->off_flags = o;  o = al(o + FL_COUNT * kMaxTp * 4);
    m->arena_bytes = o;
    struct Rec {
        int ok;
        int pad[3];
        cudaIpcMemHandle_t h;
    };
    Rec mine;
    memset(&mine, 0, sizeof mine);
    const char* mode = getenv("ALJ_TP_EXCHANGE");
    const bool want = T <= kMaxTp && mode && strcmp(mode, "p2p") == 0 && matvec_lut_supported(FMT_NF4, m->H, m->group) &&
                      matvec_lut_supported(FMT_NF4, m->Hq * m->D, m->group) &&
                      matvec_lut_supported(FMT_NF4, m->F, m->group);
    if (want && cudaMalloc(&m->arena, m->arena_bytes) == cudaSuccess &&
        cudaMemset(m->arena, 0, m->arena_bytes) == cudaSuccess && cudaIpcGetMemHandle(&mine.h, m->arena) == cudaSuccess)
        mine.ok = 1;
    cudaGetLastError();
    Rec* d = nullptr;
    std::vector<Rec> all(T);
    auto gather = [&](const Rec& r) {
        if (cudaMemcpy(d + R, &r, sizeof(Rec), cudaMemcpyHostToDevice) != cudaSuccess) return false;
        if (g_nccl.allGather(d + R, d, sizeof(Rec), ncclChar, m->comm, m->stream) != ncclSuccess) return false;
        if (cudaStreamSynchronize(m->stream) != cudaSuccess) return false;
        return cudaMemcpy(all.data(), d, T * sizeof(Rec), cudaMemcpyDeviceToHost) == cudaSuccess;
    };
    bool ok = cudaMalloc(&d, T * sizeof(Rec)) == cudaSuccess && gather(mine);
    for (int r = 0; ok && r < T; ++r) ok = all[r].ok != 0;
    m->peer_arena[R] = m->arena;
    for (int r = 0; ok && r < T; ++r) {
        if (r == R) continue;
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[r].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) ok = false;
        else m->peer_arena[r] = static_cast<uint8_t*>(ptr);
    }
    cudaGetLastError();
    // second round: every rank must have opened every mapping
    Rec agree;
    memset(&agree, 0, sizeof agree);
    agree.ok = ok ? 1 : 0;
    bool agreed = d != nullptr && gather(agree);
    for (int r = 0; agreed && r < T; ++r) agreed = all[r].ok != 0;
    if (d) cudaFree(d);
    if (!agreed) {
        for (int r = 0; r < T; ++r)
            if (r != R && m->peer_arena[r]) cudaIpcCloseMemHandle(m->peer_arena[r]);
        for (int r = 0; r < kMaxTp; ++r) m->peer_arena[r] = nullptr;
        if (m->arena) cudaFree(m->arena);
        m->arena = nullptr;
        cudaGetLastError();
        return false;
    }
    m->x = reinterpret_cast<float*>(m->arena + m->off_x);
    m->att = reinterpret_cast<float*>(m->arena + m->off_att);
    m->hh = reinterpret_cast<float*>(m->arena + m->off_hh);
    m->logits = reinterpret_cast<float*>(m->arena + m->off_logits);
    return true;
}

void destroy(DecodeModel* m) {
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    for (int r = 0; r < kMaxTp; ++r)
        if (r != m->rank && m->peer_arena[r]) cudaIpcCloseMemHandle(m->peer_arena[r]);
    if (m->arena) cudaFree(m->arena);
    if (m->comm) g_nccl.commDestroy(m->comm);
    cudaFree(m->kc);
    cudaFree(m->vc);
    cudaFree(m->act_base);
    cudaFree(m->norms);
    cudaFree(m->rope);
    cudaFree(m->io);
    cudaFree(m->tokens);
    cudaFreeHost(m->host_io);
    cudaFreeHost(m->host_logits);
    if (m->stream) cudaStreamDestroy(m->stream);
}

}  // namespace

// Helpers shared with capi.cu.
int decode_fail(int code, const char* msg);
const void* decode_resolve(const void* p);

}  // namespace alj

using namespace alj;

extern "C" {

int aljabr_blackwell_nccl_unique_id(void* out, int out_len) {
    if (!out || out_len < static_cast<int>(sizeof(ncclUniqueId))) return decode_fail(ALJ_ERR_BAD_ARG, "need a 128-byte buffer");
    if (!nccl_load()) return decode_fail(ALJ_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    if (g_nccl.getUniqueId(&id) != ncclSuccess) return decode_fail(ALJ_ERR_CUDA, "ncclGetUniqueId failed");
    memcpy(out, &id, sizeof id);
    return ALJ_OK;
}

int aljabr_blackwell_decode_model_create(const int* dims, float eps, float rope_theta, int tp_world, int tp_rank,
                                         const void* nccl_id, unsigned long long* handle) {
    if (!dims || !handle) return decode_fail(ALJ_ERR_BAD_ARG, "null dims or handle");
    auto m = std::make_unique<DecodeModel>();
    cudaGetDevice(&m->device);
    m->layers = dims[0]; m->H = dims[1]; m->Hq = dims[2]; m->Hkv = dims[3]; m->D = dims[4];
    m->F = dims[5]; m->V = dims[6]; m->max_ctx = dims[7]; m->group = dims[8]; m->kv_dtype = dims[9];
    m->eps = eps;
    m->theta = rope_theta;
    m->T = tp_world < 1 ? 1 : tp_world;
    m->rank = tp_rank;
    const int T = m->T;
    if (m->layers <= 0 || m->H <= 0 || m->Hq <= 0 || m->Hkv <= 0 || m->D <= 0 || m->F <= 0 || m->V <= 0 ||
        m->max_ctx <= 0 || m->Hq % m->Hkv)
        return decode_fail(ALJ_ERR_BAD_DIMS, "invalid model dimensions");
    if (m->Hkv % T || m->Hq % T || m->F % T || m->H % T || m->V % T || tp_rank < 0 || tp_rank >= T)
        return decode_fail(ALJ_ERR_BAD_DIMS, "heads, hidden, ffn and vocab must divide by the TP world size");
    if (m->H % 256 || m->F % 256 || (m->Hq * m->D) % 256 || !matvec_tma_supported(FMT_NF4, m->H, m->group) ||
        !matvec_tma_supported(FMT_NF4, m->F, m->group) || !matvec_tma_supported(FMT_NF4, m->Hq * m->D, m->group))
        return decode_fail(ALJ_ERR_UNSUPPORTED, "decode step needs hidden, ffn, heads*head_dim multiples of 256 and NF4 group 64/128");
    if (m->kv_dtype != ALJ_KV_BF16 && m->kv_dtype != ALJ_KV_F32) return decode_fail(ALJ_ERR_UNSUPPORTED, "kv dtype");
    const int G = m->Hq / m->Hkv;
    if (!(m->D == 64 || m->D == 128 || m->D == 256) || !(G == 1 || G == 2 || G == 4 || G == 8))
        return decode_fail(ALJ_ERR_UNSUPPORTED, "decode attention needs head_dim 64/128/256 and group 1/2/4/8");
    if (m->D / 32 * (32 / G) > 64 || (G * m->D / 32) > 32)
        return decode_fail(ALJ_ERR_UNSUPPORTED, "decode attention register budget exceeded for this head_dim/group");
    m->hq = m->Hq / T; m->hkv = m->Hkv / T; m->f = m->F / T; m->h = m->H / T; m->v = m->V / T;
    m->w.resize(m->layers);
    m->layer_set.assign(m->layers, false);
    m->splits = attention_splits(m->max_ctx, m->hkv, sm_count_for_current_device());
    if (T > 1) m->splits = std::max(m->splits, 2);   // the tensor-parallel push lives in the split merge
    // The RMSNorm scale moves to the consuming matvec when every launch that
    // produces or consumes a normed vector runs on the NF4 table kernel.
    m->defer_norm = T == 1 && matvec_lut_supported(FMT_NF4, m->H, m->group) &&
                    matvec_lut_supported(FMT_NF4, m->Hq * m->D, m->group) &&
                    matvec_lut_supported(FMT_NF4, m->F, m->group);

    auto ok = [&](cudaError_t e) { return e == cudaSuccess; };
    const size_t kvb = static_cast<size_t>(m->layers) * m->kv_layer_elems() * m->kv_elem();
    const size_t acts = static_cast<size_t>(m->H) + m->hq * m->D + 2 * m->hkv * m->D + m->hq * m->D + m->Hq * m->D +
                        m->h + m->H + m->f + m->F + m->v + m->V + m->H + matvec_max_ctas() + 4 +
                        attention_scratch_floats(m->hq, m->D, m->splits) + 64;
    if (!ok(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking)) || !ok(cudaMalloc(&m->kc, kvb)) ||
        !ok(cudaMalloc(&m->vc, kvb)) || !ok(cudaMalloc(&m->act_base, acts * 4)) ||
        !ok(cudaMalloc(&m->norms, (static_cast<size_t>(m->layers) * 2 + 1) * m->H * 4)) ||
        !ok(cudaMalloc(&m->io, 8 * sizeof(int))) || !ok(cudaMallocHost(&m->host_io, 8 * sizeof(int))) ||
        !ok(cudaMalloc(&m->rope, static_cast<size_t>(m->max_ctx) * (m->D / 2) * sizeof(float2))) ||
        !ok(cudaMalloc(&m->tokens, static_cast<size_t>(m->max_ctx) * sizeof(int))) ||
        !ok(cudaMallocHost(&m->host_logits, static_cast<size_t>(m->V) * 4))) {
        cudaGetLastError();
        destroy(m.get());
        return decode_fail(ALJ_ERR_NO_MEMORY, "allocating the decode model's KV cache / activations failed");
    }
    cudaMemsetAsync(m->kc, 0, kvb, m->stream);
    cudaMemsetAsync(m->vc, 0, kvb, m->stream);
    cudaMemsetAsync(m->act_base, 0, acts * 4, m->stream);
    {
        // RoPE angle table exactly as GGUFVectorOps.rope (GGUFVectorOps.java:425-431):
        // invFreq = (float) pow(base, -2f*i/rotaryDim); theta = (pos * invFreq) / 1f;
        // cos / sin in double, cast to float.
        const int half = m->D / 2;
        std::vector<float2> tab(static_cast<size_t>(m->max_ctx) * half);
        for (int i = 0; i < half; ++i) {
            const float expo = -2.0f * static_cast<float>(i) / static_cast<float>(m->D);
            const float inv = static_cast<float>(std::pow(static_cast<double>(m->theta), static_cast<double>(expo)));
            for (int pos = 0; pos < m->max_ctx; ++pos) {
                const float ang = static_cast<float>(pos) * inv;
                tab[static_cast<size_t>(pos) * half + i] =
                    make_float2(static_cast<float>(std::cos(static_cast<double>(ang))),
                                static_cast<float>(std::sin(static_cast<double>(ang))));
            }
        }
        if (!ok(cudaMemcpy(m->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice))) {
            destroy(m.get());
            return decode_fail(ALJ_ERR_CUDA, "uploading the RoPE table failed");
        }
    }
    float* p = m->act_base;
    auto take = [&](size_t n) { float* r = p; p += (n + 3) / 4 * 4; return r; };
    m->x = take(m->H); m->q = take(m->hq * m->D); m->k = take(m->hkv * m->D); m->vv = take(m->hkv * m->D);
    m->att_l = take(m->hq * m->D); m->att = take(m->Hq * m->D); m->delta_l = take(m->h); m->delta = take(m->H);
    m->h_l = take(m->f); m->hh = take(m->F);
    m->logits_l = take(m->v); m->logits = take(m->V);
    m->xn = take(m->H);
    m->norm_partials = take(matvec_max_ctas());
    m->norm_counter = reinterpret_cast<unsigned int*>(take(4));   // zeroed by the memset above
    m->scratch = take(attention_scratch_floats(m->hq, m->D, m->splits));
    if (T > 1) {
        if (!nccl_id) { destroy(m.get()); return decode_fail(ALJ_ERR_BAD_ARG, "TP > 1 needs an NCCL unique id"); }
        if (!nccl_load()) { destroy(m.get()); return decode_fail(ALJ_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded"); }
        ncclUniqueId id;
        memcpy(&id, nccl_id, sizeof id);
        if (g_nccl.commInitRank(&m->comm, T, id, tp_rank) != ncclSuccess) {
            m->comm = nullptr;
            destroy(m.get());
            return decode_fail(ALJ_ERR_CUDA, "ncclCommInitRank failed");
        }
        m->p2p = setup_p2p(m.get());
    }
    {
        const int init[8] = {0, 0, 0, 0, 0, 0, 1, 0};   // token counter starts at 1 (flags start at 0)
        if (!ok(cudaMemcpy(m->io, init, sizeof init, cudaMemcpyHostToDevice))) {
            destroy(m.get());
            return decode_fail(ALJ_ERR_CUDA, "initialising the step state failed");
        }
    }
    if (!ok(cudaStreamSynchronize(m->stream))) { destroy(m.get()); return decode_fail(ALJ_ERR_CUDA, "model init failed"); }
    std::lock_guard<std::mutex> g(g_models_mu);
    *handle = g_next_handle++;
    g_models[*handle] = std::move(m);
    return ALJ_OK;
}

}  // extern "C"

namespace {
// ALJ_TYPE_* of a decode-step weight -> WeightFormat, or -1.
int decode_fmt(int type) {
    switch (type) {
        case ALJ_TYPE_Q4_0: return FMT_Q4_0;
        case ALJ_TYPE_Q8_0: return FMT_Q8_0;
        case ALJ_TYPE_Q4_K: return FMT_Q4_K;
        case ALJ_TYPE_Q6_K: return FMT_Q6_K;
        case ALJ_TYPE_NF4: return FMT_NF4;
        default: return -1;
    }
}

// Resolve one weight (and, for NF4, its absmax) into `out`; marks the model
// typed for a GGUF format (one GPU only: the tensor-parallel exchange fuses
// the NF4 kernels' epilogues).
int bind_weight(DecodeModel* m, Weight& out, const void* w, int type, const void* absmax) {
    const int fmt = decode_fmt(type);
    if (fmt < 0) return decode_fail(ALJ_ERR_UNSUPPORTED, "decode weights must be Q4_0, Q8_0, Q4_K, Q6_K or NF4");
    if (fmt != FMT_NF4 && m->T > 1)
        return decode_fail(ALJ_ERR_UNSUPPORTED, "GGUF-typed decode weights need tp_world 1 (NF4 for tensor parallel)");
    Weight r;
    r.fmt = fmt;
    r.codes = static_cast<const uint8_t*>(decode_resolve(w));
    r.absmax = fmt == FMT_NF4 ? static_cast<const float*>(decode_resolve(absmax)) : nullptr;
    if (!r.codes || (fmt == FMT_NF4 && !r.absmax))
        return decode_fail(ALJ_ERR_NOT_REGISTERED, "decode weights must be device or registered memory");
    out = r;
    if (fmt != FMT_NF4) {
        m->typed = true;
        m->defer_norm = false;
    }
    return ALJ_OK;
}

int register_layer(unsigned long long handle, int layer, const void* const* w, const int* types,
                   const void* const* absmax, const float* attn_norm, const float* ffn_norm) {
    DecodeModel* m = find(handle);
    if (!m) return decode_fail(ALJ_ERR_BAD_ARG, "unknown decode model handle");
    if (layer < 0 || layer >= m->layers) return decode_fail(ALJ_ERR_BAD_DIMS, "layer index out of range");
    if (!w || !attn_norm || !ffn_norm) return decode_fail(ALJ_ERR_BAD_ARG, "null layer pointer");
    std::lock_guard<std::mutex> g(m->mu);
    cudaSetDevice(m->device);
    std::array<Weight, W_COUNT> ws;
    for (int i = 0; i < W_COUNT; ++i) {
        const int type = types ? types[i] : ALJ_TYPE_NF4;
        if (type == ALJ_TYPE_NF4 && !absmax) return decode_fail(ALJ_ERR_BAD_ARG, "NF4 weights need absmax");
        const int rc = bind_weight(m, ws[i], w[i], type, absmax ? absmax[i] : nullptr);
        if (rc != ALJ_OK) return rc;
    }
    m->w[layer] = ws;
    float* dst = m->norms + static_cast<size_t>(layer) * 2 * m->H;
    if (cudaMemcpy(dst, attn_norm, m->H * 4, cudaMemcpyDefault) != cudaSuccess ||
        cudaMemcpy(dst + m->H, ffn_norm, m->H * 4, cudaMemcpyDefault) != cudaSuccess)
        return decode_fail(ALJ_ERR_CUDA, "copying layer norms failed");
    m->layer_set[layer] = true;
    if (m->exec) { cudaGraphExecDestroy(m->exec); m->exec = nullptr; }
    return ALJ_OK;
}

int register_output(unsigned long long handle, const void* embd, int embd_type, const void* embd_absmax,
                    const void* head, int head_type, const void* head_absmax, const float* output_norm) {
    DecodeModel* m = find(handle);
    if (!m) return decode_fail(ALJ_ERR_BAD_ARG, "unknown decode model handle");
    if (!output_norm) return decode_fail(ALJ_ERR_BAD_ARG, "null output norm");
    std::lock_guard<std::mutex> g(m->mu);
    cudaSetDevice(m->device);
    Weight e, h;
    int rc = bind_weight(m, e, embd, embd_type, embd_absmax);
    if (rc == ALJ_OK) rc = bind_weight(m, h, head, head_type, head_absmax);
    if (rc != ALJ_OK) return rc;
    m->embd = e;
    m->head = h;
    if (cudaMemcpy(m->norms + static_cast<size_t>(m->layers) * 2 * m->H, output_norm, m->H * 4, cudaMemcpyDefault) !=
        cudaSuccess)
        return decode_fail(ALJ_ERR_CUDA, "copying the output norm failed");
    m->output_set = true;
    if (m->exec) { cudaGraphExecDestroy(m->exec); m->exec = nullptr; }
    return ALJ_OK;
}
}  // namespace

extern "C" {

int aljabr_blackwell_register_decode_layer(unsigned long long handle, int layer, const void* const* codes,
                                           const void* const* absmax, const float* attn_norm, const float* ffn_norm) {
    if (!codes || !absmax) return decode_fail(ALJ_ERR_BAD_ARG, "null layer pointer");
    return register_layer(handle, layer, codes, nullptr, absmax, attn_norm, ffn_norm);
}

int aljabr_blackwell_register_decode_layer_typed(unsigned long long handle, int layer, const void* const* weights,
                                                 const int* types, const void* const* absmax, const float* attn_norm,
                                                 const float* ffn_norm) {
    if (!types) return decode_fail(ALJ_ERR_BAD_ARG, "null type list");
    return register_layer(handle, layer, weights, types, absmax, attn_norm, ffn_norm);
}

int aljabr_blackwell_register_output(unsigned long long handle, const void* embd_codes, const void* embd_absmax,
                                     const void* head_codes, const void* head_absmax, const float* output_norm) {
    return register_output(handle, embd_codes, ALJ_TYPE_NF4, embd_absmax, head_codes, ALJ_TYPE_NF4, head_absmax,
                           output_norm);
}

int aljabr_blackwell_register_output_typed(unsigned long long handle, const void* embd, int embd_type,
                                           const void* embd_absmax, const void* head, int head_type,
                                           const void* head_absmax, const float* output_norm) {
    return register_output(handle, embd, embd_type, embd_absmax, head, head_type, head_absmax, output_norm);
}

int aljabr_blackwell_decode_step_token(unsigned long long handle, int token, int pos, float* logits_out,
                                       int* argmax_out) {
    DecodeModel* m = find(handle);
    if (!m) return decode_fail(ALJ_ERR_BAD_ARG, "unknown decode model handle");
    if (pos < 0 || pos >= m->max_ctx) return decode_fail(ALJ_ERR_BAD_DIMS, "position outside the KV cache");
    if (token < 0 || token >= m->V) return decode_fail(ALJ_ERR_BAD_DIMS, "token id outside the vocabulary");
    std::lock_guard<std::mutex> g(m->mu);
    cudaSetDevice(m->device);
    if (!m->output_set) return decode_fail(ALJ_ERR_NOT_INITIALIZED, "output weights not registered");
    for (int l = 0; l < m->layers; ++l)
        if (!m->layer_set[l]) return decode_fail(ALJ_ERR_NOT_INITIALIZED, "decode layer not registered");
    m->host_io[0] = pos;
    m->host_io[1] = token;
    cudaError_t e = cudaMemcpyAsync(m->io, m->host_io, 2 * sizeof(int), cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = enqueue_steps(*m, 1);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(m->host_io + 2, m->io + 2, sizeof(int), cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess && logits_out)
        e = cudaMemcpyAsync(m->host_logits, m->logits, static_cast<size_t>(m->V) * 4, cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return decode_fail(ALJ_ERR_CUDA, cudaGetErrorString(e));
    }
    if (argmax_out) *argmax_out = m->host_io[2];
    if (logits_out) memcpy(logits_out, m->host_logits, static_cast<size_t>(m->V) * 4);
    return ALJ_OK;
}

int aljabr_blackwell_decode_run(unsigned long long handle, int token, int pos, int n_tokens, int* tokens_out) {
    DecodeModel* m = find(handle);
    if (!m) return decode_fail(ALJ_ERR_BAD_ARG, "unknown decode model handle");
    if (n_tokens <= 0 || pos < 0 || pos + n_tokens > m->max_ctx)
        return decode_fail(ALJ_ERR_BAD_DIMS, "positions [pos, pos + n_tokens) must lie inside the KV cache");
    if (token < 0 || token >= m->V) return decode_fail(ALJ_ERR_BAD_DIMS, "token id outside the vocabulary");
    std::lock_guard<std::mutex> g(m->mu);
    cudaSetDevice(m->device);
    if (!m->output_set) return decode_fail(ALJ_ERR_NOT_INITIALIZED, "output weights not registered");
    for (int l = 0; l < m->layers; ++l)
        if (!m->layer_set[l]) return decode_fail(ALJ_ERR_NOT_INITIALIZED, "decode layer not registered");
    m->host_io[0] = pos;
    m->host_io[1] = token;
    cudaError_t e = cudaMemcpyAsync(m->io, m->host_io, 2 * sizeof(int), cudaMemcpyHostToDevice, m->stream);
    if (e == cudaSuccess) e = enqueue_steps(*m, n_tokens);
    if (e == cudaSuccess && tokens_out)
        e = cudaMemcpyAsync(tokens_out, m->tokens + pos, static_cast<size_t>(n_tokens) * sizeof(int),
                            cudaMemcpyDeviceToHost, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return decode_fail(ALJ_ERR_CUDA, cudaGetErrorString(e));
    }
    return ALJ_OK;
}

int aljabr_blackwell_sync_kv_cache(unsigned long long handle, int layer, int seq_len, const void* k, const void* v) {
    DecodeModel* m = find(handle);
    if (!m) return decode_fail(ALJ_ERR_BAD_ARG, "unknown decode model handle");
    if (layer < 0 || layer >= m->layers || seq_len < 0 || seq_len > m->max_ctx)
        return decode_fail(ALJ_ERR_BAD_DIMS, "layer or sequence length out of range");
    if (!k || !v) return decode_fail(ALJ_ERR_BAD_ARG, "null K or V");
    std::lock_guard<std::mutex> g(m->mu);
    cudaSetDevice(m->device);
    const size_t bytes = static_cast<size_t>(seq_len) * m->hkv * m->D * m->kv_elem();
    const size_t off = static_cast<size_t>(layer) * m->kv_layer_elems() * m->kv_elem();
    cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(m->kc) + off, k, bytes, cudaMemcpyDefault, m->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(static_cast<uint8_t*>(m->vc) + off, v, bytes, cudaMemcpyDefault, m->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(m->stream);
    if (e != cudaSuccess) return decode_fail(ALJ_ERR_CUDA, cudaGetErrorString(e));
    return ALJ_OK;
}

int aljabr_blackwell_decode_read_state(unsigned long long handle, float* x_out, void* k_cache_out, void* v_cache_out) {
    DecodeModel* m = find(handle);
    if (!m) return decode_fail(ALJ_ERR_BAD_ARG, "unknown decode model handle");
    std::lock_guard<std::mutex> g(m->mu);
    cudaSetDevice(m->device);
    const size_t kvb = static_cast<size_t>(m->layers) * m->kv_layer_elems() * m->kv_elem();
    cudaError_t e = cudaStreamSynchronize(m->stream);
    if (e == cudaSuccess && x_out) e = cudaMemcpy(x_out, m->x, static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && k_cache_out) e = cudaMemcpy(k_cache_out, m->kc, kvb, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && v_cache_out) e = cudaMemcpy(v_cache_out, m->vc, kvb, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return decode_fail(ALJ_ERR_CUDA, cudaGetErrorString(e));
    return ALJ_OK;
}

int aljabr_blackwell_decode_model_destroy(unsigned long long handle) {
    std::unique_ptr<DecodeModel> m;
    {
        std::lock_guard<std::mutex> g(g_models_mu);
        auto it = g_models.find(handle);
        if (it == g_models.end()) return decode_fail(ALJ_ERR_BAD_ARG, "unknown decode model handle");
        m = std::move(it->second);
        g_models.erase(it);
    }
    destroy(m.get());
    return ALJ_OK;
}

}  // extern "C"
