// C-ABI of libaljabr_blackwell.so (declared in include/aljabr_blackwell.h):
// per-device state, the registry of model buffers copied to HBM, host-buffer
// staging for the Metal-shaped "tb" entry points, and argument validation.
// No entry point falls back to the CPU: anything the kernels cannot run is
// reported as an error code.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <array>
#include <thread>
#include <tuple>
#include <vector>

#include "aljabr_blackwell_internal.h"

namespace alj {

extern __device__ unsigned int g_fault_word;

namespace {

thread_local std::string t_last_error;
thread_local int t_device = -1;
thread_local bool t_pdl = false;
thread_local const void* t_prefetch = nullptr;   // one-shot L2 prefetch hint (device address)
thread_local size_t t_prefetch_bytes = 0;
int g_verbose = 0;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_last_error = buf;
    if (g_verbose) fprintf(stderr, "[aljabr_blackwell] error %d: %s\n", code, buf);
    return code;
}

#define ALJ_CUDA(expr)                                                                               \
    do {                                                                                             \
        cudaError_t _e = (expr);                                                                     \
        if (_e != cudaSuccess) return fail(ALJ_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                                           __FILE__, __LINE__);                                      \
    } while (0)

struct Registered {
    size_t bytes;
    void* dev;
};

// Grow-only device staging buffer.
struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    // Attention scratch: how many leading counter words are known to be zero
    // on every stream (0 after an allocation or a reported device fault).
    int zeroed_words = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        zeroed_words = 0;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e == cudaSuccess) cap = bytes;
        return e;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        zeroed_words = 0;
    }
};
// Grow-only pinned host staging buffer, mapped into the device's address
// space: kernels read inputs from it and store results into it directly.
struct HostBuf {
    void* p = nullptr;
    void* dev = nullptr;   // the device address of p
    size_t cap = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap) return cudaSuccess;
        if (p) cudaFreeHost(p);
        p = dev = nullptr;
        cap = 0;
        cudaError_t e = cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
        if (e == cudaSuccess) e = cudaHostGetDevicePointer(&dev, p, 0);
        if (e == cudaSuccess) {
            cap = bytes;
        } else if (p) {
            cudaFreeHost(p);
            p = dev = nullptr;
        }
        return e;
    }
    void release() {
        if (p) cudaFreeHost(p);
        p = dev = nullptr;
        cap = 0;
    }
};

// A Q4_0 / Q8_0 matrix packed for the batched GEMM (gemm_q.cu).
struct PackedQ {
    void* p = nullptr;
    bool finite = true;       // every block scale finite (else the batch runs per row)
};
using PackKey = std::tuple<uintptr_t, int, int, int>;   // device weights, type, rows, K

struct DeviceState {
    int device = 0;
    int sms = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;                          // serialises the staging buffers of tb calls
    std::map<uintptr_t, Registered> reg;    // host base -> HBM copy
    std::mutex reg_mu;
    DevBuf dx, dy, dtmp, dscratch, dgemm;
    HostBuf hx, hy;
    std::map<PackKey, PackedQ> qpack;       // guarded by mu
    // host-buffer matvec calls replayed as one CUDA graph (x pull + matvecs)
    // per shape, weights and staging buffers; guarded by mu
    std::map<std::array<uintptr_t, 20>, std::pair<int, cudaGraphExec_t>> tb_graphs;
    void* upload_bounce[2] = {nullptr, nullptr};   // pinned, for model uploads (guarded by upload_mu)
    cudaEvent_t upload_done[2] = {nullptr, nullptr};
    std::mutex upload_mu;
};

std::mutex g_mu;
std::vector<std::unique_ptr<DeviceState>> g_dev;

int current_device() {
    if (t_device >= 0) return t_device;
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

// State of the calling thread's device, created on first use.
DeviceState* state(int* err) {
    const int d = current_device();
    std::lock_guard<std::mutex> g(g_mu);
    if (static_cast<int>(g_dev.size()) <= d) g_dev.resize(d + 1);
    if (!g_dev[d]) {
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
            *err = fail(ALJ_ERR_NOT_INITIALIZED, "no CUDA device visible");
            return nullptr;
        }
        if (d >= count) {
            *err = fail(ALJ_ERR_BAD_ARG, "device %d out of range (%d devices)", d, count);
            return nullptr;
        }
        cudaSetDevice(d);
        auto s = std::make_unique<DeviceState>();
        s->device = d;
        cudaDeviceGetAttribute(&s->sms, cudaDevAttrMultiProcessorCount, d);
        if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess) {
            *err = fail(ALJ_ERR_CUDA, "stream creation failed on device %d", d);
            return nullptr;
        }
        g_dev[d] = std::move(s);
    }
    cudaSetDevice(d);
    return g_dev[d].get();
}

// Map a weight pointer to device memory: a registered host address, or a
// pointer that is already device-accessible.
const void* resolve(DeviceState* st, const void* p) {
    if (!p) return nullptr;
    {
        std::lock_guard<std::mutex> g(st->reg_mu);
        const uintptr_t a = reinterpret_cast<uintptr_t>(p);
        auto it = st->reg.upper_bound(a);
        if (it != st->reg.begin()) {
            --it;
            if (a - it->first < it->second.bytes) return static_cast<const uint8_t*>(it->second.dev) + (a - it->first);
        }
    }
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) return p;
    if (attr.type == cudaMemoryTypeHost && attr.devicePointer) return attr.devicePointer;
    return nullptr;
}

int fmt_of(int type) {
    switch (type) {
        case ALJ_TYPE_Q4_0: return FMT_Q4_0;
        case ALJ_TYPE_Q8_0: return FMT_Q8_0;
        case ALJ_TYPE_NF4: return FMT_NF4;
        case ALJ_TYPE_Q4_K: return FMT_Q4_K;
        case ALJ_TYPE_Q6_K: return FMT_Q6_K;
    }
    return -1;
}

int check_dims(int type, long long K, long long N) {
    if (K <= 0 || N <= 0) return fail(ALJ_ERR_BAD_DIMS, "K=%lld N=%lld must be positive", K, N);
    if (K > (1 << 24) || N > (1 << 28)) return fail(ALJ_ERR_BAD_DIMS, "K=%lld N=%lld too large", K, N);
    if ((type == ALJ_TYPE_Q4_0 || type == ALJ_TYPE_Q8_0) && K % 32 != 0)
        return fail(ALJ_ERR_BAD_DIMS, "K=%lld is not a multiple of the 32-value block", K);
    if ((type == ALJ_TYPE_Q4_K || type == ALJ_TYPE_Q6_K) && K % 256 != 0)
        return fail(ALJ_ERR_BAD_DIMS, "K=%lld is not a multiple of the 256-value super-block", K);
    if (fmt_of(type) < 0) return fail(ALJ_ERR_UNSUPPORTED, "weight type %d has no Blackwell kernel", type);
    return ALJ_OK;
}

int launch_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return ALJ_OK;
    if (e == cudaErrorNotSupported) return fail(ALJ_ERR_UNSUPPORTED, "%s: shape not supported", what);
    return fail(ALJ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

cudaStream_t pick_stream(DeviceState* st, void* stream) {
    return stream ? static_cast<cudaStream_t>(stream) : st->stream;
}

struct MatSpec {
    int type;
    const void* w;        // device
    const float* absmax;  // device (NF4)
    const float* bias;    // device
    float* y;             // device
    int N;
};

// One fused launch when every matrix shares the format; otherwise one per matrix.
int run_matvecs(DeviceState* st, const MatSpec* m, int n, const float* dx, int K, int group, cudaStream_t stream,
                bool pdl = false) {
    bool same = true;
    for (int i = 1; i < n; ++i) same = same && m[i].type == m[0].type;
    if (same) {
        MatvecParams p = {};
        p.nseg = n;
        p.K = K;
        p.group = group;
        p.x = dx;
        for (int i = 0; i < n; ++i) {
            p.seg[i].w = static_cast<const uint8_t*>(m[i].w);
            p.seg[i].absmax = m[i].absmax;
            p.seg[i].bias = m[i].bias;
            p.seg[i].y = m[i].y;
            p.seg[i].rows = m[i].N;
            p.total_rows += m[i].N;
        }
        p.prefetch = t_prefetch;
        p.prefetch_bytes = t_prefetch_bytes;
        t_prefetch = nullptr;
        t_prefetch_bytes = 0;
        return launch_status(launch_matvec(fmt_of(m[0].type), p, stream, pdl), "matvec");
    }
    for (int i = 0; i < n; ++i) {
        int rc = run_matvecs(st, m + i, 1, dx, K, group, stream, pdl);
        if (rc) return rc;
    }
    return ALJ_OK;
}

// Host-buffer path shared by every tb entry point: stage A, run, copy C out.
struct HostOut {
    void* C;
    int N;
};

// Packed copy of a Q4_0 / Q8_0 matrix for the batched GEMM: made on first use
// (on st->stream, with one blocking read of its max-scale word) and kept until
// the model buffer holding the matrix is unregistered.  Caller holds st->mu.
int packed_q(DeviceState* st, int type, const void* w, int rows, int K, const PackedQ** out) {
    const PackKey key{reinterpret_cast<uintptr_t>(w), type, rows, K};
    auto it = st->qpack.find(key);
    if (it == st->qpack.end()) {
        const int fmt = fmt_of(type);
        PackedQ pq;
        ALJ_CUDA(cudaMalloc(&pq.p, gemm_q_packed_bytes(fmt, rows, K)));
        unsigned int maxbits = 0u;
        cudaError_t e = launch_gemm_q_pack(fmt, pq.p, w, rows, K, st->stream);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(&maxbits, static_cast<const uint8_t*>(pq.p) + 4, 4, cudaMemcpyDeviceToHost, st->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st->stream);
        if (e != cudaSuccess) {
            cudaFree(pq.p);
            return fail(ALJ_ERR_CUDA, "gemm_q_pack: %s", cudaGetErrorString(e));
        }
        pq.finite = maxbits < 0x7F800000u;
        it = st->qpack.emplace(key, pq).first;
    }
    *out = &it->second;
    return ALJ_OK;
}

// A batch of Q4_0 / Q8_0 rows through the tcgen05 GEMM, every matrix at once:
// x through the pull kernel, outputs [matrix][b][N] straight into the mapped
// buffer.  *ran stays false when a matrix has a non-finite block scale (the
// caller then runs the rows one at a time, as the reference would).  Caller
// holds st->mu.
int tb_gemm_q(DeviceState* st, int nmat, int type, const MatSpec* spec, const HostOut* outs, const void* A, int K,
              int batch, bool* ran) {
    *ran = false;
    GemmQArgs a;
    memset(&a, 0, sizeof a);
    size_t ytotal = 0;
    for (int i = 0; i < nmat; ++i) {
        const PackedQ* pq = nullptr;
        const int rc = packed_q(st, type, spec[i].w, outs[i].N, K, &pq);
        if (rc) return rc;
        if (!pq->finite) return ALJ_OK;
        a.packed[i] = pq->p;
        a.rows[i] = outs[i].N;
        a.ldy[i] = outs[i].N;
        ytotal += static_cast<size_t>(outs[i].N) * batch;
    }
    const size_t xfloats = static_cast<size_t>(K) * batch;
    const size_t ws = gemm_q_workspace_bytes(batch, K);
    ALJ_CUDA(st->dx.ensure(xfloats * 4));
    ALJ_CUDA(st->hx.ensure(xfloats * 4));
    ALJ_CUDA(st->hy.ensure(ytotal * 4));
    ALJ_CUDA(st->dgemm.ensure(ws));
    memcpy(st->hx.p, A, xfloats * 4);
    float* dx = static_cast<float*>(st->dx.p);
    ALJ_CUDA(launch_host_pull(dx, static_cast<const float*>(st->hx.dev), xfloats, st->sms, st->stream));
    size_t off = 0;
    for (int i = 0; i < nmat; ++i) {
        a.y[i] = static_cast<float*>(st->hy.dev) + off;
        off += static_cast<size_t>(outs[i].N) * batch;
    }
    a.fmt = fmt_of(type);
    a.nseg = nmat;
    a.x = dx;
    a.M = batch;
    a.K = K;
    a.workspace = st->dgemm.p;
    a.workspace_bytes = ws;
    const int rc = launch_status(launch_gemm_q(a, st->stream), "gemm_q");
    if (rc) return rc;
    ALJ_CUDA(cudaStreamSynchronize(st->stream));
    off = 0;
    for (int i = 0; i < nmat; ++i) {
        const size_t n = static_cast<size_t>(outs[i].N) * batch;
        memcpy(outs[i].C, static_cast<const float*>(st->hy.p) + off, n * 4);
        off += n;
    }
    *ran = true;
    return ALJ_OK;
}
int tb_matvec(int nmat, const int* types, const void* const* B, const float* const* absmax_host, const float* bias_host,
              const HostOut* outs, const void* A, int K, int group, int batch) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!A) return fail(ALJ_ERR_BAD_ARG, "A is null");
    for (int i = 0; i < nmat; ++i) {
        if (!outs[i].C || !B[i]) return fail(ALJ_ERR_BAD_ARG, "null C or B pointer (matrix %d)", i);
        int rc = check_dims(types[i], K, outs[i].N);
        if (rc) return rc;
        if (types[i] == ALJ_TYPE_NF4 && (group <= 0 || !absmax_host[i]))
            return fail(ALJ_ERR_BAD_ARG, "NF4 needs absmax and a positive block size");
    }
    MatSpec spec[3];
    size_t ytotal = 0;
    for (int i = 0; i < nmat; ++i) {
        spec[i].type = types[i];
        spec[i].w = resolve(st, B[i]);
        if (!spec[i].w) return fail(ALJ_ERR_NOT_REGISTERED, "weight pointer %p is neither registered nor device memory", B[i]);
        spec[i].absmax = nullptr;
        if (types[i] == ALJ_TYPE_NF4) {
            spec[i].absmax = static_cast<const float*>(resolve(st, absmax_host[i]));
            if (!spec[i].absmax) return fail(ALJ_ERR_NOT_REGISTERED, "absmax pointer %p is neither registered nor device memory", absmax_host[i]);
        }
        spec[i].N = outs[i].N;
        ytotal += static_cast<size_t>(outs[i].N);
    }
    std::lock_guard<std::mutex> g(st->mu);
    if (batch >= 2 && !bias_host) {
        bool same = true;
        for (int i = 1; i < nmat; ++i) same = same && types[i] == types[0];
        const int f0 = fmt_of(types[0]);
        if (same && (f0 == FMT_Q4_0 || f0 == FMT_Q8_0) && gemm_q_supported(f0, batch, K)) {
            bool ran = false;
            const int rc = tb_gemm_q(st, nmat, types[0], spec, outs, A, K, batch, &ran);
            if (rc || ran) return rc;
        }
    }
    // x (and the bias) go to the device through a pull kernel that reads the
    // mapped staging buffer; the matvecs store y straight into the mapped
    // output buffer.  No copy-engine transfer: at these sizes its set-up
    // (several µs each way) costs more than the PCIe traffic.
    const size_t xfloats = static_cast<size_t>(K) * batch;
    const size_t nb = nmat == 1 && bias_host ? static_cast<size_t>(outs[0].N) : 0;
    const size_t ybytes = ytotal * batch * 4;
    ALJ_CUDA(st->dx.ensure((xfloats + nb) * 4));
    ALJ_CUDA(st->hx.ensure((xfloats + nb) * 4));
    ALJ_CUDA(st->hy.ensure(ybytes));
    memcpy(st->hx.p, A, xfloats * 4);
    if (nb) memcpy(static_cast<float*>(st->hx.p) + xfloats, bias_host, nb * 4);
    float* dx = static_cast<float*>(st->dx.p);
    const float* dbias = nb ? dx + xfloats : nullptr;
    float* ydev = static_cast<float*>(st->hy.dev);
    // the x pull and the matvecs, as launched on st->stream
    auto enqueue = [&]() -> int {
        if (launch_host_pull(dx, static_cast<const float*>(st->hx.dev), xfloats + nb, st->sms, st->stream) !=
            cudaSuccess)
            return fail(ALJ_ERR_CUDA, "x pull launch failed");
        for (int b = 0; b < batch; ++b) {
            size_t off = 0;
            for (int i = 0; i < nmat; ++i) {
                spec[i].y = ydev + static_cast<size_t>(b) * ytotal + off;
                spec[i].bias = (i == 0) ? dbias : nullptr;
                off += static_cast<size_t>(outs[i].N);
            }
            int rc = run_matvecs(st, spec, nmat, dx + static_cast<size_t>(b) * K, K, group, st->stream, true);
            if (rc) return rc;
        }
        return ALJ_OK;
    };
    // A shape seen before (same matrices, sizes and staging buffers) is
    // replayed as one CUDA graph: one launch instead of two or more, with
    // the tensor maps encoded once.  Captured on its second call (the first
    // sets the kernels' attributes); not while a prefetch hint is pending,
    // which belongs to the next launch only.
    std::array<uintptr_t, 20> key{};
    key[0] = static_cast<uintptr_t>(nmat);
    key[1] = static_cast<uintptr_t>(K);
    key[2] = static_cast<uintptr_t>(group);
    key[3] = static_cast<uintptr_t>(batch);
    key[4] = static_cast<uintptr_t>(nb);
    for (int i = 0; i < nmat; ++i) {
        key[5 + i] = reinterpret_cast<uintptr_t>(spec[i].w);
        key[8 + i] = reinterpret_cast<uintptr_t>(spec[i].absmax);
        key[11 + i] = static_cast<uintptr_t>(spec[i].N);
        key[14 + i] = static_cast<uintptr_t>(spec[i].type);
    }
    key[17] = reinterpret_cast<uintptr_t>(st->hx.dev);
    key[18] = reinterpret_cast<uintptr_t>(st->dx.p);
    key[19] = reinterpret_cast<uintptr_t>(st->hy.dev);
    cudaGraphExec_t ge = nullptr;
    if (!t_prefetch) {
        auto it = st->tb_graphs.find(key);
        if (it == st->tb_graphs.end()) {
            if (st->tb_graphs.size() < 256) st->tb_graphs.emplace(key, std::make_pair(1, nullptr));
        } else if (it->second.second) {
            ge = it->second.second;
        } else if (++it->second.first >= 2) {
            cudaGraph_t graph = nullptr;
            if (cudaStreamBeginCapture(st->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
                const int rc = enqueue();
                const cudaError_t e = cudaStreamEndCapture(st->stream, &graph);
                if (rc == ALJ_OK && e == cudaSuccess && graph &&
                    cudaGraphInstantiate(&ge, graph, 0) == cudaSuccess) {
                    it->second.second = ge;
                } else {
                    ge = nullptr;
                    it->second.first = -(1 << 30);   // this shape runs direct from now on
                }
                if (graph) cudaGraphDestroy(graph);
            }
            cudaGetLastError();   // a failed capture leaves no error behind; the direct path runs
        }
    }
    if (ge) {
        ALJ_CUDA(cudaGraphLaunch(ge, st->stream));
    } else {
        const int rc = enqueue();
        if (rc) return rc;
    }
    ALJ_CUDA(cudaStreamSynchronize(st->stream));
    // scatter [b][matrix][N] staging into the callers' buffers
    for (int i = 0, off = 0; i < nmat; off += outs[i].N, ++i)
        for (int b = 0; b < batch; ++b)
            memcpy(static_cast<float*>(outs[i].C) + static_cast<size_t>(b) * outs[i].N,
                   static_cast<const float*>(st->hy.p) + static_cast<size_t>(b) * ytotal + off,
                   static_cast<size_t>(outs[i].N) * 4);
    return ALJ_OK;
}

int tb_dequant(int type, void* dst, const void* src, const void* scales, long long numel, int group) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!dst || !src) return fail(ALJ_ERR_BAD_ARG, "null dst or src");
    if (numel <= 0) return fail(ALJ_ERR_BAD_DIMS, "numel=%lld must be positive", numel);
    if (type != ALJ_TYPE_NF4 && numel % 32) return fail(ALJ_ERR_BAD_DIMS, "numel=%lld is not a multiple of 32", numel);
    if (type == ALJ_TYPE_NF4 && (group <= 0 || !scales)) return fail(ALJ_ERR_BAD_ARG, "NF4 needs scales and group > 0");
    const void* dsrc = resolve(st, src);
    if (!dsrc) return fail(ALJ_ERR_NOT_REGISTERED, "src %p is neither registered nor device memory", src);
    const float* dscale = nullptr;
    if (type == ALJ_TYPE_NF4) {
        dscale = static_cast<const float*>(resolve(st, scales));
        if (!dscale) return fail(ALJ_ERR_NOT_REGISTERED, "scales %p is neither registered nor device memory", scales);
    }
    std::lock_guard<std::mutex> g(st->mu);
    ALJ_CUDA(st->dtmp.ensure(static_cast<size_t>(numel) * 4));
    int rc = launch_status(launch_dequant(fmt_of(type), static_cast<float*>(st->dtmp.p), static_cast<const uint8_t*>(dsrc),
                                          dscale, numel, group, st->stream),
                           "dequantize");
    if (rc) return rc;
    ALJ_CUDA(cudaMemcpyAsync(dst, st->dtmp.p, static_cast<size_t>(numel) * 4, cudaMemcpyDeviceToHost, st->stream));
    ALJ_CUDA(cudaStreamSynchronize(st->stream));
    return ALJ_OK;
}

int attn_check(const void* k, const void* v, int kv_dtype, int stride, int kv_heads, int q_heads, int head_dim,
               int seq_len, int start_pos) {
    if (!k || !v) return fail(ALJ_ERR_BAD_ARG, "null K or V cache");
    if (kv_dtype != ALJ_KV_F32 && kv_dtype != ALJ_KV_BF16) return fail(ALJ_ERR_UNSUPPORTED, "kv dtype %d", kv_dtype);
    if (kv_heads <= 0 || head_dim <= 0 || q_heads <= 0 || q_heads % kv_heads)
        return fail(ALJ_ERR_BAD_DIMS, "query heads must be a positive multiple of KV heads");
    if (stride < kv_heads * head_dim) return fail(ALJ_ERR_BAD_DIMS, "stride %d < kv_heads*head_dim", stride);
    if (start_pos < 0 || start_pos >= seq_len) return fail(ALJ_ERR_BAD_DIMS, "start %d outside [0, %d)", start_pos, seq_len);
    return ALJ_OK;
}

int run_attention(DeviceState* st, float* dout, const float* dq, const void* k, const void* v, int kv_dtype, int stride,
                  long long head_stride, int kv_heads, int q_heads, int head_dim, int seq_len, int start_pos, float scale, cudaStream_t stream,
                  DevBuf* scratch) {
    AttnParams p = {};
    p.out = dout;
    p.q = dq;
    p.k = k;
    p.v = v;
    p.kv_dtype = kv_dtype;
    p.stride = stride;
    p.head_stride = head_stride;
    p.kv_heads = kv_heads;
    p.q_heads = q_heads;
    p.head_dim = head_dim;
    p.seq_len = seq_len;
    p.start_pos = start_pos;
    p.scale = scale;
    p.splits = attention_splits(seq_len - start_pos, kv_heads, st->sms);
    if (p.splits > 1) {
        ALJ_CUDA(scratch->ensure(attention_scratch_floats(q_heads, head_dim, p.splits) * 4));
        attention_bind_scratch(p, static_cast<float*>(scratch->p));
        // The split merge's arrival counters must start at zero.  Each merge
        // returns its counter to zero, so after a call the first q_heads words
        // stay zero -- but a call with fewer heads lays partials over the
        // words past its own counters.  Clear them when this call needs more
        // than that (or the buffer is new, or a fault was reported), on the
        // launch stream itself: the stream may be non-blocking (the library's
        // own) or the caller's, so a memset on any other stream would not be
        // ordered before the kernel.
        if (q_heads > scratch->zeroed_words)
            ALJ_CUDA(cudaMemsetAsync(p.split_counter, 0, static_cast<size_t>(q_heads) * sizeof(unsigned int), stream));
        scratch->zeroed_words = q_heads;
    }
    // Programmatic dependent launch: the kernel reads q, the cache and its
    // scratch only after the previous kernel on the stream has completed, so
    // only its launch and set-up overlap that kernel's tail.
    return launch_status(launch_attention(p, stream, true), "decode attention");
}

// The binding's elementwise glue (rmsnorm, silu_ffn): operands that are
// device, managed or registered memory are used in place; plain host
// operands are staged through the device scratch.  Blocks until out is
// written.  kind 0: out = rmsnorm(a; weight b, eps); kind 1: out = silu(a) * b.
int glue_call(int kind, float* out, const float* a, const float* b, int n, float eps) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!out || !a || !b) return fail(ALJ_ERR_BAD_ARG, "null pointer argument");
    if (n <= 0 || n > (1 << 24)) return fail(ALJ_ERR_BAD_DIMS, "N=%d must be in [1, 2^24]", n);
    const float* da = static_cast<const float*>(resolve(st, a));
    const float* db = static_cast<const float*>(resolve(st, b));
    float* dout = const_cast<float*>(static_cast<const float*>(resolve(st, out)));
    std::lock_guard<std::mutex> g(st->mu);
    const size_t bytes = static_cast<size_t>(n) * 4;
    ALJ_CUDA(st->dtmp.ensure(3 * bytes));
    float* slot = static_cast<float*>(st->dtmp.p);
    if (!da) {
        ALJ_CUDA(cudaMemcpyAsync(slot, a, bytes, cudaMemcpyHostToDevice, st->stream));
        da = slot;
    }
    if (!db) {
        ALJ_CUDA(cudaMemcpyAsync(slot + n, b, bytes, cudaMemcpyHostToDevice, st->stream));
        db = slot + n;
    }
    float* dst = dout ? dout : slot + 2 * static_cast<size_t>(n);
    const cudaError_t e = kind == 0 ? launch_rmsnorm(dst, da, db, n, eps, st->stream)
                                    : launch_silu_ffn(dst, da, db, n, st->sms, st->stream);
    int rc = launch_status(e, kind == 0 ? "rmsnorm" : "silu_ffn");
    if (rc) return rc;
    if (!dout) ALJ_CUDA(cudaMemcpyAsync(out, dst, bytes, cudaMemcpyDeviceToHost, st->stream));
    ALJ_CUDA(cudaStreamSynchronize(st->stream));
    return ALJ_OK;
}

}  // namespace

int sm_count_for_current_device() {
    int err = 0;
    DeviceState* st = state(&err);
    return st && st->sms > 0 ? st->sms : 148;
}

int decode_fail(int code, const char* msg) { return fail(code, "%s", msg); }
void noalloc_forget_scratch();   // noalloc.cu

const void* decode_resolve(const void* p) {
    int err = 0;
    DeviceState* st = state(&err);
    return st ? resolve(st, p) : nullptr;
}

}  // namespace alj

using namespace alj;

namespace {
// Shared host-buffer path of the prefill attention entry points: q, then k
// and v compacted to kv_heads * head_dim floats per position, through the
// mapped staging buffer and the pull kernel; the output is stored straight
// into the mapped output buffer.
int run_prefill_host(float* out, const float* q, const float* k, const float* v, int B, int T, int S, int Hq, int Hkv,
                     int D, int kv_stride, float scale, int causal, int causal_offset, int window, float soft_cap) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!out || !q || !k || !v) return fail(ALJ_ERR_BAD_ARG, "prefill attention: null pointer");
    if (B < 1 || T < 1 || S < 1 || !prefill_attention_supported(Hq, Hkv, D) || kv_stride < Hkv * D)
        return fail(ALJ_ERR_BAD_DIMS, "prefill attention: B=%d T=%d S=%d H=%d H_kv=%d D=%d kv_stride=%d (D %% 32, D <= 256)",
                    B, T, S, Hq, Hkv, D, kv_stride);
    const size_t nq = static_cast<size_t>(B) * T * Hq * D;
    const size_t row = static_cast<size_t>(Hkv) * D;
    const size_t nk = static_cast<size_t>(B) * S * row;
    std::lock_guard<std::mutex> g(st->mu);
    ALJ_CUDA(st->dx.ensure((nq + 2 * nk) * 4));
    ALJ_CUDA(st->hx.ensure((nq + 2 * nk) * 4));
    ALJ_CUDA(st->hy.ensure(nq * 4));
    float* hq = static_cast<float*>(st->hx.p);
    memcpy(hq, q, nq * 4);
    float* hk = hq + nq;
    float* hv = hk + nk;
    for (size_t p = 0; p < static_cast<size_t>(B) * S; ++p) {
        memcpy(hk + p * row, k + p * kv_stride, row * 4);
        memcpy(hv + p * row, v + p * kv_stride, row * 4);
    }
    float* d = static_cast<float*>(st->dx.p);
    ALJ_CUDA(launch_host_pull(d, static_cast<const float*>(st->hx.dev), nq + 2 * nk, st->sms, st->stream));
    PrefillArgs a;
    a.out = static_cast<float*>(st->hy.dev);
    a.q = d;
    a.k = d + nq;
    a.v = d + nq + nk;
    a.B = B;
    a.T = T;
    a.S = S;
    a.Hq = Hq;
    a.Hkv = Hkv;
    a.D = D;
    a.kv_stride = static_cast<int>(row);
    a.causal = causal;
    a.causal_offset = causal_offset;
    a.window = window;
    a.scale = scale;
    a.soft_cap = soft_cap;
    const int rc = launch_status(launch_prefill_attention(a, st->stream), "prefill attention");
    if (rc) return rc;
    ALJ_CUDA(cudaStreamSynchronize(st->stream));
    memcpy(out, st->hy.p, nq * 4);
    return ALJ_OK;
}
}  // namespace

namespace {
// memcpy spread over host threads (the mapped file's pages are read by
// several cores at once; one core's copy runs well below the PCIe rate).
void parallel_copy(void* dst, const void* src, size_t n) {
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t nthr = std::min<size_t>(std::min(4u, hw), std::max<size_t>(1, n >> 22));   // >= 4 MB each
    if (nthr <= 1) {
        memcpy(dst, src, n);
        return;
    }
    std::vector<std::thread> th;
    const size_t part = (n / nthr + 4095) & ~size_t(4095);
    for (size_t t = 0; t < nthr; ++t) {
        const size_t off = t * part;
        if (off >= n) break;
        const size_t len = std::min(part, n - off);
        th.emplace_back([=] { memcpy(static_cast<uint8_t*>(dst) + off, static_cast<const uint8_t*>(src) + off, len); });
    }
    for (auto& x : th) x.join();
}

// Copies a (mapped, pageable) model file to HBM.  Up to 64 MB: one pageable
// cudaMemcpy.  Larger: 32 MB chunks through two pinned bounce buffers kept
// per device (pinning costs ~0.4 ms per MB, paid once), the host copy of a
// chunk spread over host threads while the DMA of the previous chunk runs on
// `stream`.  Measured on B200 hosts: pageable copies ~10 GB/s, one host thread
// into pinned memory ~14 GB/s, pinned DMA ~55 GB/s.
int upload_model(DeviceState* st, void* dev, const void* src, size_t bytes) {
    constexpr size_t kSmall = size_t(64) << 20;
    constexpr size_t kChunk = size_t(32) << 20;
    if (bytes <= kSmall) {
        const cudaError_t e = cudaMemcpy(dev, src, bytes, cudaMemcpyHostToDevice);
        return e == cudaSuccess ? ALJ_OK : fail(ALJ_ERR_CUDA, "model upload: %s", cudaGetErrorString(e));
    }
    std::lock_guard<std::mutex> g(st->upload_mu);
    for (int b = 0; b < 2; ++b) {
        if (!st->upload_bounce[b] && cudaHostAlloc(&st->upload_bounce[b], kChunk, cudaHostAllocPortable) != cudaSuccess) {
            st->upload_bounce[b] = nullptr;
            cudaGetLastError();
            return fail(ALJ_ERR_NO_MEMORY, "pinned bounce buffers for the model upload (2 x %zu bytes)", kChunk);
        }
        if (!st->upload_done[b] && cudaEventCreateWithFlags(&st->upload_done[b], cudaEventDisableTiming) != cudaSuccess) {
            st->upload_done[b] = nullptr;
            cudaGetLastError();
            return fail(ALJ_ERR_CUDA, "model upload: event creation failed");
        }
    }
    int rc = ALJ_OK;
    size_t i = 0;
    for (size_t off = 0; off < bytes && rc == ALJ_OK; off += kChunk, ++i) {
        const int b = static_cast<int>(i & 1);
        const size_t n = std::min(kChunk, bytes - off);
        cudaError_t e = i >= 2 ? cudaEventSynchronize(st->upload_done[b]) : cudaSuccess;   // its previous DMA is done
        if (e == cudaSuccess) {
            parallel_copy(st->upload_bounce[b], static_cast<const uint8_t*>(src) + off, n);
            e = cudaMemcpyAsync(static_cast<uint8_t*>(dev) + off, st->upload_bounce[b], n, cudaMemcpyHostToDevice,
                                st->stream);
        }
        if (e == cudaSuccess) e = cudaEventRecord(st->upload_done[b], st->stream);
        if (e != cudaSuccess) rc = fail(ALJ_ERR_CUDA, "model upload at byte %zu: %s", off, cudaGetErrorString(e));
    }
    const cudaError_t e = cudaStreamSynchronize(st->stream);
    if (rc == ALJ_OK && e != cudaSuccess) rc = fail(ALJ_ERR_CUDA, "model upload: %s", cudaGetErrorString(e));
    return rc;
}
}  // namespace

extern "C" {

int aljabr_blackwell_init(int device_id) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(ALJ_ERR_NOT_INITIALIZED, "no CUDA device visible");
    }
    if (device_id < 0 || device_id >= count) return fail(ALJ_ERR_BAD_ARG, "device %d out of range (%d devices)", device_id, count);
    t_device = device_id;
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_id);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device_id);
    if (major != 10) return fail(ALJ_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device_id, major, minor);
    return ALJ_OK;
}

int aljabr_blackwell_device_count(void) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return count;
}

int aljabr_blackwell_device_get(int device_id) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(ALJ_ERR_NOT_INITIALIZED, "no CUDA device visible");
    }
    if (device_id < 0 || device_id >= count) return fail(ALJ_ERR_BAD_ARG, "device %d out of range (%d devices)", device_id, count);
    t_device = device_id;
    int err = 0;
    return state(&err) ? ALJ_OK : err;
}

int aljabr_blackwell_device_name(char* buf, int buf_len, int device_id) {
    if (!buf || buf_len <= 0) return fail(ALJ_ERR_BAD_ARG, "null buffer");
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        buf[0] = '\0';
        return fail(ALJ_ERR_NOT_INITIALIZED, "no CUDA device visible");
    }
    if (device_id < 0 || device_id >= count) return fail(ALJ_ERR_BAD_ARG, "device %d out of range (%d devices)", device_id, count);
    cudaDeviceProp prop;
    ALJ_CUDA(cudaGetDeviceProperties(&prop, device_id));
    snprintf(buf, static_cast<size_t>(buf_len), "%s", prop.name);
    return ALJ_OK;
}

long long aljabr_blackwell_tmem_size(int device_id) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(ALJ_ERR_NOT_INITIALIZED, "no CUDA device visible");
    }
    if (device_id < 0 || device_id >= count) return fail(ALJ_ERR_BAD_ARG, "device %d out of range (%d devices)", device_id, count);
    int major = 0, sms = 0;
    ALJ_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_id));
    ALJ_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device_id));
    if (major != 10) return fail(ALJ_ERR_UNSUPPORTED, "device %d has no tensor memory (sm_%d)", device_id, major);
    return static_cast<long long>(sms) * 128 * 512 * 4;   // 128 lanes x 512 columns x 32 bit per SM
}

int aljabr_blackwell_compute_capability(int device_id) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device_id) != cudaSuccess) return ALJ_ERR_CUDA;
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device_id);
    return major * 10 + minor;
}

long long aljabr_blackwell_free_memory(void) {
    int err = 0;
    if (!state(&err)) return err;
    size_t f = 0, t = 0;
    if (cudaMemGetInfo(&f, &t) != cudaSuccess) return ALJ_ERR_CUDA;
    return static_cast<long long>(f);
}

const char* aljabr_blackwell_last_error(void) { return t_last_error.c_str(); }

int aljabr_blackwell_set_pdl(int enable) {
    t_pdl = enable != 0;
    return ALJ_OK;
}

int aljabr_blackwell_prefetch_hint(const void* next_weights, size_t bytes) {
    if (!next_weights || bytes == 0) {
        t_prefetch = nullptr;
        t_prefetch_bytes = 0;
        return ALJ_OK;
    }
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    const void* d = resolve(st, next_weights);
    if (!d) return fail(ALJ_ERR_NOT_REGISTERED, "prefetch hint: not device or registered memory");
    t_prefetch = d;
    t_prefetch_bytes = bytes;
    return ALJ_OK;
}

void aljabr_blackwell_set_verbose(int enable) { g_verbose = enable; }

int aljabr_blackwell_device_status(unsigned int* fault_bits) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    unsigned int v = 0, zero = 0;
    ALJ_CUDA(cudaMemcpyFromSymbol(&v, g_fault_word, sizeof v));
    ALJ_CUDA(cudaMemcpyToSymbol(g_fault_word, &zero, sizeof zero));
    if (fault_bits) *fault_bits = v;
    if (v) {
        // a kernel that gave up may have left split-merge counters non-zero
        std::lock_guard<std::mutex> g(st->mu);
        st->dscratch.zeroed_words = 0;
    }
    return v & ALJ_FAULT_TIMEOUT ? ALJ_ERR_TIMEOUT : ALJ_OK;
}

int aljabr_blackwell_shutdown(void) {
    noalloc_forget_scratch();
    std::lock_guard<std::mutex> g(g_mu);
    for (auto& s : g_dev) {
        if (!s) continue;
        cudaSetDevice(s->device);
        cudaStreamSynchronize(s->stream);
        for (auto& kv : s->reg) cudaFree(kv.second.dev);
        s->reg.clear();
        s->dx.release(); s->dy.release(); s->dtmp.release(); s->dscratch.release(); s->dgemm.release();
        s->hx.release(); s->hy.release();
        for (auto& kv : s->qpack) cudaFree(kv.second.p);
        s->qpack.clear();
        for (auto& kv : s->tb_graphs)
            if (kv.second.second) cudaGraphExecDestroy(kv.second.second);
        s->tb_graphs.clear();
        for (int b = 0; b < 2; ++b) {
            if (s->upload_bounce[b]) cudaFreeHost(s->upload_bounce[b]);
            if (s->upload_done[b]) cudaEventDestroy(s->upload_done[b]);
        }
        cudaStreamDestroy(s->stream);
        s.reset();
    }
    g_dev.clear();
    return ALJ_OK;
}

int aljabr_blackwell_register_model_buffer(const void* base_ptr, size_t total_bytes) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!base_ptr || total_bytes == 0) return fail(ALJ_ERR_BAD_ARG, "null or empty model buffer");
    {
        std::lock_guard<std::mutex> g(st->reg_mu);
        auto it = st->reg.find(reinterpret_cast<uintptr_t>(base_ptr));
        if (it != st->reg.end()) {
            if (it->second.bytes >= total_bytes) return ALJ_OK;
            cudaFree(it->second.dev);
            st->reg.erase(it);
        }
    }
    void* dev = nullptr;
    cudaError_t e = cudaMalloc(&dev, total_bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ALJ_ERR_NO_MEMORY, "cudaMalloc(%zu) for the model buffer: %s", total_bytes, cudaGetErrorString(e));
    }
    const int rc = upload_model(st, dev, base_ptr, total_bytes);
    if (rc != ALJ_OK) {
        cudaFree(dev);
        return rc;
    }
    std::lock_guard<std::mutex> g(st->reg_mu);
    st->reg[reinterpret_cast<uintptr_t>(base_ptr)] = Registered{total_bytes, dev};
    return ALJ_OK;
}

int aljabr_blackwell_unregister_model_buffer(const void* base_ptr) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    std::lock_guard<std::mutex> g(st->reg_mu);
    auto it = st->reg.find(reinterpret_cast<uintptr_t>(base_ptr));
    if (it == st->reg.end()) return fail(ALJ_ERR_NOT_REGISTERED, "buffer %p is not registered", base_ptr);
    cudaStreamSynchronize(st->stream);
    {
        // packed GEMM copies of matrices inside this buffer
        std::lock_guard<std::mutex> gm(st->mu);
        const uintptr_t lo = reinterpret_cast<uintptr_t>(it->second.dev), hi = lo + it->second.bytes;
        for (auto q = st->qpack.begin(); q != st->qpack.end();) {
            const uintptr_t w = std::get<0>(q->first);
            if (w >= lo && w < hi) {
                cudaFree(q->second.p);
                q = st->qpack.erase(q);
            } else {
                ++q;
            }
        }
        // replay graphs of host-buffer calls on matrices inside this buffer
        for (auto q = st->tb_graphs.begin(); q != st->tb_graphs.end();) {
            bool inside = false;
            for (int i = 0; i < 3; ++i) inside = inside || (q->first[5 + i] >= lo && q->first[5 + i] < hi);
            if (inside) {
                if (q->second.second) cudaGraphExecDestroy(q->second.second);
                q = st->tb_graphs.erase(q);
            } else {
                ++q;
            }
        }
    }
    cudaFree(it->second.dev);
    st->reg.erase(it);
    return ALJ_OK;
}

void* aljabr_blackwell_device_address(const void* host_ptr) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return nullptr;
    return const_cast<void*>(resolve(st, host_ptr));
}

int aljabr_blackwell_matvec_tb_q4_0(void* C, const void* A, const void* B, int K, int N) {
    const int t = ALJ_TYPE_Q4_0;
    const void* b[1] = {B};
    const float* am[1] = {nullptr};
    HostOut o[1] = {{C, N}};
    return tb_matvec(1, &t, b, am, nullptr, o, A, K, 0, 1);
}

int aljabr_blackwell_matvec_tb_q8_0(void* C, const void* A, const void* B, int K, int N) {
    const int t = ALJ_TYPE_Q8_0;
    const void* b[1] = {B};
    const float* am[1] = {nullptr};
    HostOut o[1] = {{C, N}};
    return tb_matvec(1, &t, b, am, nullptr, o, A, K, 0, 1);
}

int aljabr_blackwell_matvec_tb_q4_k(void* C, const void* A, const void* B, int K, int N) {
    const int t = ALJ_TYPE_Q4_K;
    const void* b[1] = {B};
    const float* am[1] = {nullptr};
    HostOut o[1] = {{C, N}};
    return tb_matvec(1, &t, b, am, nullptr, o, A, K, 0, 1);
}

int aljabr_blackwell_matvec_tb_q6_k(void* C, const void* A, const void* B, int K, int N) {
    const int t = ALJ_TYPE_Q6_K;
    const void* b[1] = {B};
    const float* am[1] = {nullptr};
    HostOut o[1] = {{C, N}};
    return tb_matvec(1, &t, b, am, nullptr, o, A, K, 0, 1);
}

int aljabr_blackwell_matvec_tb_nf4(void* C, const void* A, const void* B_packed, const void* absmax, int K, int N,
                                   int blockSize) {
    return aljabr_blackwell_linear_nf4(C, A, B_packed, absmax, nullptr, K, N, blockSize);
}

int aljabr_blackwell_linear_nf4(void* C, const void* A, const void* B_packed, const void* absmax, const void* bias,
                                int K, int N, int blockSize) {
    const int t = ALJ_TYPE_NF4;
    const void* b[1] = {B_packed};
    const float* am[1] = {static_cast<const float*>(absmax)};
    HostOut o[1] = {{C, N}};
    return tb_matvec(1, &t, b, am, static_cast<const float*>(bias), o, A, K, blockSize, 1);
}

int aljabr_blackwell_matvec_tb_pair(void* C0, void* C1, const void* A, const void* B0, const void* B1, int K, int N0,
                                    int N1, int type0, int type1) {
    const int t[2] = {type0, type1};
    const void* b[2] = {B0, B1};
    const float* am[2] = {nullptr, nullptr};
    if (type0 == ALJ_TYPE_NF4 || type1 == ALJ_TYPE_NF4) return fail(ALJ_ERR_UNSUPPORTED, "NF4 pairs need absmax: use linear_nf4");
    HostOut o[2] = {{C0, N0}, {C1, N1}};
    return tb_matvec(2, t, b, am, nullptr, o, A, K, 0, 1);
}

int aljabr_blackwell_matvec_tb_triple(void* C0, void* C1, void* C2, const void* A, const void* B0, const void* B1,
                                      const void* B2, int K, int N0, int N1, int N2, int type0, int type1, int type2) {
    const int t[3] = {type0, type1, type2};
    const void* b[3] = {B0, B1, B2};
    const float* am[3] = {nullptr, nullptr, nullptr};
    if (type0 == ALJ_TYPE_NF4 || type1 == ALJ_TYPE_NF4 || type2 == ALJ_TYPE_NF4)
        return fail(ALJ_ERR_UNSUPPORTED, "NF4 triples need absmax: use linear_nf4");
    HostOut o[3] = {{C0, N0}, {C1, N1}, {C2, N2}};
    return tb_matvec(3, t, b, am, nullptr, o, A, K, 0, 1);
}

int aljabr_blackwell_matvec_tb_batch(void* C, const void* A, const void* B, int K, int N, int type, int batchSize) {
    if (batchSize <= 0) return fail(ALJ_ERR_BAD_DIMS, "batchSize=%d", batchSize);
    if (type == ALJ_TYPE_NF4) return fail(ALJ_ERR_UNSUPPORTED, "NF4 batches need absmax: use linear_nf4");
    const void* b[1] = {B};
    const float* am[1] = {nullptr};
    HostOut o[1] = {{C, N}};
    return tb_matvec(1, &type, b, am, nullptr, o, A, K, 0, batchSize);
}

int aljabr_blackwell_matvec_tb_triple_batch(void* C0, void* C1, void* C2, const void* A, const void* B0,
                                            const void* B1, const void* B2, int K, int N0, int N1, int N2,
                                            int type0, int type1, int type2, int batchSize) {
    if (batchSize <= 0) return fail(ALJ_ERR_BAD_DIMS, "batchSize=%d", batchSize);
    const int types[3] = {type0, type1, type2};
    for (int i = 0; i < 3; ++i)
        if (types[i] == ALJ_TYPE_NF4) return fail(ALJ_ERR_UNSUPPORTED, "NF4 batches need absmax: use linear_nf4");
    const void* b[3] = {B0, B1, B2};
    const float* am[3] = {nullptr, nullptr, nullptr};
    HostOut o[3] = {{C0, N0}, {C1, N1}, {C2, N2}};
    return tb_matvec(3, types, b, am, nullptr, o, A, K, 0, batchSize);
}

int aljabr_blackwell_dequantize_nf4(void* dst, const void* src, const void* scales, long long numel, int groupSize) {
    return tb_dequant(ALJ_TYPE_NF4, dst, src, scales, numel, groupSize);
}
int aljabr_blackwell_dequantize_q4_0(void* dst, const void* blocks, long long numel) {
    return tb_dequant(ALJ_TYPE_Q4_0, dst, blocks, nullptr, numel, 0);
}
int aljabr_blackwell_dequantize_q8_0(void* dst, const void* blocks, long long numel) {
    return tb_dequant(ALJ_TYPE_Q8_0, dst, blocks, nullptr, numel, 0);
}

int aljabr_blackwell_decode_attention(float* out, const float* q, const void* k_cache, const void* v_cache, int kv_dtype,
                                      int cache_head_stride, int kv_heads, int q_heads, int head_dim, int seq_len,
                                      int start_pos, float scale) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!out || !q) return fail(ALJ_ERR_BAD_ARG, "null q or out");
    int rc = attn_check(k_cache, v_cache, kv_dtype, cache_head_stride, kv_heads, q_heads, head_dim, seq_len, start_pos);
    if (rc) return rc;
    const void* dk = resolve(st, k_cache);
    const void* dv = resolve(st, v_cache);
    if (!dk || !dv) return fail(ALJ_ERR_NOT_REGISTERED, "K/V caches must be device or registered memory");
    std::lock_guard<std::mutex> g(st->mu);
    const size_t n = static_cast<size_t>(q_heads) * head_dim;
    ALJ_CUDA(st->dx.ensure(n * 4));
    ALJ_CUDA(st->hx.ensure(n * 4));
    ALJ_CUDA(st->hy.ensure(n * 4));
    memcpy(st->hx.p, q, n * 4);
    // q through the pull kernel, the output stored straight into the mapped buffer
    ALJ_CUDA(launch_host_pull(static_cast<float*>(st->dx.p), static_cast<const float*>(st->hx.dev), n, st->sms,
                              st->stream));
    rc = run_attention(st, static_cast<float*>(st->hy.dev), static_cast<const float*>(st->dx.p), dk, dv, kv_dtype,
                       cache_head_stride, head_dim, kv_heads, q_heads, head_dim, seq_len, start_pos, scale, st->stream, &st->dscratch);
    if (rc) return rc;
    ALJ_CUDA(cudaStreamSynchronize(st->stream));
    memcpy(out, st->hy.p, n * 4);
    return ALJ_OK;
}


int aljabr_blackwell_prefill_attention(float* out, const float* q, const float* k, const float* v, int tokens,
                                       int q_heads, int kv_heads, int head_dim, float scale, int sliding_window,
                                       int kv_stride) {
    return run_prefill_host(out, q, k, v, 1, tokens, tokens, q_heads, kv_heads, head_dim, kv_stride, scale, 1, 0,
                            sliding_window > 0 ? sliding_window : 0, 0.0f);
}

int aljabr_blackwell_fa4_attention(void* output, void* query, void* key, void* value, int B, int T, int S, int H,
                                   int H_kv, int D, float scale, int is_causal, int use_bf16, float soft_cap) {
    (void)use_bf16;   // the arithmetic is fp32 either way
    return run_prefill_host(static_cast<float*>(output), static_cast<const float*>(query),
                            static_cast<const float*>(key), static_cast<const float*>(value), B, T, S, H, H_kv, D,
                            H_kv * D, scale, is_causal ? 1 : 0, S > T ? S - T : 0, 0, soft_cap > 0.0f ? soft_cap : 0.0f);
}

int aljabr_blackwell_fa4_sdpa_available(void) { return 1; }
int aljabr_blackwell_fa4_bf16_available(void) { return 0; }

int aljabr_blackwell_prefill_attention_dev(float* out, const float* q, const float* k, const float* v, int B, int T,
                                           int S, int q_heads, int kv_heads, int head_dim, int kv_stride, float scale,
                                           int causal, int window, float soft_cap, void* stream) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!out || !q || !k || !v) return fail(ALJ_ERR_BAD_ARG, "prefill attention: null pointer");
    if (B < 1 || T < 1 || S < 1 || !prefill_attention_supported(q_heads, kv_heads, head_dim) ||
        kv_stride < kv_heads * head_dim || kv_stride % 4)
        return fail(ALJ_ERR_BAD_DIMS, "prefill attention: B=%d T=%d S=%d H=%d H_kv=%d D=%d kv_stride=%d", B, T, S,
                    q_heads, kv_heads, head_dim, kv_stride);
    if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
         reinterpret_cast<uintptr_t>(v)) & 15)
        return fail(ALJ_ERR_BAD_ARG, "prefill attention: pointers must be 16-byte aligned");
    PrefillArgs a;
    a.out = out;
    a.q = q;
    a.k = k;
    a.v = v;
    a.B = B;
    a.T = T;
    a.S = S;
    a.Hq = q_heads;
    a.Hkv = kv_heads;
    a.D = head_dim;
    a.kv_stride = kv_stride;
    a.causal = causal ? 1 : 0;
    a.causal_offset = S > T ? S - T : 0;
    a.window = window > 0 ? window : 0;
    a.scale = scale;
    a.soft_cap = soft_cap > 0.0f ? soft_cap : 0.0f;
    return launch_status(launch_prefill_attention(a, pick_stream(st, stream)), "prefill attention");
}

int aljabr_blackwell_matvec_dev(int type, float* y, const float* x, const void* w, const float* absmax, int K, int N,
                                int group, const float* bias, void* stream) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    int rc = check_dims(type, K, N);
    if (rc) return rc;
    if (!y || !x || !w) return fail(ALJ_ERR_BAD_ARG, "null y, x or w");
    if (type == ALJ_TYPE_NF4 && (!absmax || group <= 0)) return fail(ALJ_ERR_BAD_ARG, "NF4 needs absmax and group > 0");
    MatSpec m = {type, w, absmax, bias, y, N};
    return run_matvecs(st, &m, 1, x, K, group, pick_stream(st, stream), t_pdl);
}

long long aljabr_blackwell_gemm_nf4_workspace_size(int M, int K, int nseg, const int* rows) {
    if (M < 1 || K < 1 || nseg < 1 || nseg > 3 || !rows) return fail(ALJ_ERR_BAD_ARG, "bad gemm_nf4 shape");
    for (int s = 0; s < nseg; ++s)
        if (rows[s] < 1) return fail(ALJ_ERR_BAD_DIMS, "rows[%d]=%d", s, rows[s]);
    const int sms = sm_count_for_current_device();
    return static_cast<long long>(gemm_nf4_workspace_bytes(M, K, gemm_nf4_tiles(M, nseg, rows), sms > 0 ? sms : 1));
}

long long aljabr_blackwell_gemm_nf4_packed_size(int rows, int K, int blockSize) {
    if (rows < 1 || !gemm_nf4_supported(1, K, blockSize))
        return fail(ALJ_ERR_UNSUPPORTED, "gemm_nf4: rows=%d K=%d blockSize=%d (K %% 256, blockSize 64/128)", rows, K,
                    blockSize);
    return static_cast<long long>(gemm_nf4_packed_bytes(rows, K, blockSize));
}

int aljabr_blackwell_gemm_nf4_pack(void* packed, const void* codes, const void* absmax, int rows, int K, int blockSize,
                                   void* stream) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!packed || !codes || !absmax) return fail(ALJ_ERR_BAD_ARG, "gemm_nf4_pack: null pointer");
    if (rows < 1 || !gemm_nf4_supported(1, K, blockSize))
        return fail(ALJ_ERR_UNSUPPORTED, "gemm_nf4_pack: rows=%d K=%d blockSize=%d", rows, K, blockSize);
    if ((reinterpret_cast<uintptr_t>(packed) & 255) || (reinterpret_cast<uintptr_t>(codes) & 15))
        return fail(ALJ_ERR_BAD_ARG, "gemm_nf4_pack: packed must be 256-byte and codes 16-byte aligned");
    return launch_status(launch_gemm_nf4_pack(packed, codes, absmax, rows, K, blockSize, pick_stream(st, stream)),
                         "gemm_nf4_pack");
}

int aljabr_blackwell_gemm_nf4_dev(int nseg, float* const* y, const int* ldy, const void* const* packed,
                                  const int* rows, const void* x_bf16, int M, int K, int blockSize, void* workspace,
                                  long long workspace_bytes, void* stream) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (nseg < 1 || nseg > 3 || !y || !ldy || !packed || !rows || !x_bf16 || !workspace)
        return fail(ALJ_ERR_BAD_ARG, "gemm_nf4: null argument or nseg=%d", nseg);
    if (M < 1 || K < 1) return fail(ALJ_ERR_BAD_DIMS, "gemm_nf4: M=%d K=%d", M, K);
    if (reinterpret_cast<uintptr_t>(x_bf16) & 15) return fail(ALJ_ERR_BAD_ARG, "gemm_nf4: x not 16-byte aligned");
    if (!gemm_nf4_supported(M, K, blockSize))
        return fail(ALJ_ERR_UNSUPPORTED, "gemm_nf4: K=%d blockSize=%d (K %% 256, blockSize 64/128)", K, blockSize);
    GemmNf4Args a;
    memset(&a, 0, sizeof a);
    a.nseg = nseg;
    for (int s = 0; s < nseg; ++s) {
        if (!y[s] || !packed[s]) return fail(ALJ_ERR_BAD_ARG, "gemm_nf4: null segment %d", s);
        if (reinterpret_cast<uintptr_t>(packed[s]) & 255)
            return fail(ALJ_ERR_BAD_ARG, "gemm_nf4: packed weights %d not 256-byte aligned", s);
        if (rows[s] < 1 || ldy[s] < rows[s]) return fail(ALJ_ERR_BAD_DIMS, "gemm_nf4: rows=%d ldy=%d", rows[s], ldy[s]);
        a.y[s] = y[s];
        a.ldy[s] = ldy[s];
        a.packed[s] = packed[s];
        a.rows[s] = rows[s];
    }
    a.x = x_bf16;
    a.M = M;
    a.K = K;
    a.group = blockSize;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes > 0 ? static_cast<size_t>(workspace_bytes) : 0;
    const size_t need = gemm_nf4_workspace_bytes(M, K, gemm_nf4_tiles(M, nseg, rows), sm_count_for_current_device());
    if (a.workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(ALJ_ERR_BAD_ARG, "gemm_nf4: workspace %lld bytes (need %zu, 256-byte aligned)", workspace_bytes, need);
    return launch_status(launch_gemm_nf4(a, pick_stream(st, stream)), "gemm_nf4");
}

long long aljabr_blackwell_gemm_q_packed_size(int type, int rows, int K) {
    const int fmt = fmt_of(type);
    if (rows < 1 || !gemm_q_supported(fmt, 2, K))
        return fail(ALJ_ERR_UNSUPPORTED, "gemm_q: type=%d rows=%d K=%d (Q4_0/Q8_0, K %% 256, K <= 32768)", type, rows, K);
    return static_cast<long long>(gemm_q_packed_bytes(fmt, rows, K));
}

int aljabr_blackwell_gemm_q_pack(int type, void* packed, const void* weights, int rows, int K, void* stream) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!packed || !weights) return fail(ALJ_ERR_BAD_ARG, "gemm_q_pack: null pointer");
    const int fmt = fmt_of(type);
    if (rows < 1 || !gemm_q_supported(fmt, 2, K))
        return fail(ALJ_ERR_UNSUPPORTED, "gemm_q_pack: type=%d rows=%d K=%d", type, rows, K);
    if (reinterpret_cast<uintptr_t>(packed) & 255) return fail(ALJ_ERR_BAD_ARG, "gemm_q_pack: packed not 256-byte aligned");
    return launch_status(launch_gemm_q_pack(fmt, packed, weights, rows, K, pick_stream(st, stream)), "gemm_q_pack");
}

long long aljabr_blackwell_gemm_q_workspace_size(int M, int K) {
    if (M < 1 || K < 1) return fail(ALJ_ERR_BAD_ARG, "bad gemm_q shape");
    return static_cast<long long>(gemm_q_workspace_bytes(M, K));
}

int aljabr_blackwell_gemm_q_dev(int type, int nseg, float* const* y, const int* ldy, const void* const* packed,
                                const int* rows, const float* x, int M, int K, void* workspace,
                                long long workspace_bytes, void* stream) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (nseg < 1 || nseg > 3 || !y || !ldy || !packed || !rows || !x || !workspace)
        return fail(ALJ_ERR_BAD_ARG, "gemm_q: null argument or nseg=%d", nseg);
    if (M < 1 || K < 1) return fail(ALJ_ERR_BAD_DIMS, "gemm_q: M=%d K=%d", M, K);
    if (reinterpret_cast<uintptr_t>(x) & 15) return fail(ALJ_ERR_BAD_ARG, "gemm_q: x not 16-byte aligned");
    const int fmt = fmt_of(type);
    if (!gemm_q_supported(fmt, M, K))
        return fail(ALJ_ERR_UNSUPPORTED, "gemm_q: type=%d K=%d (Q4_0/Q8_0, K %% 256, K <= 32768)", type, K);
    GemmQArgs a;
    memset(&a, 0, sizeof a);
    a.fmt = fmt;
    a.nseg = nseg;
    for (int s = 0; s < nseg; ++s) {
        if (!y[s] || !packed[s]) return fail(ALJ_ERR_BAD_ARG, "gemm_q: null segment %d", s);
        if (reinterpret_cast<uintptr_t>(packed[s]) & 255)
            return fail(ALJ_ERR_BAD_ARG, "gemm_q: packed weights %d not 256-byte aligned", s);
        if (rows[s] < 1 || ldy[s] < rows[s]) return fail(ALJ_ERR_BAD_DIMS, "gemm_q: rows=%d ldy=%d", rows[s], ldy[s]);
        a.y[s] = y[s];
        a.ldy[s] = ldy[s];
        a.packed[s] = packed[s];
        a.rows[s] = rows[s];
    }
    a.x = x;
    a.M = M;
    a.K = K;
    a.workspace = workspace;
    a.workspace_bytes = workspace_bytes > 0 ? static_cast<size_t>(workspace_bytes) : 0;
    const size_t need = gemm_q_workspace_bytes(M, K);
    if (a.workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(ALJ_ERR_BAD_ARG, "gemm_q: workspace %lld bytes (need %zu, 256-byte aligned)", workspace_bytes, need);
    return launch_status(launch_gemm_q(a, pick_stream(st, stream)), "gemm_q");
}

int aljabr_blackwell_dequantize_dev(int type, float* dst, const void* src, const float* absmax, long long numel, int group,
                                    void* stream) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!dst || !src) return fail(ALJ_ERR_BAD_ARG, "null dst or src");
    if (fmt_of(type) < 0) return fail(ALJ_ERR_UNSUPPORTED, "type %d", type);
    if (numel <= 0 || (type != ALJ_TYPE_NF4 && numel % 32)) return fail(ALJ_ERR_BAD_DIMS, "numel=%lld", numel);
    if (type == ALJ_TYPE_NF4 && (!absmax || group <= 0)) return fail(ALJ_ERR_BAD_ARG, "NF4 needs absmax and group > 0");
    return launch_status(launch_dequant(fmt_of(type), dst, static_cast<const uint8_t*>(src), absmax, numel, group,
                                        pick_stream(st, stream)),
                         "dequantize");
}

int aljabr_blackwell_decode_attention_dev(float* out, const float* q, const void* k_cache, const void* v_cache,
                                          int kv_dtype, int cache_head_stride, int kv_heads, int q_heads, int head_dim,
                                          int seq_len, int start_pos, float scale, void* stream) {
    int err = 0;
    DeviceState* st = state(&err);
    if (!st) return err;
    if (!out || !q) return fail(ALJ_ERR_BAD_ARG, "null q or out");
    int rc = attn_check(k_cache, v_cache, kv_dtype, cache_head_stride, kv_heads, q_heads, head_dim, seq_len, start_pos);
    if (rc) return rc;
    std::lock_guard<std::mutex> g(st->mu);   // the split scratch is shared per device
    return run_attention(st, out, q, k_cache, v_cache, kv_dtype, cache_head_stride, head_dim, kv_heads, q_heads, head_dim,
                         seq_len, start_pos, scale, pick_stream(st, stream), &st->dscratch);
}

int aljabr_blackwell_rmsnorm(float* out, const float* x, const float* weight, int N, float eps) {
    return glue_call(0, out, x, weight, N, eps);
}

int aljabr_blackwell_silu_ffn(float* out, const float* gate, const float* up, int N) {
    return glue_call(1, out, gate, up, N, 0.0f);
}

}  // extern "C"
