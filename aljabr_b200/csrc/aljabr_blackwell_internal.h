// Internal (library-private) declarations shared by the .cu translation units
// of libaljabr_blackwell.so.  The public C-ABI lives in include/aljabr_blackwell.h.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/aljabr_blackwell.h"

// Bits of the device fault word.
#define ALJ_FAULT_TIMEOUT 0x1u      // an mbarrier / flag wait ran out of its limit
#define ALJ_FAULT_BOUNDS 0x2u       // a checked index fell outside its buffer

namespace alj {

enum WeightFormat : int { FMT_Q4_0 = 0, FMT_Q8_0 = 1, FMT_NF4 = 2, FMT_Q4_K = 3, FMT_Q6_K = 4 };

// Output-side fusions of a matvec (decode-step fusion).
enum Epilogue : int {
    EPI_STORE = 0,         // y = W x (+ bias) (+ residual)
    EPI_SWIGLU_PAIR = 1,   // segments 0 (gate) and 1 (up) of equal rows: seg[0].y = silu(W_g x) * (W_u x)
};

// Tensor-parallel exchange of a kernel's output slice over NVLink (decode
// step on 2..8 GPUs).  A kernel with tp > 1 stores each output row into every
// rank's copy (push_y[r] + row), and the CTA that finishes last publishes,
// after a system-scope fence, the rank's sum of squares of its rows into
// push_part[r] (if set) and the flag value (*seq) * push_mul + push_add into
// push_flag[r] on every rank.  A kernel whose input is such a gathered buffer
// first waits (bounded) until its local wait_flags[0..tp) all reach
// (*seq) * wait_mul + wait_add.
constexpr int kMaxTp = 8;
struct TpLink {
    int tp;                              // <= 1: no exchange
    float* push_y[kMaxTp];
    float* push_part[kMaxTp];
    unsigned int* push_flag[kMaxTp];
    unsigned int* counter;               // local last-CTA counter: 0 before and after
    const unsigned int* wait_flags;      // local [tp], or null
    const int* seq;                      // device token counter
    int push_mul, push_add, wait_mul, wait_add;
};

struct MatvecSegment {
    const uint8_t* w;        // Q4_0 / Q8_0 blocks, or NF4 packed codes (row-major [rows][K])
    const float* absmax;     // NF4 per-group fp32 scales, else null
    const float* bias;       // optional, y += bias[row]
    const float* residual;   // optional, y = residual[row] + W x (may alias y)
    float* y;
    int rows;
};

struct MatvecParams {
    MatvecSegment seg[3];
    int nseg;
    int K;
    int total_rows;          // rows of all segments (EPI_SWIGLU_PAIR: rows of one segment)
    int group;               // NF4 group size
    const float* x;
    int epilogue;
    // Optional RMSNorm of the finished output (single segment): the last CTA
    // to finish writes norm_out = y * rsqrt(mean(y^2) + eps) * norm_w.
    // norm_partials holds one float per CTA (>= 2 * SM count); norm_counter
    // starts at 0 and is left at 0.
    float* norm_out;
    const float* norm_w;
    float norm_eps;
    float* norm_partials;
    unsigned int* norm_counter;
    // Deferred RMSNorm (NF4 table and integer tensor-core kernels).
    // norm_defer: instead of the last-CTA pass, write norm_out = y * norm_w
    // (unscaled) and this CTA's sum of squares of y to norm_partials[CTA]; the
    // consuming launch applies the scale.  in_parts (consuming side): x is
    // such an unscaled vector whose producer left in_nparts partials; the
    // table kernel multiplies every output by rsqrt(sum(partials) / in_rows +
    // in_eps), the integer kernel scales x by it while converting x.
    int norm_defer;
    const float* in_parts;
    int in_nparts;
    int in_rows;
    float in_eps;
    // Optional L2 prefetch of the weights the following launch reads (each CTA
    // its 1/grid share, after its own copies are issued).
    const void* prefetch;
    size_t prefetch_bytes;
    TpLink tpl;              // tensor-parallel push / wait (NF4 table kernel only)
};
// CTAs a TMA matvec launches (the size norm_partials must have).
int matvec_max_ctas();

// Kernel launchers (return cudaError_t of the launch).  `pdl` enables
// programmatic dependent launch on the stream.
cudaError_t launch_matvec(int fmt, const MatvecParams& p, cudaStream_t stream, bool pdl);
bool matvec_tma_supported(int fmt, int K, int group);
// Integer tensor-core path (Q4_0 / Q8_0 / Q4_K / Q6_K, K a multiple of 2048,
// plain store epilogue with bias / residual and the deferred RMSNorm);
// launch_matvec picks it first.
bool matvec_imma_supported(int fmt, int K);
cudaError_t launch_matvec_imma(int fmt, const MatvecParams& p, cudaStream_t stream, bool pdl);
// fp16 tensor-core path (Q4_0 / Q8_0, K a multiple of 2048) with the fused
// SwiGLU-pair and RMSNorm epilogues; picked when the integer path declines.
bool matvec_mma_supported(int fmt, int K);
cudaError_t launch_matvec_mma(int fmt, const MatvecParams& p, cudaStream_t stream, bool pdl);
// NF4 table path (K a multiple of 2048, group 64 or 128); picked second.
bool matvec_lut_supported(int fmt, int K, int group);
cudaError_t launch_matvec_lut(int fmt, const MatvecParams& p, cudaStream_t stream, bool pdl);
int matvec_lut_grid(int total_rows);   // CTAs (and norm partials) of a table-kernel launch
// GGUF K-quants (Q4_K / Q6_K, K a multiple of 256): one warp per row, plain
// store epilogue (+ bias / residual).
bool matvec_k_supported(int fmt, int K);
cudaError_t launch_matvec_k(int fmt, const MatvecParams& p, cudaStream_t stream, bool pdl);

cudaError_t launch_dequant(int fmt, float* dst, const uint8_t* src, const float* absmax, int64_t numel,
                           int group, cudaStream_t stream);

// GQA decode attention (split-K flash decoding).  kv_dtype: ALJ_KV_F32 / ALJ_KV_BF16.
struct AttnParams {
    float* out;              // [q_heads * head_dim]
    const float* q;          // [q_heads * head_dim]
    const void* k;           // cache rows [pos][stride]
    const void* v;
    int kv_dtype;
    int stride;              // elements between consecutive positions
    long long head_stride;   // elements between consecutive kv heads (head_dim for [pos][kvh][d])
    int kv_heads, q_heads, head_dim;
    int seq_len, start_pos;
    float scale;
    float* part_o;           // scratch [q_heads][splits][head_dim]
    float* part_ml;          // scratch [q_heads][splits][2]  (running max, running sum)
    int splits;
    const int* dev_pos;      // if set, seq_len = *dev_pos + 1 is read on the device (graph replay)
    TpLink tpl;              // tensor-parallel push of `out` (split merge; needs splits >= 2)
    unsigned int* split_counter;   // [kv_heads] arrival counters of the fused split merge: 0 before and after
};
int attention_splits(int seq_len, int kv_heads, int sm_count);
// Scratch of attention_scratch_floats() floats, zeroed once when allocated
// and then owned by one stream: attention_bind_scratch points part_o,
// part_ml and split_counter into it for p.q_heads / p.head_dim / p.splits.
size_t attention_scratch_floats(int q_heads, int head_dim, int splits);
void attention_bind_scratch(AttnParams& p, float* scratch);
cudaError_t launch_attention(const AttnParams& p, cudaStream_t stream, bool pdl);

// Batched NF4 GEMM on tcgen05 (gemm_nf4.cu): y_s[m * ldy_s + n] =
// sum_k x[m][k] * W_s[n][k] for up to 3 weight matrices sharing x (bf16).
struct GemmNf4Args {
    int nseg;
    float* y[3];
    int ldy[3];
    const void* packed[3];   // weights packed by launch_gemm_nf4_pack
    int rows[3];
    const void* x;           // bf16 [M][K]
    int M, K, group;
    void* workspace;
    size_t workspace_bytes;
};
bool gemm_nf4_supported(int M, int K, int group);
size_t gemm_nf4_packed_bytes(int rows, int K, int group);
cudaError_t launch_gemm_nf4_pack(void* packed, const void* codes, const void* absmax, int rows, int K, int group,
                                 cudaStream_t stream);
int gemm_nf4_tiles(int M, int nseg, const int* rows);
size_t gemm_nf4_workspace_bytes(int M, int K, int total_tiles, int grid);
cudaError_t launch_gemm_nf4(const GemmNf4Args& a, cudaStream_t stream);

// Batched GGUF Q4_0 / Q8_0 GEMM on tcgen05 (gemm_q.cu): y_s[m * ldy_s + n] =
// sum_k x[m * K + k] * W_s[n][k] for fp32 x, every segment one format, the
// weights packed by launch_gemm_q_pack.
struct GemmQArgs {
    int fmt;                 // FMT_Q4_0 or FMT_Q8_0
    int nseg;
    float* y[3];
    int ldy[3];
    const void* packed[3];
    int rows[3];
    const float* x;          // [M][K] fp32, 16-byte aligned
    int M, K;
    void* workspace;
    size_t workspace_bytes;
};
bool gemm_q_supported(int fmt, int M, int K);
size_t gemm_q_packed_bytes(int fmt, int rows, int K);
cudaError_t launch_gemm_q_pack(int fmt, void* packed, const void* w, int rows, int K, cudaStream_t stream);
int gemm_q_tiles(int M, int nseg, const int* rows);
size_t gemm_q_workspace_bytes(int M, int K);
cudaError_t launch_gemm_q(const GemmQArgs& a, cudaStream_t stream);

// Prefill attention (prefill_attention.cu): q / out [B][T][Hq][D], k / v
// [B][S][kv_stride floats per position] with KV head h at h * D; fp32, all
// 16-byte aligned.  Token t sees keys [max(0, hi - window + 1), hi] with
// hi = causal ? min(S - 1, t + causal_offset) : S - 1 (window 0: from 0).
struct PrefillArgs {
    float* out;
    const float* q;
    const float* k;
    const float* v;
    int B, T, S, Hq, Hkv, D, kv_stride;
    int causal, causal_offset, window;
    float scale, soft_cap;
};
bool prefill_attention_supported(int Hq, int Hkv, int D);
cudaError_t launch_prefill_attention(const PrefillArgs& a, cudaStream_t stream);

// Decode glue of the FFM binding (glue.cu): one-CTA RMSNorm and the
// elementwise SiLU-gated product.
cudaError_t launch_rmsnorm(float* out, const float* x, const float* w, int n, float eps, cudaStream_t stream);
// Copies n floats from mapped pinned host memory (its device address) into
// device memory with a small kernel that releases its programmatic
// dependent launch at once (glue.cu).
cudaError_t launch_host_pull(float* dst, const float* src_mapped, size_t n, int sms, cudaStream_t stream);
cudaError_t launch_silu_ffn(float* out, const float* gate, const float* up, int n, int sms, cudaStream_t stream);

int sm_count_for_current_device();

}  // namespace alj
