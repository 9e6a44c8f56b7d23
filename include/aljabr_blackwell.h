/*
 * aljabr_blackwell.h -- C-ABI of libaljabr_blackwell.so, the B200 (sm_100a)
 * provider for Aljabr's quantized decode path.
 *
 * This is the native library that the reference's Blackwell FFM binding
 * loads (backend/blackwell/aljabr-kernel-blackwell/src/main/java/tech/kayys/
 * aljabr/blackwell/binding/BlackwellBinding.java:52-78 names the library
 * and its `aljabr_blackwell_*` symbols; the source it expects under
 * src/main/cpp/blackwell does not exist in the reference).  The matvec and
 * model-buffer entry points keep the shapes of the Metal provider's C API
 * (backend/metal/aljabr-backend-metal/src/main/cpp/metal/
 * aljabr_metal_matvec_api.h), so GgufExecutionDispatcher's bridge can call
 * either provider the same way.
 *
 * Conventions
 *  - Every entry point returns int: 0 on success, a negative ALJ_ERR_* code
 *    otherwise (the Metal API's 0 / negative convention), with a message in
 *    aljabr_blackwell_last_error() for the calling thread.  Nothing falls
 *    back to the CPU: an unsupported type or shape is an error.
 *  - "tb" (host-buffer) entry points take host float buffers for the
 *    activation A and the result C, exactly like aljabr_metal_matvec_tb_*.
 *    The weight pointer B is a host address inside a buffer previously given
 *    to aljabr_blackwell_register_model_buffer (the mmap'd GGUF file), which
 *    the library copied to HBM once; a device pointer is accepted as well.
 *    They block until C is written.  A call whose matrices, sizes and
 *    types were seen before is replayed as one cached CUDA graph (captured
 *    on the second such call; at most 256 shapes per device, dropped when
 *    their weights are unregistered); a call made while a prefetch hint is
 *    pending runs its launches directly.
 *  - "_dev" entry points take device pointers for everything and are
 *    stream-ordered (stream = cudaStream_t, NULL = the library's stream for
 *    the current device); they do not synchronize.
 *  - Weight layouts: Q4_0 and Q8_0 are ggml blocks (GgmlType ids 2 and 8,
 *    18 and 34 bytes per 32 values; element j of a Q4_0 block is the low
 *    nibble of code byte j, element j+16 the high nibble).  NF4 is the
 *    safetensors/bitsandbytes layout of DequantizationKernel.java:84-102:
 *    two codes per byte, high nibble first, one fp32 absmax per
 *    `block_size` consecutive elements of the flattened [N][K] tensor.
 *  - Threads: calls are thread-safe; each thread uses the device made
 *    current by aljabr_blackwell_init (default 0).
 */
#ifndef ALJABR_BLACKWELL_H
#define ALJABR_BLACKWELL_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (negative; mirrors the Metal provider's convention) ---- */
#define ALJ_OK                  0
#define ALJ_ERR_NOT_INITIALIZED (-1)
#define ALJ_ERR_BAD_DIMS        (-2)
#define ALJ_ERR_UNSUPPORTED     (-3)   /* no kernel for this type / shape     */
#define ALJ_ERR_NOT_REGISTERED  (-4)   /* B is neither registered nor device  */
#define ALJ_ERR_CUDA            (-5)
#define ALJ_ERR_TIMEOUT         (-6)   /* a device-side bounded wait gave up  */
#define ALJ_ERR_BAD_ARG         (-7)   /* null pointer, bad alignment, range  */
#define ALJ_ERR_NO_MEMORY       (-8)

/* ---- weight type ids (GgmlType.java ids; NF4 has no ggml id) ------------ */
#define ALJ_TYPE_Q4_0 2
#define ALJ_TYPE_Q8_0 8
#define ALJ_TYPE_NF4  100
/* GGUF K-quants, 256-value super-blocks (GgmlType ids; block sizes in
 * engine/gguf/aljabr-gguf-core/.../runtime/GgufQuantFormats.java:51-53):
 * Q4_K 144 B (GgufQ4RawDot.dotRowQ4K, GgufQ4RawDot.java:38-141), Q6_K 210 B
 * (GgufQ6RawDot.dotRowQ6K, GgufQ6RawDot.java:33-133).  Accepted by the typed
 * matvec entry points (aljabr_blackwell_matvec_dev, _tb_pair, _tb_triple) and
 * by aljabr_blackwell_matvec_tb_q4_k / _q6_k; K a multiple of 256. */
#define ALJ_TYPE_Q4_K 12
#define ALJ_TYPE_Q6_K 14

/* ---- KV-cache element types --------------------------------------------- */
#define ALJ_KV_F32  0   /* the reference's fp32 cache (KVCache.java:22-23)  */
#define ALJ_KV_BF16 1   /* bf16 cache (half the bytes)                      */

/* ---- lifecycle (BlackwellBinding.java:52-78 names) ----------------------- */
/* Select `device_id` for the calling thread and create its state.  Replaces
 * the binding's FN_INIT ("aljabr_blackwell_init"). */
int aljabr_blackwell_init(int device_id);
/* Number of CUDA devices (FN_DEVICE_COUNT). */
int aljabr_blackwell_device_count(void);
/* Select `device_id` for the calling thread's later calls, like
 * aljabr_blackwell_init (FN_DEVICE_GET, BlackwellBinding.java:153-157,
 * bound at :465-466 as (JAVA_INT) -> JAVA_INT).  Returns 0 or an error. */
int aljabr_blackwell_device_get(int device_id);
/* Device name into buf, NUL-terminated and truncated to buf_len bytes
 * (FN_DEVICE_NAME; argument order as bound at BlackwellBinding.java:469-470:
 * (ADDRESS buf, JAVA_INT bufSz, JAVA_INT deviceId)).  Returns 0 or an error. */
int aljabr_blackwell_device_name(char* buf, int buf_len, int device_id);
/* major*10+minor, e.g. 100 for B200 (FN_COMPUTE_CAP). */
int aljabr_blackwell_compute_capability(int device_id);
/* Tensor memory of the device in bytes (FN_TMEM_SIZE,
 * BlackwellBinding.java:185-189, bound at :477-478): 128 lanes x 512
 * columns x 4 bytes = 256 KiB per SM, times the SM count (37,879,808 on a
 * 148-SM B200).  Negative error code on a device without TMEM (not sm_100). */
long long aljabr_blackwell_tmem_size(int device_id);
/* Free device memory in bytes for the current device (FN_FREE_MEM). */
long long aljabr_blackwell_free_memory(void);
/* Message for the last failing call on this thread ("" if none). */
const char* aljabr_blackwell_last_error(void);
/* Verbose diagnostics to stderr (aljabr_metal_set_verbose). */
void aljabr_blackwell_set_verbose(int enable);
/* Read and clear the device fault word (bit 0: a bounded wait timed out). */
int aljabr_blackwell_device_status(unsigned int* fault_bits);
/* Release every buffer and stream the library holds on every device. */
int aljabr_blackwell_shutdown(void);
/* Programmatic dependent launch for the stream-ordered (_dev) calls of this
 * thread (default off).  When on, a matvec may begin streaming its weights
 * while the previous kernel on the same stream is still running; it still
 * waits for that kernel before reading x or writing y.  Only enable it when
 * weight buffers are not written by the kernel immediately preceding a call
 * (true for weights loaded once, as in a decode loop). */
int aljabr_blackwell_set_pdl(int enable);

/* Scheduling hint, no counterpart in the reference: the next matvec launched
 * from this thread (any entry point) prefetches, once its own weight copies
 * are issued, the weights the launch after it will read -- [next_weights,
 * next_weights + bytes), device or registered memory -- into L2, each CTA its
 * share, so that launch starts on L2 hits while this one drains.  One-shot:
 * the hint is consumed by that launch.  Pass NULL to clear. */
int aljabr_blackwell_prefetch_hint(const void* next_weights, size_t bytes);

/* ---- model buffers (aljabr_metal_buffers.h:15) ---------------------------- */
/* Copy [base, base+bytes) to HBM once; later calls may pass host pointers
 * inside this range as weight pointers.  Re-registering the same base is a
 * no-op. */
int aljabr_blackwell_register_model_buffer(const void* base_ptr, size_t total_bytes);
int aljabr_blackwell_unregister_model_buffer(const void* base_ptr);
/* Device address that a registered host address maps to (NULL if none). */
void* aljabr_blackwell_device_address(const void* host_ptr);

/* ---- host-buffer matvec, y = W x (aljabr_metal_matvec_api.h:56-95) -------- */
/* Replaces GgufTensorOps.matVecParallel for Q4_0 (GgufQ32RawDot.dotRowQ4_0,
 * engine/gguf/aljabr-gguf-core/.../runtime/GgufQ32RawDot.java:34-67).
 * C: float[N] (host), A: float[K] (host), B: N rows of K/32 Q4_0 blocks. */
int aljabr_blackwell_matvec_tb_q4_0(void* C, const void* A, const void* B, int K, int N);
/* Q8_0 (GgufQ8RawDot.dotRowQ8_0, .../runtime/GgufQ8RawDot.java:40-50);
 * same shape as aljabr_metal_matvec_tb_q8_0. */
int aljabr_blackwell_matvec_tb_q8_0(void* C, const void* A, const void* B, int K, int N);
/* Q4_K / Q6_K (GgufRawDot.q4K / q6K, .../runtime/GgufRawDot.java:79-149);
 * same shapes as aljabr_metal_matvec_tb_q4_k / _q6_k
 * (backend/metal/.../cpp/metal/aljabr_metal_matvec_api.h:48-53).
 * B: N rows of K/256 super-blocks (144 / 210 bytes); K a multiple of 256. */
int aljabr_blackwell_matvec_tb_q4_k(void* C, const void* A, const void* B, int K, int N);
int aljabr_blackwell_matvec_tb_q6_k(void* C, const void* A, const void* B, int K, int N);
/* NF4: AccelOps.linear's dequantise-then-sgemv for M == 1
 * (engine/safetensor/.../tensor/AccelOps.java:392-451); same shape as
 * aljabr_metal_matvec_tb_nf4.  absmax: float[N*K/blockSize]. */
int aljabr_blackwell_matvec_tb_nf4(void* C, const void* A, const void* B_packed, const void* absmax,
                                   int K, int N, int blockSize);
/* NF4 with an optional bias (AccelOps.java:465-467); bias may be NULL. */
int aljabr_blackwell_linear_nf4(void* C, const void* A, const void* B_packed, const void* absmax,
                                const void* bias, int K, int N, int blockSize);
/* Two / three projections of one input (GgufExecutionDispatcher
 * dispatchMatVecPair / dispatchMatVecTriple, GgufExecutionDispatcher.java:37-55;
 * aljabr_metal_matvec_tb_pair / _triple).  typeN: ALJ_TYPE_Q4_0 / Q8_0. */
int aljabr_blackwell_matvec_tb_pair(void* C0, void* C1, const void* A, const void* B0, const void* B1,
                                    int K, int N0, int N1, int type0, int type1);
int aljabr_blackwell_matvec_tb_triple(void* C0, void* C1, void* C2, const void* A, const void* B0,
                                      const void* B1, const void* B2, int K, int N0, int N1, int N2,
                                      int type0, int type1, int type2);
/* batchSize inputs A[b][K] -> C[b][N] (dispatchMatVecBatch,
 * GgufExecutionDispatcher.java:57-72; aljabr_metal_matvec_tb_batch). */
int aljabr_blackwell_matvec_tb_batch(void* C, const void* A, const void* B, int K, int N, int type,
                                     int batchSize);
/* batchSize inputs A[b][K] against three matrices: Cs[b][Ns]
 * (dispatchMatVecTripleBatch, GgufExecutionDispatcher.java:74-98;
 * aljabr_metal_matvec_tb_triple_batch).  For Q4_0 / Q8_0 with batchSize >= 2
 * and K a multiple of 256 both batch entry points run the tcgen05 GEMM
 * (weights packed on first use and cached until their model buffer is
 * unregistered); other types and shapes run one matvec per input row. */
int aljabr_blackwell_matvec_tb_triple_batch(void* C0, void* C1, void* C2, const void* A, const void* B0,
                                            const void* B1, const void* B2, int K, int N0, int N1, int N2,
                                            int type0, int type1, int type2, int batchSize);

/* ---- host-buffer dequantisation (bit-exact with the reference) ----------- */
/* DequantizationKernel.dequantizeNf4(src, dst, scales, numel, groupSize),
 * .../tensor/DequantizationKernel.java:84-102.  dst: float[numel] host. */
int aljabr_blackwell_dequantize_nf4(void* dst, const void* src, const void* scales, long long numel,
                                    int groupSize);
/* GgufBlockDequantizer.dequantizeQ4_0Block over numel/32 blocks
 * (.../runtime/GgufBlockDequantizer.java:33-37). */
int aljabr_blackwell_dequantize_q4_0(void* dst, const void* blocks, long long numel);
/* Q8_0 rows (.../runtime/GgufRowDequantizer.java:142-151). */
int aljabr_blackwell_dequantize_q8_0(void* dst, const void* blocks, long long numel);

/* ---- decode glue bound by the FFM class (BlackwellBinding.java:574-583) ---
 * Both take float buffers that are device memory, registered memory, or
 * plain host memory (staged through the library's buffers), may alias
 * elementwise (out == x, out == gate == up as BlackwellRunner.java:586
 * calls it), and block until `out` is written.
 *
 * aljabr_blackwell_rmsnorm: out[i] = (x[i] / rms) * weight[i] with
 * rms = sqrt(sum(x^2) / N + eps), the arithmetic of the binding's own
 * contract (BlackwellCpuFallback.rmsNorm, BlackwellCpuFallback.java:50-64);
 * fp32 throughout, IEEE division and square root; the sum of squares is a
 * fixed-order tree, not the Java loop's sequential order.  1 <= N <= 2^24. */
int aljabr_blackwell_rmsnorm(float* out, const float* x, const float* weight, int N, float eps);
/* aljabr_blackwell_silu_ffn: out[i] = gate[i] / (1 + exp(-gate[i])) * up[i]
 * (BlackwellCpuFallback.siluFfn, BlackwellCpuFallback.java:70-79); exp is
 * the CUDA single-precision expf, within 2 ulp of the Java double exp. */
int aljabr_blackwell_silu_ffn(float* out, const float* gate, const float* up, int N);

/* ---- GQA decode attention ------------------------------------------------ */
/* GgufDecodeAttentionExecution.execute(query, output, scores, keyCache,
 * valueCache, cacheHeadStride, kvHeads, queryHeads, headDimension,
 * sequenceLength, startPosition, scale)
 * (engine/gguf/aljabr-gguf-java/.../javabackend/GgufDecodeAttentionExecution.java:70-106).
 * out, q: host float[q_heads*head_dim]; k_cache, v_cache: device or
 * registered memory, rows of `cache_head_stride` elements per position of
 * type kv_dtype.  Attends positions [start_pos, seq_len). */
int aljabr_blackwell_decode_attention(float* out, const float* q, const void* k_cache, const void* v_cache,
                                      int kv_dtype, int cache_head_stride, int kv_heads, int q_heads,
                                      int head_dim, int seq_len, int start_pos, float scale);

/* ---- prefill attention (fp32, GQA) ----------------------------------------
 * GgufPrefillAttentionExecution.execute's Java loop
 * (engine/gguf/aljabr-gguf-java/.../javabackend/GgufPrefillAttentionExecution.java:44-82):
 * out, q: host float[tokens][q_heads*head_dim]; k, v: host
 * float[tokens][kv_stride] with KV head h at h*head_dim.  Token t attends
 * positions [t - sliding_window + 1, t] (sliding_window > 0) or [0, t]. */
int aljabr_blackwell_prefill_attention(float* out, const float* q, const float* k, const float* v, int tokens,
                                       int q_heads, int kv_heads, int head_dim, float scale, int sliding_window,
                                       int kv_stride);
/* The FlashAttention-4 seam (aljabr_metal_fa4_attention, backend/metal/
 * aljabr-backend-metal/.../binding/MetalFlashAttentionBinding.java:221-285;
 * CPU contract MetalFlashAttentionCpuFallback.java:46-104): output, query:
 * host float[B][T][H][D]; key, value: host float[B][S][H_kv][D].  Causal
 * masks keys s > max(0, S - T) + t; soft_cap > 0 applies tanh(x/cap)*cap.
 * use_bf16 is accepted and ignored: the arithmetic is fp32.  head_dim D a
 * multiple of 32 up to 256, H a multiple of H_kv with H / H_kv <= 64.
 * Returns 0 on success. */
int aljabr_blackwell_fa4_attention(void* output, void* query, void* key, void* value, int B, int T, int S, int H,
                                   int H_kv, int D, float scale, int is_causal, int use_bf16, float soft_cap);
/* aljabr_metal_fa4_sdpa_available / _bf16_available: 1 / 0 here. */
int aljabr_blackwell_fa4_sdpa_available(void);
int aljabr_blackwell_fa4_bf16_available(void);
/* Device pointers, stream-ordered: q / out [B][T][q_heads*head_dim], k / v
 * [B][S][kv_stride] (kv_stride a multiple of 4), all 16-byte aligned; the
 * causal limit of token t is t + max(0, S - T); window 0 = none. */
int aljabr_blackwell_prefill_attention_dev(float* out, const float* q, const float* k, const float* v, int B, int T,
                                           int S, int q_heads, int kv_heads, int head_dim, int kv_stride, float scale,
                                           int causal, int window, float soft_cap, void* stream);

/* ---- device-pointer, stream-ordered variants ----------------------------- */
/* y[N] = W x (+ bias); type ALJ_TYPE_*; absmax/group only for NF4. */
int aljabr_blackwell_matvec_dev(int type, float* y, const float* x, const void* w, const float* absmax,
                                int K, int N, int group, const float* bias, void* stream);
int aljabr_blackwell_dequantize_dev(int type, float* dst, const void* src, const float* absmax,
                                    long long numel, int group, void* stream);
/* Decode attention on device pointers.  Its split partials live in one
 * scratch buffer per device that the library allocates on first use and
 * reuses.  The split merge's arrival counters sit at the head of that
 * buffer; every merge returns its counter to zero, and a call clears them on
 * `stream` before its kernel when they may not be zero (a new buffer, more
 * query heads than the previous call, or a fault reported by
 * aljabr_blackwell_device_status).  Calls whose kernels may overlap on the
 * GPU (different streams, or several threads) share that buffer and must be
 * ordered by the caller (an event or one stream). */
int aljabr_blackwell_decode_attention_dev(float* out, const float* q, const void* k_cache,
                                          const void* v_cache, int kv_dtype, int cache_head_stride,
                                          int kv_heads, int q_heads, int head_dim, int seq_len,
                                          int start_pos, float scale, void* stream);

/* ---- batched NF4 linear on the tensor cores (prefill / batched decode) ----
 * AccelOps.linear for M > 1 (engine/safetensor/aljabr-safetensor-core/.../
 * tensor/AccelOps.java:453-456: cblas_sgemm(RowMajor, NoTrans, Trans, M, N,
 * K, 1, X, K, W, K, 0, Y, N) on the dequantised weight), bf16 activations:
 *     y_s[m * ldy_s + n] = sum_k X[m][k] * W_s[n][k]        (fp32 out)
 * for nseg (1..3) weight matrices W_s sharing X (q/k/v, gate/up).
 *
 * The weights are packed once per matrix (at registration, like the
 * reference's prepared Q4_0 cache, GgufQ32Build): gemm_nf4_pack reads codes
 * (device NF4 [rows][K/2], two codes per byte, high nibble first; 16-byte
 * aligned) and absmax (device fp32 [rows][K/blockSize]) and writes `packed`
 * (device, 256-byte aligned, gemm_nf4_packed_size bytes): each 128-row x
 * 256-column block of codes and each 128-row x 16-group block of absmax is
 * contiguous.  K a multiple of 256; blockSize 64 or 128.
 *
 * gemm_nf4_dev: x_bf16 device bf16 [M][K] (16-byte aligned); workspace
 * device memory, 256-byte aligned, at least gemm_nf4_workspace_size bytes,
 * used by one call at a time (no reference counterpart: the reference's
 * sgemm runs on the host).  Stream-ordered on `stream` (NULL = the
 * library's stream). */
long long aljabr_blackwell_gemm_nf4_packed_size(int rows, int K, int blockSize);
int aljabr_blackwell_gemm_nf4_pack(void* packed, const void* codes, const void* absmax, int rows, int K,
                                   int blockSize, void* stream);
long long aljabr_blackwell_gemm_nf4_workspace_size(int M, int K, int nseg, const int* rows);
int aljabr_blackwell_gemm_nf4_dev(int nseg, float* const* y, const int* ldy, const void* const* packed,
                                  const int* rows, const void* x_bf16, int M, int K, int blockSize,
                                  void* workspace, long long workspace_bytes, void* stream);

/* ---- batched GGUF Q4_0 / Q8_0 GEMM on tcgen05 (prefill projections) -------
 * dispatchMatVecBatch / dispatchMatVecTripleBatch for batchSize >= 2
 * (engine/gguf/aljabr-gguf-java/.../javabackend/GgufExecutionDispatcher.java:
 * 57-98; the Metal seam's aljabr_metal_matvec_tb_batch / _tb_triple_batch,
 * backend/metal/.../cpp/metal/aljabr_metal_matvec_api.h:93-106), fp32
 * activations:
 *     y_s[m * ldy_s + n] = sum_k X[m][k] * W_s[n][k]        (fp32 out)
 * for nseg (1..3) matrices W_s of one type sharing X (q/k/v, gate/up).
 *
 * gemm_q_pack reads `weights` (device GGUF blocks of `type`, ALJ_TYPE_Q4_0
 * or ALJ_TYPE_Q8_0, [rows][K/32]) and writes `packed` (device, 256-byte
 * aligned, gemm_q_packed_size bytes): a header with the matrix's scale
 * exponent, then per 128-row x 256-column block the codes and the block
 * scales contiguous.  K a multiple of 256, at most 32768.
 *
 * gemm_q_dev: x device fp32 [M][K] (16-byte aligned); workspace device
 * memory, 256-byte aligned, at least gemm_q_workspace_size bytes, used by one
 * call at a time.  Stream-ordered on `stream` (NULL = the library's stream).
 * Block scales that are Inf or NaN make the whole matrix's outputs NaN here;
 * the host-buffer batch entry points route such matrices to the per-row
 * matvec instead. */
long long aljabr_blackwell_gemm_q_packed_size(int type, int rows, int K);
int aljabr_blackwell_gemm_q_pack(int type, void* packed, const void* weights, int rows, int K, void* stream);
long long aljabr_blackwell_gemm_q_workspace_size(int M, int K);
int aljabr_blackwell_gemm_q_dev(int type, int nseg, float* const* y, const int* ldy, const void* const* packed,
                                const int* rows, const float* x, int M, int K, void* workspace,
                                long long workspace_bytes, void* stream);

/* Same computation as aljabr_blackwell_decode_attention_dev, for callers that
 * may not allocate device memory at call time.  No counterpart in the
 * reference: its attention runs on the host and needs no device scratch.
 * The split partials live in a static device array of 1,048,576 floats
 * (4 MiB) compiled into the library; shapes whose scratch,
 * q_heads * splits * (head_dim + 2) floats plus one counter word per query
 * head (rounded up to 4), exceeds it are rejected with ALJ_ERR_BAD_DIMS.  Calls no cudaMalloc / cudaFree and needs no prior
 * aljabr_blackwell_init: it runs on the current device and on `stream`
 * (NULL = the legacy default stream).  The first call on a device looks up
 * the array's device address (cudaGetSymbolAddress) with that device
 * current; make it before any stream capture.  A device reset may move the
 * array: call aljabr_blackwell_shutdown after one, so the next call looks
 * the address up again.  All calls share the array,
 * so calls whose kernels may overlap (other streams, other threads) race
 * and must be ordered by the caller.  The split merge's arrival counters
 * must start at zero; each call clears them on `stream` before its kernel. */
int aljabr_blackwell_decode_attention_noalloc(float* out, const float* q, const void* k_cache,
                                              const void* v_cache, int kv_dtype, int cache_head_stride,
                                              int kv_heads, int q_heads, int head_dim, int seq_len,
                                              int start_pos, float scale, void* stream);

/* ---- full decode step (Llama-shaped, NF4 or GGUF weights, one CUDA graph/token) ---
 * The device-resident form of GgufDecodePass.forward's layer loop
 * (engine/gguf/aljabr-gguf-java/.../GgufDecodePass.java:297-545), shaped like
 * the Metal provider's registered decode step (aljabr_metal_matvec_api.h:
 * aljabr_metal_init_kv_cache / register_decode_layer / register_output /
 * register_token_embd / decode_step_token), but handle-based so several
 * models can coexist.
 *
 * dims = {layers, hidden, q_heads, kv_heads, head_dim, ffn, vocab, max_ctx,
 *         nf4_group, kv_dtype}.  With tp_world > 1 every weight passed in is
 * this rank's contiguous row block ([rows/tp_world] of each matrix; the
 * q/k/v row blocks are whole heads), the KV cache holds this rank's heads,
 * and nccl_id is the 128-byte id from aljabr_blackwell_nccl_unique_id,
 * shared by all ranks; one call per rank, each with its own current device. */
int aljabr_blackwell_nccl_unique_id(void* out, int out_len);
int aljabr_blackwell_decode_model_create(const int* dims, float eps, float rope_theta, int tp_world, int tp_rank,
                                         const void* nccl_id, unsigned long long* handle);
/* codes[7] / absmax[7]: q, k, v, o, gate, up, down (device or registered
 * memory, referenced, not copied); norms are host or device float[hidden]. */
int aljabr_blackwell_register_decode_layer(unsigned long long handle, int layer, const void* const* codes,
                                           const void* const* absmax, const float* attn_norm, const float* ffn_norm);
/* Token embedding [vocab][hidden] (full on every rank) and lm_head rows. */
int aljabr_blackwell_register_output(unsigned long long handle, const void* embd_codes, const void* embd_absmax,
                                     const void* head_codes, const void* head_absmax, const float* output_norm);
/* The same two registrations with one GGUF type per tensor, as the Metal
 * provider's aljabr_metal_register_decode_layer (typeQ .. typeDown) and
 * aljabr_metal_register_output / register_token_embd (typeOutputW,
 * typeEmbdW) take them (aljabr_metal_matvec_api.h:244-268).
 * types[7] / embd_type / head_type: ALJ_TYPE_Q4_0, _Q8_0, _Q4_K, _Q6_K or
 * _NF4; weights are row-major ggml blocks (NF4: packed codes); absmax may be
 * NULL, its entries are read only for NF4 tensors.  Any GGUF-typed tensor
 * makes the step run its residual adds, RMSNorms and SwiGLU as separate
 * small launches; it needs tp_world 1 (ALJ_ERR_UNSUPPORTED otherwise). */
int aljabr_blackwell_register_decode_layer_typed(unsigned long long handle, int layer, const void* const* weights,
                                                 const int* types, const void* const* absmax, const float* attn_norm,
                                                 const float* ffn_norm);
int aljabr_blackwell_register_output_typed(unsigned long long handle, const void* embd, int embd_type,
                                           const void* embd_absmax, const void* head, int head_type,
                                           const void* head_absmax, const float* output_norm);
/* One token at position `pos` (its K/V are written at pos; attention covers
 * [0, pos]).  logits_out: host float[vocab] or NULL; argmax_out: host int or
 * NULL (greedy next token). */
int aljabr_blackwell_decode_step_token(unsigned long long handle, int token, int pos, float* logits_out,
                                       int* argmax_out);
/* n_tokens greedy steps entirely on the device: the argmax of each step is
 * the next step's token, positions pos .. pos+n_tokens-1; the emitted tokens
 * go to tokens_out (host int[n_tokens], may be NULL).  One synchronisation
 * at the end. */
int aljabr_blackwell_decode_run(unsigned long long handle, int token, int pos, int n_tokens, int* tokens_out);
/* Load positions [0, seq_len) of one layer's K and V cache (prompt prefill
 * or a restored session; aljabr_metal_sync_kv_cache).  k, v: host or device
 * memory holding seq_len x (kv_heads/tp * head_dim) elements of kv_dtype. */
int aljabr_blackwell_sync_kv_cache(unsigned long long handle, int layer, int seq_len, const void* k, const void* v);
/* Copy the residual stream x (float[hidden]) and this rank's KV caches
 * ([layers][max_ctx][kv_heads/tp*head_dim] of kv_dtype) to host memory;
 * any pointer may be NULL. */
int aljabr_blackwell_decode_read_state(unsigned long long handle, float* x_out, void* k_cache_out, void* v_cache_out);
int aljabr_blackwell_decode_model_destroy(unsigned long long handle);

#ifdef __cplusplus
}
#endif

#endif /* ALJABR_BLACKWELL_H */
