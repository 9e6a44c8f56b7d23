/*
 * aljabr_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference's arithmetic for the quantized decode
 * path (NF4 / GGUF Q4_0 / Q8_0 dequantise-and-matvec, GQA decode attention,
 * and the decode-step glue).  It is the checker for the CUDA path and the
 * timed CPU baseline; nothing in the product links, loads or calls it.
 *
 * Paths in citations are relative to the reference project root
 * (andalus-ai/aljabr).  Abbreviations used below:
 *   RT  = engine/gguf/aljabr-gguf-core/src/main/java/tech/kayys/aljabr/gguf/runtime
 *   VO  = engine/gguf/aljabr-gguf-core/src/main/java/tech/kayys/aljabr/gguf/loader/tensor/GGUFVectorOps.java
 *   GW  = engine/gguf/aljabr-gguf-core/src/main/java/tech/kayys/aljabr/gguf/writer/GGUFWriter.java
 *   DK  = engine/safetensor/aljabr-safetensor-core/src/main/java/tech/kayys/aljabr/safetensor/core/tensor/DequantizationKernel.java
 *   AT  = engine/gguf/aljabr-gguf-java/src/main/java/tech/kayys/aljabr/gguf/javabackend/GgufDecodeAttentionExecution.java
 *   DP  = engine/gguf/aljabr-gguf-java/src/main/java/tech/kayys/aljabr/gguf/javabackend/GgufDecodePass.java
 *   PA  = engine/gguf/aljabr-gguf-java/src/main/java/tech/kayys/aljabr/gguf/javabackend/GgufPrefillAttentionExecution.java
 *   FA  = backend/metal/aljabr-backend-metal/src/main/java/tech/kayys/aljabr/backend/metal/binding/MetalFlashAttentionCpuFallback.java
 *
 * Parity status: the GGUF and attention restatements are pinned by the
 * reference's own known-answer tests (restated as fixtures under
 * tests/golden/).  The NF4 fp32 GEMV half follows Apple Accelerate
 * cblas_sgemv, which is closed and macOS-only, and the NF4 quantizer lives
 * in an external project: both are "parity unpinned"; NF4 *dequantisation*
 * is pinned by its in-repo table and nibble order.
 */
#ifndef ALJABR_ORACLE_H
#define ALJABR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar conversions ------------------------------------------------ */
float    orc_f16_to_f32(uint16_t half);          /* RT/GgufQuantTables.java:143-165 */
uint16_t orc_f32_to_f16_bits(float value);       /* GW:360-387 (floatToHalfBits)   */
int      orc_java_round(float value);            /* java.lang.Math.round(float)     */
uint16_t orc_f32_to_bf16_rne(float value);       /* bf16 KV-cache store rounding    */

/* ---- encoders (fixture generators) ------------------------------------- */
void orc_encode_q4_0(const float* values, int64_t n, uint8_t* out);   /* GW:179-194 */
void orc_encode_q8_0(const float* values, int64_t n, uint8_t* out);   /* GW:163-177 */
/* Own NF4 quantizer (the reference's lives in an external project):
 * per-group fp32 absmax, nearest codebook entry, high nibble = even index. */
void orc_quantize_nf4(const float* values, int64_t n, int group_size,
                      uint8_t* codes, float* absmax);

/* ---- dequantisation (bit-exact targets) -------------------------------- */
void orc_dequantize_nf4(const uint8_t* src, float* dst, const float* scales,
                        int64_t numel, int group_size);               /* DK:84-102 */
void orc_dequantize_q4_0(const uint8_t* blocks, float* dst, int64_t numel); /* RT/GgufBlockDequantizer.java:33-37,366-415 */
void orc_dequantize_q8_0(const uint8_t* blocks, float* dst, int64_t numel); /* RT/GgufRowDequantizer.java:142-151 */

/* ---- row dots in the reference's summation order ------------------------ */
float orc_dot_row_q4_0(const uint8_t* row, int columns, const float* x);          /* RT/GgufQ32RawDot.java:34-67 */
/* Q4_0 in the prepared-cache order (the reference's default for >= 32 rows):
 * RT/GgufQ32Build.java:78-91, RT/GgufQuantUnpacker.java:365-367,414-448,
 * RT/GgufQ32Dot.java:627-670, RT/GgufDot.java:1046-1058. */
float orc_dot_row_q4_0_prepared(const uint8_t* row, int columns, const float* x);
float orc_dot_row_q8_0_scalar(const uint8_t* row, int columns, const float* x);   /* RT/GgufQ8RawDot.java:138-185 */
float orc_dot_row_q8_0_vector(const uint8_t* row, int columns, const float* x);   /* RT/GgufQ8RawDot.java:63-121 */
float orc_dot_row_q4_k(const uint8_t* row, int columns, const float* x);          /* RT/GgufQ4RawDot.java:38-141 */
float orc_dot_row_q6_k(const uint8_t* row, int columns, const float* x);          /* RT/GgufQ6RawDot.java:33-133,403-513 */
void  orc_dequantize_k_row(int type, const uint8_t* row, int columns, double* out); /* element formulas, fp64 */

/* ---- matvec (rows parallel over `threads` host threads, 2 chunks each) -- */
enum { ORC_Q4_0 = 2, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14, ORC_NF4 = 100, ORC_Q4_0_PREPARED = 1002 };
void orc_matvec_q4_0(const uint8_t* w, const float* x, float* y, int K, int N, int threads);
void orc_matvec_q4_0_prepared(const uint8_t* w, const float* x, float* y, int K, int N, int threads);
void orc_matvec_q8_0(const uint8_t* w, const float* x, float* y, int K, int N, int vector_order, int threads);
void orc_matvec_k(int type, const uint8_t* w, const float* x, float* y, int K, int N, int threads);   /* Q4_K / Q6_K */
/* NF4: dequantise (DK:84-102) then a plain fp32 row dot (stands in for the
 * closed cblas_sgemv at engine/safetensor/.../AccelOps.java:444-451). */
void orc_matvec_nf4(const uint8_t* codes, const float* absmax, const float* x, float* y,
                    int K, int N, int group_size, const float* bias, int threads);
/* fp64 ground truth on the dequantised weights (type = ORC_*). */
void orc_matvec_f64(int type, const void* w, const float* absmax, const float* x, double* y,
                    int K, int N, int group_size, int threads);

/* ---- decode attention --------------------------------------------------- */
/* AT:70-106 with VO:43-55 (dot), VO:302-317 (softmax), VO:165-174 (axpy).
 * K/V are fp32 [position][kvHeads*headDim] with `stride` floats/position. */
void orc_gqa_decode_attention(const float* q, float* out, float* scores,
                              const float* k_cache, const float* v_cache, int stride,
                              int kv_heads, int q_heads, int head_dim,
                              int seq_len, int start_pos, float scale);

/* ---- prefill attention --------------------------------------------------- */
/* PA:44-82: causal (or sliding-window) attention of `tokens` queries
 * [token][q_heads*head_dim] over the same tokens' keys / values
 * [position][kv_stride] (head h at (h / (q_heads/kv_heads)) * head_dim),
 * with VO:302-317 (softmax); sequential fp32 dots and axpys as written
 * there.  window > 0 limits token t to positions [t - window + 1, t]
 * (PA:48-51, slidingWindowAttention && slidingWindow > 0).  `scores` holds
 * `tokens` floats. */
void orc_prefill_attention(float* out, const float* q, const float* k, const float* v, float* scores, int tokens,
                           int q_heads, int kv_heads, int head_dim, float scale, int window, int kv_stride);
/* FA:46-104, the FlashAttention-4 seam's CPU contract: q / out [B][T][H][D],
 * k / v [B][S][H_kv][D]; causal masks s > max(0, S - T) + t; soft_cap > 0
 * applies tanh(score / cap) * cap.  `scores` holds S floats. */
void orc_fa4_attention(float* out, const float* q, const float* k, const float* v, float* scores, int B, int T,
                       int S, int H, int H_kv, int D, float scale, int causal, float soft_cap);

/* ---- decode-step glue --------------------------------------------------- */
float orc_vec_dot(const float* a, const float* b, int len);                      /* VO:43-55   */
void  orc_rms_norm(const float* x, const float* w, float* out, int len, float eps); /* VO:211-234 */
void  orc_rope(float* x, int n_heads, int head_dim, int rotary_dim, int pos, float freq_base); /* VO:383-440 */
void  orc_swiglu(const float* gate, const float* up, float* dst, int len);       /* VO:333-338 */
void  orc_softmax(float* a, int len);                                            /* VO:302-317 */
/* The FFM binding's own glue contract (backend/blackwell/aljabr-kernel-
 * blackwell/.../binding/BlackwellCpuFallback.java:50-64 and :70-79). */
void  orc_rmsnorm_binding(const float* x, const float* w, float* out, int n, float eps);
void  orc_silu_ffn_binding(const float* gate, const float* up, float* out, int n);

/* One batch-1 decode step of a Llama-shaped model with NF4 linear weights,
 * following DP:297-545 (pre-norm, q/k/v, split-half RoPE, KV store,
 * attention, o-proj + residual, SwiGLU FFN + residual) and the logits
 * projection.  The KV cache is [layer][max_ctx][kvH*D] of either fp32
 * (kv_bf16 = 0, the reference's cache) or bf16 bit patterns (kv_bf16 = 1:
 * the current token's k/v are rounded to bf16, RNE, when stored).
 *
 * Weight layout per layer l (NF4, group g, row-major [N][K]):
 *   wq [Hq*D][H], wk [Hkv*D][H], wv [Hkv*D][H], wo [H][Hq*D],
 *   wg [F][H], wu [F][H], wd [H][F]; embedding [V][H]; lm_head [V][H].
 * Codes/absmax of all tensors are passed as arrays of pointers in that
 * order: 7 per layer, then embedding, then lm_head. */
typedef struct {
    int layers, hidden, q_heads, kv_heads, head_dim, ffn, vocab, max_ctx, group;
    float eps, rope_theta;
} orc_llama_cfg;
void orc_decode_step_nf4(const orc_llama_cfg* cfg,
                         const uint8_t* const* codes, const float* const* absmax,
                         const float* norms,   /* [layers][2][H] (attn, ffn) then [H] output norm */
                         void* k_cache, void* v_cache, int kv_bf16,
                         int token, int pos, float* x_out, float* logits);
/* Host threads the two decode-step restatements use for their matvecs
 * (rows split among threads; results do not depend on the count). */
void orc_set_decode_threads(int threads);
/* One GGUF row (Q4_0 / Q8_0 / Q4_K / Q6_K) in the reference's dequantiser
 * float order (GgufBlockDequantizer, GgufKBlockDequantizer). */
void orc_dequantize_row_ref(int type, const uint8_t* row, int cols, float* out);

/* The same step with one GGUF type per tensor (types[7*layers + 2], ORC_*;
 * absmax entries only for ORC_NF4 tensors): RawDot row order per type, the
 * reference's dequantiser order for the embedding row. */
void orc_decode_step_typed(const orc_llama_cfg* cfg, const uint8_t* const* w, const int* types,
                           const float* const* absmax, const float* norms, void* k_cache, void* v_cache,
                           int kv_bf16, int token, int pos, float* x_out, float* logits);

#ifdef __cplusplus
}
#endif
#endif
