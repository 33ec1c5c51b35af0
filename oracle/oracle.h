/* CPU oracle for the arctic-embed-s int8 W8A8 forward pass: a C++ restatement of the reference
 * crate's x86_64 path (mdlockyer/snowflake-arctic-embed-s-rust, src/{quantize,gemm,simd_math,
 * model,lib}.rs). TEST INFRASTRUCTURE ONLY: the tests, the smoke check and the CPU-baseline leg of
 * the benchmark call it as the checker; the product path never links or calls it.
 *
 * Parity status: the reference crate (Rust) cannot be built in this environment and its golden
 * vectors are tied to model weights that are not available, so this restatement is "parity
 * unpinned" against the reference binary. It is checked instead against the reference's own
 * invariants (backend equivalence, ragged == single, pruned layer 11) and against an independent
 * float64 NumPy forward of the same synthetic model (tests/test_oracle.py).
 */
#ifndef ARCTIC_ORACLE_H
#define ARCTIC_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GEMM backends of the reference (src/gemm.rs:19-27), the x86_64 subset. */
enum { OR_BACKEND_AVX_VNNI = 5, OR_BACKEND_AVX2 = 6, OR_BACKEND_SCALAR = 7 };

typedef struct or_model or_model;

/* SimdBackend::detect (src/gemm.rs:100-125) on this host. */
int or_detect_backend(void);
/* 1 if the host has AVX2+FMA (selects the AVX2 simd_math kernels, as the reference does). */
int or_has_avx2_fma(void);

/* QuantizedModelRaw::load_ae8 (src/quantize.rs:76-137) + PackedModel::from_raw (src/model.rs:49-84).
 * Returns NULL on error; *err receives a message pointer (static storage). */
or_model* or_model_load(const char* path, int backend, const char** err);
or_model* or_model_load_mem(const uint8_t* buf, uint64_t len, int backend, const char** err);
void or_model_free(or_model* m);
int or_model_backend(const or_model* m);

/* PackedModel::forward_cls (src/model.rs:185-513). */
void or_forward_cls(const or_model* m, const uint16_t* ids, uint32_t len, float* out384);
/* PackedModel::forward_ragged_cls (src/model.rs:521-914): cu_seqlens[n+1] offsets into ids. */
void or_forward_ragged(const or_model* m, const uint16_t* ids, const uint32_t* cu, uint32_t n, float* out);
/* embed_batch (src/lib.rs:138-260) over pre-tokenised sequences, `threads` workers. */
void or_embed_batch(const or_model* m, const uint16_t* ids, const uint32_t* cu, uint32_t n, uint32_t threads,
                    float* out);

/* forward_cls with intermediate dumps (any pointer may be NULL), L = min(len, 512):
 *   gemm_in_q   [12][L][384]  int8 input of each layer's QKV (layer 11: of kv_only)
 *   gemm_in_s   [12][L]       its row scales
 *   qkv_out     [11][L][1152] fp32 QKV GEMM output of layers 0..10
 *   ctx         [11][L][384]  fp32 attention context of layers 0..10
 *   hidden      [11][L][384]  fp32 hidden state after LN2 of layers 0..10
 *   down_in_q   [11][L][1536] int8 input of each FFN-down
 *   down_in_s   [11][L]       its row scales */
void or_forward_trace(const or_model* m, const uint16_t* ids, uint32_t len, int8_t* gemm_in_q, float* gemm_in_s,
                      float* qkv_out, float* ctx, float* hidden, int8_t* down_in_q, float* down_in_s);

/* The embedding rows of one sequence of L = min(len, 512) ids: hidden [L][384] after the embedding
 * LayerNorm, q [L][384] / scale [L] its quantization with layers[0].qkv.inv_smooth
 * (src/simd_math.rs:1827-1881, src/model.rs:196-219). */
void or_embed_rows(const or_model* m, const uint16_t* ids, uint32_t len, float* hidden, int8_t* q, float* scale);

/* gemm_int8_fused (src/gemm.rs:630-671) with a row-major [N,K] weight packed for `backend`;
 * acc_out (nullable) receives the int32 accumulators. */
void or_gemm(int backend, uint32_t M, uint32_t K, uint32_t N, const int8_t* a_q, const float* a_scale,
             const int8_t* w, const float* w_scale, const float* bias, const float* res, float* out,
             int32_t* acc_out);

/* Row kernels (src/simd_math.rs), dispatched as the reference dispatches them on this host. */
float or_layernorm_smooth_quantize_row(float* x, const float* g, const float* b, const float* inv_s, int8_t* q,
                                       uint32_t n);
float or_smooth_quantize_row(const float* x, const float* inv_s, int8_t* q, uint32_t n);
float or_gelu_smooth_quantize_row(float* x, const float* inv_s, int8_t* q, uint32_t n);
void or_layernorm_inplace_row(float* x, const float* g, const float* b, uint32_t n);
void or_l2_normalize(float* x, uint32_t n);
/* One attention head for one query: compute_scores_head32 + softmax_inplace + weighted_sum_head32. */
void or_attention_query(const float* q32, const float* k_head, const float* v_head, uint32_t seq_len,
                        float* out32);
/* Attention of layers 0-10: the reference's x86 fp32 kernels (OR_ATTENTION_EXACT, the default), or
 * its int8 scheme (attention_heads_sme, src/simd_math.rs:1933-2186) for every sequence of at least
 * 16 tokens (OR_ATTENTION_INT8; shorter ones and the layer-11 [CLS] row stay fp32, as in
 * src/model.rs:245 and :427-450), with scales over each sequence's own keys. Returns -1 for an
 * unknown mode. */
enum { OR_ATTENTION_EXACT = 0, OR_ATTENTION_INT8 = 1 };
int or_model_set_attention_mode(or_model* m, int mode);
/* The int8 scheme on one sequence: qkv [L][1152] row-major (Q | K | V) -> ctx [L][384]. */
void or_attention_i8(const float* qkv, uint32_t L, float* ctx);
/* The AVX2 GELU approximation of the reference (avx2_gelu_f32), elementwise. */
void or_gelu_ref(const float* x, float* y, uint32_t n);

#ifdef __cplusplus
}
#endif
#endif
