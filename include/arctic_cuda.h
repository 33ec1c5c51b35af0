/* arctic_cuda.h — C ABI of the B200 (sm_100a) backend for the arctic-embed-s int8 W8A8 encoder.
 *
 * This is the boundary a host crate binds through FFI in place of the reference crate's CPU
 * kernels (mdlockyer/snowflake-arctic-embed-s-rust). Plain pointers and sizes only. Every function
 * returns 0 on success or a negative AE_ERR_* code; ae_last_error() gives the message of the last
 * failure on a context. No exception, abort or panic crosses this boundary.
 *
 * Threading: one ae_ctx drives one GPU. A context is NOT thread-safe (it owns its workspace,
 * like the reference's `&mut Workspace`); different contexts may be driven from different host
 * threads at the same time. ae_embed_batch_multi drives several contexts itself.
 *
 * Units: a "sequence" is a list of token ids ([CLS] ... [SEP] as produced by the WordPiece
 * tokenizer); sequences longer than 512 are truncated to their first 512 ids, as the reference
 * does (src/model.rs:191, src/tokenizer.rs:98-101). Outputs are L2-normalised 384-d [CLS]
 * embeddings, row-major float32.
 */
#ifndef ARCTIC_CUDA_H
#define ARCTIC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AE_HIDDEN 384
#define AE_MAX_POSITIONS 512

enum {
  AE_OK = 0,
  AE_ERR_INVALID_ARG = -1,  /* null pointer, bad size, empty sequence */
  AE_ERR_CUDA = -2,         /* CUDA runtime error (message has the CUDA error string) */
  AE_ERR_NO_MODEL = -3,     /* forward called before ae_model_load */
  AE_ERR_BAD_PACK = -4,     /* malformed .ae8 pack or model descriptor */
  AE_ERR_TOKEN_RANGE = -5,  /* token id >= 30522 (the reference panics on a slice index) */
  AE_ERR_DEVICE = -6,       /* a kernel reported an error (bounded wait ran out, bad shape) */
  AE_ERR_CAPACITY = -7,     /* request larger than the reserved workspace */
};

typedef struct ae_ctx ae_ctx;

/* One int8 linear layer: QuantizedLinearRaw (src/quantize.rs:22-30) /
 * PackedLinearInt8::from_raw_row_major (src/gemm.rs:186-246). Host pointers; copied to the GPU by
 * ae_model_load. n_out == 0 means "pruned": only inv_smooth is kept (src/gemm.rs:195-205). */
typedef struct {
  uint64_t n_out;
  uint64_t k_in;
  const int8_t* w_q;        /* [n_out * k_in] row-major (out_features x in_features) */
  const float* w_scale;     /* [n_out] */
  const float* bias;        /* [n_out] */
  const float* inv_smooth;  /* [k_in] */
} ae_linear_desc;

/* QuantizedLayerRaw (src/quantize.rs:46-58). */
typedef struct {
  ae_linear_desc qkv;
  int32_t has_split;        /* 1 on layer 11: q_only / kv_only are valid */
  ae_linear_desc q_only;
  ae_linear_desc kv_only;
  ae_linear_desc attn_out;
  const float* ln1_weight;
  const float* ln1_bias;
  ae_linear_desc ffn_inter;
  ae_linear_desc ffn_out;
  const float* ln2_weight;
  const float* ln2_bias;
} ae_layer_desc;

/* QuantizedModelRaw (src/quantize.rs:60-72): what QuantizedModelRaw::load_ae8 produces. */
typedef struct {
  const int8_t* word_emb_q;   const float* word_emb_scale;  /* [30522*384], [30522] */
  const int8_t* pos_emb_q;    const float* pos_emb_scale;   /* [512*384],   [512]   */
  const int8_t* type_emb_q;   const float* type_emb_scale;  /* [2*384],     [2]     */
  const float* emb_ln_weight; const float* emb_ln_bias;     /* [384] */
  ae_layer_desc layers[12];
} ae_model_desc;

/* Context on CUDA device `device` (its own stream and device error word).
 * Replaces: nothing in the reference (the CPU crate has no device); pairs with Workspace::new
 * (src/model.rs:146-173) for the memory it owns. */
int ae_ctx_create(int device, ae_ctx** out);
int ae_ctx_destroy(ae_ctx* ctx);
/* Message of the last failure on ctx (or of the last ae_ctx_create failure when ctx is NULL). */
const char* ae_last_error(const ae_ctx* ctx);
/* Stream the context launches on (a cudaStream_t); NULL selects the context's own stream, a
 * blocking stream (ordered with work on the legacy default stream). */
int ae_ctx_set_stream(ae_ctx* ctx, void* cuda_stream);
int ae_ctx_device(const ae_ctx* ctx);

/* Uploads the model. Replaces PackedModel::from_raw (src/model.rs:49-84), which repacks the
 * weights for a CPU SIMD backend; here the row-major int8 weights are already the K-major
 * tcgen05 operand layout and are copied as they are. Validates every size. */
int ae_model_load(ae_ctx* ctx, const ae_model_desc* desc);
/* Convenience: QuantizedModelRaw::load_ae8 (src/quantize.rs:76-137) + ae_model_load. */
int ae_model_load_file(ae_ctx* ctx, const char* path);

/* Reserves the device workspace for batches of up to max_tokens packed rows and max_seqs
 * sequences (Workspace::new, src/model.rs:146-173, sized for a token budget instead of 512).
 * Called implicitly (growing) by the forward functions. */
int ae_reserve(ae_ctx* ctx, uint32_t max_tokens, uint32_t max_seqs);

/* PackedModel::forward_cls (src/model.rs:185-513) / ArcticEmbedS::embed_tokens (src/lib.rs:96-102):
 * one sequence -> out[384]. Host buffers. Latency mode: replays a CUDA graph per length. */
int ae_forward_cls(ae_ctx* ctx, const uint16_t* ids, uint32_t len, float* out384);

/* PackedModel::forward_ragged_cls (src/model.rs:521-914) without its 64-sequence / 512-row limits:
 * n_seqs sequences packed back to back in ids, sequence i = ids[cu_seqlens[i] .. cu_seqlens[i+1]),
 * each truncated to 512 ids on its own. out: [n_seqs * 384]. Host buffers (copied in/out inside). */
int ae_forward_ragged(ae_ctx* ctx, const uint16_t* ids, const uint32_t* cu_seqlens, uint32_t n_seqs, float* out);

/* Same as ae_forward_ragged with every buffer already in device memory of ctx's GPU and every
 * sequence already 1..512 ids long (a kernel checks and reports AE_ERR_DEVICE otherwise);
 * max_len bounds the longest sequence. Asynchronous on the context's stream; no host sync. */
int ae_forward_ragged_device(ae_ctx* ctx, const uint16_t* d_ids, const uint32_t* d_cu_seqlens, uint32_t n_seqs,
                             uint32_t total_tokens, uint32_t max_len, float* d_out);

/* ArcticEmbedS::embed_batch (src/lib.rs:138-260) over pre-tokenised sequences, sharded across
 * n_ctx contexts (GPUs) by token-weighted greedy assignment, one host thread per context; results
 * in input order. `max_batch_tokens` (0 = 65536) bounds the rows of one device batch. */
int ae_embed_batch_multi(ae_ctx* const* ctxs, int n_ctx, const uint16_t* ids, const uint32_t* cu_seqlens,
                         uint32_t n_seqs, uint32_t max_batch_tokens, float* out);

/* The sharding plan ae_embed_batch_multi uses (host only, no GPU needed): shard_of[i] in
 * [0, n_shards) for every sequence, token-weighted greedy (longest first) over the cost
 * 19,759,104 L + 8,448 L^2 MACs of an L-token sequence. Replaces the work-stealing counter of
 * embed_batch (src/lib.rs:163-167), which balances threads dynamically on one CPU. */
int ae_plan_shards(const uint32_t* cu_seqlens, uint32_t n_seqs, int n_shards, int32_t* shard_of);

/* gemm_int8_fused (src/gemm.rs:630-671) on device buffers, for tests and the kernel microbench:
 *   epi 0: out = fma(float(A W^T), a_scale * w_scale, bias (+ res))              [M, N] f32
 *   epi 1: epi 0 with res, then LayerNorm(gamma, beta) -> out (the new residual) and the
 *          SmoothQuant row quantization with inv_smooth -> out_q [M, 384], out_scale [M]  (N = 384)
 *   epi 2: GELU(epi 0) * inv_smooth, row-quantized -> out_q [M, 1536], out_scale [M]    (N = 1536)
 *   epi 3: epi 0 with res, then layernorm_inplace_row + l2_normalize_inplace -> out     (N = 384)
 * A [M, K] int8, W [N, K] int8 row-major; K a multiple of 128. acc (nullable) receives the raw
 * int32 accumulators [M, N]. Every pointer must be 16-byte aligned (AE_ERR_INVALID_ARG otherwise).
 * Epilogues 1 and 3 run fused into the GEMM from 74 row tiles of 128 (M >= 9,345); below, as a
 * GEMM into a context-owned scratch buffer (grown on demand) followed by a row kernel, with the
 * same results. out may alias res, and out_q / out_scale may alias A / a_scale. */
int ae_gemm_i8(ae_ctx* ctx, int epi, uint32_t M, uint32_t N, uint32_t K, const int8_t* d_a, const float* d_a_scale,
               const int8_t* d_w, const float* d_w_scale, const float* d_bias, const float* d_res,
               const float* d_gamma, const float* d_beta, const float* d_inv_smooth, float* d_out, int8_t* d_out_q,
               float* d_out_scale, int32_t* d_acc);

/* The attention of one layer (src/model.rs:294-321 per segment) on device buffers:
 * qkv [total, 1152] f32 (Q | K | V, head h at columns 32h..32h+31 of each third) -> ctx [total, 384]. */
int ae_attention_f32(ae_ctx* ctx, const float* d_qkv, const uint32_t* d_cu_seqlens, uint32_t n_seqs,
                     uint32_t max_len, float* d_ctx);

/* Attention of layers 0-10 (no counterpart in the reference's API: the crate picks its attention by
 * SIMD backend, src/model.rs:245 and :608):
 *   AE_ATTENTION_EXACT (default): fp32 in the operation order of the reference's x86 kernels.
 *   AE_ATTENTION_INT8: the reference's int8 scheme of its SME backend (attention_heads_sme,
 *     src/simd_math.rs:1933-2186: per-token int8 Q / K, per-column int8 V, 14-bit integer exp2
 *     probabilities, int32 products) for every sequence of at least 16 tokens, with scales taken
 *     over each sequence's own keys (what forward_cls computes for it alone); shorter sequences and
 *     the layer-11 [CLS] row stay fp32, as in the reference. Results differ from the fp32 mode by
 *     about 4e-5 in cosine.
 * The environment variable ARCTIC_ATTN=int8 selects the int8 scheme for new contexts.
 * Changing the mode drops the context's captured single-sequence graphs. */
enum { AE_ATTENTION_EXACT = 0, AE_ATTENTION_INT8 = 1 };
int ae_set_attention_mode(ae_ctx* ctx, int mode);
int ae_get_attention_mode(const ae_ctx* ctx);

/* The int8 scheme on device buffers, every sequence (any length 1..512), same layout as
 * ae_attention_f32. */
int ae_attention_i8(ae_ctx* ctx, const float* d_qkv, const uint32_t* d_cu_seqlens, uint32_t n_seqs,
                    uint32_t max_len, float* d_ctx);

/* Allocation-free variant of the single-sequence forward, for callers that cannot call cudaMalloc
 * when they embed: hosts that hand out device memory once at start-up from their own pool (a
 * service with a fixed memory budget), and latency paths that must not block on the allocator
 * (cudaMalloc / cudaFree can synchronise the device). No counterpart in the reference (the CPU
 * crate gets the same effect from a reusable Workspace).
 * d_ids: 1..512 token ids in device memory of ctx's GPU (longer inputs are rejected with
 * AE_ERR_CAPACITY: truncate to the first 512 first); d_out384: device float[384]. Asynchronous on
 * the context's stream. The model must already be loaded (ae_model_load allocates; this call
 * does not). Scratch: a file-scope 8 MiB device array in the library, which every GPU that loads
 * the library holds until the process exits. The first call on a device (and the first call after
 * a device reset, which moves the array) looks up that array's device address
 * (cudaGetSymbolAddress) and builds its tensor maps; make that first call before any stream
 * capture. Every call shares the one array, which keeps the last call's contents: nothing in it
 * has to start at zero, because every row a kernel's result depends on is written by this call
 * first (the GEMMs load whole 128-row tiles, so rows past len still hold an earlier call's data;
 * rows are independent and those rows' results are never stored). Calls that overlap on the GPU,
 * from any context on the same device, race on the array. Per-kernel profiling (ae_profile) does
 * not record this call. */
int ae_forward_cls_noalloc(ae_ctx* ctx, const uint16_t* d_ids, uint32_t len, float* d_out384);

/* Test hook (no counterpart in the reference's API; it exposes what the reference computes inside
 * forward_ragged_cls, src/model.rs:521-914): runs the forward pass of a packed batch of host
 * sequences, as ae_forward_ragged does, up to `stage` and copies rows of the device workspace back,
 * in the caller's order (T = the sum of the sequences' lengths, each truncated to 512):
 *   AE_TRACE_EMBED: f32 [T, 384] = the hidden state after the embedding LayerNorm; q [T, 384] and
 *     scale [T] = its quantization for layer 0's QKV GEMM (dequant_add_embeddings_row,
 *     src/simd_math.rs:1827-1881, + layernorm_smooth_quantize_row, src/model.rs:196-219);
 *   AE_TRACE_ATTN0: f32 = layer 0's attention context; q / scale = its SmoothQuant row quantization
 *     with attn_out.inv_smooth (smooth_quantize_row, src/simd_math.rs:584-649), the attention-out
 *     GEMM's input, from whichever kernel the forward pass used for it (a separate kernel, or the
 *     attention kernel itself for short single sequences). */
enum { AE_TRACE_EMBED = 0, AE_TRACE_ATTN0 = 1 };
int ae_trace_forward(ae_ctx* ctx, const uint16_t* ids, const uint32_t* cu_seqlens, uint32_t n_seqs, int stage,
                     float* f32, int8_t* q, float* scale);

/* Per-kernel timing of the forward pass (CUDA events around every launch on the context's stream).
 * Kinds, in the order of the forward pass: */
enum {
  AE_KERNEL_ROW_META = 0,   /* positions and [CLS] rows of a packed batch */
  AE_KERNEL_EMBED = 1,      /* embedding + LayerNorm + quantization */
  AE_KERNEL_QKV = 2,        /* QKV GEMM (layers 0-10), KV GEMM (layer 11) */
  AE_KERNEL_ATTENTION = 3,  /* attention of all rows (layers 0-10) */
  AE_KERNEL_CTX_QUANT = 4,  /* attention-context quantization */
  AE_KERNEL_ATTN_OUT = 5,   /* attention-out GEMM + residual + LayerNorm + quantization */
  AE_KERNEL_FFN_UP = 6,     /* FFN-up GEMM + GELU + quantization */
  AE_KERNEL_FFN_DOWN = 7,   /* FFN-down GEMM + residual + LayerNorm + quantization */
  AE_KERNEL_CLS = 8,        /* layer-11 [CLS] tail: gather, Q GEMM, attention, quantization, GEMMs */
  AE_KERNEL_KINDS = 9
};
/* enable != 0 starts recording (and clears earlier records); 0 stops. */
int ae_profile(ae_ctx* ctx, int enable);
/* After ae_sync: total milliseconds and launch counts per kind over everything recorded. */
int ae_profile_read(ae_ctx* ctx, float* total_ms, uint32_t* launches);

/* Number of this library's kernels the context has launched so far (graph replays included). */
uint64_t ae_kernel_launches(const ae_ctx* ctx);

/* Waits for the context's stream; reports a device-side error (AE_ERR_DEVICE) if one was raised. */
int ae_sync(ae_ctx* ctx);

/* Measured int8 tensor-core throughput of this GPU (no counterpart in the reference; the roofline
 * denominator of the GEMMs): one CTA per SM issues `iters` (1..1,000,000) rounds of tcgen05.mma
 * kind::i8 (M = 128, N = 256, K = 128 per round) on operands resident in shared memory, after one
 * shorter warm-up launch. *ms = CUDA-event time of the timed launch, *tops = its int8 ops / time
 * in 10^12 ops/s. */
int ae_measure_int8_peak(ae_ctx* ctx, uint32_t iters, float* ms, double* tops);

/* Self-test of failure detection (no reference counterpart): launches a kernel whose bounded wait
 * on an mbarrier can never complete, with a limit of limit_us microseconds (1..1,000,000) instead
 * of the kernels' 2 s. Returns AE_ERR_DEVICE ("epilogue wait timed out"); the context stays usable.
 * No GPU fault or hang is involved. */
int ae_selftest_wait_timeout(ae_ctx* ctx, uint32_t limit_us);

/* ---------------------------------------------------------------------------------------------
 * WordPiece tokenizer (host only, no GPU needed): BertTokenizer, src/tokenizer.rs:25-327.
 * Text is UTF-8 (AE_ERR_INVALID_ARG on invalid UTF-8, which a Rust &str cannot hold). Outputs are
 * [CLS] (+ the query prefix) + WordPiece ids + [SEP], truncated to 512 ids as encode_into does
 * (src/tokenizer.rs:90-101). A tokenizer is immutable after creation and may be shared by threads.
 * ------------------------------------------------------------------------------------------- */
typedef struct ae_tokenizer ae_tokenizer;

#define AE_QUERY_PREFIX "Represent this sentence for searching relevant passages: "

/* BertTokenizer::from_vocab_file / from_vocab_str (src/tokenizer.rs:35-68): one token per line,
 * id = line index (at most 65,536 lines). */
int ae_tokenizer_create_from_file(const char* vocab_path, ae_tokenizer** out);
int ae_tokenizer_create_from_vocab(const char* vocab_text, size_t len, ae_tokenizer** out);
int ae_tokenizer_destroy(ae_tokenizer* tok);
/* BertTokenizer::vocab_size (src/tokenizer.rs:70-73). */
uint32_t ae_tokenizer_vocab_size(const ae_tokenizer* tok);
/* Message of the last failure of ae_tokenizer_create_* on this thread. */
const char* ae_tokenizer_last_error(void);

/* encode (is_query = 0) / encode_query (is_query = 1), src/tokenizer.rs:74-101. Writes n <= 512
 * ids to ids[0..n) and *n_ids = n; AE_ERR_CAPACITY if cap < n. */
int ae_tokenize(const ae_tokenizer* tok, const char* text, size_t len, int is_query, uint16_t* ids,
                uint32_t cap, uint32_t* n_ids);

/* The tokenization step of ArcticEmbedS::embed_batch (src/lib.rs:138-160) over n texts on
 * host threads: packed ids (ids_cap >= total) and cu_seqlens [n + 1], ready for
 * ae_forward_ragged / ae_embed_batch_multi. texts[i] has lens[i] bytes. */
int ae_tokenize_batch(const ae_tokenizer* tok, const char* const* texts, const size_t* lens, uint32_t n,
                      int is_query, uint16_t* ids, size_t ids_cap, uint32_t* cu_seqlens);

#ifdef __cplusplus
}
#endif
#endif /* ARCTIC_CUDA_H */
