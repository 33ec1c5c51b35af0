// Launch interfaces of the row, metadata and attention kernels (rowops.cu, attention.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace ae {

struct EmbedArgs {
  int T;                      // rows
  const uint16_t* ids;        // [T] token ids
  const uint16_t* pos;        // [T] position of each row inside its sequence
  const int8_t* word_q;       // [30522, 384]
  const float* word_s;        // [30522]
  const int8_t* pos_q;        // [512, 384]
  const float* pos_s;         // [512]
  const float* type0;         // [384] dequantized token_type_embeddings[0]
  const float* gamma;         // embedding LayerNorm
  const float* beta;
  const float* inv_smooth;    // layers[0].qkv.inv_smooth
  float* hidden;              // [T, 384] out, tile-transposed
  int8_t* act_q;              // [T, 384] out
  float* act_s;               // [T] out
  int* err;
};

struct AttnArgs {
  // Q: tile-transposed [rows, q_C] when q_tt, else row-major with row stride q_C; head h of the
  // query at columns q_col + 32h ... + 31.
  const float* q;
  int q_C, q_col, q_tt;
  // K and V: columns k_col + 32h and v_col + 32h of kv ([rows, kv_C], tile-transposed when kv_tt,
  // else row-major with row stride kv_C); rows of sequence s are cu[s] .. cu[s+1]-1.
  const float* kv;
  int kv_C, k_col, v_col, kv_tt;
  float* out;                 // context rows, row-major [rows, 384] (row of the query)
  const uint32_t* cu;         // [n_seqs + 1] row offsets of the sequences
  int max_len;                // upper bound of any sequence length (<= 512)
  int cls_mode;               // 1: one query per sequence, at row s of q / out
  int* err;
  // optional: where a launch that can quantize the context rows itself (the SmoothQuant row
  // quantization of the next GEMM's input) writes them; see launch_attention_exact
  const float* quant_inv_s;   // [384] inverse smoothing factors, or nullptr
  int8_t* quant_q;            // [rows, 384]
  float* quant_scale;         // [rows]
  int skip_from;              // > 0: the exact kernels leave sequences of at least this many keys alone
  int few_mode;               // few long sequences: 0 the faster kernel, 1 the TMEM kernels, 2 32-query
                              // tiles, 3 eight lanes per query, 4 32-query tiles with dim-major K / V
                              // (all the same results; for tests)
};

// Launch with programmatic stream serialization (the kernel calls pdl_wait before it touches data
// that earlier kernels produced).
template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, static_cast<Args&&>(args)...);
}

int launch_embed(const EmbedArgs& a, cudaStream_t st);
int launch_wait_selftest(int* err, uint64_t limit_ns, cudaStream_t st);
int launch_ln_quant_rows(const float* h_in, int M, const float* gamma, const float* beta, const float* inv_s,
                         float* hidden, int hidden_tt, int8_t* q, float* scale, cudaStream_t st);
int launch_ln_final_rows(const float* h_in, int M, const float* gamma, const float* beta, float* out,
                         cudaStream_t st);
int launch_smooth_quant(const float* x, const float* inv_s, int8_t* q, float* scale, int rows, cudaStream_t st);
int launch_row_meta(const uint32_t* cu, int n_seqs, uint16_t* pos, int32_t* cls_row, int* err, cudaStream_t st);
int launch_gather_cls(const int32_t* cls_row, int n, const int8_t* act_q, const float* act_s, const float* hidden,
                      int8_t* cq, float* cs, float* ch, cudaStream_t st);
int attention_prime();
// A run of consecutive packed sequences [first, first + count) whose lengths are at most max_len
// and fall in one attention length class.
struct AttnSegment {
  int first;
  int count;
  int max_len;
  int min_len;
};
// Length classes of the attention launch: 1-32, 33-64, 65-128, 129-256, 257-512 keys (the TMEM
// columns a CTA allocates for its scores).
constexpr int kAttnClasses = 5;
inline int attn_class(int len) { return len <= 32 ? 0 : len <= 64 ? 1 : len <= 128 ? 2 : len <= 256 ? 3 : 4; }
// quantized (optional): set to 1 when the launch also wrote the quantized context rows
// (a.quant_*; the single-sequence path for at most 64 keys), else 0 (the caller quantizes).
int launch_attention_exact(const AttnArgs& a, int n_seqs, cudaStream_t st, int* quantized = nullptr);
// The reference's int8 attention scheme (no cls_mode) for the sequences of at least min_len keys;
// the context rows of shorter ones are left as they are.
int launch_attention_i8(const AttnArgs& a, int n_seqs, int min_len, cudaStream_t st);

// QKV projection fused with the attention (sequences of at most 128 keys): the int8 GEMM
// fma(float(acc), a_scale[row] * w_scale[n], bias[n]) of one sequence's 128-row tile against the
// Q, K and V weight rows of two heads (tcgen05 kind::i8, the same arithmetic as the QKV GEMM's plain
// epilogue), dequantized straight into shared memory, then k_attention_rows2's attention. The
// projection never goes to global memory.
struct QkvAttnArgs {
  AttnArgs a;               // out, cu, max_len (<= 128), err; the q / kv fields are unused
  const float* a_scale;     // [rows] row scales of the int8 activations
  const float* w_scale;     // [1152] per-output-channel scales of the QKV weights
  const float* bias;        // [1152]
};
// tm_act: the [rows, 384] int8 activations (128-row boxes); tm_w: the [1152, 384] int8 QKV weights
// (64-row boxes).
int launch_qkv_attention(const CUtensorMap& tm_act, const CUtensorMap& tm_w, const QkvAttnArgs& a, int n_seqs,
                         cudaStream_t st);

}  // namespace ae
