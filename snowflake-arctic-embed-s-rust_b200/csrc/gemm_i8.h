// Host interface of the tcgen05 int8 GEMM (gemm_i8.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace ae {

enum GemmEpilogue : int {
  EPI_F32 = 0,
  EPI_LN_QUANT = 1,
  EPI_GELU_QUANT = 2,
  EPI_LN_FINAL = 3,
};

struct GemmArgs {
  int M, N, K;
  const float* a_scale;     // [M]
  const float* w_scale;     // [N]
  const float* bias;        // [N]
  const float* res;         // [M, ldr] residual or nullptr
  int ldr;
  const float* gamma;       // [384] LayerNorm weight (LN epilogues)
  const float* beta;        // [384] LayerNorm bias
  const float* inv_smooth;  // [N] SmoothQuant inverse scale of the next GEMM's input (quant epilogues)
  float* out_f32;           // [M, ldo] fp32 output (F32 / LN epilogues)
  int ldo;
  int8_t* out_q;            // [M, N] int8 output (quant epilogues)
  float* out_scale;         // [M] row scale of out_q
  int32_t* acc_dbg;         // [M, N] raw int32 accumulators, or nullptr
  int* err;                 // device error word
  int gelu_erf;             // EPI_GELU_QUANT: 0 = the reference's rational GELU, 1 = exact erf
  int out_tt;               // out_f32 in the tile-transposed layout (ldo = its column count)
  int res_tt;               // res in the tile-transposed layout (ldr = its column count)
};

int gemm_i8_prime();
// Tensor map of a [rows, K] row-major int8 matrix with boxes of box_rows x 128 bytes: 128 for
// activations (A operands), 64 for weights (B operands, loaded in 64-row slices).
int make_tmap_i8(CUtensorMap* map, const void* base, int rows, int K, int box_rows);
constexpr int kBoxA = 128;
constexpr int kBoxB = 64;
int gemm_i8_launch(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t st);

// int8 tensor-pipe throughput probe: one CTA per SM issuing `iters` rounds of resident-operand
// tcgen05.mma kind::i8 (M = 128, N = 256, K = 128 per round); i8_peak_ops gives its int8 ops.
int i8_peak_launch(int iters, int* err, cudaStream_t st, int* ctas_out);
double i8_peak_ops(int iters, int ctas);

}  // namespace ae
