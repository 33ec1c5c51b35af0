// Row kernels of the forward pass: token embedding + LayerNorm + SmoothQuant quantization, the
// attention-context quantization, per-row metadata of a packed (ragged) batch and the gather of
// the [CLS] rows for the pruned last layer.
//
// LayerNorm and quantization reproduce the reference's AVX2 row kernels bit for bit: 16 lanes
// hold the 16 partial sums (element j goes to lane j % 16, as the two 8-wide AVX2 accumulators
// do), combined with the hsum256 tree; every product and sum rounds as in the reference.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"
#include "rowmath.cuh"

namespace ae {

// Combines the 16 per-lane partial sums held by the 16 lanes of a half-warp exactly as
// hsum256_ps(sum0 + sum1) does; the result is returned on all 16 lanes.
__device__ __forceinline__ float halfwarp_tree16(float p, unsigned mask) {
  // v[l] = p[l] + p[8 + l]            (lanes 0..7)
  float v = p + __shfl_down_sync(mask, p, 8, 16);
  // t[l] = v[l] + v[l + 4]            (lanes 0..3)
  float t = v + __shfl_down_sync(mask, v, 4, 16);
  // u0 = t0 + t1, u2 = t2 + t3        (lanes 0, 2)
  float u = t + __shfl_down_sync(mask, t, 1, 16);
  // (t0 + t1) + (t2 + t3)             (lane 0)
  float r = u + __shfl_down_sync(mask, u, 2, 16);
  return __shfl_sync(mask, r, 0, 16);
}

__device__ __forceinline__ float halfwarp_max(float v, unsigned mask) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(mask, v, o, 16));
  return v;
}

// One half-warp per token row, 16 rows per block: dequant_add_embeddings_row
// (src/simd_math.rs:1827-1881, generic path) + layernorm_smooth_quantize_row (src/simd_math.rs:369-477)
// with the embedding LayerNorm and layers[0].qkv.inv_smooth (src/model.rs:196-219). The hidden
// rows go through a shared-memory tile so that the tile-transposed store of a column covers the
// block's 16 consecutive rows (64 contiguous bytes).
__global__ void __launch_bounds__(256) k_embed_ln_quant(EmbedArgs a) {
  pdl_trigger();
  // model constants, staged before the dependency wait
  __shared__ float s_type0[kHidden], s_gamma[kHidden], s_beta[kHidden], s_invs[kHidden];
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    s_type0[i] = a.type0[i];
    s_gamma[i] = a.gamma[i];
    s_beta[i] = a.beta[i];
    s_invs[i] = a.inv_smooth[i];
  }
  __syncthreads();
  pdl_wait();
  __shared__ float tile[kHidden][17];
  const int r0 = blockIdx.x * 16;
  const int lr = threadIdx.x >> 4;  // row within the block
  const int row = r0 + lr;
  const int l = threadIdx.x & 15;
  const unsigned mask = 0xffffffffu;  // both half-warps stay converged (inactive rows compute row T-1)
  const bool active = row < a.T;
  const int hw = active ? row : a.T - 1;
  int tok = a.ids[hw];
  const int pos = min(int(a.pos[hw]), kMaxPos - 1);
  if (tok >= kVocab) {
    if (l == 0) record_err(a.err, DEV_ERR_BAD_TOKEN);
    tok = 0;
  }
  const int8_t* wq = a.word_q + size_t(tok) * kHidden;
  const int8_t* pq = a.pos_q + size_t(pos) * kHidden;
  const float ws = a.word_s[tok], ps = a.pos_s[pos];
  float h[24];
  float p = 0.0f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const int j = l + 16 * i;
    h[i] = (float(wq[j]) * ws + float(pq[j]) * ps) + s_type0[j];
    p = p + h[i];
  }
  const float mean = halfwarp_tree16(p, mask) / float(kHidden);
  p = 0.0f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const float d = h[i] - mean;
    p = fmaf(d, d, p);
  }
  const float var = halfwarp_tree16(p, mask) / float(kHidden);
  const float rstd = 1.0f / sqrtf(var + kLnEps);
  float vmax = 1e-8f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const int j = l + 16 * i;
    h[i] = fmaf((h[i] - mean) * rstd, s_gamma[j], s_beta[j]);
    tile[j][lr] = h[i];
    vmax = fmaxf(vmax, fabsf(h[i] * s_invs[j]));
  }
  const float max_abs = halfwarp_max(vmax, mask);
  const float inv_scale = 127.0f / max_abs;
  int8_t* qrow = a.act_q + size_t(hw) * kHidden;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const int j = l + 16 * i;
    const int8_t qv = int8_t(quant_i8(h[i] * (s_invs[j] * inv_scale)));
    if (active) qrow[j] = qv;
  }
  if (active && l == 0) a.act_s[hw] = max_abs / 127.0f;
  __syncthreads();
  // tile-transposed store: thread -> (column, row), rows fastest
  for (int i = threadIdx.x; i < kHidden * 16; i += blockDim.x) {
    const int j = i >> 4, rr = i & 15;
    if (r0 + rr < a.T) a.hidden[tt_index(r0 + rr, j, kHidden)] = tile[j][rr];
  }
}

// One half-warp per row: layernorm_smooth_quantize_row_avx2 (src/simd_math.rs:369-477) on rows of
// h = fma(acc, a_scale * w_scale, bias + residual) that a GEMM with the plain epilogue wrote
// (row-major [M, 384]); the LayerNorm output goes to hidden (tile-transposed when hidden_tt, else
// row-major), the quantized row to q / scale. Used when a batch has too few row tiles for the fused
// LayerNorm epilogue to fill the GPU.
__global__ void __launch_bounds__(256) k_ln_quant_rows(const float* __restrict__ h_in, int M,
                                                       const float* __restrict__ gamma,
                                                       const float* __restrict__ beta,
                                                       const float* __restrict__ inv_s, float* __restrict__ hidden,
                                                       int hidden_tt, int8_t* __restrict__ q,
                                                       float* __restrict__ scale) {
  pdl_trigger();
  // the LayerNorm and SmoothQuant vectors are model constants: staged before the dependency wait
  __shared__ float s_gamma[kHidden], s_beta[kHidden], s_invs[kHidden];
  // the block's 16 output rows, staged so that the stores are contiguous: hidden as [column][row]
  // (a tile-transposed column of the 16 rows is 64 contiguous bytes), int8 rows as [row][column]
  __shared__ float tile[kHidden][17];
  __shared__ __align__(16) int8_t qtile[16][kHidden];
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    s_gamma[i] = gamma[i];
    s_beta[i] = beta[i];
    s_invs[i] = inv_s[i];
  }
  __syncthreads();
  pdl_wait();
  const int r0 = blockIdx.x * 16;
  const int lr = threadIdx.x >> 4;  // row within the block
  const int row = r0 + lr;
  const int l = threadIdx.x & 15;
  const unsigned mask = 0xffffffffu;
  const bool active = row < M;
  const int hw = active ? row : M - 1;
  const float* x = h_in + size_t(hw) * kHidden;
  float h[24];
  float p = 0.0f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    h[i] = x[l + 16 * i];
    p = p + h[i];
  }
  const float mean = halfwarp_tree16(p, mask) / float(kHidden);
  p = 0.0f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const float d = h[i] - mean;
    p = fmaf(d, d, p);
  }
  const float var = halfwarp_tree16(p, mask) / float(kHidden);
  const float rstd = 1.0f / sqrtf(var + kLnEps);
  float vmax = 1e-8f;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const int j = l + 16 * i;
    h[i] = fmaf((h[i] - mean) * rstd, s_gamma[j], s_beta[j]);
    tile[j][lr] = h[i];
    vmax = fmaxf(vmax, fabsf(h[i] * s_invs[j]));
  }
  const float max_abs = halfwarp_max(vmax, mask);
  const float inv_scale = 127.0f / max_abs;
#pragma unroll
  for (int i = 0; i < 24; ++i) {
    const int j = l + 16 * i;
    qtile[lr][j] = int8_t(quant_i8(h[i] * (s_invs[j] * inv_scale)));
  }
  if (active && l == 0) scale[hw] = max_abs / 127.0f;
  __syncthreads();
  const int rows = M - r0 < 16 ? M - r0 : 16;
  if (hidden_tt) {
    for (int i = threadIdx.x; i < kHidden * 16; i += blockDim.x) {  // rows fastest
      const int j = i >> 4, rr = i & 15;
      if (rr < rows) hidden[tt_index(r0 + rr, j, kHidden)] = tile[j][rr];
    }
  } else {
    for (int i = threadIdx.x; i < kHidden * 16; i += blockDim.x) {  // columns fastest
      const int rr = i / kHidden, j = i - rr * kHidden;
      if (rr < rows) hidden[size_t(r0 + rr) * kHidden + j] = tile[j][rr];
    }
  }
  for (int i = threadIdx.x; i < 16 * (kHidden / 16); i += blockDim.x) {  // 16-byte pieces of the int8 rows
    const int rr = i / (kHidden / 16), c = i - rr * (kHidden / 16);
    if (rr < rows)
      *reinterpret_cast<uint4*>(q + size_t(r0 + rr) * kHidden + 16 * c) =
          *reinterpret_cast<const uint4*>(&qtile[rr][16 * c]);
  }
}

// layernorm_inplace_row + l2_normalize_inplace (src/simd_math.rs:481-497, :2892-2903) on rows of
// h (row-major [M, 384]). Their sums are sequential over the 384 elements, so one thread owns a
// row; a block stages 16 rows in shared memory with coalesced loads (rows padded to 385 floats, so
// the 16 owners read 16 different banks) and writes the results back the same way.
constexpr int kLnFinalRows = 16;
constexpr int kLnFinalPitch = kHidden + 1;

__global__ void __launch_bounds__(128) k_ln_final_rows(const float* __restrict__ h_in, int M,
                                                       const float* __restrict__ gamma,
                                                       const float* __restrict__ beta, float* __restrict__ out) {
  pdl_trigger();
  __shared__ float s_gamma[kHidden], s_beta[kHidden];  // model constants, staged before the wait
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
    s_gamma[i] = gamma[i];
    s_beta[i] = beta[i];
  }
  pdl_wait();
  extern __shared__ float xs[];  // [kLnFinalRows][kLnFinalPitch]
  const int r0 = blockIdx.x * kLnFinalRows;
  const int rows = M - r0 < kLnFinalRows ? M - r0 : kLnFinalRows;
  for (int i = threadIdx.x; i < rows * kHidden; i += blockDim.x) {
    const int r = i / kHidden, j = i - r * kHidden;
    xs[r * kLnFinalPitch + j] = h_in[size_t(r0 + r) * kHidden + j];
  }
  __syncthreads();
  const int r = threadIdx.x;
  if (r < rows) {
    float* x = xs + r * kLnFinalPitch;
    float sum = 0.0f;
    for (int j = 0; j < kHidden; ++j) sum = sum + x[j];
    const float mean = sum / float(kHidden);
    float var = 0.0f;
    for (int j = 0; j < kHidden; ++j) {
      const float d = x[j] - mean;
      var = var + d * d;
    }
    const float rstd = 1.0f / sqrtf(var / float(kHidden) + kLnEps);
    float ss = 0.0f;
    for (int j = 0; j < kHidden; ++j) {
      const float y = (x[j] - mean) * rstd * s_gamma[j] + s_beta[j];
      x[j] = y;
      ss = ss + y * y;
    }
    if (ss > 0.0f) {
      const float inv = 1.0f / sqrtf(ss);
      for (int j = 0; j < kHidden; ++j) x[j] = x[j] * inv;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows * kHidden; i += blockDim.x) {
    const int rr = i / kHidden, j = i - rr * kHidden;
    out[size_t(r0 + rr) * kHidden + j] = xs[rr * kLnFinalPitch + j];
  }
}

// One warp per row: smooth_quantize_row_avx2 (src/simd_math.rs:584-649), the quantization of the
// attention context with attn_out.inv_smooth (src/model.rs:324-328).
// Grid-stride over the rows: a block's warps keep the lane's 12 inverse smoothing factors in
// registers (loaded once, before the dependency wait) and take rows two at a time, the loads of
// both rows in flight together.
__global__ void __launch_bounds__(256) k_smooth_quant(const float* __restrict__ x, const float* __restrict__ inv_s,
                                                      int8_t* __restrict__ q, float* __restrict__ scale, int rows) {
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  float s[12];  // element 4 (lane + 32 i) + e of the row
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const float4 t = reinterpret_cast<const float4*>(inv_s)[lane + 32 * i];
    s[4 * i] = t.x;
    s[4 * i + 1] = t.y;
    s[4 * i + 2] = t.z;
    s[4 * i + 3] = t.w;
  }
  pdl_wait();
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += 2 * nwarps) {
    const int rr[2] = {r, r + nwarps < rows ? r + nwarps : -1};
    float v[2][12];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float4* xr = reinterpret_cast<const float4*>(x + size_t(rr[u] < 0 ? r : rr[u]) * kHidden);
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        const float4 t = xr[lane + 32 * i];
        v[u][4 * i] = t.x;
        v[u][4 * i + 1] = t.y;
        v[u][4 * i + 2] = t.z;
        v[u][4 * i + 3] = t.w;
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (rr[u] < 0) continue;
      float vmax = 1e-8f;
#pragma unroll
      for (int i = 0; i < 12; ++i) vmax = fmaxf(vmax, fabsf(v[u][i] * s[i]));
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
      const float inv_scale = 127.0f / vmax;
      int8_t* qr = q + size_t(rr[u]) * kHidden;
#pragma unroll
      for (int i = 0; i < 3; ++i) {
        uint32_t w = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          w |= (uint32_t(quant_i8(v[u][4 * i + e] * (s[4 * i + e] * inv_scale))) & 0xFFu) << (8 * e);
        reinterpret_cast<uint32_t*>(qr)[lane + 32 * i] = w;
      }
      if (lane == 0) scale[rr[u]] = vmax / 127.0f;
    }
  }
}

// Per-row metadata of a packed batch: position of each row inside its sequence (positions restart
// at 0 for every sequence, src/model.rs:557-567) and the row of each sequence's [CLS] token.
// One block per sequence. Sequences must have 1..512 rows.
__global__ void k_row_meta(const uint32_t* __restrict__ cu, int n_seqs, uint16_t* __restrict__ pos,
                           int32_t* __restrict__ cls_row, int* err) {
  pdl_trigger();
  pdl_wait();
  const int s = blockIdx.x;
  if (s >= n_seqs) return;
  const uint32_t b = cu[s], e = cu[s + 1];
  if (e <= b || e - b > uint32_t(kMaxPos)) {
    if (threadIdx.x == 0) record_err(err, DEV_ERR_BAD_SHAPE);
    return;
  }
  for (uint32_t r = b + threadIdx.x; r < e; r += blockDim.x) pos[r] = uint16_t(r - b);
  if (threadIdx.x == 0) cls_row[s] = int32_t(b);
}

// Gathers the [CLS] rows (act_q, act_scale, hidden) of every sequence into rows 0..n-1
// (the compaction of src/model.rs:786-800, into separate buffers); hidden is tile-transposed,
// the gathered rows are row-major.
__global__ void k_gather_cls(const int32_t* __restrict__ cls_row, int n, const int8_t* __restrict__ act_q,
                             const float* __restrict__ act_s, const float* __restrict__ hidden,
                             int8_t* __restrict__ cq, float* __restrict__ cs, float* __restrict__ ch) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  if (b >= n) return;
  const int r = cls_row[b];
  const int t = threadIdx.x;  // 96 threads
#pragma unroll
  for (int e = 0; e < 4; ++e) ch[size_t(b) * kHidden + 4 * t + e] = hidden[tt_index(r, 4 * t + e, kHidden)];
  reinterpret_cast<uint32_t*>(cq + size_t(b) * kHidden)[t] =
      reinterpret_cast<const uint32_t*>(act_q + size_t(r) * kHidden)[t];
  if (t == 0) cs[b] = act_s[r];
}

// Self-test of the bounded device waits: one thread waits for a phase of an mbarrier that nothing
// ever completes, through the same mbar_wait the GEMM pipeline uses; the wait gives up after
// limit_ns and records DEV_ERR_TIMEOUT_EPILOGUE. Nothing faults or hangs.
__global__ void k_wait_selftest(int* err, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, err, DEV_ERR_TIMEOUT_EPILOGUE, limit_ns);
}

int launch_wait_selftest(int* err, uint64_t limit_ns, cudaStream_t st) {
  k_wait_selftest<<<1, 32, 0, st>>>(err, limit_ns);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_embed(const EmbedArgs& a, cudaStream_t st) {
  if (a.T <= 0) return 0;
  const int rows_per_block = 16;
  const dim3 grid((a.T + rows_per_block - 1) / rows_per_block);
  return launch_pdl(k_embed_ln_quant, grid, dim3(256), 0, st, a) == cudaSuccess ? 0 : -1;
}

int launch_ln_quant_rows(const float* h_in, int M, const float* gamma, const float* beta, const float* inv_s,
                         float* hidden, int hidden_tt, int8_t* q, float* scale, cudaStream_t st) {
  if (M <= 0) return 0;
  return launch_pdl(k_ln_quant_rows, dim3((M + 15) / 16), dim3(256), 0, st, h_in, M, gamma, beta, inv_s, hidden,
                    hidden_tt, q, scale) == cudaSuccess ? 0 : -1;
}

int launch_ln_final_rows(const float* h_in, int M, const float* gamma, const float* beta, float* out,
                         cudaStream_t st) {
  if (M <= 0) return 0;
  return launch_pdl(k_ln_final_rows, dim3((M + kLnFinalRows - 1) / kLnFinalRows), dim3(128),
                    size_t(kLnFinalRows * kLnFinalPitch * 4), st, h_in, M, gamma, beta, out) == cudaSuccess ? 0 : -1;
}

int launch_smooth_quant(const float* x, const float* inv_s, int8_t* q, float* scale, int rows, cudaStream_t st) {
  if (rows <= 0) return 0;
  // enough warps for every row of a small batch, at most 8 blocks of 8 warps per SM
  const int blocks = (rows + 7) / 8 < 148 * 8 ? (rows + 7) / 8 : 148 * 8;
  return launch_pdl(k_smooth_quant, dim3(blocks), dim3(256), 0, st, x, inv_s, q, scale, rows) == cudaSuccess ? 0 : -1;
}

int launch_row_meta(const uint32_t* cu, int n_seqs, uint16_t* pos, int32_t* cls_row, int* err, cudaStream_t st) {
  if (n_seqs <= 0) return 0;
  return launch_pdl(k_row_meta, dim3(n_seqs), dim3(128), 0, st, cu, n_seqs, pos, cls_row, err) == cudaSuccess ? 0 : -1;
}

int launch_gather_cls(const int32_t* cls_row, int n, const int8_t* act_q, const float* act_s, const float* hidden,
                      int8_t* cq, float* cs, float* ch, cudaStream_t st) {
  if (n <= 0) return 0;
  return launch_pdl(k_gather_cls, dim3(n), dim3(96), 0, st, cls_row, n, act_q, act_s, hidden, cq, cs, ch) == cudaSuccess ? 0 : -1;
}

}  // namespace ae
