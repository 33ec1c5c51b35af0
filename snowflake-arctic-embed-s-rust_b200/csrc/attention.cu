// Segment-masked multi-head attention (12 heads x d32, <= 512 keys per sequence) in fp32 on the
// CUDA cores, in the exact operation order of the reference's AVX2 kernels:
//   compute_scores_head32_avx2   src/simd_math.rs:2953-2984  (q pre-scaled by 1/sqrt(32),
//                                 dot32x4 + hadd tree for keys in groups of 4, hsum256 for the rest)
//   softmax_inplace_avx2         src/simd_math.rs:2989-3042  (Cody-Waite exp on 8-wide chunks with
//                                 two 8-lane accumulators, scalar exp for the tail, then * 1/sum)
//   weighted_sum_head32_avx2     src/simd_math.rs:3047-3070  (two accumulators, even/odd keys)
// driven as in src/model.rs:294-321 (all rows) and :814-843 ([CLS] rows of the pruned layer 11).
//
// One CTA per (sequence, head, query tile of 128); one thread per query. The sequence's K and V
// head slices are staged in shared memory and read as broadcasts. Scores are recomputed in each
// of the three softmax passes instead of being stored, which keeps shared memory at 2 x L x 128 B.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "ptx.cuh"
#include "rowmath.cuh"

namespace ae {

// One score in the reference order; `grouped` selects the hadd-tree order used for keys inside a
// complete group of four.
__device__ __forceinline__ float score_ref(const float (&q)[32], const float* __restrict__ k, bool grouped) {
  float s8[8];
  const float4* k4 = reinterpret_cast<const float4*>(k);
  float kk[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 t = k4[i];
    kk[4 * i] = t.x;
    kk[4 * i + 1] = t.y;
    kk[4 * i + 2] = t.z;
    kk[4 * i + 3] = t.w;
  }
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    const float a = fmaf(q[8 + l], kk[8 + l], q[l] * kk[l]);
    const float b = fmaf(q[24 + l], kk[24 + l], q[16 + l] * kk[16 + l]);
    s8[l] = a + b;
  }
  if (grouped) return ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
  return ((s8[0] + s8[4]) + (s8[1] + s8[5])) + ((s8[2] + s8[6]) + (s8[3] + s8[7]));
}

__global__ void __launch_bounds__(128) k_attention_exact(AttnArgs a) {
  extern __shared__ float4 smem4[];
  const int s = blockIdx.x;
  const int h = blockIdx.y;
  const int tile = blockIdx.z;
  const int tid = threadIdx.x;
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  if (L <= 0 || L > a.max_len) {
    if (tid == 0 && tile == 0 && h == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  const int nq = a.cls_mode ? 1 : L;
  if (tile * 128 >= nq) return;

  float* ks = reinterpret_cast<float*>(smem4);
  float* vs = ks + size_t(L) * 32;
  for (int i = tid; i < L * 8; i += blockDim.x) {
    const int t = i >> 3, c = (i & 7) * 4;
    const size_t base = size_t(s0 + t) * a.kv_stride + h * 32 + c;
    *reinterpret_cast<float4*>(ks + t * 32 + c) = *reinterpret_cast<const float4*>(a.k + base);
    *reinterpret_cast<float4*>(vs + t * 32 + c) = *reinterpret_cast<const float4*>(a.v + base);
  }
  __syncthreads();

  const int qi = tile * 128 + tid;
  if (qi >= nq) return;
  const int qrow = a.cls_mode ? s : s0 + qi;
  const float scale = 1.0f / sqrtf(32.0f);
  float q[32];
  {
    const float4* qp = reinterpret_cast<const float4*>(a.q + size_t(qrow) * a.q_stride + h * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 t = qp[i];
      q[4 * i] = t.x * scale;
      q[4 * i + 1] = t.y * scale;
      q[4 * i + 2] = t.z * scale;
      q[4 * i + 3] = t.w * scale;
    }
  }
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;

  // pass 1: row max
  float mx = -INFINITY;
  for (int t = 0; t < L; ++t) mx = fmaxf(mx, score_ref(q, ks + t * 32, t < L4));

  // pass 2: sum of exponentials in the reference's accumulation order
  float vs0[8], vs1[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) vs0[j] = vs1[j] = 0.0f;
  for (int t0 = 0; t0 < L16; t0 += 16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) vs0[j] = vs0[j] + cw_exp(score_ref(q, ks + (t0 + j) * 32, t0 + j < L4) - mx);
#pragma unroll
    for (int j = 0; j < 8; ++j) vs1[j] = vs1[j] + cw_exp(score_ref(q, ks + (t0 + 8 + j) * 32, t0 + 8 + j < L4) - mx);
  }
  if (L8 > L16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) vs0[j] = vs0[j] + cw_exp(score_ref(q, ks + (L16 + j) * 32, L16 + j < L4) - mx);
  }
  float v8[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) v8[j] = vs0[j] + vs1[j];
  float sum = tree8(v8);
  for (int t = L8; t < L; ++t) sum = sum + scalar_expf(score_ref(q, ks + t * 32, t < L4) - mx);
  const float inv = 1.0f / sum;

  // pass 3: probabilities and the weighted sum of V (accumulator a: even keys, b: odd keys)
  float acc_a[32], acc_b[32];
#pragma unroll
  for (int d = 0; d < 32; ++d) acc_a[d] = acc_b[d] = 0.0f;
  auto prob = [&](int t) {
    const float x = score_ref(q, ks + t * 32, t < L4) - mx;
    return (t < L8 ? cw_exp(x) : scalar_expf(x)) * inv;
  };
  int t = 0;
  for (; t + 2 <= L; t += 2) {
    const float pa = prob(t), pb = prob(t + 1);
    const float* va = vs + t * 32;
    const float* vb = va + 32;
#pragma unroll
    for (int d = 0; d < 32; ++d) {
      acc_a[d] = fmaf(va[d], pa, acc_a[d]);
      acc_b[d] = fmaf(vb[d], pb, acc_b[d]);
    }
  }
  if (t < L) {
    const float pa = prob(t);
    const float* va = vs + t * 32;
#pragma unroll
    for (int d = 0; d < 32; ++d) acc_a[d] = fmaf(va[d], pa, acc_a[d]);
  }
  float4* o = reinterpret_cast<float4*>(a.out + size_t(qrow) * a.out_stride + h * 32);
#pragma unroll
  for (int i = 0; i < 8; ++i)
    o[i] = make_float4(acc_a[4 * i] + acc_b[4 * i], acc_a[4 * i + 1] + acc_b[4 * i + 1],
                       acc_a[4 * i + 2] + acc_b[4 * i + 2], acc_a[4 * i + 3] + acc_b[4 * i + 3]);
}

int attention_prime() {
  return cudaFuncSetAttribute(k_attention_exact, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxPos * 32 * 4 * 2) ==
                 cudaSuccess
             ? 0
             : -1;
}

int launch_attention_exact(const AttnArgs& a, int n_seqs, cudaStream_t st) {
  if (n_seqs <= 0) return 0;
  if (a.max_len <= 0 || a.max_len > kMaxPos) return -1;
  const size_t smem = size_t(a.max_len) * 32 * 4 * 2;
  const int nq = a.cls_mode ? 1 : a.max_len;
  dim3 grid(n_seqs, kHeads, (nq + 127) / 128);
  k_attention_exact<<<grid, 128, smem, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

}  // namespace ae
