// The attention of one query over at most 64 keys with four (or eight) lanes per query, in the
// reference's exact operation order (compute_scores_head32_avx2 + softmax_inplace_avx2 +
// weighted_sum_head32_avx2, src/simd_math.rs:2953-3070). Shared by the short-sequence attention
// kernel (attention.cu, k_attention_lat) and the single-sequence cluster forward (latency.cu, eight
// lanes), so both compute the same bits.
//
// Sub-lane sl (0..3) of a query computes the scores and exponentials of the keys whose softmax-sum
// slots it owns -- in every full 16-key chunk t0 the keys t0 + 2sl, t0 + 2sl + 1 (slots 2sl, 2sl + 1
// of the first 8-lane accumulator) and t0 + 8 + 2sl, t0 + 9 + 2sl (the second), in the trailing
// 8-key chunk L16 + 2sl, L16 + 2sl + 1, and the tail keys L8 + sl + 4k (scalar exp, added after the
// tree) -- so each of the reference's 16 sum chains stays in one thread, in order; the hsum256 tree
// of the 8 lanes runs over two shuffles. The weighted sum: sub-lane sl owns dims 8sl .. 8sl + 7,
// both the even- and odd-key accumulators, over all keys in order.
#pragma once
#include <cstdint>

#include "rowmath.cuh"

namespace ae {

// q: the query pre-scaled by 1/sqrt(32); kd / vd: K and V dim-major (dim d of key t at d * P + t);
// er: this query's row of P floats for its scores, then exponentials; cx: dims 8sl .. 8sl + 7 of the
// context row. The four lanes of a query are consecutive lanes 4k .. 4k + 3 of a warp, and every
// lane of the warp calls this function (full-warp shuffles).
__device__ __forceinline__ void attend_query_lanes4(const float (&q)[32], const float* __restrict__ kd,
                                                    const float* __restrict__ vd, int P, float* er, int L, int sl,
                                                    float (&cx)[8]) {
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;
  const unsigned full = 0xffffffffu;

  auto score = [&](int t) -> float {  // score_pair's order for one key
    float s8[8];
#pragma unroll
    for (int l = 0; l < 8; ++l)
      s8[l] = fmaf(q[8 + l], kd[(8 + l) * P + t], q[l] * kd[l * P + t]) +
              fmaf(q[24 + l], kd[(24 + l) * P + t], q[16 + l] * kd[(16 + l) * P + t]);
    return (t < L4) ? ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]))
                    : ((s8[0] + s8[4]) + (s8[1] + s8[5])) + ((s8[2] + s8[6]) + (s8[3] + s8[7]));
  };

  // pass 1: scores of the owned keys, their max over the query's four sub-lanes
  float mx = -INFINITY;
  for (int t0 = 0; t0 < L16; t0 += 16) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int t = t0 + 2 * sl + (k & 1) + 8 * (k >> 1);
      const float sv = score(t);
      er[t] = sv;
      mx = fmaxf(mx, sv);
    }
  }
  for (int t = L16 + 2 * sl; t < L16 + 2 * sl + 2 && t < L8; ++t) {
    const float sv = score(t);
    er[t] = sv;
    mx = fmaxf(mx, sv);
  }
  for (int t = L8 + sl; t < L; t += 4) {
    const float sv = score(t);
    er[t] = sv;
    mx = fmaxf(mx, sv);
  }
  mx = fmaxf(mx, __shfl_xor_sync(full, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(full, mx, 2));

  // pass 2: exponentials of the owned keys and the owned sum chains (slots 2sl, 2sl + 1 of both
  // 8-lane accumulators), in chunk order
  float c0a = 0.0f, c0b = 0.0f, c1a = 0.0f, c1b = 0.0f;
  for (int t0 = 0; t0 < L16; t0 += 16) {
    const int t = t0 + 2 * sl;
    const float e0 = cw_exp(er[t] - mx), e1 = cw_exp(er[t + 1] - mx);
    const float e2 = cw_exp(er[t + 8] - mx), e3 = cw_exp(er[t + 9] - mx);
    er[t] = e0;
    er[t + 1] = e1;
    er[t + 8] = e2;
    er[t + 9] = e3;
    c0a = c0a + e0;
    c0b = c0b + e1;
    c1a = c1a + e2;
    c1b = c1b + e3;
  }
  if (L16 + 2 * sl < L8) {  // the trailing 8-key chunk feeds the first accumulator
    const int t = L16 + 2 * sl;
    const float e0 = cw_exp(er[t] - mx), e1 = cw_exp(er[t + 1] - mx);
    er[t] = e0;
    er[t + 1] = e1;
    c0a = c0a + e0;
    c0b = c0b + e1;
  }
  for (int t = L8 + sl; t < L; t += 4) er[t] = scalar_expf(er[t] - mx);
  // hsum256 of v[m] = acc0[m] + acc1[m]: sub-lane sl holds v[2sl], v[2sl + 1]
  const float vx = c0a + c1a, vy = c0b + c1b;
  const float ax = vx + __shfl_down_sync(full, vx, 2);  // v0 + v4 | v2 + v6
  const float ay = vy + __shfl_down_sync(full, vy, 2);  // v1 + v5 | v3 + v7
  const float tt = ax + ay;
  float sum = tt + __shfl_down_sync(full, tt, 1);
  __syncwarp();
  if (sl == 0)
    for (int t = L8; t < L; ++t) sum = sum + er[t];  // the tail keys in order, after the tree
  const float inv = __shfl_sync(full, 1.0f / sum, (threadIdx.x & 31) & ~3);

  // pass 3: weighted sum of V, dims 8sl .. 8sl + 7; even keys to the first accumulator
  float acc_e[8], acc_o[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc_e[k] = acc_o[k] = 0.0f;
  const float* vrow = vd + 8 * sl * P;
  int t = 0;
  for (; t + 1 < L; t += 2) {
    const float p0 = er[t] * inv, p1 = er[t + 1] * inv;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      acc_e[k] = fmaf(vrow[k * P + t], p0, acc_e[k]);
      acc_o[k] = fmaf(vrow[k * P + t + 1], p1, acc_o[k]);
    }
  }
  if (t < L) {
    const float p0 = er[t] * inv;
#pragma unroll
    for (int k = 0; k < 8; ++k) acc_e[k] = fmaf(vrow[k * P + t], p0, acc_e[k]);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) cx[k] = acc_e[k] + acc_o[k];
}

// The same with eight lanes per query (consecutive lanes 8k .. 8k + 7 of a warp; every lane of the
// warp calls it): sub-lane s owns slot s of both 8-lane sum accumulators -- in every full 16-key
// chunk t0 the keys t0 + s (first accumulator) and t0 + 8 + s (second), key L16 + s of the trailing
// 8-key chunk (first), and tail key L8 + s (scalar exp, added in order after the tree by sub-lane 0)
// -- and dims 4s .. 4s + 3 of the even / odd weighted-sum accumulators. Every chain the reference
// keeps runs in one thread in the reference's order, so the result is the same bits as
// attend_query_lanes4. cx: dims 4s .. 4s + 3 of the context row.
__device__ __forceinline__ void attend_query_lanes8(const float (&q)[32], const float* __restrict__ kd,
                                                    const float* __restrict__ vd, int P, float* er, int L, int s,
                                                    float (&cx)[4]) {
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;
  const unsigned full = 0xffffffffu;

  auto score = [&](int t) -> float {  // score_pair's order for one key
    float s8[8];
#pragma unroll
    for (int l = 0; l < 8; ++l)
      s8[l] = fmaf(q[8 + l], kd[(8 + l) * P + t], q[l] * kd[l * P + t]) +
              fmaf(q[24 + l], kd[(24 + l) * P + t], q[16 + l] * kd[(16 + l) * P + t]);
    return (t < L4) ? ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]))
                    : ((s8[0] + s8[4]) + (s8[1] + s8[5])) + ((s8[2] + s8[6]) + (s8[3] + s8[7]));
  };

  // pass 1: scores of the owned keys, their max over the query's eight sub-lanes
  float mx = -INFINITY;
  for (int t0 = 0; t0 < L16; t0 += 16) {
    const float a = score(t0 + s), b = score(t0 + 8 + s);
    er[t0 + s] = a;
    er[t0 + 8 + s] = b;
    mx = fmaxf(mx, fmaxf(a, b));
  }
  if (L16 + s < L8) {
    const float a = score(L16 + s);
    er[L16 + s] = a;
    mx = fmaxf(mx, a);
  }
  if (L8 + s < L) {
    const float a = score(L8 + s);
    er[L8 + s] = a;
    mx = fmaxf(mx, a);
  }
  mx = fmaxf(mx, __shfl_xor_sync(full, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(full, mx, 2));
  mx = fmaxf(mx, __shfl_xor_sync(full, mx, 4));

  // pass 2: exponentials of the owned keys and the owned sum chains (slot s of both accumulators)
  float c0 = 0.0f, c1 = 0.0f;
  for (int t0 = 0; t0 < L16; t0 += 16) {
    const float e0 = cw_exp(er[t0 + s] - mx), e1 = cw_exp(er[t0 + 8 + s] - mx);
    er[t0 + s] = e0;
    er[t0 + 8 + s] = e1;
    c0 = c0 + e0;
    c1 = c1 + e1;
  }
  if (L16 + s < L8) {  // the trailing 8-key chunk feeds the first accumulator
    const float e0 = cw_exp(er[L16 + s] - mx);
    er[L16 + s] = e0;
    c0 = c0 + e0;
  }
  if (L8 + s < L) er[L8 + s] = scalar_expf(er[L8 + s] - mx);
  // hsum256 of v[m] = acc0[m] + acc1[m]: sub-lane s holds v[s]
  const float v = c0 + c1;
  const float a = v + __shfl_down_sync(full, v, 4);  // v0 + v4 | v1 + v5 | v2 + v6 | v3 + v7
  const float b = a + __shfl_down_sync(full, a, 1);  // (v0 + v4) + (v1 + v5) | ... (sub-lanes 0, 2)
  float sum = b + __shfl_down_sync(full, b, 2);      // sub-lane 0
  __syncwarp();
  if (s == 0)
    for (int t = L8; t < L; ++t) sum = sum + er[t];  // the tail keys in order, after the tree
  const float inv = __shfl_sync(full, 1.0f / sum, (threadIdx.x & 31) & ~7);

  // pass 3: weighted sum of V, dims 4s .. 4s + 3; even keys to the first accumulator
  float acc_e[4], acc_o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) acc_e[k] = acc_o[k] = 0.0f;
  const float* vrow = vd + 4 * s * P;
  int t = 0;
  for (; t + 1 < L; t += 2) {
    const float p0 = er[t] * inv, p1 = er[t + 1] * inv;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      acc_e[k] = fmaf(vrow[k * P + t], p0, acc_e[k]);
      acc_o[k] = fmaf(vrow[k * P + t + 1], p1, acc_o[k]);
    }
  }
  if (t < L) {
    const float p0 = er[t] * inv;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc_e[k] = fmaf(vrow[k * P + t], p0, acc_e[k]);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) cx[k] = acc_e[k] + acc_o[k];
}

}  // namespace ae
