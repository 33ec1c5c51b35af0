// Segment-masked multi-head attention (12 heads x d32, <= 512 keys per sequence) in fp32 on the
// CUDA cores, in the exact operation order of the reference's AVX2 kernels:
//   compute_scores_head32_avx2   src/simd_math.rs:2953-2984  (q pre-scaled by 1/sqrt(32),
//                                 dot32x4 + hadd tree for keys in complete groups of 4, hsum256
//                                 for the rest)
//   softmax_inplace_avx2         src/simd_math.rs:2989-3042  (Cody-Waite exp on 8-wide chunks with
//                                 two 8-lane accumulators, scalar exp for the tail, then * 1/sum)
//   weighted_sum_head32_avx2     src/simd_math.rs:3047-3070  (two accumulators: even / odd keys)
// driven as in src/model.rs:294-321 (all rows) and :814-843 ([CLS] rows of the pruned layer 11).
//
// k_attention_rows: one CTA per (sequence, head, tile of QT queries), one thread per query. The
// head's K and V are staged in shared memory as key pairs (k[2i][d], k[2i+1][d]) so that every
// operation works on two keys at once with the sm_100 packed f32x2 instructions: each lane of a
// packed FMA / add / multiply is an ordinary IEEE single-precision operation, so the results are
// the same bits as the scalar sequence, and the reference's even/odd weighted-sum accumulators are
// exactly the two lanes. Each thread keeps the scores, then the exponentials, of its query in its
// TMEM lane (column t = key t), so every score is computed once and shared memory holds only K / V.
//
// k_attention_wide: the same with two or four warpgroups on one tile's TMEM lanes, for sequences
// of more than 128 keys (whose score columns leave room for only 1-2 CTAs per SM).
//
// k_attention_rows2: two queries per thread and two heads per CTA for wide batches of 65-128 keys
// (every staged K / V load feeds both queries).
//
// k_attention_lat: single sequences of at most 64 keys: four lanes per query, no TMEM, and
// optionally the context quantization of the next GEMM's input (clusters of the 12 heads).
//
// For few tiles (single sequences) the TMEM kernels split a tile's weighted sum by dims over 2-4
// CTAs, each repeating the tile's scores and exponentials, to spread the work over more SMs.
//
// k_attention_cls: one CTA per (sequence, head) for the single [CLS] query of layer 11: threads
// split the keys for the scores (all K / V loads of a thread in flight at once), 16 lanes run the
// 16 exp-sum chains, 64 threads the even / odd weighted-sum accumulators of the 32 dims.
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "attn_lanes.cuh"
#include "kernels.h"
#include "ptx.cuh"
#include "rowmath.cuh"

namespace ae {

#ifndef ATTN_WIDE_256_NWG
#define ATTN_WIDE_256_NWG 2
#define ATTN_WIDE_256_MINB 2
#endif
#define ATTN_WIDE_256 ATTN_WIDE_256_NWG, ATTN_WIDE_256_MINB

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// Scores of the key pair (2i, 2i+1). K pairs are staged with the dims that one 8-lane partial
// sum of the reference's dot32x4 uses side by side: kp[4l + j] = (k[2i][l + 8j], k[2i+1][l + 8j]),
// so lane l's four products come from two 128-bit shared loads.
__device__ __forceinline__ float2 score_pair(const float (&q)[32], const float2* __restrict__ kp, bool grouped) {
  const float4* k4 = reinterpret_cast<const float4*>(kp);
  float2 s8[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    const float4 t0 = k4[2 * l];      // dims l, l + 8 of both keys
    const float4 t1 = k4[2 * l + 1];  // dims l + 16, l + 24
    const float2 a = fma2(f2(q[8 + l], q[8 + l]), f2(t0.z, t0.w), mul2(f2(q[l], q[l]), f2(t0.x, t0.y)));
    const float2 b = fma2(f2(q[24 + l], q[24 + l]), f2(t1.z, t1.w), mul2(f2(q[16 + l], q[16 + l]), f2(t1.x, t1.y)));
    s8[l] = add2(a, b);
  }
  if (grouped)
    return add2(add2(add2(s8[0], s8[1]), add2(s8[2], s8[3])), add2(add2(s8[4], s8[5]), add2(s8[6], s8[7])));
  return add2(add2(add2(s8[0], s8[4]), add2(s8[1], s8[5])), add2(add2(s8[2], s8[6]), add2(s8[3], s8[7])));
}

// cw_exp (rowmath.cuh) on two lanes. The rounding add after the packed product y * log2(e) is two
// scalar adds by default: a packed product feeding a packed add has been seen to come out of the
// compiler with a single rounding (in the key-pair kernel, 25 of 737,280 outputs of 30 sequences
// of 64 keys then differed from the reference by up to 7.5e-8); PACKED_ROUND = true keeps the packed add
// where the compiled kernel has been checked against the reference bit for bit on 100 M
// exponentials (attend_rows_dm, config 3), one instruction less per key pair.
template <bool PACKED_ROUND = false>
__device__ __forceinline__ float2 cw_exp2(float2 x) {
  const float2 y = f2(fmaxf(fminf(x.x, 88.0f), -87.3f), fmaxf(fminf(x.y, 88.0f), -87.3f));
  const float2 t = mul2(y, f2(1.44269504088896341f, 1.44269504088896341f));
  const float2 big = PACKED_ROUND ? add2(t, f2(kRoundMagic, kRoundMagic))  // round half to even
                                  : f2(t.x + kRoundMagic, t.y + kRoundMagic);  // (rowmath.cuh)
  const float2 n = add2(big, f2(-kRoundMagic, -kRoundMagic));
  const float2 nn = f2(-n.x, -n.y);
  const float2 r = fma2(nn, f2(1.428606765330187e-6f, 1.428606765330187e-6f),
                        fma2(nn, f2(0.693145751953125f, 0.693145751953125f), y));
  float2 p = fma2(r, f2(0.008333334f, 0.008333334f), f2(0.041666668f, 0.041666668f));
  p = fma2(r, p, f2(0.16666667f, 0.16666667f));
  p = fma2(r, p, f2(0.5f, 0.5f));
  p = fma2(r, p, f2(1.0f, 1.0f));
  p = fma2(r, p, f2(1.0f, 1.0f));
  const float2 pw = f2(__int_as_float(((__float_as_int(big.x) - kRoundMagicBits) + 127) << 23),
                       __int_as_float(((__float_as_int(big.y) - kRoundMagicBits) + 127) << 23));
  return mul2(p, pw);
}

// (sequence, head, z) of a block of a (sequences, heads, z) grid, numbered so that z varies fastest
// in launch order: the query-tile CTAs of one (sequence, head), which all stage the same K / V, are
// dispatched together, and all but the first find K / V in L2 (launched with the sequence fastest,
// the tiles of a pair were thousands of CTAs apart and re-read K / V from DRAM).
__device__ __forceinline__ void tile_major_block(int& s, int& h, int& z) {
  const unsigned lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  z = int(lin % gridDim.z);
  const unsigned rest = lin / gridDim.z;
  h = int(rest % gridDim.y);
  s = int(rest / gridDim.y);
}

constexpr int KPS = 34;  // float2 per staged key pair (32 dims + 2 pad: 16-byte aligned, fewer bank conflicts)

__device__ __forceinline__ float ld_act(const float* p, int C, int tt, int t, int c) {
  return tt ? p[tt_index(t, c, C)] : p[size_t(t) * C + c];
}

// Stages the head's K and V of rows [s0, s0 + L) as key pairs (k[2p][d], k[2p+1][d]), K dims in
// score_pair's order, V dims in order (odd L: the last pair's second key is 0). A warp covers
// 8 pairs x 4 dims per step, so the tile-transposed rows it reads are contiguous.
__device__ __forceinline__ void stage_kv_pairs(const AttnArgs& a, int s0, int L, int h, float2* kp, float2* vp) {
  const int pairs = (L + 1) >> 1;
  const int kc = a.k_col + 32 * h, vc = a.v_col + 32 * h;
  if (a.kv_tt && !(s0 & 1)) {
    // tile-transposed rows with an even first row: keys (2p, 2p+1) of one dim are 8 adjacent bytes
    // in the same 128-row block, copied asynchronously (all in flight at once); lanes take
    // consecutive pairs of one dim. The second key of an odd L's last pair is zero-filled.
    for (int i = threadIdx.x; i < pairs * 32; i += blockDim.x) {
      const int d = i / pairs, p = i - d * pairs;
      const int t = s0 + 2 * p;
      const uint32_t bytes = (2 * p + 1 < L) ? 8u : 4u;
      cp_async8(kp + p * KPS + (d & 7) * 4 + (d >> 3), a.kv + tt_index(t, kc + d, a.kv_C), bytes);
      cp_async8(vp + p * KPS + d, a.kv + tt_index(t, vc + d, a.kv_C), bytes);
    }
    cp_async_wait_all();
    return;
  }
  if (!a.kv_tt) {
    // row-major rows: one key's 32 dims of a head are 128 contiguous bytes; an item takes dims
    // 4g .. 4g + 3 of both keys of a pair as 16-byte loads (eight items cover a key row)
    for (int i = threadIdx.x; i < pairs * 8; i += blockDim.x) {
      const int p = i >> 3, g = i & 7;
      const size_t r0 = size_t(s0 + 2 * p) * a.kv_C;
      const bool two = 2 * p + 1 < L;
      const float4 ka = *reinterpret_cast<const float4*>(a.kv + r0 + kc + 4 * g);
      const float4 va = *reinterpret_cast<const float4*>(a.kv + r0 + vc + 4 * g);
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 kb = two ? *reinterpret_cast<const float4*>(a.kv + r0 + a.kv_C + kc + 4 * g) : z;
      const float4 vb = two ? *reinterpret_cast<const float4*>(a.kv + r0 + a.kv_C + vc + 4 * g) : z;
      const float k0[4] = {ka.x, ka.y, ka.z, ka.w}, k1[4] = {kb.x, kb.y, kb.z, kb.w};
      const float v0[4] = {va.x, va.y, va.z, va.w}, v1[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = 4 * g + e;
        kp[p * KPS + (d & 7) * 4 + (d >> 3)] = f2(k0[e], k1[e]);  // score_pair's order
        vp[p * KPS + d] = f2(v0[e], v1[e]);
      }
    }
    return;
  }
  const int groups = (pairs + 7) >> 3;  // 8-pair groups
  for (int i = threadIdx.x; i < groups * 256; i += blockDim.x) {
    const int w = i >> 5, l = i & 31;
    const int g = w >> 3, dgrp = w & 7;  // warp-step: pair group g, dims 4*dgrp .. 4*dgrp+3
    const int p = 8 * g + (l & 7), d = 4 * dgrp + (l >> 3);
    if (p >= pairs) continue;
    const int t0 = 2 * p, t1 = t0 + 1;
    const float k0 = ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t0, kc + d);
    const float v0 = ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t0, vc + d);
    float k1 = 0.0f, v1 = 0.0f;
    if (t1 < L) {
      k1 = ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t1, kc + d);
      v1 = ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t1, vc + d);
    }
    kp[p * KPS + (d & 7) * 4 + (d >> 3)] = f2(k0, k1);  // score_pair's order
    vp[p * KPS + d] = f2(v0, v1);
  }
}

__device__ __forceinline__ void load_query(const AttnArgs& a, int qrow, int h, float (&q)[32]) {
  const float scale = 1.0f / sqrtf(32.0f);
  if (a.q_tt) {
    const float* qp = a.q + tt_index(qrow, a.q_col + 32 * h, a.q_C);
#pragma unroll
    for (int d = 0; d < 32; ++d) q[d] = qp[size_t(d) << 7] * scale;
  } else {
    const float4* qp = reinterpret_cast<const float4*>(a.q + size_t(qrow) * a.q_C + a.q_col + 32 * h);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 t = qp[i];
      q[4 * i] = t.x * scale;
      q[4 * i + 1] = t.y * scale;
      q[4 * i + 2] = t.z * scale;
      q[4 * i + 3] = t.w * scale;
    }
  }
}

// TMEM columns of one CTA: the scores of a sequence of L keys (power of two, >= 32).
__host__ __device__ constexpr uint32_t tmem_cols_for_len(int L) {
  return L <= 32 ? 32 : L <= 64 ? 64 : L <= 128 ? 128 : L <= 256 ? 256 : 512;
}

// One CTA per (sequence, head, tile of QT queries); thread = query = TMEM lane. Every thread keeps
// the scores, then the exponentials, of its query in its TMEM lane (column t = key t), so shared
// memory holds only the head's K / V pairs. Threads whose query lies past the sequence still take
// part in the warp-collective TMEM loads and stores and write nothing.
//
// DSPLIT > 1 (few tiles: single sequences): z = tile * DSPLIT + part, and CTA `part`
// repeats the scores and exponentials of its tile but runs the weighted sum only for dims
// part * 32 / DSPLIT .. + 32 / DSPLIT - 1.
template <int QT, int DSPLIT = 1>
__global__ void __launch_bounds__(QT, 512 / QT) k_attention_rows(AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  constexpr int DN = 32 / DSPLIT;  // dims of this CTA's weighted sum
  extern __shared__ float4 smem4[];
  __shared__ uint32_t tmem_slot;
  int s, h, bz;
  tile_major_block(s, h, bz);
  const int tile = bz / DSPLIT;
  const int dbase = (bz % DSPLIT) * DN;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  if (a.skip_from > 0 && L >= a.skip_from) return;  // another kernel takes these sequences
  if (L <= 0 || L > a.max_len) {
    if (tid == 0 && tile == 0 && h == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  if (tile * QT >= L) return;
  const uint32_t cols = tmem_cols_for_len(L);
  if (warp == 0) {
    tmem_alloc(&tmem_slot, cols);
    tmem_relinquish();
  }
  const int qi = tile * QT + tid;
  const bool active = qi < L;
  const int qrow = s0 + (active ? qi : L - 1);
  float q[32];
  load_query(a, qrow, h, q);  // requested before the K / V staging, in flight with it
  const int pairs = (L + 1) >> 1;
  float2* kp = reinterpret_cast<float2*>(smem4);
  float2* vp = kp + pairs * KPS;
  stage_kv_pairs(a, s0, L, h, kp, vp);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tl = tmem_slot + (uint32_t(warp * 32) << 16);  // this warp's 32 lanes
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;
  uint32_t r[16];

  // pass 1: scores -> TMEM (16 keys per store) and their max (order-independent)
  float mx = -INFINITY;
  for (int t0 = 0; t0 < L; t0 += 16) {
    if (t0 + 16 <= L4) {  // a full chunk of complete 4-key groups: no bounds, pairs interleave freely
      float2 ma = f2(-INFINITY, -INFINITY), mb = ma;  // two max chains (even / odd pairs)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 sp = score_pair(q, kp + ((t0 >> 1) + j) * KPS, true);
        if (j & 1) mb = f2(fmaxf(mb.x, sp.x), fmaxf(mb.y, sp.y));
        else ma = f2(fmaxf(ma.x, sp.x), fmaxf(ma.y, sp.y));
        r[2 * j] = __float_as_uint(sp.x);
        r[2 * j + 1] = __float_as_uint(sp.y);
      }
      mx = fmaxf(mx, fmaxf(fmaxf(ma.x, ma.y), fmaxf(mb.x, mb.y)));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t = t0 + 2 * j;
        float2 sp = f2(0.0f, 0.0f);
        if (t < L) {
          sp = score_pair(q, kp + (t >> 1) * KPS, t < L4);
          mx = fmaxf(mx, sp.x);
          if (t + 1 < L) mx = fmaxf(mx, sp.y);
        }
        r[2 * j] = __float_as_uint(sp.x);
        r[2 * j + 1] = __float_as_uint(sp.y);
      }
    }
    tmem_st16(tl + t0, r);
  }
  tmem_st_wait();
  const float2 neg_mx = f2(-mx, -mx);

  // pass 2: exponentials (back into TMEM) and their sum in the reference's accumulation order:
  // full 16-key chunks feed the two 8-lane accumulators, a trailing 8-key chunk the first one,
  // the last L % 8 keys a scalar exp added in order after the tree
  float2 vs0[4], vs1[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) vs0[j] = vs1[j] = f2(0.0f, 0.0f);
  for (int t0 = 0; t0 < L; t0 += 16) {
    tmem_ld16(tl + t0, r);
    tmem_ld_wait();
    if (t0 + 16 <= L16) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 e = cw_exp2(add2(f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), neg_mx));
        if (j < 4) vs0[j] = add2(vs0[j], e);
        else vs1[j - 4] = add2(vs1[j - 4], e);
        r[2 * j] = __float_as_uint(e.x);
        r[2 * j + 1] = __float_as_uint(e.y);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t = t0 + 2 * j;
        const float2 x = add2(f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), neg_mx);
        float2 e;
        if (j < 4 && t + 1 < L8) {  // the trailing 8-key chunk (keys L16 .. L16 + 7)
          e = cw_exp2(x);
          vs0[j & 3] = add2(vs0[j & 3], e);
        } else {  // the last L % 8 keys: scalar exp, summed after the tree
          e = f2(t < L ? scalar_expf(x.x) : 0.0f, t + 1 < L ? scalar_expf(x.y) : 0.0f);
        }
        r[2 * j] = __float_as_uint(e.x);
        r[2 * j + 1] = __float_as_uint(e.y);
      }
    }
    tmem_st16(tl + t0, r);
  }
  tmem_st_wait();
  float v8[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 t = add2(vs0[j], vs1[j]);
    v8[2 * j] = t.x;
    v8[2 * j + 1] = t.y;
  }
  float sum = tree8(v8);
  if (L8 < L) {  // ((tree + e[L8]) + e[L8 + 1]) + ..., the keys re-read from TMEM
    tmem_ld16(tl + L16, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (L16 + j >= L8 && L16 + j < L) sum = sum + __uint_as_float(r[j]);
  }
  const float inv = 1.0f / sum;
  const float2 inv2 = f2(inv, inv);

  // pass 3: probabilities and the weighted sum of V; lane x = even keys (a), lane y = odd keys (b)
  float2 acc[DN];
#pragma unroll
  for (int d = 0; d < DN; ++d) acc[d] = f2(0.0f, 0.0f);
  for (int t0 = 0; t0 < L; t0 += 16) {
    tmem_ld16(tl + t0, r);
    tmem_ld_wait();
    if (t0 + 16 <= L) {  // a full chunk: no bounds
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 p = mul2(f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), inv2);
        const float4* v4 = reinterpret_cast<const float4*>(vp + ((t0 >> 1) + j) * KPS + dbase);
#pragma unroll
        for (int i = 0; i < DN / 2; ++i) {
          const float4 vv = v4[i];
          acc[2 * i] = fma2(f2(vv.x, vv.y), p, acc[2 * i]);
          acc[2 * i + 1] = fma2(f2(vv.z, vv.w), p, acc[2 * i + 1]);
        }
      }
      continue;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = t0 + 2 * j;
      if (t + 1 < L) {
        const float2 p = mul2(f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), inv2);
        const float4* v4 = reinterpret_cast<const float4*>(vp + (t >> 1) * KPS + dbase);
#pragma unroll
        for (int i = 0; i < DN / 2; ++i) {
          const float4 vv = v4[i];
          acc[2 * i] = fma2(f2(vv.x, vv.y), p, acc[2 * i]);
          acc[2 * i + 1] = fma2(f2(vv.z, vv.w), p, acc[2 * i + 1]);
        }
      } else if (t < L) {  // odd L: the last key goes to the even accumulator
        const float pa = __uint_as_float(r[2 * j]) * inv;
        const float2* v = vp + (t >> 1) * KPS + dbase;
#pragma unroll
        for (int d = 0; d < DN; ++d) acc[d].x = fmaf(v[d].x, pa, acc[d].x);
      }
    }
  }
  if (active) {
    float4* o = reinterpret_cast<float4*>(a.out + size_t(s0 + qi) * kHidden + h * 32 + dbase);
#pragma unroll
    for (int i = 0; i < DN / 4; ++i)
      o[i] = make_float4(acc[4 * i].x + acc[4 * i].y, acc[4 * i + 1].x + acc[4 * i + 1].y,
                         acc[4 * i + 2].x + acc[4 * i + 2].y, acc[4 * i + 3].x + acc[4 * i + 3].y);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_slot, cols);
}

// ---------------------------------------------------------------------------------------------
// Dim-major staging: K (and V) of a head as 32 rows (dims) of RS floats, key t at column t -- the
// tile-transposed activation layout itself, so a sequence that starts a 128-row tile arrives by
// one bulk copy. A float4 holds one dim of four keys (a "quad"), which feeds the same packed
// operations as the key-pair layout: lanes (x, y) are the pair (4i, 4i+1), (z, w) the pair
// (4i+2, 4i+3).

// Scores of keys 4i .. 4i+3 (kq = column 4i of dim row 0) for NQ queries, in score_pair's order:
// each float4 loaded from shared memory feeds 2 pairs x NQ queries. grouped: the four keys form a
// complete group (dot32x4 + hadd tree); otherwise each pair takes the hsum256 order.
template <int NQ>
__device__ __forceinline__ void score_quad(const float (&q)[NQ][32], const float* __restrict__ kq, int rs,
                                           bool grouped, float2 (&sp)[NQ][2]) {
  float2 s8[NQ][2][8];
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    const float4 A = *reinterpret_cast<const float4*>(kq + l * rs);
    const float4 B = *reinterpret_cast<const float4*>(kq + (l + 8) * rs);
    const float4 C = *reinterpret_cast<const float4*>(kq + (l + 16) * rs);
    const float4 D = *reinterpret_cast<const float4*>(kq + (l + 24) * rs);
#pragma unroll
    for (int u = 0; u < NQ; ++u) {
      const float2 ql = f2(q[u][l], q[u][l]), ql8 = f2(q[u][l + 8], q[u][l + 8]);
      const float2 ql16 = f2(q[u][l + 16], q[u][l + 16]), ql24 = f2(q[u][l + 24], q[u][l + 24]);
      s8[u][0][l] = add2(fma2(ql8, f2(B.x, B.y), mul2(ql, f2(A.x, A.y))), fma2(ql24, f2(D.x, D.y), mul2(ql16, f2(C.x, C.y))));
      s8[u][1][l] = add2(fma2(ql8, f2(B.z, B.w), mul2(ql, f2(A.z, A.w))), fma2(ql24, f2(D.z, D.w), mul2(ql16, f2(C.z, C.w))));
    }
  }
#pragma unroll
  for (int u = 0; u < NQ; ++u)
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      const float2* x = s8[u][pr];
      sp[u][pr] = grouped ? add2(add2(add2(x[0], x[1]), add2(x[2], x[3])), add2(add2(x[4], x[5]), add2(x[6], x[7])))
                          : add2(add2(add2(x[0], x[4]), add2(x[1], x[5])), add2(add2(x[2], x[6]), add2(x[3], x[7])));
    }
}

// score_quad (grouped order) for the eight keys 8i .. 8i+7 (two quads): dims outer, so that every
// step of the loop has eight independent key-pair chains per query, and the dot32x4 + hadd tree
// ((x0 + x1) + (x2 + x3)) + ((x4 + x5) + (x6 + x7)) built as its terms arrive (the same additions in
// the same order). sp[u][k]: keys (8i + 2k, 8i + 2k + 1).
template <int NQ>
__device__ __forceinline__ void score_oct(const float (&q)[NQ][32], const float* __restrict__ kq, int rs,
                                          float2 (&sp)[NQ][4]) {
  float2 h[NQ][4], a[NQ][4], b[NQ][4];
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    float4 A[2], B[2], C[2], D[2];
#pragma unroll
    for (int o = 0; o < 2; ++o) {
      A[o] = *reinterpret_cast<const float4*>(kq + 4 * o + l * rs);
      B[o] = *reinterpret_cast<const float4*>(kq + 4 * o + (l + 8) * rs);
      C[o] = *reinterpret_cast<const float4*>(kq + 4 * o + (l + 16) * rs);
      D[o] = *reinterpret_cast<const float4*>(kq + 4 * o + (l + 24) * rs);
    }
#pragma unroll
    for (int u = 0; u < NQ; ++u) {
      const float2 ql = f2(q[u][l], q[u][l]), ql8 = f2(q[u][l + 8], q[u][l + 8]);
      const float2 ql16 = f2(q[u][l + 16], q[u][l + 16]), ql24 = f2(q[u][l + 24], q[u][l + 24]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int o = k >> 1;
        const float2 av = (k & 1) ? f2(A[o].z, A[o].w) : f2(A[o].x, A[o].y);
        const float2 bv = (k & 1) ? f2(B[o].z, B[o].w) : f2(B[o].x, B[o].y);
        const float2 cv = (k & 1) ? f2(C[o].z, C[o].w) : f2(C[o].x, C[o].y);
        const float2 dv = (k & 1) ? f2(D[o].z, D[o].w) : f2(D[o].x, D[o].y);
        const float2 x = add2(fma2(ql8, bv, mul2(ql, av)), fma2(ql24, dv, mul2(ql16, cv)));
        // ((x0 + x1) + (x2 + x3)) + ((x4 + x5) + (x6 + x7))
        if ((l & 1) == 0) {
          if (l & 2) b[u][k] = x; else a[u][k] = x;
        } else {
          if (l & 2) {
            b[u][k] = add2(b[u][k], x);
            const float2 t = add2(a[u][k], b[u][k]);
            if (l == 3) h[u][k] = t; else sp[u][k] = add2(h[u][k], t);
          } else {
            a[u][k] = add2(a[u][k], x);
          }
        }
      }
    }
  }
}

// k_attention_rows' three passes for NQ queries per thread over one head's dim-major K / V
// (row stride rs): every shared-memory load of K or V feeds NQ queries. Query u keeps its scores,
// then exponentials, in TMEM columns tl + u * qcols .. + L - 1 of the thread's lane. q: pre-scaled
// by 1/sqrt(32); out[u] = nullptr for a query past the sequence (which still takes part in the
// warp-collective TMEM loads and stores). Columns L .. (L + 3) & ~3 of K / V must hold finite
// values (their lanes are computed and discarded).
template <int NQ>
__device__ __forceinline__ void attend_rows_dm(const float (&q)[NQ][32], const float* __restrict__ kd,
                                               const float* __restrict__ vd, int rs, int L, uint32_t tl,
                                               uint32_t qcols, float* const (&out)[NQ]) {
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;
  uint32_t r[NQ][16];

  // pass 1: scores -> TMEM and their max (order-independent)
  float mx[NQ];
#pragma unroll
  for (int u = 0; u < NQ; ++u) mx[u] = -INFINITY;
  for (int t0 = 0; t0 < L; t0 += 16) {
    if (t0 + 16 <= L4) {
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float2 sp[NQ][4];
        score_oct<NQ>(q, kd + t0 + 8 * c, rs, sp);
#pragma unroll
        for (int u = 0; u < NQ; ++u)
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            mx[u] = fmaxf(mx[u], fmaxf(sp[u][k].x, sp[u][k].y));
            r[u][8 * c + 2 * k] = __float_as_uint(sp[u][k].x);
            r[u][8 * c + 2 * k + 1] = __float_as_uint(sp[u][k].y);
          }
      }
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int t = t0 + 4 * c;
        float2 sp[NQ][2];
#pragma unroll
        for (int u = 0; u < NQ; ++u) sp[u][0] = sp[u][1] = f2(0.0f, 0.0f);
        if (t < L) {
          score_quad<NQ>(q, kd + t, rs, t < L4, sp);
#pragma unroll
          for (int u = 0; u < NQ; ++u) {
            // keys past the sequence: 0, outside the max
            if (t + 1 >= L) sp[u][0].y = 0.0f;
            if (t + 2 >= L) sp[u][1].x = 0.0f;
            if (t + 3 >= L) sp[u][1].y = 0.0f;
            mx[u] = fmaxf(mx[u], sp[u][0].x);
            if (t + 1 < L) mx[u] = fmaxf(mx[u], sp[u][0].y);
            if (t + 2 < L) mx[u] = fmaxf(mx[u], sp[u][1].x);
            if (t + 3 < L) mx[u] = fmaxf(mx[u], sp[u][1].y);
          }
        }
#pragma unroll
        for (int u = 0; u < NQ; ++u) {
          r[u][4 * c] = __float_as_uint(sp[u][0].x);
          r[u][4 * c + 1] = __float_as_uint(sp[u][0].y);
          r[u][4 * c + 2] = __float_as_uint(sp[u][1].x);
          r[u][4 * c + 3] = __float_as_uint(sp[u][1].y);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < NQ; ++u) tmem_st16(tl + u * qcols + t0, r[u]);
  }
  tmem_st_wait();

  // pass 2: exponentials (back into TMEM) and their sums, in k_attention_rows' order per query
  float inv[NQ];
  {
    float2 vs0[NQ][4], vs1[NQ][4];
#pragma unroll
    for (int u = 0; u < NQ; ++u)
#pragma unroll
      for (int j = 0; j < 4; ++j) vs0[u][j] = vs1[u][j] = f2(0.0f, 0.0f);
    for (int t0 = 0; t0 < L; t0 += 16) {
#pragma unroll
      for (int u = 0; u < NQ; ++u) tmem_ld16(tl + u * qcols + t0, r[u]);
      tmem_ld_wait();
#pragma unroll
      for (int u = 0; u < NQ; ++u) {
        const float2 neg_mx = f2(-mx[u], -mx[u]);
        if (t0 + 16 <= L16) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float2 e =
                cw_exp2<true>(add2(f2(__uint_as_float(r[u][2 * j]), __uint_as_float(r[u][2 * j + 1])), neg_mx));
            if (j < 4) vs0[u][j] = add2(vs0[u][j], e);
            else vs1[u][j - 4] = add2(vs1[u][j - 4], e);
            r[u][2 * j] = __float_as_uint(e.x);
            r[u][2 * j + 1] = __float_as_uint(e.y);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int t = t0 + 2 * j;
            const float2 x = add2(f2(__uint_as_float(r[u][2 * j]), __uint_as_float(r[u][2 * j + 1])), neg_mx);
            float2 e;
            if (j < 4 && t + 1 < L8) {
              e = cw_exp2<true>(x);
              vs0[u][j & 3] = add2(vs0[u][j & 3], e);
            } else {
              e = f2(t < L ? scalar_expf(x.x) : 0.0f, t + 1 < L ? scalar_expf(x.y) : 0.0f);
            }
            r[u][2 * j] = __float_as_uint(e.x);
            r[u][2 * j + 1] = __float_as_uint(e.y);
          }
        }
        tmem_st16(tl + u * qcols + t0, r[u]);
      }
    }
    tmem_st_wait();
#pragma unroll
    for (int u = 0; u < NQ; ++u) {
      float v8[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 t = add2(vs0[u][j], vs1[u][j]);
        v8[2 * j] = t.x;
        v8[2 * j + 1] = t.y;
      }
      float sum = tree8(v8);
      if (L8 < L) {
        tmem_ld16(tl + u * qcols + L16, r[u]);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (L16 + j >= L8 && L16 + j < L) sum = sum + __uint_as_float(r[u][j]);
      }
      inv[u] = 1.0f / sum;
    }
  }

  // pass 3: probabilities and the weighted sum of V; lane x = even keys, lane y = odd keys
  float2 acc[NQ][32];
#pragma unroll
  for (int u = 0; u < NQ; ++u)
#pragma unroll
    for (int d = 0; d < 32; ++d) acc[u][d] = f2(0.0f, 0.0f);
  for (int t0 = 0; t0 < L; t0 += 16) {
#pragma unroll
    for (int u = 0; u < NQ; ++u) tmem_ld16(tl + u * qcols + t0, r[u]);
    tmem_ld_wait();
    if (t0 + 16 <= L) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float2 p01[NQ], p23[NQ];
#pragma unroll
        for (int u = 0; u < NQ; ++u) {
          p01[u] = mul2(f2(__uint_as_float(r[u][4 * c]), __uint_as_float(r[u][4 * c + 1])), f2(inv[u], inv[u]));
          p23[u] = mul2(f2(__uint_as_float(r[u][4 * c + 2]), __uint_as_float(r[u][4 * c + 3])), f2(inv[u], inv[u]));
        }
        const float* vq = vd + t0 + 4 * c;
#pragma unroll
        for (int d = 0; d < 32; ++d) {
          const float4 vv = *reinterpret_cast<const float4*>(vq + d * rs);
#pragma unroll
          for (int u = 0; u < NQ; ++u) {
            acc[u][d] = fma2(f2(vv.x, vv.y), p01[u], acc[u][d]);
            acc[u][d] = fma2(f2(vv.z, vv.w), p23[u], acc[u][d]);
          }
        }
      }
      continue;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = t0 + 2 * j;
      if (t + 1 < L) {
        float2 p[NQ];
#pragma unroll
        for (int u = 0; u < NQ; ++u)
          p[u] = mul2(f2(__uint_as_float(r[u][2 * j]), __uint_as_float(r[u][2 * j + 1])), f2(inv[u], inv[u]));
#pragma unroll
        for (int d = 0; d < 32; ++d) {
          const float2 vv = *reinterpret_cast<const float2*>(vd + d * rs + t);
#pragma unroll
          for (int u = 0; u < NQ; ++u) acc[u][d] = fma2(vv, p[u], acc[u][d]);
        }
      } else if (t < L) {  // odd L: the last key goes to the even accumulator
#pragma unroll
        for (int u = 0; u < NQ; ++u) {
          const float pa = __uint_as_float(r[u][2 * j]) * inv[u];
#pragma unroll
          for (int d = 0; d < 32; ++d) acc[u][d].x = fmaf(vd[d * rs + t], pa, acc[u][d].x);
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < NQ; ++u) {
    if (out[u]) {
      float4* o = reinterpret_cast<float4*>(out[u]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        o[i] = make_float4(acc[u][4 * i].x + acc[u][4 * i].y, acc[u][4 * i + 1].x + acc[u][4 * i + 1].y,
                           acc[u][4 * i + 2].x + acc[u][4 * i + 2].y, acc[u][4 * i + 3].x + acc[u][4 * i + 3].y);
    }
  }
}

// Stages K and V of heads 2y, 2y + 1 (64 columns each) of rows [s0, s0 + L) dim-major with row
// stride rs (>= L rounded up to 4; columns L .. rs - 1 zero) by per-thread asynchronous copies of
// 16 bytes (four keys; s0 a multiple of 4, tile-transposed rows) or 4 bytes, or plain loads for
// row-major activations. Complete after cp_async_wait_all.
__device__ __forceinline__ void stage_kv_dim_major(const AttnArgs& a, int s0, int L, int y, int rs, float* kd,
                                                   float* vd) {
  const int kc = a.k_col + 64 * y, vc = a.v_col + 64 * y;
  if (a.kv_tt && !(s0 & 3)) {
    const int quads = rs >> 2;
    for (int i = threadIdx.x; i < 128 * quads; i += blockDim.x) {
      const int row = i / quads, c = i - row * quads;  // row: 0-63 K dims, 64-127 V dims
      const int t = 4 * c;
      const int col = row < 64 ? kc + row : vc + row - 64;
      float* dst = (row < 64 ? kd + row * rs : vd + (row - 64) * rs) + t;
      const int valid = L - t < 4 ? (L - t > 0 ? L - t : 0) : 4;
      cp_async16(dst, a.kv + tt_index(s0 + (valid ? t : 0), col, a.kv_C), uint32_t(valid) * 4u);
    }
    return;
  }
  if (!a.kv_tt) {
    // row-major rows: an item takes dims 4g .. 4g + 3 of one key (K or V of one of the two heads)
    // as one 16-byte load; the columns L .. rs - 1 are zero
    for (int i = threadIdx.x; i < 32 * rs; i += blockDim.x) {  // keys fastest: conflict-free stores
      const int g = i / rs, t = i - g * rs;  // g: K dims 4g (g < 16), V dims 4 (g - 16) (g >= 16)
      const int dd = 4 * (g & 15);
      const int col = (g < 16 ? kc : vc) + dd;
      float* dst = (g < 16 ? kd : vd) + dd * rs + t;
      const float4 x = t < L ? *reinterpret_cast<const float4*>(a.kv + size_t(s0 + t) * a.kv_C + col)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      dst[0] = x.x;
      dst[rs] = x.y;
      dst[2 * rs] = x.z;
      dst[3 * rs] = x.w;
    }
    return;
  }
  for (int i = threadIdx.x; i < 128 * rs; i += blockDim.x) {
    const int row = i / rs, t = i - row * rs;
    const int col = row < 64 ? kc + row : vc + row - 64;
    float* dst = (row < 64 ? kd + row * rs : vd + (row - 64) * rs) + t;
    if (a.kv_tt) {
      cp_async4(dst, a.kv + tt_index(s0 + (t < L ? t : 0), col, a.kv_C), t < L ? 4u : 0u);
    } else {
      *dst = t < L ? ld_act(a.kv, a.kv_C, 0, s0 + t, col) : 0.0f;
    }
  }
}

// Sequences of 65..128 keys in wide batches: one CTA per (sequence, pair of heads), 128 threads.
// Warps 0-1 take head 2y, warps 2-3 head 2y + 1 (TMEM lanes 0-63 / 64-127); thread j of a head
// takes queries j and j + 64, so every staged K / V load feeds two queries. The scores of query
// j + 64 sit 128 TMEM columns after those of query j (256 columns: two CTAs per SM). K / V are
// staged dim-major: a sequence that starts a 128-row tile by bulk copies (the 64 K columns of the
// two heads are 32 KB in a row, as are the V columns and the Q columns), any other by per-thread
// copies.
__global__ void __launch_bounds__(128, 2) k_attention_rows2(AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float4 smem4[];
  __shared__ uint32_t tmem_slot;
  __shared__ uint64_t kv_bar;
  const int s = blockIdx.x;
  const int y = blockIdx.y;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int unit = warp >> 1;
  const int h = 2 * y + unit;
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  if (a.skip_from > 0 && L >= a.skip_from) return;  // another kernel takes these sequences
  if (L <= 0 || L > a.max_len || L > 128) {
    if (tid == 0 && y == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  const bool bulk = a.kv_tt && !(s0 & 127);
  const int rs = bulk ? 128 : (L + 3) & ~3;
  float* kd = reinterpret_cast<float*>(smem4);  // [64][rs]: K dims of heads 2y, 2y + 1
  float* vd = kd + 64 * rs;                     // [64][rs]: V dims
  float* qd = vd + 64 * rs;                     // [64][128]: Q dims (bulk staging only)
  const bool bulk_q = bulk && a.q_tt && a.q == a.kv && a.q_C == a.kv_C;
  if (bulk) {
    if (tid == 0) {
      mbar_init(&kv_bar, 1);
      fence_mbar_init();
      mbar_arrive_expect_tx(&kv_bar, (bulk_q ? 3 : 2) * 64 * 128 * 4);
      const float* tile = a.kv + size_t(s0 >> 7) * a.kv_C * 128;
      bulk_load(kd, tile + size_t(a.k_col + 64 * y) * 128, 64 * 128 * 4, &kv_bar);
      bulk_load(vd, tile + size_t(a.v_col + 64 * y) * 128, 64 * 128 * 4, &kv_bar);
      if (bulk_q) bulk_load(qd, tile + size_t(a.q_col + 64 * y) * 128, 64 * 128 * 4, &kv_bar);
    }
  } else {
    stage_kv_dim_major(a, s0, L, y, rs, kd, vd);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 256);
    tmem_relinquish();
  }

  const int j = (warp & 1) * 32 + (tid & 31);
  float q[2][32];
  float* out[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int qi = j + 64 * u;
    const bool active = qi < L;
    if (!bulk_q) load_query(a, s0 + (active ? qi : L - 1), h, q[u]);
    out[u] = active ? a.out + size_t(s0 + qi) * kHidden + h * 32 : nullptr;
  }
  bool ok = true;
  if (bulk) {
    __syncthreads();  // kv_bar initialised
    ok = mbar_wait(&kv_bar, 0, a.err, DEV_ERR_TIMEOUT_PRODUCER);
  } else {
    cp_async_wait_all();
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok && bulk_q) {  // query qi of head h: column qi of dim rows 32 unit .. 32 unit + 31
    const float scale = 1.0f / sqrtf(32.0f);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int qi = j + 64 * u < L ? j + 64 * u : L - 1;
#pragma unroll
      for (int d = 0; d < 32; ++d) q[u][d] = qd[(unit * 32 + d) * 128 + qi] * scale;
    }
  }
  if (ok)
    attend_rows_dm<2>(q, kd + unit * 32 * rs, vd + unit * 32 * rs, rs, L, tmem_slot + (uint32_t(warp * 32) << 16), 128,
                      out);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_slot, 256);
}

// QKV projection + attention of one sequence of at most 128 keys and one pair of heads (2y, 2y + 1):
// one CTA, 128 threads, two CTAs per SM.
//   1. thread 0 loads the 192 weight rows of the pair (Q, K, V rows 64y .. 64y + 63 of each of the
//      three 384-row blocks of the [1152, 384] QKV weights; k-blocks 0 and 1 before the dependency
//      wait, they are model constants) and the sequence's 128-row activation tile (rows s0 ..
//      s0 + 127, whatever sequences they hold beyond s0 + L), then issues the 128 x 192 x 384
//      tcgen05 kind::i8 MMA into TMEM columns 0 .. 191;
//   2. warp w dequantizes rows 32w .. 32w + 31 (its TMEM lanes) as the QKV GEMM's plain epilogue
//      does, h = fma(float(acc), a_scale * w_scale, bias), into shared memory, dim-major: column n of
//      the 192 at row n of a [192][128] array, so that Q, K and V of the pair are the [64][128]
//      blocks k_attention_rows2 stages by bulk copies (rows past the sequence: a_scale 0, h = bias);
//   3. k_attention_rows2's attention on those blocks, the scores in the same TMEM columns.
// Shared memory: A (3 k-blocks x 16 KB) and a 2-stage ring of weight k-blocks (24 KB each): 96 KB,
// which the dequantized [192][128] fp32 block reuses once the MMA has completed.
constexpr int kQaStageA = 128 * 128;                 // one k-block of the activation tile
constexpr int kQaStageW = 192 * 128;                 // one k-block of the pair's weight rows
constexpr int kQaAlias = 3 * kQaStageA + 2 * kQaStageW;  // 96 KB
static_assert(kQaAlias == 192 * 128 * 4, "the dequantized block reuses exactly the MMA operands' memory");
constexpr size_t kQaSmem = 1024 + kQaAlias + 2 * 192 * 4 + 8 * 8;

__global__ void __launch_bounds__(128, 2)
    k_qkv_attention(const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_w,
                    QkvAttnArgs qa) {
  pdl_trigger();
  extern __shared__ uint8_t qa_raw[];
  __shared__ uint32_t tmem_slot;
  // 1024-byte aligned (128-byte swizzle atoms) by pointer arithmetic on the shared array itself, so
  // that the compiler keeps every access below in the shared address space
  uint8_t* sm = qa_raw + ((1024u - (smem_u32(qa_raw) & 1023u)) & 1023u);
  uint8_t* sa = sm;                                   // A: k-block kb at kb * 16 KB
  uint8_t* sw = sm + 3 * kQaStageA;                   // weight ring: stage st at st * 24 KB
  float* dm = reinterpret_cast<float*>(sm);           // after the MMA: [192][128] Q | K | V, dim-major
  float* s_ws = reinterpret_cast<float*>(sm + kQaAlias);
  float* s_bias = s_ws + 192;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_bias + 192);
  uint64_t* w_full = bars;       // [2] weight stage loaded
  uint64_t* a_full = bars + 2;   // activation tile loaded
  uint64_t* w_free = bars + 3;   // stage 0 read by the MMAs of k-block 0
  uint64_t* acc_full = bars + 4; // accumulator complete
  const AttnArgs& a = qa.a;
  const int s = blockIdx.x;
  const int y = blockIdx.y;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  for (int i = tid; i < 192; i += 128) {  // column i of the pair = column gc of the QKV output
    const int gc = (i >> 6) * kHidden + 64 * y + (i & 63);
    s_ws[i] = qa.w_scale[gc];
    s_bias[i] = qa.bias[gc];
  }
  if (tid == 0) {
    tma_prefetch_desc(&tm_act);
    tma_prefetch_desc(&tm_w);
    for (int i = 0; i < 5; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    for (int kb = 0; kb < 2; ++kb) {
      mbar_arrive_expect_tx(&w_full[kb], kQaStageW);
      for (int p = 0; p < 3; ++p)
        tma_load_2d(sw + kb * kQaStageW + p * 64 * 128, &tm_w, &w_full[kb], kb * 128, p * kHidden + 64 * y);
    }
  }
  pdl_wait();
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  const bool shape_ok = L > 0 && L <= a.max_len && L <= 128;
  if (!shape_ok && tid == 0 && y == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
  if (tid == 0 && shape_ok) {
    mbar_arrive_expect_tx(a_full, 3 * kQaStageA);
    for (int kb = 0; kb < 3; ++kb) tma_load_2d(sa + kb * kQaStageA, &tm_act, a_full, kb * 128, s0);
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 256);
    tmem_relinquish();
  }
  const float as = (shape_ok && tid < L) ? qa.a_scale[s0 + tid] : 0.0f;  // requested while the MMA runs
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (tid == 0) {
    if (shape_ok) {
      constexpr uint32_t idesc = idesc_i8(128, 192);
      bool good = mbar_wait(a_full, 0, a.err, DEV_ERR_TIMEOUT_PRODUCER);
      for (int kb = 0; kb < 3 && good; ++kb) {
        const int st = kb & 1;
        if (kb == 2) {  // k-block 2 reuses stage 0 once the MMAs of k-block 0 have read it
          if (!(good = mbar_wait(w_free, 0, a.err, DEV_ERR_TIMEOUT_MMA))) break;
          mbar_arrive_expect_tx(&w_full[0], kQaStageW);
          for (int p = 0; p < 3; ++p) tma_load_2d(sw + p * 64 * 128, &tm_w, &w_full[0], 2 * 128, p * kHidden + 64 * y);
        }
        if (!(good = mbar_wait(&w_full[st], kb >> 1, a.err, DEV_ERR_TIMEOUT_MMA))) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(sa + kb * kQaStageA);
        const uint32_t b_addr = smem_u32(sw + st * kQaStageW);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_i8(tmem, sdesc_sw128(a_addr + ks * 32), sdesc_sw128(b_addr + ks * 32), idesc, (kb | ks) != 0);
        if (kb == 0) mma_commit(w_free);
      }
      if (good) mma_commit(acc_full);
    } else {  // no MMA: the weight copies in flight complete before the CTA exits
      mbar_wait(&w_full[0], 0, a.err, DEV_ERR_TIMEOUT_PRODUCER);
      mbar_wait(&w_full[1], 0, a.err, DEV_ERR_TIMEOUT_PRODUCER);
    }
  }
  bool ok = shape_ok && mbar_wait(acc_full, 0, a.err, DEV_ERR_TIMEOUT_EPILOGUE);
  ok = __all_sync(0xffffffffu, ok);  // the TMEM loads below are warp-collective
  tc_fence_after();
  fence_proxy_async();  // the MMAs' reads of A and the weights precede the writes that reuse that memory
  if (ok && warp * 32 < ((L + 3) & ~3)) {  // rows the attention reads: keys 0 .. L rounded up to 4
    const uint32_t tl = tmem + (uint32_t(warp * 32) << 16);
    for (int c0 = 0; c0 < 192; c0 += 32) {
      uint32_t r[32];
      tmem_ld16(tl + c0, r);
      tmem_ld16(tl + c0 + 16, r + 16);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = c0 + j;
        dm[n * 128 + tid] = fmaf(float(int(r[j])), as * s_ws[n], s_bias[n]);
      }
    }
  }
  tc_fence_before();
  ok = __syncthreads_and(ok);
  tc_fence_after();

  const int unit = warp >> 1;  // warps 0-1: head 2y, warps 2-3: head 2y + 1
  const int h = 2 * y + unit;
  const int j = (warp & 1) * 32 + (tid & 31);
  if (ok) {
    const float scale = 1.0f / sqrtf(32.0f);
    float q[2][32];
    float* out[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int qi = j + 64 * u;
      const bool active = qi < L;
      const int qc = active ? qi : L - 1;
#pragma unroll
      for (int d = 0; d < 32; ++d) q[u][d] = dm[(unit * 32 + d) * 128 + qc] * scale;
      out[u] = active ? a.out + size_t(s0 + qi) * kHidden + h * 32 : nullptr;
    }
    attend_rows_dm<2>(q, dm + (64 + unit * 32) * 128, dm + (128 + unit * 32) * 128, 128, L,
                      tmem + (uint32_t(warp * 32) << 16), 128, out);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// Attention for few (sequence, head) pairs (single sequences: the latency path). The TMEM kernels
// hold one query per thread, so a 32-token sequence gives 12 CTAs of one warp and a 512-token one 48
// CTAs; here four lanes share a query, so each CTA (one sequence, one head, QT queries) has 4 QT
// threads and no TMEM. Sub-lane sl of a query computes the scores and exponentials of the keys
// whose softmax-sum slots it owns -- in every full 16-key chunk t0 the keys t0 + 2sl, t0 + 2sl + 1
// (slots 2sl, 2sl + 1 of the first 8-lane accumulator) and t0 + 8 + 2sl, t0 + 9 + 2sl (the second),
// in the trailing 8-key chunk L16 + 2sl, L16 + 2sl + 1, and the tail keys L8 + sl + 4k (scalar exp,
// added after the tree) -- so each of the reference's 16 sum chains stays in one thread, in order;
// the hsum256 tree of the 8 lanes runs over two shuffles. The weighted sum: sub-lane sl owns dims
// 8sl .. 8sl + 7, both the even- and odd-key accumulators, over all keys in order. K and V are
// staged dim-major with an odd-stride pitch P = 4k + 1, so that the four sub-lanes' reads fall in
// different banks; the scores, then exponentials, of the CTA's queries live in shared memory.
// Longest sequence the kernel takes: at 96-128 keys the TMEM kernels' one query per thread is faster
// for a single sequence, at 512 keys much faster (48 CTAs of 16 warps against 192 of 4).
constexpr int kLatMaxLen = 64;
__host__ __device__ constexpr int lat_pitch(int L) { return ((L + 3) & ~3) + 1; }
__host__ __device__ constexpr size_t lat_smem_bytes(int L, int QT) { return size_t(64 + QT) * lat_pitch(L) * 4; }

//
// QUANT: launched as clusters of the 12 heads of one (sequence, tile); the context rows are also
// quantized here (smooth_quantize_row, src/simd_math.rs:584-649, as k_smooth_quant does): each
// CTA sends its heads' partial row maxima max|ctx * inv_s| into every peer's shared memory with
// st.async, then quantizes its 32 columns with the row's maximum over all 384.
template <int QT, bool QUANT>
__global__ void __launch_bounds__(4 * QT) k_attention_lat(AttnArgs a) {
  pdl_trigger();
  extern __shared__ float4 smem4[];
  __shared__ float rmx[QUANT ? kHeads : 1][QT];  // QUANT: partial row maxima of the 12 heads
  __shared__ uint64_t rbar;
  const int s = blockIdx.x;
  const int h = blockIdx.y;
  const int tile = blockIdx.z;
  const int tid = threadIdx.x;
  if constexpr (QUANT) {  // the peers' barriers exist before any st.async
    if (tid == 0) {
      mbar_init(&rbar, 1);
      fence_mbar_init();
    }
    cluster_arrive_release();
    cluster_wait_acquire();
  }
  pdl_wait();
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  // the 12 CTAs of a cluster share the sequence and the tile: these exits are cluster-uniform
  if (a.skip_from > 0 && L >= a.skip_from) return;  // another kernel takes these sequences
  if (L <= 0 || L > a.max_len) {
    if (tid == 0 && tile == 0 && h == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  if (tile * QT >= L) return;
  const int P = lat_pitch(L);
  float* kd = reinterpret_cast<float*>(smem4);  // [32][P]: dim d of key t at d * P + t
  float* vd = kd + 32 * P;                      // [32][P]
  float* es = vd + 32 * P;                      // [QT][P]: scores, then exponentials, of the tile's queries
  const int kc = a.k_col + 32 * h, vc = a.v_col + 32 * h;
  for (int i = tid; i < 32 * L; i += 4 * QT) {  // keys fastest: coalesced in the tile-transposed layout
    const int d = i / L, t = i - d * L;
    kd[d * P + t] = ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t, kc + d);
    vd[d * P + t] = ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t, vc + d);
  }
  const int ql = tid >> 2, sl = tid & 3;
  const int qi = tile * QT + ql;
  const bool active = qi < L;
  float q[32];
  load_query(a, s0 + (active ? qi : L - 1), h, q);
  __syncthreads();
  float* er = es + ql * P;
  const unsigned full = 0xffffffffu;
  float cx[8];
  attend_query_lanes4(q, kd, vd, P, er, L, sl, cx);
  if constexpr (!QUANT) {
    if (active) {
      float4* o = reinterpret_cast<float4*>(a.out + size_t(s0 + qi) * kHidden + h * 32 + 8 * sl);
      o[0] = make_float4(cx[0], cx[1], cx[2], cx[3]);
      o[1] = make_float4(cx[4], cx[5], cx[6], cx[7]);
    }
  } else {
    const float* ivs = a.quant_inv_s + h * 32 + 8 * sl;
    float vmax = 1e-8f;
#pragma unroll
    for (int k = 0; k < 8; ++k) vmax = fmaxf(vmax, fabsf(cx[k] * ivs[k]));
    vmax = fmaxf(vmax, __shfl_xor_sync(full, vmax, 1));
    vmax = fmaxf(vmax, __shfl_xor_sync(full, vmax, 2));
    if (tid == 0) mbar_arrive_expect_tx(&rbar, kHeads * QT * 4);
    if (sl == 0)
      for (uint32_t pr = 0; pr < uint32_t(kHeads); ++pr)
        st_async_f32(map_peer(&rmx[h][ql], pr), vmax, map_peer(&rbar, pr));
    const bool got = mbar_wait(&rbar, 0, a.err, DEV_ERR_TIMEOUT_EPILOGUE);
    float max_abs = rmx[0][ql];
#pragma unroll
    for (int g = 1; g < kHeads; ++g) max_abs = fmaxf(max_abs, rmx[g][ql]);
    const float inv_scale = 127.0f / max_abs;
    if (active && got) {
      uint32_t w0 = 0, w1 = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        w0 |= (uint32_t(quant_i8(cx[k] * (ivs[k] * inv_scale))) & 0xFFu) << (8 * k);
        w1 |= (uint32_t(quant_i8(cx[4 + k] * (ivs[4 + k] * inv_scale))) & 0xFFu) << (8 * k);
      }
      *reinterpret_cast<uint2*>(a.quant_q + size_t(s0 + qi) * kHidden + h * 32 + 8 * sl) = make_uint2(w0, w1);
      if (h == 0 && sl == 0) a.quant_scale[s0 + qi] = max_abs / 127.0f;
    }
    // no CTA leaves while a peer may still write into it
    cluster_arrive_release();
    cluster_wait_acquire();
  }
}

// Few (sequence, head) pairs of more than 64 keys (single sequences of 65-512 tokens and small
// batches on the latency path): eight lanes per query, one CTA per (sequence, head, tile of qt
// queries), qt chosen by the launch so that the tiles of all pairs fill the SMs about once. The
// TMEM kernels keep one query per thread and so give a 512-token sequence 48 tiles of 128 queries;
// here 12 tiles of 44 queries per head are 144 CTAs of 11 warps.
//
// The chains are attend_query_lanes8's (so the same bits as every other exact kernel): sub-lane s
// owns slot s of both 8-lane sum accumulators (keys t0 + s and t0 + 8 + s of every full 16-key
// chunk, L16 + s of the trailing 8-key chunk, tail key L8 + s) and dims 4s .. 4s + 3 of the even /
// odd weighted-sum accumulators. K and V are staged key-major (32 dims of a key in a row of 128
// bytes) with the row's 16-byte chunks XOR-swizzled by the key's low 3 bits, so that a lane reads 4
// dims in one 16-byte load: the 8 sub-lanes reading 8 consecutive keys at one dim chunk, or one key's
// 8 chunks, touch 8 different bank groups. The scores, then exponentials, of the CTA's queries use a
// pitch of 8 mod 32 floats (the 4 queries of a warp read 4 different banks).
__host__ __device__ constexpr int lat8_er_pitch(int L) { return ((L + 31) & ~31) + 8; }
__host__ __device__ constexpr size_t lat8_smem_bytes(int L, int qt) {
  return (size_t(64) * ((L + 7) & ~7) + size_t(qt) * lat8_er_pitch(L)) * 4;
}
// float index of dims 4j .. 4j + 3 of key t in a key-major swizzled K / V block
__device__ __forceinline__ int km_index(int t, int j) { return t * 32 + ((j ^ (t & 7)) << 2); }

__device__ __forceinline__ void attend_query_lanes8_km(const float (&q)[32], const float* __restrict__ kk,
                                                       const float* __restrict__ vv, float* er, int L, int s,
                                                       float (&cx)[4]) {
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;
  const unsigned full = 0xffffffffu;

  auto score = [&](int t) -> float {  // score_pair's order for one key
    float k[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 c = *reinterpret_cast<const float4*>(kk + km_index(t, j));
      k[4 * j] = c.x;
      k[4 * j + 1] = c.y;
      k[4 * j + 2] = c.z;
      k[4 * j + 3] = c.w;
    }
    float s8[8];
#pragma unroll
    for (int l = 0; l < 8; ++l)
      s8[l] = fmaf(q[8 + l], k[8 + l], q[l] * k[l]) + fmaf(q[24 + l], k[24 + l], q[16 + l] * k[16 + l]);
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
  const float v = c0 + c1;  // hsum256 of v[m] = acc0[m] + acc1[m]: sub-lane s holds v[s]
  const float a = v + __shfl_down_sync(full, v, 4);
  const float b = a + __shfl_down_sync(full, a, 1);
  float sum = b + __shfl_down_sync(full, b, 2);
  __syncwarp();
  if (s == 0)
    for (int t = L8; t < L; ++t) sum = sum + er[t];  // the tail keys in order, after the tree
  const float inv = __shfl_sync(full, 1.0f / sum, (threadIdx.x & 31) & ~7);

  // pass 3: weighted sum of V, dims 4s .. 4s + 3; even keys to the first accumulator
  float acc_e[4], acc_o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) acc_e[k] = acc_o[k] = 0.0f;
  int t = 0;
  for (; t + 1 < L; t += 2) {
    const float2 e2 = *reinterpret_cast<const float2*>(er + t);
    const float p0 = e2.x * inv, p1 = e2.y * inv;
    const float4 v0 = *reinterpret_cast<const float4*>(vv + km_index(t, s));
    const float4 v1 = *reinterpret_cast<const float4*>(vv + km_index(t + 1, s));
    acc_e[0] = fmaf(v0.x, p0, acc_e[0]);
    acc_e[1] = fmaf(v0.y, p0, acc_e[1]);
    acc_e[2] = fmaf(v0.z, p0, acc_e[2]);
    acc_e[3] = fmaf(v0.w, p0, acc_e[3]);
    acc_o[0] = fmaf(v1.x, p1, acc_o[0]);
    acc_o[1] = fmaf(v1.y, p1, acc_o[1]);
    acc_o[2] = fmaf(v1.z, p1, acc_o[2]);
    acc_o[3] = fmaf(v1.w, p1, acc_o[3]);
  }
  if (t < L) {
    const float p0 = er[t] * inv;
    const float4 v0 = *reinterpret_cast<const float4*>(vv + km_index(t, s));
    acc_e[0] = fmaf(v0.x, p0, acc_e[0]);
    acc_e[1] = fmaf(v0.y, p0, acc_e[1]);
    acc_e[2] = fmaf(v0.z, p0, acc_e[2]);
    acc_e[3] = fmaf(v0.w, p0, acc_e[3]);
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) cx[k] = acc_e[k] + acc_o[k];
}

__global__ void __launch_bounds__(512) k_attention_lat8(AttnArgs a, int qt) {
  pdl_trigger();
  extern __shared__ float4 smem4[];
  const int s = blockIdx.x;
  const int h = blockIdx.y;
  const int tile = blockIdx.z;
  const int tid = threadIdx.x;
  pdl_wait();
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  if (a.skip_from > 0 && L >= a.skip_from) return;  // another kernel takes these sequences
  if (L <= 0 || L > a.max_len) {
    if (tid == 0 && tile == 0 && h == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  if (tile * qt >= L) return;
  const int rows = (L + 7) & ~7;
  float* kk = reinterpret_cast<float*>(smem4);  // [rows][32] key-major, swizzled
  float* vv = kk + rows * 32;                   // [rows][32]
  float* es = vv + rows * 32;                   // [qt][Pe]: scores, then exponentials
  const int Pe = lat8_er_pitch(L);
  const int kc = a.k_col + 32 * h, vc = a.v_col + 32 * h;
  // warp w copies columns w, w + nwarps, ... (K dims 0-31, then V dims), its lanes consecutive keys
  // (coalesced in the tile-transposed layout): 4-byte asynchronous copies, all in flight at once
  const int nwarps = blockDim.x >> 5, lane = tid & 31;
  for (int c = tid >> 5; c < 64; c += nwarps) {
    const int d = c & 31;
    float* dst = (c < 32 ? kk : vv) + (d & 3);
    const int col = (c < 32 ? kc : vc) + d;
    for (int t = lane; t < L; t += 32) {
      const float* src = a.kv_tt ? a.kv + tt_index(s0 + t, col, a.kv_C) : a.kv + size_t(s0 + t) * a.kv_C + col;
      cp_async4(dst + km_index(t, d >> 2), src, 4u);
    }
  }
  cp_async_wait_all();
  const int ql = tid >> 3, sl = tid & 7;
  const int qi = tile * qt + ql;
  const bool active = qi < L;
  float q[32];
  load_query(a, s0 + (active ? qi : L - 1), h, q);
  __syncthreads();
  float cx[4];
  attend_query_lanes8_km(q, kk, vv, es + ql * Pe, L, sl, cx);
  if (active)
    *reinterpret_cast<float4*>(a.out + size_t(s0 + qi) * kHidden + h * 32 + 4 * sl) =
        make_float4(cx[0], cx[1], cx[2], cx[3]);
}

// NWG warpgroups per 128-query tile: warps w, w + 4, ... share TMEM lane quadrant w & 3 (the same
// queries). Scores and exponentials: group g takes keys t0 + g KPG .. t0 + (g + 1) KPG - 1 of
// every 16-key chunk (KPG = 16 / NWG), so each of the reference's 16 sum slots is summed in order
// by one group; P.V: group g accumulates dims g DPG .. (g + 1) DPG - 1 (DPG = 32 / NWG) over all
// keys in order.
// DSPLIT > 1 (few (sequence, head) pairs: single sequences): z = tile * DSPLIT + part,
// and CTA `part` runs the scores and exponentials of its tile (the same work in every part) but the
// weighted sum only for dims part * 32 / DSPLIT .. + 32 / DSPLIT - 1, so a tile's attention spreads
// over DSPLIT SMs.
template <int NWG, int MINB, int DSPLIT = 1>
__global__ void __launch_bounds__(128 * NWG, MINB) k_attention_wide(AttnArgs a) {
  pdl_trigger();
  pdl_wait();
  constexpr int KPG = 16 / NWG;           // keys of a 16-key chunk per group (8 or 4)
  constexpr int DPG = 32 / NWG / DSPLIT;  // dims of V per group
  static_assert(DPG >= 4, "a group's dims are stored as float4");
  extern __shared__ float4 smem4[];
  __shared__ uint32_t tmem_slot;
  __shared__ float xmx[NWG][128];
  __shared__ float xsl[16][128];  // the 16 slot sums of every query
  int s, h, bz;
  tile_major_block(s, h, bz);
  const int tile = bz / DSPLIT;
  const int dbase = (bz % DSPLIT) * (32 / DSPLIT);  // first dim of this CTA's weighted sum
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int grp = warp >> 2;
  const int qt = tid & 127;
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  if (a.skip_from > 0 && L >= a.skip_from) return;  // another kernel takes these sequences
  if (L <= 0 || L > a.max_len) {
    if (tid == 0 && tile == 0 && h == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  if (tile * 128 >= L) return;
  const uint32_t cols = tmem_cols_for_len(L);
  if (warp == 0) {
    tmem_alloc(&tmem_slot, cols);
    tmem_relinquish();
  }
  const int qi = tile * 128 + qt;
  const bool active = qi < L;
  const int qrow = s0 + (active ? qi : L - 1);
  float q[32];
  load_query(a, qrow, h, q);  // requested before the K / V staging, in flight with it
  const int pairs = (L + 1) >> 1;
  float2* kp = reinterpret_cast<float2*>(smem4);
  float2* vp = kp + pairs * KPS;
  stage_kv_pairs(a, s0, L, h, kp, vp);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tl = tmem_slot + (uint32_t((warp & 3) * 32) << 16);
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;
  const int ko = KPG * grp;  // this group's keys within a 16-key chunk
  uint32_t r[16];

  // pass 1: scores -> TMEM and their max
  float mx = -INFINITY;
  {
    for (int t0 = 0; t0 < L; t0 += 16) {
#pragma unroll
      for (int j = 0; j < KPG / 2; ++j) {
        const int t = t0 + ko + 2 * j;
        float2 sp = f2(0.0f, 0.0f);
        if (t < L) {
          sp = score_pair(q, kp + (t >> 1) * KPS, t < L4);
          mx = fmaxf(mx, sp.x);
          if (t + 1 < L) mx = fmaxf(mx, sp.y);
        }
        r[2 * j] = __float_as_uint(sp.x);
        r[2 * j + 1] = __float_as_uint(sp.y);
      }
      if constexpr (KPG == 8) tmem_st8(tl + t0 + ko, r);
      else tmem_st4(tl + t0 + ko, r);
    }
  }
  tmem_st_wait();
  xmx[grp][qt] = mx;
  __syncthreads();
#pragma unroll
  for (int g = 0; g < NWG; ++g) mx = fmaxf(mx, xmx[g][qt]);
  const float2 neg_mx = f2(-mx, -mx);

  // pass 2: exponentials -> TMEM; this group's sum slots (and, for slots 0-7, the trailing
  // 8-key chunk) accumulated in chunk order
  float2 vs[KPG / 2];
#pragma unroll
  for (int j = 0; j < KPG / 2; ++j) vs[j] = f2(0.0f, 0.0f);
  int t0 = 0;
  for (; t0 + 64 <= L16; t0 += 64) {  // four full chunks per TMEM round trip, summed in chunk order
    uint32_t rq[4][KPG];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if constexpr (KPG == 8) tmem_ld8(tl + t0 + 16 * c + ko, rq[c]);
      else tmem_ld4(tl + t0 + 16 * c + ko, rq[c]);
    }
    tmem_ld_wait();
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int j = 0; j < KPG / 2; ++j) {
        const float2 e = cw_exp2(add2(f2(__uint_as_float(rq[c][2 * j]), __uint_as_float(rq[c][2 * j + 1])), neg_mx));
        vs[j] = add2(vs[j], e);
        rq[c][2 * j] = __float_as_uint(e.x);
        rq[c][2 * j + 1] = __float_as_uint(e.y);
      }
      if constexpr (KPG == 8) tmem_st8(tl + t0 + 16 * c + ko, rq[c]);
      else tmem_st4(tl + t0 + 16 * c + ko, rq[c]);
    }
  }
  for (; t0 < L; t0 += 16) {
    if constexpr (KPG == 8) tmem_ld8(tl + t0 + ko, r);
    else tmem_ld4(tl + t0 + ko, r);
    tmem_ld_wait();
    if (t0 + 16 <= L16) {
#pragma unroll
      for (int j = 0; j < KPG / 2; ++j) {
        const float2 e = cw_exp2(add2(f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), neg_mx));
        vs[j] = add2(vs[j], e);
        r[2 * j] = __float_as_uint(e.x);
        r[2 * j + 1] = __float_as_uint(e.y);
      }
    } else {
#pragma unroll
      for (int j = 0; j < KPG / 2; ++j) {
        const int t = t0 + ko + 2 * j;
        const float2 x = add2(f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), neg_mx);
        float2 e;
        if (ko < 8 && t + 1 < L8) {  // the trailing 8-key chunk (keys L16 .. L16 + 7): slots 0-7
          e = cw_exp2(x);
          vs[j] = add2(vs[j], e);
        } else {  // the last L % 8 keys: scalar exp, summed after the tree
          e = f2(t < L ? scalar_expf(x.x) : 0.0f, t + 1 < L ? scalar_expf(x.y) : 0.0f);
        }
        r[2 * j] = __float_as_uint(e.x);
        r[2 * j + 1] = __float_as_uint(e.y);
      }
    }
    if constexpr (KPG == 8) tmem_st8(tl + t0 + ko, r);
    else tmem_st4(tl + t0 + ko, r);
  }
  tmem_st_wait();
#pragma unroll
  for (int j = 0; j < KPG / 2; ++j) {
    xsl[ko + 2 * j][qt] = vs[j].x;
    xsl[ko + 2 * j + 1][qt] = vs[j].y;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (grp == 0) {
    float v8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v8[j] = xsl[j][qt] + xsl[8 + j][qt];  // acc0 + acc1
    float sum = tree8(v8);
    if (L8 < L) {  // ((tree + e[L8]) + e[L8 + 1]) + ..., the keys re-read from TMEM
      tmem_ld16(tl + L16, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (L16 + j >= L8 && L16 + j < L) sum = sum + __uint_as_float(r[j]);
    }
    xmx[0][qt] = 1.0f / sum;
  }
  __syncthreads();
  const float inv = xmx[0][qt];
  const float2 inv2 = f2(inv, inv);

  // pass 3: probabilities and the weighted sum of this group's dims of V
  float2 acc[DPG];
#pragma unroll
  for (int d = 0; d < DPG; ++d) acc[d] = f2(0.0f, 0.0f);
  for (t0 = 0; t0 + 32 <= L; t0 += 32) {  // two full chunks per TMEM round trip, keys in order
    uint32_t rq[32];
    tmem_ld16(tl + t0, rq);
    tmem_ld16(tl + t0 + 16, rq + 16);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 p = mul2(f2(__uint_as_float(rq[2 * j]), __uint_as_float(rq[2 * j + 1])), inv2);
      const float4* v4 = reinterpret_cast<const float4*>(vp + ((t0 >> 1) + j) * KPS + dbase + DPG * grp);
#pragma unroll
      for (int i = 0; i < DPG / 2; ++i) {
        const float4 vv = v4[i];
        acc[2 * i] = fma2(f2(vv.x, vv.y), p, acc[2 * i]);
        acc[2 * i + 1] = fma2(f2(vv.z, vv.w), p, acc[2 * i + 1]);
      }
    }
  }
  for (; t0 < L; t0 += 16) {
    tmem_ld16(tl + t0, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int t = t0 + 2 * j;
      if (t + 1 < L) {
        const float2 p = mul2(f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), inv2);
        const float4* v4 = reinterpret_cast<const float4*>(vp + (t >> 1) * KPS + dbase + DPG * grp);
#pragma unroll
        for (int i = 0; i < DPG / 2; ++i) {
          const float4 vv = v4[i];
          acc[2 * i] = fma2(f2(vv.x, vv.y), p, acc[2 * i]);
          acc[2 * i + 1] = fma2(f2(vv.z, vv.w), p, acc[2 * i + 1]);
        }
      } else if (t < L) {  // odd L: the last key goes to the even accumulator
        const float pa = __uint_as_float(r[2 * j]) * inv;
        const float2* v = vp + (t >> 1) * KPS + dbase + DPG * grp;
#pragma unroll
        for (int d = 0; d < DPG; ++d) acc[d].x = fmaf(v[d].x, pa, acc[d].x);
      }
    }
  }
  if (active) {
    float4* o = reinterpret_cast<float4*>(a.out + size_t(s0 + qi) * kHidden + h * 32 + dbase + DPG * grp);
#pragma unroll
    for (int i = 0; i < DPG / 4; ++i)
      o[i] = make_float4(acc[4 * i].x + acc[4 * i].y, acc[4 * i + 1].x + acc[4 * i + 1].y,
                         acc[4 * i + 2].x + acc[4 * i + 2].y, acc[4 * i + 3].x + acc[4 * i + 3].y);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem_slot, cols);
}

// One CTA (128 threads) per (sequence, head): the single [CLS] query (row s of q / out) over the
// sequence's keys. Thread t takes keys t, t + 128, ...: it loads each key's K and V row (the 32 dims
// of a key are 32 coalesced loads across the CTA's threads in the tile-transposed layout, all in
// flight together), computes the score in the reference's order and stages V in shared memory.
// Warp 0 then runs the reference's 16 exp-sum chains and tree; the weighted sum takes 64 threads,
// one per (dim, even / odd key) accumulator, each over its keys in order.
// Shared memory: q (32), scores / exponentials (max_len), V rows (max_len x 33), two reduction slots.
__host__ __device__ constexpr size_t cls_smem_floats(int max_len) { return 32 + 8 + size_t(max_len) * 34 + 64; }

// Few (sequence, head) pairs of long sequences: k_attention_wide's passes on tiles of 32 queries
// (thread = query, so every K / V load is a warp-wide broadcast), with the scores, then
// exponentials, in shared memory instead of TMEM: a 512-token sequence gives 12 x 16 CTAs
// instead of 48. NW = 8 warps: warp g takes the key pair t0 + 2g, t0 + 2g + 1 of every 16-key
// chunk in the scores pass and in the exponentials pass -- the sum slots 2g, 2g + 1, in chunk
// order, as k_attention_wide's groups do -- and dims 4g .. 4g + 3 of the weighted sum, over all
// keys in order. NW = 16 (twice the warps to hide shared-memory latency): warps g and g + 8 take
// key pair g of alternate chunks for the scores, warp g alone sum slot g (key t0 + g of every
// chunk) for the exponentials, and dims 2g, 2g + 1 of the weighted sum. Either way every chain the
// reference keeps runs in one thread in its order, so the same bits. Score rows use a pitch of
// 2 mod 32 floats (a warp's 32 float2 accesses take the minimum two wavefronts).
__host__ __device__ constexpr int narrow_er_pitch(int L) { return ((L + 31) & ~31) + 2; }
__host__ __device__ constexpr size_t narrow_smem_bytes(int L) {
  return size_t((L + 1) >> 1) * KPS * 8 * 2 + size_t(32) * narrow_er_pitch(L) * 4;
}

template <int NW>
__global__ void __launch_bounds__(32 * NW) k_attention_narrow(AttnArgs a) {
  static_assert(NW == 8 || NW == 16, "8 or 16 warps");
  constexpr int DPG = 32 / NW;  // dims of the weighted sum per warp
  pdl_trigger();
  pdl_wait();
  extern __shared__ float4 smem4[];
  __shared__ float xmx[NW][32];
  __shared__ float xsl[16][32];  // the 16 slot sums of every query
  const int s = blockIdx.x;
  const int h = blockIdx.y;
  const int tile = blockIdx.z;
  const int tid = threadIdx.x;
  const int g = tid >> 5;
  const int lane = tid & 31;
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  if (a.skip_from > 0 && L >= a.skip_from) return;  // another kernel takes these sequences
  if (L <= 0 || L > a.max_len) {
    if (tid == 0 && tile == 0 && h == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  if (tile * 32 >= L) return;
  const int qi = tile * 32 + lane;
  const bool active = qi < L;
  float q[32];
  load_query(a, s0 + (active ? qi : L - 1), h, q);  // in flight with the K / V staging
  const int pairs = (L + 1) >> 1;
  float2* kp = reinterpret_cast<float2*>(smem4);
  float2* vp = kp + pairs * KPS;
  float* er = reinterpret_cast<float*>(vp + pairs * KPS) + lane * narrow_er_pitch(L);
  stage_kv_pairs(a, s0, L, h, kp, vp);
  __syncthreads();
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;

  // pass 1: scores and their max (key pair ko of the chunks this warp takes)
  const int ko = 2 * (g & 7);
  const int c_first = 16 * (g >> 3), c_step = 16 * (NW / 8);
  float mx = -INFINITY;
  int t0 = c_first;
#pragma unroll 4
  for (; t0 + 16 <= L4; t0 += c_step) {  // both keys inside complete groups of 4
    const float2 sp = score_pair(q, kp + ((t0 + ko) >> 1) * KPS, true);
    mx = fmaxf(mx, fmaxf(sp.x, sp.y));
    *reinterpret_cast<float2*>(er + t0 + ko) = sp;
  }
  for (; t0 < L; t0 += c_step) {
    const int t = t0 + ko;
    if (t < L) {
      const float2 sp = score_pair(q, kp + (t >> 1) * KPS, t < L4);
      mx = fmaxf(mx, sp.x);
      if (t + 1 < L) mx = fmaxf(mx, sp.y);
      *reinterpret_cast<float2*>(er + t) = sp;
    }
  }
  xmx[g][lane] = mx;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < NW; ++w) mx = fmaxf(mx, xmx[w][lane]);

  // pass 2: exponentials; this warp's sum slots (and, for slots 0-7, the trailing 8-key chunk)
  // accumulated in chunk order; the last L % 8 keys by scalar exp, summed after the tree
  if constexpr (NW == 8) {
    const float2 neg_mx = f2(-mx, -mx);
    float2 vs = f2(0.0f, 0.0f);
#pragma unroll 4
    for (t0 = 0; t0 + 16 <= L16; t0 += 16) {
      float2* ep = reinterpret_cast<float2*>(er + t0 + ko);
      const float2 e = cw_exp2(add2(*ep, neg_mx));
      vs = add2(vs, e);
      *ep = e;
    }
    const int t = t0 + ko;  // t0 == L16: the partial chunk
    if (t < L) {
      float2* ep = reinterpret_cast<float2*>(er + t);
      const float2 x = add2(*ep, neg_mx);
      float2 e;
      if (ko < 8 && t + 1 < L8) {  // the trailing 8-key chunk (keys L16 .. L16 + 7): slots 0-7
        e = cw_exp2(x);
        vs = add2(vs, e);
      } else {
        e = f2(scalar_expf(x.x), t + 1 < L ? scalar_expf(x.y) : 0.0f);
      }
      *ep = e;
    }
    xsl[ko][lane] = vs.x;
    xsl[ko + 1][lane] = vs.y;
  } else {
    float vs = 0.0f;
#pragma unroll 4
    for (t0 = 0; t0 + 16 <= L16; t0 += 16) {
      const float e = cw_exp(er[t0 + g] - mx);
      vs = vs + e;
      er[t0 + g] = e;
    }
    const int t = t0 + g;  // t0 == L16: the partial chunk
    if (t < L) {
      const float x = er[t] - mx;
      float e;
      if (g < 8 && t < L8) {  // the trailing 8-key chunk: slots 0-7
        e = cw_exp(x);
        vs = vs + e;
      } else {
        e = scalar_expf(x);
      }
      er[t] = e;
    }
    xsl[g][lane] = vs;
  }
  __syncthreads();
  if (g == 0) {
    float v8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v8[j] = xsl[j][lane] + xsl[8 + j][lane];  // acc0 + acc1
    float sum = tree8(v8);
    for (int t = L8; t < L; ++t) sum = sum + er[t];  // the tail keys in order, after the tree
    xmx[0][lane] = 1.0f / sum;
  }
  __syncthreads();
  const float inv = xmx[0][lane];
  const float2 inv2 = f2(inv, inv);

  // pass 3: probabilities and the weighted sum of this warp's dims; lane x = even keys
  float2 acc[DPG];
#pragma unroll
  for (int d = 0; d < DPG; ++d) acc[d] = f2(0.0f, 0.0f);
  const int dg = DPG * g;
  int t = 0;
#pragma unroll 4
  for (; t + 1 < L; t += 2) {
    const float2 p = mul2(*reinterpret_cast<const float2*>(er + t), inv2);
    const float4* v4 = reinterpret_cast<const float4*>(vp + (t >> 1) * KPS + dg);
#pragma unroll
    for (int i = 0; i < DPG / 2; ++i) {
      const float4 va = v4[i];
      acc[2 * i] = fma2(f2(va.x, va.y), p, acc[2 * i]);
      acc[2 * i + 1] = fma2(f2(va.z, va.w), p, acc[2 * i + 1]);
    }
  }
  if (t < L) {  // odd L: the last key goes to the even accumulator
    const float pa = er[t] * inv;
    const float2* v = vp + (t >> 1) * KPS + dg;
#pragma unroll
    for (int d = 0; d < DPG; ++d) acc[d].x = fmaf(v[d].x, pa, acc[d].x);
  }
  if (active) {
    float* o = a.out + size_t(s0 + qi) * kHidden + h * 32 + dg;
    if constexpr (DPG == 4)
      *reinterpret_cast<float4*>(o) =
          make_float4(acc[0].x + acc[0].y, acc[1].x + acc[1].y, acc[2].x + acc[2].y, acc[3].x + acc[3].y);
    else
      *reinterpret_cast<float2*>(o) = make_float2(acc[0].x + acc[0].y, acc[1].x + acc[1].y);
  }
}

// k_attention_narrow for one sequence that starts a 128-row tile of the tile-transposed Q | K | V
// (the latency path's single sequence): K and V are staged dim-major, exactly as they lie in the
// tile-transposed layout -- dims 32h .. 32h + 31 of a 128-row tile are 16 KB in a row -- by two
// bulk copies per tile (no multicast) instead of the key-pair layout's per-thread copies, whose issue
// dominated the kernel at 257-512 keys. A 16-byte load is one dim of four keys (score_quad), so the
// scores pass takes quads: warp g the quad g % 4 of the chunks it owns; the exponentials and the
// weighted sum keep k_attention_narrow's chain ownership, so the same bits.
__host__ __device__ constexpr int narrow_dm_er_pitch(int L) { return ((L + 31) & ~31) + 4; }
__host__ __device__ constexpr size_t narrow_dm_smem_bytes(int L, int qt = 32) {
  return size_t((L + 127) >> 7) * 2 * 32 * 128 * 4 + size_t(qt) * narrow_dm_er_pitch(L) * 4;
}
__device__ __forceinline__ int dm_index(int d, int t) { return ((t >> 7) << 12) + (d << 7) + (t & 127); }

// QPT = 2 (one row of warps): each thread takes the queries of slots lane and 32 + lane, so every
// staged K / V load feeds two queries (half the shared-memory loads per product of QPT = 1, whose
// passes are bound by them at 385-512 keys); a thread whose second slot lies past the tile computes
// that query's scores from a copy of its first query and discards them.
template <int NW, int ROWS, int QPT = 1>
__global__ void __launch_bounds__(32 * NW * ROWS) k_attention_narrow_dm(AttnArgs a, int qt) {
  static_assert(NW == 8 || NW == 16, "8 or 16 warps per row of queries");
  static_assert(QPT == 1 || (QPT == 2 && ROWS == 1), "two queries per thread take one row of warps");
  constexpr int DPG = 32 / NW;
  constexpr int NR = ROWS * QPT;  // rows of 32 query slots per tile
  pdl_trigger();
  pdl_wait();
  extern __shared__ float4 smem4[];
  __shared__ float xmx[NR][NW][32];
  __shared__ float xsl[NR][16][32];
  __shared__ uint64_t kv_bar;
  const int h = blockIdx.y;
  const int tile = blockIdx.z;
  const int tid = threadIdx.x;
  const int wid = tid >> 5;
  const int g = wid % NW;   // warp within its row of queries
  const int rw = wid / NW;  // row of warps (QPT = 1): slots 32 rw .. 32 rw + 31 of the tile
  const int lane = tid & 31;
  const int s0 = int(a.cu[blockIdx.x]);
  const int L = int(a.cu[blockIdx.x + 1]) - s0;
  if (a.skip_from > 0 && L >= a.skip_from) return;
  if (L <= 0 || L > a.max_len) {
    if (tid == 0 && tile == 0 && h == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  if (tile * qt >= L) return;
  const bool bulk = a.kv_tt && !(s0 & 127);
  const int ntile = (L + 127) >> 7;
  float* kd = reinterpret_cast<float*>(smem4);  // [ntile][32][128]
  float* vd = kd + ntile * 4096;
  const int Pe = narrow_dm_er_pitch(L);
  // query u of this thread: slot 32 (rw + u) + lane of the tile, row R = rw + u of xmx / xsl
  bool has[QPT], active[QPT];
  int qi[QPT];
  float* er[QPT];
#pragma unroll
  for (int u = 0; u < QPT; ++u) {
    const int slot = 32 * (rw + u) + lane;
    has[u] = slot < qt;  // the tile's last row of queries may be partial
    qi[u] = tile * qt + slot;
    active[u] = has[u] && qi[u] < L;
    er[u] = vd + ntile * 4096 + (has[u] ? slot : 0) * Pe;
  }
  if (bulk && tid == 0) {
    mbar_init(&kv_bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&kv_bar, uint32_t(ntile) * 2 * 16384);
    for (int j = 0; j < ntile; ++j) {
      const float* blk = a.kv + size_t((s0 >> 7) + j) * a.kv_C * 128;
      bulk_load(kd + j * 4096, blk + size_t(a.k_col + 32 * h) * 128, 16384, &kv_bar);
      bulk_load(vd + j * 4096, blk + size_t(a.v_col + 32 * h) * 128, 16384, &kv_bar);
    }
  }
  float q[QPT][32];
#pragma unroll
  for (int u = 0; u < QPT; ++u) {
    // a slot past the tile takes the first query's row (its results are discarded)
    const int qr = active[u] ? qi[u] : (active[0] ? qi[0] : L - 1);
    load_query(a, s0 + qr, h, q[u]);
  }
  if (!bulk) {  // a sequence inside a tile: 4-byte asynchronous copies of its rows, all in flight
    const int nwarps = blockDim.x >> 5;
    for (int c = wid; c < 64; c += nwarps) {
      const int d = c & 31;
      const int col = (c < 32 ? a.k_col : a.v_col) + 32 * h + d;
      float* dst = c < 32 ? kd : vd;
      for (int t = lane; t < L; t += 32)
        cp_async4(dst + dm_index(d, t),
                  a.kv_tt ? a.kv + tt_index(s0 + t, col, a.kv_C) : a.kv + size_t(s0 + t) * a.kv_C + col, 4u);
    }
    cp_async_wait_all();
  }
  __syncthreads();  // kv_bar initialised; per-thread copies complete
  const bool ok = !bulk || __syncthreads_and(mbar_wait(&kv_bar, 0, a.err, DEV_ERR_TIMEOUT_PRODUCER));
  if (!ok) {
    // the copies' bytes have not all landed: wait once more (bounded) before the CTA's shared
    // memory is released; nothing of this tile is written
    mbar_wait(&kv_bar, 0, a.err, DEV_ERR_TIMEOUT_PRODUCER);
    return;
  }
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;

  // pass 1: scores (quad g % 4 of the chunks this warp owns) and their max
  const int qo = 4 * (g & 3);
  const int c_first = 16 * (g >> 2), c_step = 16 * (NW / 4);
  float mx[QPT];
#pragma unroll
  for (int u = 0; u < QPT; ++u) mx[u] = -INFINITY;
  for (int t0 = c_first; has[0] && t0 < L; t0 += c_step) {
    const int t = t0 + qo;
    if (t >= L) continue;
    float2 sp[QPT][2];
    score_quad<QPT>(q, kd + dm_index(0, t), 128, t < L4, sp);
#pragma unroll
    for (int u = 0; u < QPT; ++u) {
      float4 v = make_float4(sp[u][0].x, sp[u][0].y, sp[u][1].x, sp[u][1].y);
      if (t + 4 <= L) {
        mx[u] = fmaxf(mx[u], fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
      } else {  // keys past the sequence: 0, outside the max
        mx[u] = fmaxf(mx[u], v.x);
        if (t + 1 < L) mx[u] = fmaxf(mx[u], v.y); else v.y = 0.0f;
        if (t + 2 < L) mx[u] = fmaxf(mx[u], v.z); else v.z = 0.0f;
        v.w = 0.0f;
      }
      if (u == 0 || has[u]) *reinterpret_cast<float4*>(er[u] + t) = v;
    }
  }
#pragma unroll
  for (int u = 0; u < QPT; ++u) xmx[rw + u][g][lane] = mx[u];
  __syncthreads();
#pragma unroll
  for (int u = 0; u < QPT; ++u)
#pragma unroll
    for (int w = 0; w < NW; ++w) mx[u] = fmaxf(mx[u], xmx[rw + u][w][lane]);

  // pass 2: as k_attention_narrow
  int t0;
#pragma unroll
  for (int u = 0; u < QPT; ++u) {
    const int L16r = has[u] ? L16 : 0, Lr = has[u] ? L : 0;
    if constexpr (NW == 8) {
      const int ko = 2 * g;
      const float2 neg_mx = f2(-mx[u], -mx[u]);
      float2 vs = f2(0.0f, 0.0f);
#pragma unroll 4
      for (t0 = 0; t0 + 16 <= L16r; t0 += 16) {
        float2* ep = reinterpret_cast<float2*>(er[u] + t0 + ko);
        const float2 e = cw_exp2(add2(*ep, neg_mx));
        vs = add2(vs, e);
        *ep = e;
      }
      const int t = t0 + ko;
      if (t < Lr) {
        float2* ep = reinterpret_cast<float2*>(er[u] + t);
        const float2 x = add2(*ep, neg_mx);
        float2 e;
        if (ko < 8 && t + 1 < L8) {
          e = cw_exp2(x);
          vs = add2(vs, e);
        } else {
          e = f2(scalar_expf(x.x), t + 1 < L ? scalar_expf(x.y) : 0.0f);
        }
        *ep = e;
      }
      xsl[rw + u][ko][lane] = vs.x;
      xsl[rw + u][ko + 1][lane] = vs.y;
    } else {
      float vs = 0.0f;
#pragma unroll 4
      for (t0 = 0; t0 + 16 <= L16r; t0 += 16) {
        const float e = cw_exp(er[u][t0 + g] - mx[u]);
        vs = vs + e;
        er[u][t0 + g] = e;
      }
      const int t = t0 + g;
      if (t < Lr) {
        const float x = er[u][t] - mx[u];
        float e;
        if (g < 8 && t < L8) {
          e = cw_exp(x);
          vs = vs + e;
        } else {
          e = scalar_expf(x);
        }
        er[u][t] = e;
      }
      xsl[rw + u][g][lane] = vs;
    }
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < QPT; ++u) {
    if (g == u && has[u]) {
      float v8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v8[j] = xsl[rw + u][j][lane] + xsl[rw + u][8 + j][lane];
      float sum = tree8(v8);
      for (int t = L8; t < L; ++t) sum = sum + er[u][t];
      xmx[rw + u][0][lane] = 1.0f / sum;
    }
  }
  __syncthreads();
  float2 inv2[QPT];
#pragma unroll
  for (int u = 0; u < QPT; ++u) {
    const float inv = xmx[rw + u][0][lane];
    inv2[u] = f2(inv, inv);
  }

  // pass 3: the weighted sum of dims DPG g .. DPG g + DPG - 1, four keys per 16-byte load; each
  // V load feeds the thread's QPT queries
  float2 acc[QPT][DPG];
#pragma unroll
  for (int u = 0; u < QPT; ++u)
#pragma unroll
    for (int d = 0; d < DPG; ++d) acc[u][d] = f2(0.0f, 0.0f);
  const int dg = DPG * g;
  int t = 0;
  const int L3 = has[0] ? L : 0;
#pragma unroll 2
  for (; t + 4 <= L3; t += 4) {
    float2 p01[QPT], p23[QPT];
#pragma unroll
    for (int u = 0; u < QPT; ++u) {
      const float4 e4 = (u == 0 || has[u]) ? *reinterpret_cast<const float4*>(er[u] + t) : make_float4(0.f, 0.f, 0.f, 0.f);
      p01[u] = mul2(f2(e4.x, e4.y), inv2[u]);
      p23[u] = mul2(f2(e4.z, e4.w), inv2[u]);
    }
#pragma unroll
    for (int d = 0; d < DPG; ++d) {
      const float4 vv = *reinterpret_cast<const float4*>(vd + dm_index(dg + d, t));
#pragma unroll
      for (int u = 0; u < QPT; ++u) {
        acc[u][d] = fma2(f2(vv.x, vv.y), p01[u], acc[u][d]);
        acc[u][d] = fma2(f2(vv.z, vv.w), p23[u], acc[u][d]);
      }
    }
  }
  for (; t + 1 < L3; t += 2) {
#pragma unroll
    for (int u = 0; u < QPT; ++u) {
      const float2 p = mul2(f2(er[u][t], er[u][t + 1]), inv2[u]);
#pragma unroll
      for (int d = 0; d < DPG; ++d)
        acc[u][d] = fma2(f2(vd[dm_index(dg + d, t)], vd[dm_index(dg + d, t + 1)]), p, acc[u][d]);
    }
  }
  if (t < L3) {  // odd L: the last key goes to the even accumulator
#pragma unroll
    for (int u = 0; u < QPT; ++u) {
      const float pa = er[u][t] * inv2[u].x;
#pragma unroll
      for (int d = 0; d < DPG; ++d) acc[u][d].x = fmaf(vd[dm_index(dg + d, t)], pa, acc[u][d].x);
    }
  }
#pragma unroll
  for (int u = 0; u < QPT; ++u) {
    if (active[u]) {
      float* o = a.out + size_t(s0 + qi[u]) * kHidden + h * 32 + dg;
      if constexpr (DPG == 4)
        *reinterpret_cast<float4*>(o) = make_float4(acc[u][0].x + acc[u][0].y, acc[u][1].x + acc[u][1].y,
                                                    acc[u][2].x + acc[u][2].y, acc[u][3].x + acc[u][3].y);
      else
        *reinterpret_cast<float2*>(o) = make_float2(acc[u][0].x + acc[u][0].y, acc[u][1].x + acc[u][1].y);
    }
  }
}

__global__ void __launch_bounds__(128) k_attention_cls(AttnArgs a, int n_seqs) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float4 smem4[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s = blockIdx.x / kHeads, h = blockIdx.x % kHeads;
  if (s >= n_seqs) return;
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  if (L <= 0 || L > a.max_len) {
    if (tid == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  float* qs = reinterpret_cast<float*>(smem4);  // [32] pre-scaled query
  float* red = qs + 32;                          // [8] warp maxima, then 1 / sum
  float* sc = red + 8;                           // [max_len] scores, then exponentials
  float* vs = sc + a.max_len;                    // [max_len][33] V rows
  float* accs = vs + size_t(a.max_len) * 33;     // [64] weighted-sum accumulators
  if (tid < 32) {
    const float scale = 1.0f / sqrtf(32.0f);
    qs[tid] = (a.q_tt ? a.q[tt_index(s, a.q_col + 32 * h + tid, a.q_C)]
                      : a.q[size_t(s) * a.q_C + a.q_col + 32 * h + tid]) * scale;
  }
  __syncthreads();
  const int kc = a.k_col + 32 * h, vc = a.v_col + 32 * h;
  const int L4 = L & ~3, L8 = L & ~7, L16 = L & ~15;
  float mx = -INFINITY;
  for (int t = tid; t < L; t += 128) {
    float kk[32], vv[32];
#pragma unroll
    for (int d = 0; d < 32; ++d) {
      kk[d] = ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t, kc + d);
      vv[d] = ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t, vc + d);
    }
    float s8[8];
#pragma unroll
    for (int l = 0; l < 8; ++l)
      s8[l] = fmaf(qs[8 + l], kk[8 + l], qs[l] * kk[l]) + fmaf(qs[24 + l], kk[24 + l], qs[16 + l] * kk[16 + l]);
    const float sv = (t < L4) ? ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]))
                              : ((s8[0] + s8[4]) + (s8[1] + s8[5])) + ((s8[2] + s8[6]) + (s8[3] + s8[7]));
    sc[t] = sv;
    mx = fmaxf(mx, sv);
#pragma unroll
    for (int d = 0; d < 32; ++d) vs[t * 33 + d] = vv[d];
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[warp] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));  // the max is order-independent
  for (int t = tid; t < L; t += 128) sc[t] = (t < L8) ? cw_exp(sc[t] - mx) : scalar_expf(sc[t] - mx);
  __syncthreads();
  if (warp == 0) {
    // lane l < 16 runs the chain of the reference's lane slot l (keys t0 + l of every 16-key chunk;
    // slots 0-7 then also take the trailing 8-key chunk), as the two 8-lane AVX2 accumulators do
    float part = 0.0f;
    if (lane < 16) {
      for (int t0 = 0; t0 < L16; t0 += 16) part = part + sc[t0 + lane];
      if (L8 > L16 && lane < 8) part = part + sc[L16 + lane];
    }
    const float v = part + __shfl_down_sync(0xffffffffu, part, 8);  // vs0[l] + vs1[l]
    const float t4 = v + __shfl_down_sync(0xffffffffu, v, 4);
    const float u = t4 + __shfl_down_sync(0xffffffffu, t4, 1);
    float sum = u + __shfl_down_sync(0xffffffffu, u, 2);
    if (lane == 0) {
      for (int t = L8; t < L; ++t) sum = sum + sc[t];
      red[4] = 1.0f / sum;
    }
  }
  __syncthreads();
  if (tid < 64) {  // accumulator a (even keys, threads 0-31) or b (odd keys, threads 32-63) of dim d
    const float inv = red[4];
    const int d = tid & 31;
    float acc = 0.0f;
    for (int t = tid >> 5; t < L; t += 2) acc = fmaf(vs[t * 33 + d], sc[t] * inv, acc);
    accs[tid] = acc;
  }
  __syncthreads();
  if (tid < 32) a.out[size_t(s) * kHidden + h * 32 + tid] = accs[tid] + accs[32 + tid];
}

constexpr size_t kRowsSmemMax = 220 * 1024;  // dynamic shared memory cap (static smem comes on top)

// Static shared memory of the kernels (cudaFuncGetAttributes at setup), counted by rows_smem.
static size_t g_static_rows = 0, g_static_wide2 = 0, g_static_wide4 = 0, g_static_rows2 = 0;

// Dynamic shared memory of a CTA: the K / V pairs, padded so that at most 512 / cols CTAs share an
// SM (their TMEM allocations then always fit; a CTA never waits in tcgen05.alloc). static_bytes:
// the kernel's static shared memory, which shares the SM's 228 KB with the dynamic part.
static size_t rows_smem_cap(size_t static_bytes) {  // a CTA holds at most 227 KB, static included
  const size_t cap = 227 * 1024 - static_bytes;
  return cap < kRowsSmemMax ? cap : kRowsSmemMax;
}
static size_t rows_smem(int max_len, size_t static_bytes) {
  const size_t kv = size_t((max_len + 1) / 2) * KPS * 8 * 2;
  const uint32_t cols = tmem_cols_for_len(max_len);
  const size_t per_sm = 227 * 1024;
  size_t floor_bytes = per_sm / (512 / cols) - 2048 + 1 - static_bytes;  // no more than 512 / cols CTAs fit
  if (floor_bytes > rows_smem_cap(static_bytes)) floor_bytes = rows_smem_cap(static_bytes);
  return kv > floor_bytes ? kv : floor_bytes;
}

template <int QT>
static int launch_rows(const AttnArgs& a, int n_seqs, cudaStream_t st) {
  dim3 grid(n_seqs, kHeads, (a.max_len + QT - 1) / QT);
  // few tiles (single sequences): each tile's weighted sum split by dims over 2 or 4 CTAs
  const long units = long(grid.x) * grid.y * grid.z;
  if (QT == 128 && tmem_cols_for_len(a.max_len) == 256) {  // 2 CTAs per SM: two warpgroups each
    const size_t sm = rows_smem(a.max_len, g_static_wide2);
    if (units * 4 <= 2 * 148) {
      grid.z *= 4;
      return launch_pdl(k_attention_wide<2, 2, 4>, grid, dim3(256), sm, st, a) == cudaSuccess ? 0 : -3;
    }
    if (units * 2 <= 2 * 148) {
      grid.z *= 2;
      return launch_pdl(k_attention_wide<2, 2, 2>, grid, dim3(256), sm, st, a) == cudaSuccess ? 0 : -3;
    }
    return launch_pdl(k_attention_wide<ATTN_WIDE_256>, grid, dim3(128 * ATTN_WIDE_256_NWG), sm, st, a) == cudaSuccess
               ? 0
               : -3;
  }
  if (QT == 128 && tmem_cols_for_len(a.max_len) == 512) {  // 1 CTA per SM: four warpgroups
    const size_t sm = rows_smem(a.max_len, g_static_wide4);
    if (units * 2 <= 148) {
      grid.z *= 2;
      return launch_pdl(k_attention_wide<4, 1, 2>, grid, dim3(512), sm, st, a) == cudaSuccess ? 0 : -3;
    }
    return launch_pdl(k_attention_wide<4, 1>, grid, dim3(512), sm, st, a) == cudaSuccess ? 0 : -3;
  }
  if (QT == 32 && units * 2 <= 2 * 148) {  // a 32-query tile holds 1 warp: several CTAs per SM
    grid.z *= 2;
    return launch_pdl(k_attention_rows<32, 2>, grid, dim3(32), rows_smem(a.max_len, g_static_rows), st, a) ==
                   cudaSuccess
               ? 0
               : -3;
  }
  return launch_pdl(k_attention_rows<QT>, grid, dim3(QT), rows_smem(a.max_len, g_static_rows), st, a) == cudaSuccess ? 0 : -3;
}

// k_attention_rows2: K / V of two heads; at least half an SM's shared memory, so that no
// more CTAs share an SM than its TMEM holds (2 x 256 columns).
static int launch_rows2(const AttnArgs& a, int n_seqs, cudaStream_t st) {
  const size_t kv = size_t(3) * 64 * 128 * 4;  // [64][128] K, V and Q (row stride <= 128)
  const size_t floor_bytes = 227 * 1024 / 2 - 2048 + 1 - g_static_rows2;
  const size_t bytes = kv > floor_bytes ? kv : floor_bytes;
  return launch_pdl(k_attention_rows2, dim3(n_seqs, kHeads / 2), dim3(128), bytes, st, a) == cudaSuccess ? 0 : -3;
}

// k_attention_lat8: the query tiles of all (sequence, head) pairs fill the SMs about once; qt a
// multiple of 4 (whole warps), capped by shared memory.
static size_t g_static_lat8 = 0;
static int launch_lat8(const AttnArgs& a, int n_seqs, cudaStream_t st) {
  const int L = a.max_len;
  const long pairs = long(n_seqs) * kHeads;
  int tiles = int(148 / pairs);
  if (tiles < 1) tiles = 1;
  int qt = (L + tiles - 1) / tiles;
  qt = qt > 64 ? 64 : (qt + 3) & ~3;  // at most 512 threads
  const size_t cap = 227 * 1024 - g_static_lat8;
  while (qt > 4 && lat8_smem_bytes(L, qt) > cap) qt -= 4;
  tiles = (L + qt - 1) / qt;
  return launch_pdl(k_attention_lat8, dim3(n_seqs, kHeads, tiles), dim3(8 * qt), lat8_smem_bytes(L, qt), st, a, qt) ==
                 cudaSuccess
             ? 0
             : -3;
}

static size_t g_static_narrow = 0;
#ifndef ATTN_NARROW_WARPS
#define ATTN_NARROW_WARPS 16
#endif
constexpr int kNarrowWarps = ATTN_NARROW_WARPS;
static int launch_narrow(const AttnArgs& a, int n_seqs, cudaStream_t st) {
  const dim3 grid(n_seqs, kHeads, (a.max_len + 31) / 32);
  return launch_pdl(k_attention_narrow<kNarrowWarps>, grid, dim3(32 * kNarrowWarps), narrow_smem_bytes(a.max_len), st, a) ==
                 cudaSuccess
             ? 0
             : -3;
}

static size_t g_static_narrow_dm = 0;
// one wave of 32-query tiles (16 warps each), or, where that takes two waves, tiles of up to 64
// queries sized to fill the SMs once (two rows of 8 warps, the second row partial)
static size_t g_static_narrow_dm2 = 0;
static int launch_narrow_dm(const AttnArgs& a, int n_seqs, cudaStream_t st) {
  const long heads = long(n_seqs) * kHeads;
  if (heads * ((a.max_len + 31) / 32) <= 148) {
    const dim3 grid(n_seqs, kHeads, (a.max_len + 31) / 32);
    return launch_pdl(k_attention_narrow_dm<kNarrowWarps, 1>, grid, dim3(32 * kNarrowWarps),
                      narrow_dm_smem_bytes(a.max_len), st, a, 32) == cudaSuccess
               ? 0
               : -3;
  }
  int tiles = int(148 / heads);
  if (tiles < 1) tiles = 1;
  int qt = (a.max_len + tiles - 1) / tiles;
  if (qt > 64) qt = 64;
  while (qt > 32 && narrow_dm_smem_bytes(a.max_len, qt) + g_static_narrow_dm2 > 227 * 1024) --qt;
  const dim3 grid(n_seqs, kHeads, (a.max_len + qt - 1) / qt);
  return launch_pdl(k_attention_narrow_dm<8, 1, 2>, grid, dim3(256), narrow_dm_smem_bytes(a.max_len, qt), st, a, qt) ==
                 cudaSuccess
             ? 0
             : -3;
}

static int smem_attr(const void* fn, size_t bytes) {
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes)) == cudaSuccess ? 0 : -1;
}

static int static_smem(const void* fn, size_t* out) {
  cudaFuncAttributes at{};
  if (cudaFuncGetAttributes(&at, fn) != cudaSuccess) return -1;
  *out = at.sharedSizeBytes;
  return 0;
}

int attention_prime() {
  int r = 0;
  r |= static_smem((const void*)k_attention_rows<128>, &g_static_rows);
  r |= static_smem((const void*)k_attention_wide<ATTN_WIDE_256>, &g_static_wide2);
  r |= static_smem((const void*)k_attention_wide<4, 1>, &g_static_wide4);
  r |= static_smem((const void*)k_attention_rows2, &g_static_rows2);
  r |= static_smem((const void*)k_attention_lat8, &g_static_lat8);
  r |= static_smem((const void*)k_attention_narrow<kNarrowWarps>, &g_static_narrow);
  r |= static_smem((const void*)k_attention_narrow_dm<kNarrowWarps, 1>, &g_static_narrow_dm);
  r |= static_smem((const void*)k_attention_narrow_dm<8, 1, 2>, &g_static_narrow_dm2);
  if (r) return r;
  r |= smem_attr((const void*)k_attention_narrow<kNarrowWarps>, 227 * 1024 - g_static_narrow);
  r |= smem_attr((const void*)k_attention_narrow_dm<kNarrowWarps, 1>, 227 * 1024 - g_static_narrow_dm);
  r |= smem_attr((const void*)k_attention_narrow_dm<8, 1, 2>, 227 * 1024 - g_static_narrow_dm2);
  r |= smem_attr((const void*)k_attention_lat8, 227 * 1024 - g_static_lat8);
  r |= smem_attr((const void*)k_attention_rows2, rows_smem_cap(g_static_rows2));
  r |= smem_attr((const void*)k_attention_rows<128>, rows_smem_cap(g_static_rows));
  r |= smem_attr((const void*)k_attention_rows<64>, rows_smem_cap(g_static_rows));
  r |= smem_attr((const void*)k_attention_rows<32>, rows_smem_cap(g_static_rows));
  r |= smem_attr((const void*)k_attention_rows<32, 2>, rows_smem_cap(g_static_rows));
  r |= smem_attr((const void*)k_attention_wide<ATTN_WIDE_256>, rows_smem_cap(g_static_wide2));
  r |= smem_attr((const void*)k_attention_wide<4, 1>, rows_smem_cap(g_static_wide4));
  r |= smem_attr((const void*)k_attention_wide<4, 1, 2>, rows_smem_cap(g_static_wide4));
  r |= smem_attr((const void*)k_attention_wide<2, 2, 2>, rows_smem_cap(g_static_wide2));
  r |= smem_attr((const void*)k_attention_wide<2, 2, 4>, rows_smem_cap(g_static_wide2));
  r |= smem_attr((const void*)k_attention_cls, cls_smem_floats(kMaxPos) * 4);
  r |= smem_attr((const void*)k_attention_lat<32, false>, lat_smem_bytes(kMaxPos, 32));
  r |= smem_attr((const void*)k_attention_lat<32, true>, lat_smem_bytes(kMaxPos, 32));
  // 12-CTA clusters (the heads of one sequence) exceed the portable cluster size of 8
  r |= cudaFuncSetAttribute((const void*)k_attention_lat<32, true>, cudaFuncAttributeNonPortableClusterSizeAllowed,
                            1) == cudaSuccess ? 0 : -1;
  r |= smem_attr((const void*)k_qkv_attention, kQaSmem);
  return r;
}

int launch_qkv_attention(const CUtensorMap& tm_act, const CUtensorMap& tm_w, const QkvAttnArgs& a, int n_seqs,
                         cudaStream_t st) {
  if (n_seqs <= 0) return 0;
  if (a.a.max_len <= 0 || a.a.max_len > 128) return -1;
  return launch_pdl(k_qkv_attention, dim3(n_seqs, kHeads / 2), dim3(128), kQaSmem, st, tm_act, tm_w, a) == cudaSuccess
             ? 0
             : -3;
}

// ------------------------------------------------------------------------------------------ int8 mode
// The reference's int8 attention scheme (attention_heads_sme, src/simd_math.rs:1933-2186; run by the
// crate on its SME backend for layers 0-10 of sequences of at least 16 tokens, src/model.rs:245):
//   Q and K rows of a head quantized per token (quantize_head32_row_neon :2482-2527), the K scale
//   carrying 1/sqrt(32) * log2(e); V quantized per column over the sequence's keys (:2598-2640);
//   scores s = (int32 Q.K * k_scale) * q_scale (softmax_quantize_i16_from_acc_neon :2291-2336);
//   q = round(16383 * 2^(s - max)) by exp2_q_neon (:2353-2366) for the row's complete 8-key blocks
//   and by exp2 + round for the last len % 8 keys (softmax_exp2_quantize_pass_i16_neon :2379-2410);
//   ctx = int32 (q . V) * (v_scale * (1 / sum q)).
// Every step is elementwise or an integer sum, so any order gives the reference's values: the
// integer products run as dp4a (Q.K, 4 dims a step) and dp2a (14-bit q times int8 V, 2 keys a step).
//
// k_attention_i8: one CTA per (sequence, head, 128 queries), one thread per query. The CTA
// quantizes the head's K rows and V columns into shared memory (K as 32 int8 per key, V as key
// pairs interleaved per column pair for dp2a), so that every shared load is a broadcast that
// serves the warp's 32 queries. A thread makes two passes over the keys: the scores and their
// maximum, then the same scores again (the same operations, so the same values), their 14-bit
// exponentials, the integer sum and the 32 integer column sums of P.V in registers.
constexpr int kI8Queries = 128;

struct I8Smem {
  int4 k[kMaxPos][2];          // key j: dims 0-15, 16-31 as int8
  float ks[kMaxPos];           // key scales (with 1/sqrt(32) * log2 e)
  int v[kMaxPos / 2][16];      // key pair (2p, 2p+1), word w: v[2p][2w], v[2p+1][2w], v[2p][2w+1], v[2p+1][2w+1]
  float v_scale[kHeadDim], v_inv[kHeadDim];
};

// quantize_head32_row_neon: q = sat(rn(x * (127 / m))), m = max(1e-8, max |x|); returns (m / 127) * mul.
__device__ __forceinline__ float i8_quant_head_row(const float (&x)[32], float mul, int4& lo, int4& hi) {
  float m = 0.0f;
#pragma unroll
  for (int d = 0; d < 32; ++d) m = fmaxf(m, fabsf(x[d]));
  m = fmaxf(m, 1e-8f);
  const float inv = __fdiv_rn(127.0f, m);
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = 0u;
#pragma unroll
  for (int d = 0; d < 32; ++d) {
    const int v = max(-128, min(127, __float2int_rn(__fmul_rn(x[d], inv))));
    w[d >> 2] |= (uint32_t(v) & 0xffu) << (8 * (d & 3));
  }
  lo = make_int4(int(w[0]), int(w[1]), int(w[2]), int(w[3]));
  hi = make_int4(int(w[4]), int(w[5]), int(w[6]), int(w[7]));
  return __fmul_rn(__fdiv_rn(m, 127.0f), mul);
}

// The 32 values of row t, columns c0 .. c0+31 (tile-transposed or row-major activations).
__device__ __forceinline__ void i8_load_head_row(const float* base, int C, int tt, int t, int c0, float (&x)[32]) {
  if (tt) {
    const float* p = base + tt_index(t, c0, C);
#pragma unroll
    for (int d = 0; d < 32; ++d) x[d] = p[size_t(d) << 7];
  } else {
    const float4* p = reinterpret_cast<const float4*>(base + size_t(t) * C + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = p[i];
      x[4 * i] = v.x;
      x[4 * i + 1] = v.y;
      x[4 * i + 2] = v.z;
      x[4 * i + 3] = v.w;
    }
  }
}

// exp2_q_neon(x, 16383, -16): round(16383 * 2^x), x <= 0; c[] = the polynomial's coefficients * 16383.
__device__ __forceinline__ int i8_exp2_q(float x, const float (&c)[4]) {
  x = fmaxf(x, -16.0f);
  const int n = __float2int_rd(x);
  const float f = __fsub_rn(x, __int2float_rn(n));
  float p = __fmaf_rn(f, c[3], c[2]);
  p = __fmaf_rn(f, p, c[1]);
  p = __fmaf_rn(f, p, c[0]);
  return __float2int_rn(__int_as_float(__float_as_int(p) + int(uint32_t(n) << 23)));
}

// The score of key j for a query held as (qa, qb, qsc): (int32 q.k * k_scale) * q_scale.
__device__ __forceinline__ float i8_score(const I8Smem& sm, int j, const int4& qa, const int4& qb, float qsc) {
  const int4 ka = sm.k[j][0], kb = sm.k[j][1];
  int acc = __dp4a(qa.x, ka.x, 0);
  acc = __dp4a(qa.y, ka.y, acc);
  acc = __dp4a(qa.z, ka.z, acc);
  acc = __dp4a(qa.w, ka.w, acc);
  acc = __dp4a(qb.x, kb.x, acc);
  acc = __dp4a(qb.y, kb.y, acc);
  acc = __dp4a(qb.z, kb.z, acc);
  acc = __dp4a(qb.w, kb.w, acc);
  return __fmul_rn(__fmul_rn(__int2float_rn(acc), sm.ks[j]), qsc);
}

// min_len: sequences shorter than this are left to the fp32 kernels (their context rows untouched).
__global__ void __launch_bounds__(kI8Queries, 4) k_attention_i8(AttnArgs a, int min_len) {
  pdl_trigger();
  pdl_wait();
  __shared__ I8Smem sm;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int s, h, z;
  tile_major_block(s, h, z);  // the query tiles of a (sequence, head) together: K / V from L2
  const int s0 = int(a.cu[s]);
  const int L = int(a.cu[s + 1]) - s0;
  if (L <= 0 || L > a.max_len) {
    if (tid == 0) record_err(a.err, DEV_ERR_BAD_SHAPE);
    return;
  }
  const int i0 = z * kI8Queries;
  if (L < min_len || i0 >= L) return;
  const int L8 = L & ~7, pairs = (L + 1) >> 1;
  const int qc = a.q_col + 32 * h, kc = a.k_col + 32 * h, vc = a.v_col + 32 * h;

  // K rows, quantized per token
  const float k_mul = __fmul_rn(__fdiv_rn(1.0f, __fsqrt_rn(32.0f)), 1.44269504088896341f);
  for (int j = tid; j < L; j += kI8Queries) {
    float x[32];
    i8_load_head_row(a.kv, a.kv_C, a.kv_tt, s0 + j, kc, x);
    sm.ks[j] = i8_quant_head_row(x, k_mul, sm.k[j][0], sm.k[j][1]);
  }
  // V column maxima: warp w takes columns 8w .. 8w+7, lanes split the keys
  {
    float cm[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) cm[e] = 0.0f;
    for (int j = lane; j < L; j += 32) {
#pragma unroll
      for (int e = 0; e < 8; ++e) cm[e] = fmaxf(cm[e], fabsf(ld_act(a.kv, a.kv_C, a.kv_tt, s0 + j, vc + 8 * warp + e)));
    }
    float mine = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) cm[e] = fmaxf(cm[e], __shfl_xor_sync(0xffffffffu, cm[e], o));
      if (lane == e) mine = cm[e];
    }
    if (lane < 8) {
      const float m = fmaxf(mine, 1e-8f);
      sm.v_scale[8 * warp + lane] = __fmul_rn(m, __fdiv_rn(1.0f, 127.0f));
      sm.v_inv[8 * warp + lane] = __fdiv_rn(127.0f, m);
    }
  }
  __syncthreads();
  // V as int8 key pairs per column pair (the second key of an odd L's last pair is zero); lanes take
  // consecutive key pairs of one column pair (tile-transposed rows) or consecutive column pairs of
  // one key pair (row-major rows), so that their loads are contiguous
  for (int i = tid; i < pairs * 16; i += kI8Queries) {
    const int p = a.kv_tt ? i % pairs : i >> 4;
    const int w = a.kv_tt ? i / pairs : i & 15;
    const int t0 = 2 * p, c0 = 2 * w;
    const float i0v = sm.v_inv[c0], i1v = sm.v_inv[c0 + 1];
    auto q8 = [](float x, float inv) { return uint32_t(max(-128, min(127, __float2int_rn(__fmul_rn(x, inv))))) & 0xffu; };
    const uint32_t a0 = q8(ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t0, vc + c0), i0v);
    const uint32_t a1 = q8(ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t0, vc + c0 + 1), i1v);
    uint32_t b0 = 0u, b1 = 0u;
    if (t0 + 1 < L) {
      b0 = q8(ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t0 + 1, vc + c0), i0v);
      b1 = q8(ld_act(a.kv, a.kv_C, a.kv_tt, s0 + t0 + 1, vc + c0 + 1), i1v);
    }
    sm.v[p][w] = int(a0 | (b0 << 8) | (a1 << 16) | (b1 << 24));
  }
  __syncthreads();

  const int qi = i0 + tid;
  if (qi >= L) return;  // no barrier follows
  int4 qa, qb;
  float qsc;
  {
    float x[32];
    i8_load_head_row(a.q, a.q_C, a.q_tt, s0 + qi, qc, x);
    qsc = i8_quant_head_row(x, 1.0f, qa, qb);
  }
  // pass 1: the maximum score
  float mx = -INFINITY;
  {
    int j = 0;
    for (; j + 4 <= L; j += 4) {
      const float e0 = i8_score(sm, j, qa, qb, qsc), e1 = i8_score(sm, j + 1, qa, qb, qsc);
      const float e2 = i8_score(sm, j + 2, qa, qb, qsc), e3 = i8_score(sm, j + 3, qa, qb, qsc);
      mx = fmaxf(mx, fmaxf(fmaxf(e0, e1), fmaxf(e2, e3)));
    }
    for (; j < L; ++j) mx = fmaxf(mx, i8_score(sm, j, qa, qb, qsc));
  }
  // pass 2: 14-bit exponentials, their sum and P.V (integer sums: exact in any order)
  float cexp[4];
  cexp[0] = __fmul_rn(0.999857f, 16383.0f);
  cexp[1] = __fmul_rn(0.6963853f, 16383.0f);
  cexp[2] = __fmul_rn(0.22511937f, 16383.0f);
  cexp[3] = __fmul_rn(0.07842169f, 16383.0f);
  auto prob = [&](int j) -> int {
    if (j >= L) return 0;
    const float x = __fsub_rn(i8_score(sm, j, qa, qb, qsc), mx);
    if (j < L8) return i8_exp2_q(x, cexp);
    return max(0, min(16383, int(roundf(__fmul_rn(exp2f(x), 16383.0f)))));
  };
  int acc[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) acc[c] = 0;
  int isum = 0;
  for (int p = 0; p < pairs; ++p) {
    const int p0 = prob(2 * p), p1 = prob(2 * p + 1);
    isum += p0 + p1;
    const int pp = int(uint32_t(p0) | (uint32_t(p1) << 16));
    const int4* vr = reinterpret_cast<const int4*>(sm.v[p]);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int4 wv = vr[g];
      acc[8 * g + 0] = __dp2a_lo(pp, wv.x, acc[8 * g + 0]);
      acc[8 * g + 1] = __dp2a_hi(pp, wv.x, acc[8 * g + 1]);
      acc[8 * g + 2] = __dp2a_lo(pp, wv.y, acc[8 * g + 2]);
      acc[8 * g + 3] = __dp2a_hi(pp, wv.y, acc[8 * g + 3]);
      acc[8 * g + 4] = __dp2a_lo(pp, wv.z, acc[8 * g + 4]);
      acc[8 * g + 5] = __dp2a_hi(pp, wv.z, acc[8 * g + 5]);
      acc[8 * g + 6] = __dp2a_lo(pp, wv.w, acc[8 * g + 6]);
      acc[8 * g + 7] = __dp2a_hi(pp, wv.w, acc[8 * g + 7]);
    }
  }
  const float p_scale = __fdiv_rn(1.0f, __int2float_rn(max(isum, 1)));
  float4* o = reinterpret_cast<float4*>(a.out + size_t(s0 + qi) * kHidden + h * 32);
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    float r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = 4 * g + e;
      r[e] = __fmul_rn(__int2float_rn(acc[c]), __fmul_rn(sm.v_scale[c], p_scale));
    }
    o[g] = make_float4(r[0], r[1], r[2], r[3]);
  }
}

int launch_attention_i8(const AttnArgs& a, int n_seqs, int min_len, cudaStream_t st) {
  if (n_seqs <= 0) return 0;
  if (a.max_len <= 0 || a.max_len > kMaxPos || a.cls_mode) return -1;
  const dim3 grid(n_seqs, kHeads, (a.max_len + kI8Queries - 1) / kI8Queries);
  return launch_pdl(k_attention_i8, grid, dim3(kI8Queries), 0, st, a, min_len) == cudaSuccess ? 0 : -3;
}

int launch_attention_exact(const AttnArgs& a, int n_seqs, cudaStream_t st, int* quantized) {
  if (quantized) *quantized = 0;
  if (n_seqs <= 0) return 0;
  if (a.max_len <= 0 || a.max_len > kMaxPos) return -1;
  if (a.cls_mode) {
    return launch_pdl(k_attention_cls, dim3(n_seqs * kHeads), dim3(128), cls_smem_floats(a.max_len) * 4, st, a, n_seqs) ==
                   cudaSuccess
               ? 0
               : -3;
  }
  // query tile: no wider than the sequences (32 / 64 threads for short ones, whose TMEM then packs
  // 16 / 8 CTAs per SM), and narrower while the grid has fewer than two CTAs per SM.
  // More than 128 keys: always the multi-warpgroup kernels (their score columns allow only 1-2 CTAs
  // per SM, so one-warp tiles would leave each SM one warp for L x 32 query-key pairs).
  const int cap = a.max_len <= 32 ? 32 : a.max_len <= 64 ? 64 : 128;
  const long heads = long(n_seqs) * kHeads;
  // few (sequence, head) pairs of short sequences: four lanes per query, 32-query tiles, no TMEM
  if (a.max_len <= kLatMaxLen && heads * ((a.max_len + 31) / 32) <= 2 * 148) {
    const dim3 grid(n_seqs, kHeads, (a.max_len + 31) / 32);
    if (!(quantized && a.quant_inv_s && a.quant_q && a.quant_scale))
      return launch_pdl(k_attention_lat<32, false>, grid, dim3(128), lat_smem_bytes(a.max_len, 32), st, a) ==
                     cudaSuccess
                 ? 0
                 : -3;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(128);
    cfg.dynamicSmemBytes = lat_smem_bytes(a.max_len, 32);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = kHeads;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (cudaLaunchKernelEx(&cfg, k_attention_lat<32, true>, a) != cudaSuccess) return -3;
    *quantized = 1;
    return 0;
  }
  // few pairs of longer sequences: eight lanes per query, the tiles sized to fill the SMs once
  // few pairs of longer sequences: 32-query tiles with the scores in shared memory when those
  // tiles fill the SMs in one wave, else eight lanes per query in tiles sized to fill them once
  if (a.few_mode != 1 && heads * ((a.max_len + 127) / 128) <= 148) {
    const size_t per_cta = narrow_smem_bytes(a.max_len) + g_static_narrow + 1024;
    const long fit = long(227 * 1024 / per_cta);
    const bool dm_fits = narrow_dm_smem_bytes(a.max_len) + g_static_narrow_dm + 1024 <= 227 * 1024;
    if (a.few_mode == 4 || (a.few_mode == 0 && n_seqs == 1 && dm_fits)) return launch_narrow_dm(a, n_seqs, st);
    const bool narrow = a.few_mode == 2 ? fit >= 1 : (a.few_mode == 0 && fit >= 1 && heads * ((a.max_len + 31) / 32) <= 148 * fit);
    return narrow ? launch_narrow(a, n_seqs, st) : launch_lat8(a, n_seqs, st);
  }
  if (a.max_len > 128) return launch_rows<128>(a, n_seqs, st);
#ifndef ATTN_PAIRS
#define ATTN_PAIRS 1
#endif
  if (cap == 128 && heads >= 2 * 148) return ATTN_PAIRS ? launch_rows2(a, n_seqs, st) : launch_rows<128>(a, n_seqs, st);
  if (cap >= 64 && heads * ((a.max_len + 63) / 64) >= 2 * 148) return launch_rows<64>(a, n_seqs, st);
  return launch_rows<32>(a, n_seqs, st);
}

}  // namespace ae
