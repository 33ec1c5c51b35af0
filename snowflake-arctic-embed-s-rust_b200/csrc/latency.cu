// Single-sequence forward pass (PackedModel::forward_cls, src/model.rs:185-513) of at most 32 tokens
// as one kernel: a cluster of 12 CTAs, CTA c owning attention head c and a 1/12 column slice of
// every projection. It replaces the ~90 dependent launches of the multi-kernel path (each a few
// microseconds of launch and dependency latency) with one launch; every value is computed with the
// same arithmetic, in the same order, as that path, so the embedding is the same bits.
//
// Data moves between the CTAs only by stores into the consumer's shared memory (st.shared::cluster,
// which the producer does not wait for), made visible by a cluster barrier; no step waits on a
// remote load. Row r's LayerNorm (whose 16 partial-sum chains run across all 384 columns) is
// computed by its owner CTA r % 12, which receives the row's 12 column slices and sends the
// int8 row, its scale and the residual columns back to every CTA.
//
// Per layer (L <= 32 rows, one 128-row tcgen05 tile whose rows L..127 are ignored):
//   QKV    MMA of the layer input (int8, shared memory) with the 96 weight rows of head c's Q | K |
//          V (N = 96, K = 384), dequantized as the QKV GEMM's plain epilogue does
//   attn   the head's attention in the reference's order (attend_query_lanes8); partial row maxima
//          of the context slice -> every CTA                                   | cluster barrier
//   ctx q  each CTA quantizes its own 32 context columns with the row maxima (smooth_quantize_row,
//          as the short-sequence attention kernel does) -> every CTA's A operand | cluster barrier
//   AO     N = 32 slice c: h = fma(acc, a_s * w_s, bias + residual) -> the row owners | barrier
//   LN1    owners: layernorm_smooth_quantize_row -> int8 rows, scales, residual columns | barrier
//   FFN-up N = 128 slice c, g = GELU(h) * inv_smooth, partial row maxima -> every CTA | barrier;
//          the slice quantized with the row maximum over all 1,536 columns -> every CTA's A
//          operand as k-block c                                                  | barrier
//   FFN-dn N = 32 slice c (K = 1,536) with the residual -> the row owners           | barrier
//   LN2    as LN1, quantized for the next layer                                      | barrier
// Layer 11 runs the [CLS]-pruned tail (src/model.rs:400-512): K and V of all rows and Q of row 0
// (N = 96 from the q_only / kv_only weights), the [CLS] query's attention, then the same steps for
// row 0, and CTA 0 applies the final LayerNorm and L2 normalisation (sequential sums).
//
// Weights are TMA-loaded (32-row boxes, 128-byte swizzle, no multicast) into two 48 KB buffers,
// each stage's load issued as soon as the MMA two stages earlier has released its buffer. The A
// operand uses a 4 KB k-block stride (32 rows): rows 32..127 of a k-block, which the M = 128 MMA
// also reads, are the next k-blocks' bytes and only produce accumulator rows that are never read.
//
// Every mbarrier wait is bounded (2 s, then the error word is set and the CTA stops issuing MMAs
// and waiting); every CTA executes every cluster barrier, so no CTA can wait on another for ever.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "attn_lanes.cuh"
#include "latency.h"
#include "ptx.cuh"
#include "rowmath.cuh"

namespace ae {

namespace {

constexpr int kLatCtas = kHeads;  // 12
constexpr int kLatThreads = 256;
constexpr int kR = kLatMaxTokens;   // rows held per k-block of the A operand
constexpr int kP = 33;              // pitch of the attention's dim-major K / V rows (odd: no conflicts)
constexpr int kKbBytes = kR * 128;  // 4 KB
constexpr int kOwned = (kR + kLatCtas - 1) / kLatCtas;  // rows a CTA owns for the LayerNorms (3)

// the layer's vectors and this CTA's column parameters, prefetched at the start of every layer
enum : int {
  V_AOINV = 0,             // attention-out inv_smooth [384] (context quantization)
  V_LN1W = V_AOINV + 384,  // LayerNorm 1 weight, bias [384]
  V_LN1B = V_LN1W + 384,
  V_FIINV = V_LN1B + 384,  // FFN-up inv_smooth [384]
  V_LN2W = V_FIINV + 384,  // LayerNorm 2 weight, bias [384]
  V_LN2B = V_LN2W + 384,
  V_NXINV = V_LN2B + 384,  // the next layer's QKV inv_smooth [384]
  V_FOINV = V_NXINV + 384, // FFN-down inv_smooth, this CTA's 128 FFN-up columns
  V_QKVW = V_FOINV + 128,  // w_scale / bias of the 96 Q | K | V columns of head c
  V_QKVB = V_QKVW + 96,
  V_AOW = V_QKVB + 96,     // w_scale / bias of the 32 attention-out columns of slice c
  V_AOB = V_AOW + 32,
  V_FIW = V_AOB + 32,      // of the 128 FFN-up columns
  V_FIB = V_FIW + 128,
  V_FOW = V_FIB + 128,     // of the 32 FFN-down columns
  V_FOB = V_FOW + 32,
  V_FLOATS = V_FOB + 32
};

// shared memory, offsets from a 1024-byte aligned base
constexpr int OFF_A = 0;
constexpr int SZ_A = 12 * kKbBytes + (128 - kR) * 128;  // 12 k-blocks + the rows the MMA reads past them
constexpr int OFF_B0 = OFF_A + SZ_A;
constexpr int SZ_B = 48 * 1024;
constexpr int OFF_B1 = OFF_B0 + SZ_B;
constexpr int OFF_ACC = OFF_B1 + SZ_B;                 // [32][N + 1] accumulators, then g
constexpr int SZ_ACC = kR * 129 * 4;
constexpr int OFF_KD = OFF_ACC + SZ_ACC;               // attention: kd, vd, es [32][kP], qd [32][32]
constexpr int SZ_ATT = (3 * 32 * kP + 32 * 32) * 4;
constexpr int OFF_HG = OFF_KD + SZ_ATT;                // the owned rows of h (received), then y [3][384]
constexpr int OFF_RES = OFF_HG + kOwned * kHidden * 4; // residual columns of slice c [32][32]
constexpr int OFF_XCM = OFF_RES + kR * 32 * 4;         // context partial row maxima, from each CTA [12][32]
constexpr int OFF_XGM = OFF_XCM + kLatCtas * kR * 4;   // g partial row maxima, from each CTA [12][32]
constexpr int OFF_AS = OFF_XGM + kLatCtas * kR * 4;    // row scales of the A operand [32]
constexpr int OFF_VEC = OFF_AS + kR * 4;
constexpr int OFF_BAR = OFF_VEC + V_FLOATS * 4;        // mbarriers: weights x 2, MMA
constexpr int OFF_TMEM = OFF_BAR + 3 * 8;
constexpr int kLatSmem = OFF_TMEM + 8 + 1024;          // + the alignment slack
static_assert(OFF_B0 % 1024 == 0 && OFF_B1 % 1024 == 0, "swizzle atoms are 1024-aligned");
static_assert(OFF_HG % 16 == 0 && OFF_RES % 16 == 0 && OFF_VEC % 16 == 0, "16-byte vectors");
static_assert(OFF_BAR % 8 == 0, "mbarrier alignment");
static_assert(kLatSmem <= 232448, "shared memory of one CTA exceeds the sm_100 limit");

constexpr int kStages = 4 * kLayers;  // QKV, attention-out, FFN-up, FFN-down per layer

// Byte offset of element (row r, column j) of a K-major int8 operand with k-blocks of 128 columns
// at kKbBytes stride, 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r & 7)).
__device__ __forceinline__ int a_off(int r, int j) {
  const int b = j & 127;
  return (j >> 7) * kKbBytes + r * 128 + ((((b >> 4) ^ (r & 7))) << 4) + (b & 15);
}

__device__ __forceinline__ float halfwarp_tree16(float p) {
  const unsigned m = 0xffffffffu;
  float v = p + __shfl_down_sync(m, p, 8, 16);
  float t = v + __shfl_down_sync(m, v, 4, 16);
  float u = t + __shfl_down_sync(m, t, 1, 16);
  float r = u + __shfl_down_sync(m, u, 2, 16);
  return __shfl_sync(m, r, 0, 16);
}
__device__ __forceinline__ float halfwarp_max(float v) {
#pragma unroll
  for (int o = 8; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o, 16));
  return v;
}

__device__ __forceinline__ void cluster_sync_all() {
  cluster_arrive_release();
  cluster_wait_acquire();
}

struct Smem {
  int8_t* A;
  uint8_t* B[2];
  int32_t* acc;
  float *kd, *vd, *es, *qd, *hg, *res, *xcm, *xgm, *as, *vec;
  uint64_t *bw, *bmma;
  uint32_t* tslot;
};

// Weights of stage s (layer s / 4; 0 QKV, 1 attention-out, 2 FFN-up, 3 FFN-down) for slice c into
// buffer s & 1. Called by one thread.
__device__ __forceinline__ void issue_weights(const LatModel* m, const Smem& S, int s, int c) {
  const int l = s >> 2, k = s & 3, b = s & 1;
  uint8_t* dst = S.B[b];
  uint64_t* bar = &S.bw[b];
  const CUtensorMap* tm = m->tm[l];
  if (k == 0) {  // Q | K | V rows of head c (layer 11: q_only | kv_only K | kv_only V)
    mbar_arrive_expect_tx(bar, 96 * kHidden);
    for (int kb = 0; kb < 3; ++kb) {
      uint8_t* d = dst + kb * 96 * 128;
      if (l < kLayers - 1) {
        tma_load_2d(d, &tm[LAT_QKV], bar, kb * 128, 32 * c);
        tma_load_2d(d + 4096, &tm[LAT_QKV], bar, kb * 128, kHidden + 32 * c);
        tma_load_2d(d + 8192, &tm[LAT_QKV], bar, kb * 128, 2 * kHidden + 32 * c);
      } else {
        tma_load_2d(d, &tm[LAT_Q], bar, kb * 128, 32 * c);
        tma_load_2d(d + 4096, &tm[LAT_KV], bar, kb * 128, 32 * c);
        tma_load_2d(d + 8192, &tm[LAT_KV], bar, kb * 128, kHidden + 32 * c);
      }
    }
  } else if (k == 1) {  // attention-out rows 32c .. 32c + 31
    mbar_arrive_expect_tx(bar, 32 * kHidden);
    for (int kb = 0; kb < 3; ++kb) tma_load_2d(dst + kb * 4096, &tm[LAT_AO], bar, kb * 128, 32 * c);
  } else if (k == 2) {  // FFN-up rows 128c .. 128c + 127
    mbar_arrive_expect_tx(bar, 128 * kHidden);
    for (int kb = 0; kb < 3; ++kb)
      for (int j = 0; j < 4; ++j) tma_load_2d(dst + kb * 16384 + j * 4096, &tm[LAT_FI], bar, kb * 128, 128 * c + 32 * j);
  } else {  // FFN-down rows 32c .. 32c + 31, K = 1536
    mbar_arrive_expect_tx(bar, 32 * kInter);
    for (int kb = 0; kb < 12; ++kb) tma_load_2d(dst + kb * 4096, &tm[LAT_FO], bar, kb * 128, 32 * c);
  }
}

// Layer l's vectors and this CTA's column parameters -> S.vec by 16-byte asynchronous copies
// (complete after cp_async_wait_all; every source is 16-byte aligned in the model arena).
__device__ __forceinline__ void prefetch_layer(const LatModel* m, const Smem& S, int l, int c, int tid) {
  const LatLayer& Ly = m->layer[l];
  const bool last = l == kLayers - 1;
  const LatLinear& lq = last ? Ly.q_only : Ly.qkv;
  const LatLinear& lk = last ? Ly.kv_only : Ly.qkv;
  const int ko = last ? 32 * c : kHidden + 32 * c, vo = last ? kHidden + 32 * c : 2 * kHidden + 32 * c;
  const float* nx = last ? Ly.qkv.invs : m->layer[l + 1].qkv.invs;
  struct Seg {
    int dst;
    const float* src;
    int n;
  };
  const Seg seg[] = {{V_AOINV, Ly.ao.invs, 384},       {V_LN1W, Ly.ln1w, 384},          {V_LN1B, Ly.ln1b, 384},
                     {V_FIINV, Ly.fi.invs, 384},       {V_LN2W, Ly.ln2w, 384},          {V_LN2B, Ly.ln2b, 384},
                     {V_NXINV, nx, 384},               {V_FOINV, Ly.fo.invs + 128 * c, 128},
                     {V_QKVW, lq.ws + 32 * c, 32},     {V_QKVW + 32, lk.ws + ko, 32},  {V_QKVW + 64, lk.ws + vo, 32},
                     {V_QKVB, lq.bias + 32 * c, 32},   {V_QKVB + 32, lk.bias + ko, 32}, {V_QKVB + 64, lk.bias + vo, 32},
                     {V_AOW, Ly.ao.ws + 32 * c, 32},   {V_AOB, Ly.ao.bias + 32 * c, 32},
                     {V_FIW, Ly.fi.ws + 128 * c, 128}, {V_FIB, Ly.fi.bias + 128 * c, 128},
                     {V_FOW, Ly.fo.ws + 32 * c, 32},   {V_FOB, Ly.fo.bias + 32 * c, 32}};
  // warps 1-7 (warp 0 issues the MMA and reads TMEM meanwhile)
  constexpr int kCopiers = kLatThreads - 32;
  const int t = tid - 32;
  if (t < 0) return;
  int base = 0;
#pragma unroll
  for (int k = 0; k < int(sizeof(seg) / sizeof(seg[0])); ++k) {
    const int units = seg[k].n / 4;
    for (int u = (t - base + kCopiers) % kCopiers; u < units; u += kCopiers)
      cp_async16(S.vec + seg[k].dst + 4 * u, seg[k].src + 4 * u, 16u);
    base = (base + units) % kCopiers;
  }
}

// Thread 0: waits for stage s's weights, runs the N x (128 KB) MMA of the A operand into TMEM
// columns 0..N-1, waits for it and requests the weights of stage s + 2 into the released buffer.
// Returns false when a wait ran out (the CTA then stops issuing MMAs and waiting).
__device__ __forceinline__ bool mma_stage(const LatModel* m, const Smem& S, int s, int N, int KB, uint32_t tmem,
                                          int c, int* err, bool ok) {
  if (!ok) return false;
  const int b = s & 1;
  if (!mbar_wait(&S.bw[b], uint32_t(s >> 1) & 1u, err, DEV_ERR_TIMEOUT_MMA)) return false;
  fence_proxy_async_all();  // the A operand was written by generic stores, partly by other CTAs
  tc_fence_after();
  const uint32_t idesc = idesc_i8(128, N);
  const uint32_t a0 = smem_u32(S.A), b0 = smem_u32(S.B[b]);
  for (int kb = 0; kb < KB; ++kb)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
      mma_i8(tmem, sdesc_sw128(a0 + kb * kKbBytes + ks * 32), sdesc_sw128(b0 + kb * N * 128 + ks * 32), idesc,
             (kb | ks) != 0);
  mma_commit(S.bmma);
  if (!mbar_wait(S.bmma, uint32_t(s) & 1u, err, DEV_ERR_TIMEOUT_MMA)) return false;
  if (s + 2 < kStages) issue_weights(m, S, s + 2, c);
  return true;
}

// MMA (thread 0) -> accumulators of rows 0..31 in S.acc ([32][N + 1]), copied by warps 0 and 4
// (TMEM lane quadrant 0); all threads synchronised on return.
template <int N>
__device__ __forceinline__ bool run_gemm(const LatModel* m, const Smem& S, int s, int KB, uint32_t tmem, int c,
                                         int* err, bool ok, int tid, int warp, int lane) {
  __shared__ int s_ok;
  if (tid == 0) s_ok = mma_stage(m, S, s, N, KB, tmem, c, err, ok) ? 1 : 0;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  ok = s_ok != 0;
  if (ok && (warp == 0 || warp == 4)) {
    constexpr int H = N / 2, CH = H / 16;
    const int c0 = warp == 0 ? 0 : H;
    uint32_t r[CH][16];
#pragma unroll
    for (int ch = 0; ch < CH; ++ch) tmem_ld16(tmem + uint32_t(c0 + 16 * ch), r[ch]);
    tmem_ld_wait();
    int32_t* row = S.acc + lane * (N + 1) + c0;
#pragma unroll
    for (int ch = 0; ch < CH; ++ch)
#pragma unroll
      for (int j = 0; j < 16; ++j) row[16 * ch + j] = int32_t(r[ch][j]);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  return ok;
}

// h = fma(acc, a_s * w_s, bias + residual) of the 32-column slice c (the plain GEMM epilogue with a
// residual; w_s, bias: the slice's prefetched column parameters), four columns per thread, sent to
// the row's owner CTA (r % 12) at columns 32c .. 32c + 31 of its received rows.
__device__ __forceinline__ void epilogue_residual_push(const Smem& S, const float* ws, const float* bias, int c,
                                                       int rows, int tid) {
  for (int i = tid; i < rows * 8; i += kLatThreads) {
    const int r = i >> 3, n = 4 * (i & 7);
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float bb = bias[n + e] + S.res[r * 32 + n + e];
      v[e] = fmaf(float(S.acc[r * 33 + n + e]), S.as[r] * ws[n + e], bb);
    }
    st_cluster_f32x4(map_peer(S.hg + (r / kLatCtas) * kHidden + 32 * c + n, uint32_t(r % kLatCtas)),
                     make_float4(v[0], v[1], v[2], v[3]));
  }
}

// Rows this CTA owns for the LayerNorms: r = c + 12k, k < the count (uniform over the CTA).
__device__ __forceinline__ int owned_rows(int c, int rows) { return rows > c ? (rows - 1 - c) / kLatCtas + 1 : 0; }

// layernorm_smooth_quantize_row (k_ln_quant_rows' arithmetic) on the rows this CTA owns, from the
// received h rows in S.hg; called by every thread. A half-warp per row computes the statistics
// (the reference's 16 partial-sum chains, in order); then all threads form y (the same expression,
// so the same bits), its int8 row in the A operand and y in S.hg, and send the int8 row (3 x 128
// bytes, already in the operand's swizzled layout), its scale and every CTA's 32 residual columns
// to the other CTAs.
__device__ __forceinline__ void ln_quant_owned(const Smem& S, const float* gamma, const float* beta,
                                               const float* invs, int c, int rows, int tid) {
  __shared__ float st_mean[kOwned], st_rstd[kOwned], st_inv[kOwned], st_scale[kOwned];
  const int nown = owned_rows(c, rows);
  if (tid < 64) {  // warps 0-1: half-warp k takes owned row k (the fourth runs a copy for the shuffles)
    const int k = tid >> 4, l = tid & 15;
    const bool active = k < nown;
    const float* hrow = S.hg + (active ? k : 0) * kHidden;
    float h[24];
    float p = 0.0f;
#pragma unroll
    for (int i = 0; i < 24; ++i) {
      h[i] = hrow[l + 16 * i];
      p = p + h[i];
    }
    const float mean = halfwarp_tree16(p) / float(kHidden);
    p = 0.0f;
#pragma unroll
    for (int i = 0; i < 24; ++i) {
      const float d = h[i] - mean;
      p = fmaf(d, d, p);
    }
    const float var = halfwarp_tree16(p) / float(kHidden);
    const float rstd = 1.0f / sqrtf(var + kLnEps);
    float vmax = 1e-8f;
#pragma unroll
    for (int i = 0; i < 24; ++i) {
      const int j = l + 16 * i;
      vmax = fmaxf(vmax, fabsf(fmaf((h[i] - mean) * rstd, gamma[j], beta[j]) * invs[j]));
    }
    const float max_abs = halfwarp_max(vmax);
    if (active && l == 0) {
      st_mean[k] = mean;
      st_rstd[k] = rstd;
      st_inv[k] = 127.0f / max_abs;
      st_scale[k] = max_abs / 127.0f;
    }
  }
  __syncthreads();
  for (int i = tid; i < nown * kHidden; i += kLatThreads) {
    const int k = i / kHidden, j = i - k * kHidden;
    const float y = fmaf((S.hg[i] - st_mean[k]) * st_rstd[k], gamma[j], beta[j]);
    S.A[a_off(c + kLatCtas * k, j)] = int8_t(quant_i8(y * (invs[j] * st_inv[k])));
    S.hg[i] = y;
  }
  __syncthreads();
  constexpr int kPerRow = kLatCtas * 24 + kLatCtas * 8 + kLatCtas;  // chunks, residual float4s, scales
  for (int i = tid; i < nown * kPerRow; i += kLatThreads) {
    const int k = i / kPerRow, w = i - k * kPerRow;
    const int r = c + kLatCtas * k;
    if (w < kLatCtas * 24) {  // 16-byte chunks of the int8 row -> the other CTAs' A operands
      const int p = w / 24, ch = w - p * 24;
      if (p == c) continue;
      const int off = (ch >> 3) * kKbBytes + r * 128 + (ch & 7) * 16;
      st_cluster_u32x4(map_peer(S.A + off, uint32_t(p)), *reinterpret_cast<const uint4*>(S.A + off));
    } else if (w < kLatCtas * 32) {  // residual columns 32p .. 32p + 31 -> CTA p
      const int v = w - kLatCtas * 24, p = v >> 3, q4 = v & 7;
      st_cluster_f32x4(map_peer(S.res + r * 32 + 4 * q4, uint32_t(p)),
                       *reinterpret_cast<const float4*>(S.hg + k * kHidden + 32 * p + 4 * q4));
    } else {  // the row scale -> every CTA
      st_cluster_f32(map_peer(S.as + r, uint32_t(w - kLatCtas * 32)), st_scale[k]);
    }
  }
}

// FFN-up epilogue of slice c: g = GELU(fma(acc, a_s * w_s, bias)) * inv_smooth (the GEMM's GELU
// epilogue arithmetic) back into S.acc as floats, and each row's partial maximum over the slice's 128
// columns -> every CTA. G threads per row (128 / G columns each), so short sequences spread their
// rows over all threads.
template <int G>
__device__ __forceinline__ void gelu_slice(const Smem& S, int c, int rows, int tid, int use_erf) {
  constexpr int CW = 128 / G;
  const int r = tid / G, cb = (tid % G) * CW;
  float vmax = 1e-8f;
  if (r < rows) {
    const float as = S.as[r];
    int32_t* arow = S.acc + r * 129;
    float* grow = reinterpret_cast<float*>(arow);
    const float* fws = S.vec + V_FIW + cb;
    const float* fb = S.vec + V_FIB + cb;
    const float* finv = S.vec + V_FOINV + cb;
    if (use_erf) {
#pragma unroll
      for (int j = 0; j < CW; ++j) {
        const float gv = gelu_erf(fmaf(float(arow[cb + j]), as * fws[j], fb[j])) * finv[j];
        vmax = fmaxf(vmax, fabsf(gv));
        grow[cb + j] = gv;
      }
    } else {
#pragma unroll
      for (int j = 0; j < CW; j += 2) {
        const float2 ws2 = make_float2(fws[j], fws[j + 1]);
        const float2 b2 = make_float2(fb[j], fb[j + 1]);
        const float2 iv2 = make_float2(finv[j], finv[j + 1]);
        const float2 h = __ffma2_rn(make_float2(float(arow[cb + j]), float(arow[cb + j + 1])),
                                    __fmul2_rn(make_float2(as, as), ws2), b2);
        const float2 gv = __fmul2_rn(gelu_ref2(h), iv2);
        vmax = fmaxf(vmax, fmaxf(fabsf(gv.x), fabsf(gv.y)));
        grow[cb + j] = gv.x;
        grow[cb + j + 1] = gv.y;
      }
    }
  }
#pragma unroll
  for (int o = 1; o < G; o <<= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
  const int t = tid % G;
  if (r < rows && t < kLatCtas) st_cluster_f32(map_peer(S.xgm + c * kR + r, uint32_t(t)), vmax);
  if (G == 8 && r < rows && t < 4)  // 8 threads per row: the first 4 take the remaining CTAs
    for (int p = t + 8; p < kLatCtas; p += 4) st_cluster_f32(map_peer(S.xgm + c * kR + r, uint32_t(p)), vmax);
}

__global__ void __launch_bounds__(kLatThreads, 1)
    k_forward_lat(const LatModel* __restrict__ m, const uint16_t* __restrict__ ids, int L, float* __restrict__ out,
                  int* err, int use_erf) {
  extern __shared__ uint8_t lat_raw[];
  uint8_t* sm = lat_raw + ((1024u - (smem_u32(lat_raw) & 1023u)) & 1023u);
  Smem S;
  S.A = reinterpret_cast<int8_t*>(sm + OFF_A);
  S.B[0] = sm + OFF_B0;
  S.B[1] = sm + OFF_B1;
  S.acc = reinterpret_cast<int32_t*>(sm + OFF_ACC);
  S.kd = reinterpret_cast<float*>(sm + OFF_KD);
  S.vd = S.kd + 32 * kP;
  S.es = S.vd + 32 * kP;
  S.qd = S.es + 32 * kP;
  S.hg = reinterpret_cast<float*>(sm + OFF_HG);
  S.res = reinterpret_cast<float*>(sm + OFF_RES);
  S.xcm = reinterpret_cast<float*>(sm + OFF_XCM);
  S.xgm = reinterpret_cast<float*>(sm + OFF_XGM);
  S.as = reinterpret_cast<float*>(sm + OFF_AS);
  S.vec = reinterpret_cast<float*>(sm + OFF_VEC);
  S.bw = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
  S.bmma = S.bw + 2;
  S.tslot = reinterpret_cast<uint32_t*>(sm + OFF_TMEM);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = int(cluster_ctarank());
  if (L < 1 || L > kLatMaxTokens) {  // uniform over the cluster: every CTA leaves here
    if (tid == 0 && c == 0) record_err(err, DEV_ERR_BAD_SHAPE);
    return;
  }
  if (tid == 0) {
    mbar_init(&S.bw[0], 1);
    mbar_init(&S.bw[1], 1);
    mbar_init(S.bmma, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(S.tslot, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *S.tslot;
  if (tid == 0) {
    issue_weights(m, S, 0, c);
    issue_weights(m, S, 1, c);
  }
  cluster_sync_all();  // every CTA has started before any CTA stores into another's shared memory
  bool ok = true;
  const float qscale = 1.0f / sqrtf(32.0f);

  // ---- embeddings of the owned rows (dequant_add_embeddings_row as k_embed_ln_quant computes it),
  // then their LayerNorm + quantization with layer 0's inv_smooth -> every CTA
  {
    const int nown = owned_rows(c, L);
    for (int i = tid; i < nown * kHidden; i += kLatThreads) {
      const int k = i / kHidden, j = i - k * kHidden;
      const int r = c + kLatCtas * k;
      int tok = ids[r];
      if (tok >= kVocab) {
        if (j == 0) record_err(err, DEV_ERR_BAD_TOKEN);
        tok = 0;
      }
      S.hg[i] = (float(m->word_q[size_t(tok) * kHidden + j]) * m->word_s[tok] +
                 float(m->pos_q[size_t(r) * kHidden + j]) * m->pos_s[r]) +
                m->type0[j];
    }
    __syncthreads();
    ln_quant_owned(S, m->emb_lnw, m->emb_lnb, m->layer[0].qkv.invs, c, L, tid);
  }
  fence_proxy_async_all();
  cluster_sync_all();

  for (int l = 0; l < kLayers; ++l) {
    const bool last = l == kLayers - 1;
    const int s0 = 4 * l;
    // rows from the attention output on: all L rows, except in the pruned last layer ([CLS] only)
    const int rows = last ? 1 : L;

    // ---- Q | K | V of head c (N = 96); the layer's vectors arrive meanwhile
    prefetch_layer(m, S, l, c, tid);
    ok = run_gemm<96>(m, S, s0, 3, tmem, c, err, ok, tid, warp, lane);
    cp_async_wait_all();
    __syncthreads();
    {
      const float* ws = S.vec + V_QKVW;
      const float* bias = S.vec + V_QKVB;
      for (int i = tid; i < L * 96; i += kLatThreads) {
        const int r = i / 96, n = i - r * 96;
        const float v = fmaf(float(S.acc[r * 97 + n]), S.as[r] * ws[n], bias[n]);
        if (n < 32) S.qd[r * 32 + n] = v;
        else if (n < 64) S.kd[(n - 32) * kP + r] = v;
        else S.vd[(n - 64) * kP + r] = v;
      }
    }
    __syncthreads();

    // ---- attention of head c (eight lanes per query, all 256 threads; the [CLS] query alone in
    // the last layer); the partial row maxima of the context slice -> every CTA
    float cx[4];
    const int ql = tid >> 3, sl = tid & 7;
    const bool att = warp < (last ? 1 : 8);  // warp-uniform
    const bool qactive = att && ql < rows;
    const int qi = qactive ? ql : rows - 1;
    const float* ivs = S.vec + V_AOINV + 32 * c + 4 * sl;
    if (att) {
      float q[32];
#pragma unroll
      for (int d = 0; d < 32; ++d) q[d] = S.qd[qi * 32 + d] * qscale;
      attend_query_lanes8(q, S.kd, S.vd, kP, S.es + ql * kP, L, sl, cx);
      float vmax = 1e-8f;
#pragma unroll
      for (int k = 0; k < 4; ++k) vmax = fmaxf(vmax, fabsf(cx[k] * ivs[k]));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 4));
      if (qactive) {
        st_cluster_f32(map_peer(S.xcm + c * kR + qi, uint32_t(sl)), vmax);
        if (sl < kLatCtas - 8) st_cluster_f32(map_peer(S.xcm + c * kR + qi, uint32_t(sl + 8)), vmax);
      }
    }
    cluster_sync_all();

    // ---- each CTA quantizes its own 32 context columns with the row maxima -> every CTA's A
    if (qactive) {
      float max_abs = S.xcm[qi];
#pragma unroll
      for (int p = 1; p < kLatCtas; ++p) max_abs = fmaxf(max_abs, S.xcm[p * kR + qi]);
      const float inv_scale = 127.0f / max_abs;
      uint32_t w = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) w |= (uint32_t(quant_i8(cx[k] * (ivs[k] * inv_scale))) & 0xFFu) << (8 * k);
      const int off = a_off(qi, 32 * c + 4 * sl);
#pragma unroll
      for (int p = 0; p < kLatCtas; ++p) st_cluster_u32(map_peer(S.A + off, uint32_t(p)), w);
      if (sl == 0) S.as[qi] = max_abs / 127.0f;
    }
    fence_proxy_async_all();
    cluster_sync_all();

    // ---- attention-out slice c with the residual -> the row owners
    ok = run_gemm<32>(m, S, s0 + 1, 3, tmem, c, err, ok, tid, warp, lane);
    epilogue_residual_push(S, S.vec + V_AOW, S.vec + V_AOB, c, rows, tid);
    cluster_sync_all();

    // ---- LayerNorm 1 + quantization for FFN-up (owned rows) -> every CTA
    ln_quant_owned(S, S.vec + V_LN1W, S.vec + V_LN1B, S.vec + V_FIINV, c, rows, tid);
    fence_proxy_async_all();
    cluster_sync_all();

    // ---- FFN-up slice c (N = 128): g = GELU(h) * inv_smooth; partial row maxima -> every CTA
    ok = run_gemm<128>(m, S, s0 + 2, 3, tmem, c, err, ok, tid, warp, lane);
    if (rows <= 8) gelu_slice<32>(S, c, rows, tid, use_erf);
    else if (rows <= 16) gelu_slice<16>(S, c, rows, tid, use_erf);
    else gelu_slice<8>(S, c, rows, tid, use_erf);
    cluster_sync_all();
    {  // the slice quantized with the row maximum over all 1,536 columns -> k-block c of every A
      const int r = tid >> 3, ch = tid & 7;
      if (r < rows) {
        float max_abs = S.xgm[r];
#pragma unroll
        for (int p = 1; p < kLatCtas; ++p) max_abs = fmaxf(max_abs, S.xgm[p * kR + r]);
        const float inv_scale = 127.0f / max_abs;
        const float* grow = reinterpret_cast<const float*>(S.acc + r * 129) + ch * 16;
        uint4 v;
        v.x = pack_i8x4(quant_bits_scaled(grow[0] * inv_scale), quant_bits_scaled(grow[1] * inv_scale),
                        quant_bits_scaled(grow[2] * inv_scale), quant_bits_scaled(grow[3] * inv_scale));
        v.y = pack_i8x4(quant_bits_scaled(grow[4] * inv_scale), quant_bits_scaled(grow[5] * inv_scale),
                        quant_bits_scaled(grow[6] * inv_scale), quant_bits_scaled(grow[7] * inv_scale));
        v.z = pack_i8x4(quant_bits_scaled(grow[8] * inv_scale), quant_bits_scaled(grow[9] * inv_scale),
                        quant_bits_scaled(grow[10] * inv_scale), quant_bits_scaled(grow[11] * inv_scale));
        v.w = pack_i8x4(quant_bits_scaled(grow[12] * inv_scale), quant_bits_scaled(grow[13] * inv_scale),
                        quant_bits_scaled(grow[14] * inv_scale), quant_bits_scaled(grow[15] * inv_scale));
        const int off = c * kKbBytes + r * 128 + ((ch ^ (r & 7)) << 4);
#pragma unroll
        for (int p = 0; p < kLatCtas; ++p) st_cluster_u32x4(map_peer(S.A + off, uint32_t(p)), v);
        if (ch == 0) S.as[r] = max_abs / 127.0f;
      }
    }
    fence_proxy_async_all();
    cluster_sync_all();

    // ---- FFN-down slice c (N = 32, K = 1536) with the residual -> the row owners
    ok = run_gemm<32>(m, S, s0 + 3, 12, tmem, c, err, ok, tid, warp, lane);
    epilogue_residual_push(S, S.vec + V_FOW, S.vec + V_FOB, c, rows, tid);
    cluster_sync_all();

    if (!last) {  // ---- LayerNorm 2 + quantization for the next layer (owned rows) -> every CTA
      ln_quant_owned(S, S.vec + V_LN2W, S.vec + V_LN2B, S.vec + V_NXINV, c, rows, tid);
      fence_proxy_async_all();
      cluster_sync_all();
    }
  }

  // ---- final LayerNorm + L2 normalisation of the [CLS] row (row 0, owned by CTA 0;
  // k_ln_final_rows' sequential sums)
  if (c == 0) {
    if (tid == 0) {
      float* x = S.hg;
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
        const float y = (x[j] - mean) * rstd * S.vec[V_LN2W + j] + S.vec[V_LN2B + j];
        x[j] = y;
        ss = ss + y * y;
      }
      if (ss > 0.0f) {
        const float inv = 1.0f / sqrtf(ss);
        for (int j = 0; j < kHidden; ++j) x[j] = x[j] * inv;
      }
    }
    __syncthreads();
    for (int j = tid; j < kHidden; j += kLatThreads) out[j] = S.hg[j];
  }
  // no CTA leaves while another may still store into its shared memory
  cluster_sync_all();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 128);
  (void)ok;
}

}  // namespace

bool lat_prime() {
  if (cudaFuncSetAttribute(k_forward_lat, cudaFuncAttributeMaxDynamicSharedMemorySize, kLatSmem) != cudaSuccess)
    return false;
  if (cudaFuncSetAttribute(k_forward_lat, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kLatCtas);
  cfg.blockDim = dim3(kLatThreads);
  cfg.dynamicSmemBytes = kLatSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kLatCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, k_forward_lat, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return clusters >= 1;
}

int launch_forward_lat(const LatModel* d_model, const uint16_t* d_ids, int L, float* d_out, int* err, int gelu_erf,
                       cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kLatCtas);
  cfg.blockDim = dim3(kLatThreads);
  cfg.dynamicSmemBytes = kLatSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kLatCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_forward_lat, d_model, d_ids, L, d_out, err, gelu_erf) == cudaSuccess ? 0 : -1;
}

}  // namespace ae
