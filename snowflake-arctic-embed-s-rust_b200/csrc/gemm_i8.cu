// int8 x int8 -> int32 GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8) with fused epilogues.
//
// Contract (src/gemm.rs:627-628, gemm_scalar_fused src/gemm.rs:2000-2029):
//   acc[m,n] = sum_k A[m,k] * W[n,k]                      (exact int32)
//   h[m,n]   = fma(float(acc), a_scale[m] * w_scale[n], bias[n] (+ res[m,n]))
// A is [M,K] row-major int8, W is [N,K] row-major int8 (out_features x in_features), both K-major
// operands for tcgen05.
//
// Structure: a persistent, warp-specialised kernel, one CTA per SM (576 threads).
//   warp 0      TMA producer: the CTA's slice of W (BN rows) is loaded once and stays in shared
//               memory when K = 384 ("resident"); A tiles (128 rows) stream through a STAGES-deep
//               ring of 128-byte K blocks (128-byte swizzle, no multicast).
//   warp 1      MMA issuer: one thread issues the tcgen05.mma of each tile into a TMEM accumulator;
//               two accumulators alternate when 2 x BN <= 512 TMEM columns, so the epilogue of one
//               tile overlaps the MMAs of the next.
//   warps 2-17  epilogue: 4 warps per TMEM lane quadrant (32 rows), each with a quarter of the
//               columns, so the FP32 epilogue work runs on 16 warps.
// Each CTA keeps one N slice and walks the M tiles m0 = start, start + stride, ...
//
// Epilogues:
//   EPI_F32        out[m,n] = h                                   (QKV, KV-only, Q-only projections)
//   EPI_LN_QUANT   hidden = LayerNorm(h) written back as the new residual, then the SmoothQuant
//                  dynamic row quantization for the next GEMM (attention-out and FFN-down;
//                  src/model.rs:330-353, :375-397 with layernorm_smooth_quantize_row_avx2,
//                  src/simd_math.rs:369-477). The full 384-wide row is in one CTA; warp q of a
//                  quadrant owns the reduction lanes 4q..4q+3 (columns 16k + 4q + e) so every
//                  exact-order partial-sum chain stays inside one thread, and the 16 lanes are
//                  combined through shared memory with the reference's hsum256 tree.
//   EPI_GELU_QUANT g = GELU(h) * inv_smooth, row max over all 1536 columns, row quantization
//                  (FFN-up; gelu_smooth_quantize_row_avx2, src/simd_math.rs:1371-1435). A cluster
//                  of 6 CTAs holds the 6 slices of 256 columns of the same 128 rows (12 CTAs of 128
//                  columns when the batch has at most 12 row tiles); each CTA sends
//                  its partial row maxima into its peers' shared memory with st.async, which
//                  completes on the peers' mbarriers. GELU is the reference's rational
//                  approximation (gelu_ref) or, on request, the exact erf.
//   EPI_LN_FINAL   out = l2_normalize(layernorm_inplace_row(h))  (layer-11 FFN-down of the [CLS]
//                  rows; src/model.rs:496-512, src/simd_math.rs:481-497, :2892-2903; sequential sums)
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>

#include "gemm_i8.h"
#include "ptx.cuh"
#include "rowmath.cuh"

namespace ae {

constexpr int BM = 128;            // rows per tile
constexpr int BK = 128;            // K bytes per block (one 128-byte swizzle atom wide)
constexpr int A_STAGE = BM * BK;   // 16 KB
constexpr int kEpiWarps = 16;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kTmemBar = 15;  // named barrier of the MMA and epilogue warps (the epilogues use 1..8)
constexpr int kResK = 384;         // K of the GEMMs whose weight slice stays resident
constexpr int kResKB = kResK / BK;

template <int BN, int EPI, bool RES, int STAGES>
struct Layout {
  static constexpr bool LN = EPI == EPI_LN_QUANT || EPI == EPI_LN_FINAL;
  static constexpr int NB = (2 * BN <= 512) ? 2 : 1;                   // TMEM accumulators
  static constexpr uint32_t TCOLS = (NB * BN <= 128) ? 128 : (NB * BN <= 256 ? 256 : 512);
  static constexpr int NSUB = BN <= 256 ? BN : BN / 2;                  // N of one MMA
  static constexpr int B_RES = RES ? kResKB * BN * BK : 0;
  static constexpr int STAGE = A_STAGE + (RES ? 0 : BN * BK);
  static constexpr int RING = STAGES * STAGE;
  static constexpr int PARAM_FLOATS = 3 * BN + 2 * kHidden;             // ws, bias, invs | gamma, beta
  // EPI_GELU_QUANT: the cluster holds the 1,536 columns of a tile as kInter / BN slices of BN columns
  static constexpr int GCL = EPI == EPI_GELU_QUANT ? kInter / BN : 1;
  static constexpr int XCH_FLOATS_GELU = 2 * 4 * BM + 2 * GCL * BM;
  static constexpr int STAGING_BYTES = EPI == EPI_GELU_QUANT ? kEpiWarps * 32 * 80 : 0;  // int8 output rows
  static constexpr int NBARS_ = 2 * STAGES + 1 + 2 * 2 + 2;
  // EPI_F32 with a row-major output: each epilogue warp transposes its 32 rows x STG_W columns through
  // shared memory (pitch STG_W + 1) so that the stores are whole row segments; 32 columns where
  // the memory allows, else 16, else none (per-row stores)
  static constexpr int BASE_BYTES = 1024 + B_RES + RING + 4 * PARAM_FLOATS + 8 * NBARS_ + 16;
  static constexpr int STG_W = EPI != EPI_F32 ? 0
                               : (BASE_BYTES + 4 * kEpiWarps * 32 * 33 <= 232448 && (BN / 4) % 32 == 0)
                                   ? 32
                                   : (BASE_BYTES + 4 * kEpiWarps * 32 * 17 <= 232448 ? 16 : 0);
  static constexpr int STG_FLOATS = STG_W ? kEpiWarps * 32 * (STG_W + 1) : 0;
  static constexpr int XCH_FLOATS =
      LN ? (2 * BM * 17 + BM * 5) : (EPI == EPI_GELU_QUANT ? XCH_FLOATS_GELU + STAGING_BYTES / 4 : STG_FLOATS);
  static constexpr int NBARS = NBARS_;
  static constexpr int TOTAL = 1024 + B_RES + RING + 4 * (PARAM_FLOATS + XCH_FLOATS) + 8 * NBARS + 16;
  static_assert(TOTAL <= 232448, "shared memory of one CTA exceeds the sm_100 limit");
};

template <int BN, int EPI, bool RES, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_i8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs g,
              int n_tiles_n, int m_tiles) {
  using Ly = Layout<BN, EPI, RES, STAGES>;
  constexpr int NB = Ly::NB;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned (128-byte swizzle atoms) by pointer arithmetic on the shared array itself, so
  // that the compiler keeps the parameter and exchange accesses in the shared address space
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* b_res = smem;
  uint8_t* ring = smem + Ly::B_RES;
  float* s_ws = reinterpret_cast<float*>(ring + Ly::RING);
  float* s_bias = s_ws + BN;
  float* s_invs = s_bias + BN;
  float* s_gamma = s_invs + BN;
  float* s_beta = s_gamma + kHidden;
  float* xch = s_beta + kHidden;
  uint64_t* bars = reinterpret_cast<uint64_t*>(xch + Ly::XCH_FLOATS);
  uint64_t* full = bars;
  uint64_t* empty = full + STAGES;
  uint64_t* bfull = empty + STAGES;
  uint64_t* acc_full = bfull + 1;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* rmx_bar = acc_empty + 2;  // EPI_GELU_QUANT: peers' row maxima arrived (per tile parity)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Ly::NBARS);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n_tile = blockIdx.x % n_tiles_n;
  const int n0 = n_tile * BN;
  const int m_first = blockIdx.x / n_tiles_n;
  const int m_stride = gridDim.x / n_tiles_n;
  const int my_tiles = m_first < m_tiles ? (m_tiles - 1 - m_first) / m_stride + 1 : 0;
  const int KB = g.K / BK;
  pdl_trigger();

  if (tid == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(bfull, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      // EPI_GELU_QUANT: the epilogue warps form two groups of 8 that take alternate tiles
      mbar_init(&acc_empty[b], EPI == EPI_GELU_QUANT ? kEpiWarps / 2 : kEpiWarps);
      mbar_init(&rmx_bar[b], 1);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < BN; i += blockDim.x) {
    const int n = n0 + i;
    s_ws[i] = g.w_scale[n];
    s_bias[i] = g.bias[n];
    if constexpr (EPI == EPI_LN_QUANT || EPI == EPI_GELU_QUANT) s_invs[i] = g.inv_smooth[n];
  }
  if constexpr (Ly::LN) {
    for (int i = tid; i < kHidden; i += blockDim.x) {
      s_gamma[i] = g.gamma[i];
      s_beta[i] = g.beta[i];
    }
  }
  __syncthreads();
  if constexpr (EPI == EPI_GELU_QUANT) {  // peers' barriers are initialised before any st.async
    cluster_arrive_release();
    cluster_wait_acquire();
  }
  if constexpr (RES) {  // the weights are model constants: requested before waiting for the previous kernel
    if (tid == 0) {
      mbar_arrive_expect_tx(bfull, Ly::B_RES);
      for (int kb = 0; kb < kResKB; ++kb)
        for (int j = 0; j < BN / 64; ++j)
          tma_load_2d(b_res + (kb * BN + j * 64) * BK, &tmB, bfull, kb * BK, n0 + j * 64);
    }
  }
  pdl_wait();
  // TMEM is allocated only after the wait: a CTA waiting for the previous kernel holds none, so that
  // kernel's CTAs can always allocate theirs. The producer needs no TMEM and starts loading at once;
  // the MMA warp allocates while the first stage is in flight and hands the address to the epilogue.
  uint32_t tmem = 0;
  if (warp >= 1) {
    if (warp == 1) {
      tmem_alloc(tmem_slot, Ly::TCOLS);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar(kTmemBar, kThreads - 32);
    tc_fence_after();
    tmem = *tmem_slot;
  }

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      int kc = 0;
      for (int it = 0; it < my_tiles && ok; ++it) {
        const int m0 = (m_first + it * m_stride) * BM;
        if constexpr (Ly::LN) {
          // the epilogue reads this tile's residual: one contiguous block in the tile-transposed layout
          if (g.res_tt && g.res && m0 < g.M) prefetch_l2_bulk(g.res + size_t(m0) * g.ldr, uint32_t(BM) * g.ldr * 4);
        }
        for (int kb = 0; kb < KB; ++kb, ++kc) {
          const int s = kc % STAGES;
          if (kc >= STAGES && !(ok = mbar_wait(&empty[s], ((kc / STAGES) - 1) & 1, g.err, DEV_ERR_TIMEOUT_PRODUCER)))
            break;
          uint8_t* st = ring + s * Ly::STAGE;
          mbar_arrive_expect_tx(&full[s], Ly::STAGE);
          tma_load_2d(st, &tmA, &full[s], kb * BK, m0);
          if constexpr (!RES) {
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(st + A_STAGE + j * 64 * BK, &tmB, &full[s], kb * BK, n0 + j * 64);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      if constexpr (RES) ok = mbar_wait(bfull, 0, g.err, DEV_ERR_TIMEOUT_MMA);
      constexpr uint32_t idesc = idesc_i8(BM, Ly::NSUB);
      int kc = 0;
      for (int it = 0; it < my_tiles && ok; ++it) {
        const int b = it % NB, u = it / NB;
        if (u >= 1 && !(ok = mbar_wait(&acc_empty[b], (u - 1) & 1, g.err, DEV_ERR_TIMEOUT_MMA))) break;
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(b * BN);
        for (int kb = 0; kb < KB; ++kb, ++kc) {
          const int s = kc % STAGES;
          if (!(ok = mbar_wait(&full[s], (kc / STAGES) & 1, g.err, DEV_ERR_TIMEOUT_MMA))) break;
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + s * Ly::STAGE);
          const uint32_t b_addr = RES ? smem_u32(b_res + kb * BN * BK) : a_addr + A_STAGE;
#pragma unroll
          for (int ks = 0; ks < BK / 32; ++ks) {
            const uint64_t ad = sdesc_sw128(a_addr + ks * 32);
#pragma unroll
            for (int j = 0; j < BN / Ly::NSUB; ++j)
              mma_i8(d + j * Ly::NSUB, ad, sdesc_sw128(b_addr + j * Ly::NSUB * BK + ks * 32), idesc, (kb | ks) != 0);
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ epilogue
    const int ew = warp - 2;       // 0..15
    const int Q = warp & 3;        // TMEM lane quadrant this warp may access
    const int qq = ew >> 2;        // column quarter (F32, GELU) / reduction-lane group (LN)
    const int rt = Q * 32 + lane;  // row within the tile
    const uint32_t tq = tmem + (uint32_t(Q * 32) << 16);
    // EPI_GELU_QUANT: warps 0-7 of the epilogue take the even tiles (TMEM accumulator 0), warps
    // 8-15 the odd ones (accumulator 1), two warps per lane quadrant each with half the columns, so
    // that one group's row-maximum exchange and quantization overlap the other group's GELU
    const int grp = EPI == EPI_GELU_QUANT ? ew >> 3 : 0;
    // EPI_LN_QUANT: a row-major residual whose rows are 16-byte aligned is read 16 bytes at a time
    [[maybe_unused]] const bool res_v4 =
        g.res && !g.res_tt && (reinterpret_cast<uintptr_t>(g.res) & 15) == 0 && (g.ldr & 3) == 0;
    const int it_step = EPI == EPI_GELU_QUANT ? 2 : 1;
    bool ok = true;
    for (int it = grp; it < my_tiles; it += it_step) {
      const int b = it % NB, u = it / NB;
      const int m0 = (m_first + it * m_stride) * BM;
      const int row = m0 + rt;
      // inputs that do not depend on the accumulator are requested while the MMA runs: the row
      // scale (not in the GELU epilogue, whose registers are the tighter) and, in the LayerNorm
      // epilogue, the first 16 residual values of the row
      float as_pre = 0.0f;
      if constexpr (EPI != EPI_GELU_QUANT) as_pre = row < g.M ? g.a_scale[row] : 0.0f;
      [[maybe_unused]] float rv0[16], rv1[16];
      if constexpr (EPI == EPI_LN_QUANT) {  // residual chunks 0 and 1 (column blocks 0-7)
        if (row < g.M) {
          if (g.res_tt) {
            const float* rr = g.res + tt_index(row, 0, g.ldr);
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                rv0[4 * k + e] = __ldcs(rr + size_t(16 * k + 4 * qq + e) * 128);
                rv1[4 * k + e] = __ldcs(rr + size_t(16 * (k + 4) + 4 * qq + e) * 128);
              }
          } else if (res_v4) {  // row-major: the thread's four columns of a block are one 16-byte load
            const float4* rr = reinterpret_cast<const float4*>(g.res + size_t(row) * g.ldr + 4 * qq);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float4 x0 = __ldcs(rr + 4 * k), x1 = __ldcs(rr + 4 * (k + 4));
              rv0[4 * k] = x0.x; rv0[4 * k + 1] = x0.y; rv0[4 * k + 2] = x0.z; rv0[4 * k + 3] = x0.w;
              rv1[4 * k] = x1.x; rv1[4 * k + 1] = x1.y; rv1[4 * k + 2] = x1.z; rv1[4 * k + 3] = x1.w;
            }
          } else {
            const float* rr = g.res + size_t(row) * g.ldr;
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                rv0[4 * k + e] = __ldcs(rr + 16 * k + 4 * qq + e);
                rv1[4 * k + e] = __ldcs(rr + 16 * (k + 4) + 4 * qq + e);
              }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) rv0[i] = rv1[i] = 0.0f;
        }
      }
      if (ok) ok = mbar_wait(&acc_full[b], u & 1, g.err, DEV_ERR_TIMEOUT_EPILOGUE);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const bool valid = ok && row < g.M;
      const float as = !valid ? 0.0f : (EPI == EPI_GELU_QUANT ? g.a_scale[row] : as_pre);
      const uint32_t tb = tq + uint32_t(b * BN);

      if constexpr (EPI == EPI_F32) {
        constexpr int CW = BN / 4;
        const int c0 = qq * CW;
        uint32_t r[CW];
        if (ok) {
#pragma unroll
          for (int ch = 0; ch < CW / 16; ++ch) tmem_ld16(tb + c0 + ch * 16, r + ch * 16);
          tmem_ld_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
        if (valid && g.acc_dbg) {
          int4* ad = reinterpret_cast<int4*>(g.acc_dbg + size_t(row) * g.N + n0 + c0);
#pragma unroll
          for (int q = 0; q < CW / 4; ++q)
            ad[q] = make_int4(int(r[4 * q]), int(r[4 * q + 1]), int(r[4 * q + 2]), int(r[4 * q + 3]));
        }
        if constexpr (Ly::STG_W > 0) {
          if (!g.out_tt && !g.res) {
            // row-major output through the warp's staging tile: lane = row writes SW values, then
            // lane = column stores whole row segments (SW = 32: one 128-byte line per row)
            constexpr int SW = Ly::STG_W, PITCH = SW + 1;
            float* stg = xch + ew * 32 * PITCH;
            const int rbase = m0 + Q * 32;
#pragma unroll
            for (int c1 = 0; c1 < CW; c1 += SW) {
#pragma unroll
              for (int j = 0; j < SW; ++j)
                stg[lane * PITCH + j] = fmaf(float(int(r[c1 + j])), as * s_ws[c0 + c1 + j], s_bias[c0 + c1 + j]);
              __syncwarp();
              constexpr int RPI = 32 / SW;  // rows per store instruction
              const int cl = lane % SW, rsub = lane / SW;
              float* ocol = g.out_f32 + n0 + c0 + c1 + cl;
#pragma unroll 4
              for (int r0 = 0; r0 < 32; r0 += RPI) {
                const int rr = r0 + rsub;
                if (ok && rbase + rr < g.M) ocol[size_t(rbase + rr) * g.ldo] = stg[rr * PITCH + cl];
              }
              __syncwarp();
            }
            continue;
          }
        }
        if (valid) {
          if (g.out_tt && !g.res) {  // one 128-byte line per column for the warp's 32 rows
            float* o = g.out_f32 + tt_index(row, n0 + c0, g.ldo);
#pragma unroll
            for (int j4 = 0; j4 < CW / 4; ++j4) {  // column parameters as 16-byte broadcast loads
              const float4 w4 = *reinterpret_cast<const float4*>(s_ws + c0 + 4 * j4);
              const float4 b4 = *reinterpret_cast<const float4*>(s_bias + c0 + 4 * j4);
              const float wv[4] = {w4.x, w4.y, w4.z, w4.w}, bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                o[size_t(4 * j4 + e) << 7] = fmaf(float(int(r[4 * j4 + e])), as * wv[e], bv[e]);
            }
            continue;
          }
          float* o = g.out_f32 + size_t(row) * g.ldo + n0 + c0;
          const float* rs = g.res ? g.res + size_t(row) * g.ldr + n0 + c0 : nullptr;
          const float* rs_tt = (g.res && g.res_tt) ? g.res + tt_index(row, n0 + c0, g.ldr) : nullptr;
#pragma unroll
          for (int q = 0; q < CW / 4; ++q) {
            float v[4];
            float4 rr = make_float4(0.f, 0.f, 0.f, 0.f);
            if (rs_tt)
              rr = make_float4(rs_tt[(4 * q) << 7], rs_tt[(4 * q + 1) << 7], rs_tt[(4 * q + 2) << 7],
                               rs_tt[(4 * q + 3) << 7]);
            else if (rs)
              rr = reinterpret_cast<const float4*>(rs)[q];
            const float rv[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = 4 * q + e;
              float bb = s_bias[c0 + j];
              if (rs) bb = bb + rv[e];
              v[e] = fmaf(float(int(r[j])), as * s_ws[c0 + j], bb);
            }
            reinterpret_cast<float4*>(o)[q] = make_float4(v[0], v[1], v[2], v[3]);
          }
        }
      } else if constexpr (EPI == EPI_GELU_QUANT) {
        static_assert(NB == 2, "the two epilogue groups alternate between the two accumulators");
        // 16 columns at a time: accumulators -> g = GELU(h) * inv_smooth -> back into the same TMEM
        // columns (few registers live, no spills); the accumulator buffer is released after the
        // quantization pass has read g back
        constexpr int CW = BN / 2;      // columns of this warp: half of the slice
        const int gq = (ew >> 2) & 1;   // which half
        const int c0 = gq * CW;
        const int par = it & 1;         // == grp
        const uint32_t rank = cluster_ctarank();
        // [2][BM] maxima of the column halves, alternating between two slots of the group's [4][BM],
        // so that no warp can write a slot its partner may still read
        float* xg = xch + par * 4 * BM + ((it >> 1) & 1) * 2 * BM;
        float* rmx = xch + 2 * 4 * BM + par * Ly::GCL * BM;  // [GCL][BM] maxima of the cluster CTAs
        uint32_t r[16];
        float vmax = 1e-8f;
        if (ok) {
#pragma unroll 1
          for (int ch = 0; ch < CW / 16; ++ch) {
            const int cc = c0 + 16 * ch;
            tmem_ld16(tb + cc, r);
            tmem_ld_wait();
            if (valid && g.acc_dbg) {
              int4* ad = reinterpret_cast<int4*>(g.acc_dbg + size_t(row) * g.N + n0 + cc);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                ad[q] = make_int4(int(r[4 * q]), int(r[4 * q + 1]), int(r[4 * q + 2]), int(r[4 * q + 3]));
            }
            if (g.gelu_erf) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int c = cc + j;
                const float gv = gelu_erf(fmaf(float(int(r[j])), as * s_ws[c], s_bias[c])) * s_invs[c];
                vmax = fmaxf(vmax, fabsf(gv));
                r[j] = __float_as_uint(gv);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {  // column parameters as 16-byte broadcast loads
                const int c = cc + j;
                const float4 ws4 = *reinterpret_cast<const float4*>(s_ws + c);
                const float4 b4 = *reinterpret_cast<const float4*>(s_bias + c);
                const float4 iv4 = *reinterpret_cast<const float4*>(s_invs + c);
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                  const float2 ws2 = hf ? make_float2(ws4.z, ws4.w) : make_float2(ws4.x, ws4.y);
                  const float2 b2 = hf ? make_float2(b4.z, b4.w) : make_float2(b4.x, b4.y);
                  const float2 iv2 = hf ? make_float2(iv4.z, iv4.w) : make_float2(iv4.x, iv4.y);
                  const int jj = j + 2 * hf;
                  const float2 h = __ffma2_rn(make_float2(float(int(r[jj])), float(int(r[jj + 1]))),
                                              __fmul2_rn(make_float2(as, as), ws2), b2);
                  const float2 gv = __fmul2_rn(gelu_ref2(h), iv2);
                  vmax = fmaxf(vmax, fmaxf(fabsf(gv.x), fabsf(gv.y)));
                  r[jj] = __float_as_uint(gv.x);
                  r[jj + 1] = __float_as_uint(gv.y);
                }
              }
            }
            tmem_st16(tb + cc, r);
          }
          tmem_st_wait();
        }
        xg[gq * BM + rt] = vmax;
        named_bar(1 + Q + 4 * grp, 64);  // the group's two warps of this lane quadrant
        const float cta_max = fmaxf(xg[rt], xg[BM + rt]);
        if ((ew & 7) == 0 && lane == 0) mbar_arrive_expect_tx(&rmx_bar[par], Ly::GCL * BM * 4);
        if (gq == 0) {
#pragma unroll
          for (uint32_t q = 0; q < uint32_t(Ly::GCL); ++q)
            st_async_f32(map_peer(&rmx[rank * BM + rt], q), cta_max, map_peer(&rmx_bar[par], q));
        }
        if (ok) ok = mbar_wait(&rmx_bar[par], (it >> 1) & 1, g.err, DEV_ERR_TIMEOUT_EPILOGUE);
        float max_abs = rmx[rt];
#pragma unroll
        for (int q = 1; q < Ly::GCL; ++q) max_abs = fmaxf(max_abs, rmx[q * BM + rt]);
        const float inv_scale = 127.0f / max_abs;
        {
          // quantize 64 columns at a time into this warp's staging slot (32 rows x 64 bytes, rows
          // padded to 80 bytes), then write 8 rows x 64 contiguous bytes per store instruction
          uint8_t* stg = reinterpret_cast<uint8_t*>(xch + Ly::XCH_FLOATS_GELU) + ew * (32 * 80);
#pragma unroll 1
          for (int hc = 0; hc < CW / 64; ++hc) {
            const int cb = c0 + 64 * hc;
            if (ok) {
#pragma unroll 1
              for (int ch = 0; ch < 4; ++ch) {
                tmem_ld16(tb + cb + 16 * ch, r);
                tmem_ld_wait();
                uint32_t pk[4];
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  pk[q] = pack_i8x4(quant_bits_scaled(__uint_as_float(r[4 * q]) * inv_scale),
                                    quant_bits_scaled(__uint_as_float(r[4 * q + 1]) * inv_scale),
                                    quant_bits_scaled(__uint_as_float(r[4 * q + 2]) * inv_scale),
                                    quant_bits_scaled(__uint_as_float(r[4 * q + 3]) * inv_scale));
                *reinterpret_cast<uint4*>(stg + lane * 80 + 16 * ch) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              }
            }
            if (hc + 1 == CW / 64) {  // the last read of this accumulator
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&acc_empty[b]);
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int rr = 8 * i + lane / 4, q = lane % 4;
              const int grow = m0 + Q * 32 + rr;
              const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 80 + 16 * q);
              if (ok && grow < g.M) *reinterpret_cast<uint4*>(g.out_q + size_t(grow) * g.N + n0 + cb + 16 * q) = v;
            }
            __syncwarp();
          }
          if (valid && rank == 0 && gq == 0) g.out_scale[row] = max_abs / 127.0f;
        }
      } else if constexpr (EPI == EPI_LN_QUANT) {
        static_assert(BN == kHidden, "row-LayerNorm epilogue needs the full 384-wide row");
        // rows padded to 17 and 5 floats: the 32 rows of a warp fall in 32 different banks
        float* xs = xch;                 // [BM][17] partial sums
        float* xv = xch + BM * 17;       // [BM][17] partial sums of squares
        float* xm = xch + 2 * BM * 17;   // [BM][5]  partial maxima
        const int cq = 4 * qq;           // first owned column of every 16-column block
        uint32_t r[32];
        float p[4] = {0.f, 0.f, 0.f, 0.f};
        // pass 1: h = fma(acc, as * ws, bias + res) -> TMEM; partial sums (chains of lanes cq..cq+3)
        const float* res_row = nullptr;  // column c of this row at res_row[c * rstep]
        size_t rstep = 1;
        if (valid) {
          res_row = g.res_tt ? g.res + tt_index(row, 0, g.ldr) : g.res + size_t(row) * g.ldr;
          rstep = g.res_tt ? 128 : 1;
        }
        if (ok) {
          // residual chunks triple-buffered: chunk i + 2 (16 values) is requested before chunk i is
          // used; chunks 0 and 1 were requested before the accumulator wait
          float rv2[16];
#pragma unroll
          for (int i = 0; i < 6; ++i) {
            const int k0 = 4 * i;
            float* rv = (i % 3 == 0) ? rv0 : (i % 3 == 1) ? rv1 : rv2;
            float* nx = (i % 3 == 0) ? rv2 : (i % 3 == 1) ? rv0 : rv1;
            if (i + 2 < 6) {
              if (res_v4) {  // row-major, 16-byte aligned rows: one 16-byte load per block
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const float4 x = valid ? __ldcs(reinterpret_cast<const float4*>(res_row + 16 * (k0 + 8 + k) + cq))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                  nx[4 * k] = x.x; nx[4 * k + 1] = x.y; nx[4 * k + 2] = x.z; nx[4 * k + 3] = x.w;
                }
              } else {
#pragma unroll
                for (int k = 0; k < 4; ++k)
#pragma unroll
                  for (int e = 0; e < 4; ++e)
                    nx[4 * k + e] = valid ? __ldcs(res_row + size_t(16 * (k0 + 8 + k) + cq + e) * rstep) : 0.0f;
              }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int c = 16 * (k0 + k) + cq;
              tmem_ld4(tb + c, r + 4 * k);
              tmem_ld_wait();
              if (valid && g.acc_dbg)
                *reinterpret_cast<int4*>(g.acc_dbg + size_t(row) * g.N + c) =
                    make_int4(int(r[4 * k]), int(r[4 * k + 1]), int(r[4 * k + 2]), int(r[4 * k + 3]));
              const float4 wv = *reinterpret_cast<const float4*>(s_ws + c);
              const float4 bv = *reinterpret_cast<const float4*>(s_bias + c);
              const float wsv[4] = {wv.x, wv.y, wv.z, wv.w};
              const float bsv[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float h = fmaf(float(int(r[4 * k + e])), as * wsv[e], bsv[e] + rv[4 * k + e]);
                p[e] = p[e] + h;
                r[4 * k + e] = __float_as_uint(h);
              }
              tmem_st4(tb + c, r + 4 * k);
            }
          }
          tmem_st_wait();
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) xs[rt * 17 + cq + e] = p[e];
        named_bar(1 + Q, 128);
        float pp[16];
#pragma unroll
        for (int l = 0; l < 16; ++l) pp[l] = xs[rt * 17 + l];
        const float mean = tree16(pp) / float(kHidden);
        // pass 2: variance
#pragma unroll
        for (int e = 0; e < 4; ++e) p[e] = 0.0f;
        if (ok) {
          for (int k0 = 0; k0 < 24; k0 += 6) {
#pragma unroll
            for (int k = 0; k < 6; ++k) tmem_ld4(tb + 16 * (k0 + k) + cq, r + 4 * k);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 6; ++k)
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float d = __uint_as_float(r[4 * k + e]) - mean;
                p[e] = fmaf(d, d, p[e]);
              }
          }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) xv[rt * 17 + cq + e] = p[e];
        named_bar(1 + Q, 128);
#pragma unroll
        for (int l = 0; l < 16; ++l) pp[l] = xv[rt * 17 + l];
        const float var = tree16(pp) / float(kHidden);
        const float rstd = 1.0f / sqrtf(var + kLnEps);
        // pass 3: y = LN(h) -> residual out and TMEM; max |y * inv_smooth|
        float vmax = 1e-8f;
        float* out_row = valid ? (g.out_tt ? g.out_f32 + tt_index(row, 0, g.ldo) : g.out_f32 + size_t(row) * g.ldo)
                               : nullptr;
        if (ok) {
          for (int k0 = 0; k0 < 24; k0 += 6) {
#pragma unroll
            for (int k = 0; k < 6; ++k) tmem_ld4(tb + 16 * (k0 + k) + cq, r + 4 * k);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 6; ++k) {
              const int c = 16 * (k0 + k) + cq;
              const float4 gv4 = *reinterpret_cast<const float4*>(s_gamma + c);
              const float4 bv4 = *reinterpret_cast<const float4*>(s_beta + c);
              const float4 iv4 = *reinterpret_cast<const float4*>(s_invs + c);
              const float gv[4] = {gv4.x, gv4.y, gv4.z, gv4.w};
              const float bv[4] = {bv4.x, bv4.y, bv4.z, bv4.w};
              const float iv[4] = {iv4.x, iv4.y, iv4.z, iv4.w};
              float y[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                y[e] = fmaf((__uint_as_float(r[4 * k + e]) - mean) * rstd, gv[e], bv[e]);
                vmax = fmaxf(vmax, fabsf(y[e] * iv[e]));
                r[4 * k + e] = __float_as_uint(y[e]);
              }
              if (valid) {
                if (g.out_tt) {
                  float* op = out_row + size_t(c) * 128;
#pragma unroll
                  for (int e = 0; e < 4; ++e) op[e << 7] = y[e];
                } else {
                  *reinterpret_cast<float4*>(out_row + c) = make_float4(y[0], y[1], y[2], y[3]);
                }
              }
              tmem_st4(tb + c, r + 4 * k);
            }
          }
          tmem_st_wait();
        }
        xm[rt * 5 + qq] = vmax;
        tc_fence_before();
        named_bar(1 + Q, 128);
        tc_fence_after();
        const float max_abs = fmaxf(fmaxf(xm[rt * 5], xm[rt * 5 + 1]), fmaxf(xm[rt * 5 + 2], xm[rt * 5 + 3]));
        const float inv_scale = 127.0f / max_abs;
        // pass 4: quantize. Elementwise, so this warp takes the 96 contiguous columns
        // 96 qq .. 96 qq + 95 of its rows (written to TMEM by the quadrant's four warps in pass 3)
        // and stores each row's bytes as six 16-byte pieces.
        if (ok) {
          const int c0 = 96 * qq;
          for (int ch = 0; ch < 6; ch += 2) {
            tmem_ld16(tb + c0 + 16 * ch, r);
            tmem_ld16(tb + c0 + 16 * ch + 16, r + 16);
            tmem_ld_wait();
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int c = c0 + 16 * (ch + u);
              uint32_t w[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float4 iv = *reinterpret_cast<const float4*>(s_invs + c + 4 * q);
                const uint32_t* y = r + 16 * u + 4 * q;
                w[q] = pack_i8x4(quant_bits_scaled(__uint_as_float(y[0]) * (iv.x * inv_scale)),
                                 quant_bits_scaled(__uint_as_float(y[1]) * (iv.y * inv_scale)),
                                 quant_bits_scaled(__uint_as_float(y[2]) * (iv.z * inv_scale)),
                                 quant_bits_scaled(__uint_as_float(y[3]) * (iv.w * inv_scale)));
              }
              if (valid)
                *reinterpret_cast<uint4*>(g.out_q + size_t(row) * kHidden + c) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
        if (valid && qq == 0) g.out_scale[row] = max_abs / 127.0f;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
      } else {  // EPI_LN_FINAL
        static_assert(BN == kHidden, "row-LayerNorm epilogue needs the full 384-wide row");
        const int cq = 4 * qq;
        uint32_t r[32];
        // pass 1 (all 4 warps of the quadrant): h = fma(acc, as * ws, bias + res) -> TMEM
        if (ok) {
          for (int k0 = 0; k0 < 24; k0 += 6) {
#pragma unroll
            for (int k = 0; k < 6; ++k) tmem_ld4(tb + 16 * (k0 + k) + cq, r + 4 * k);
            tmem_ld_wait();
#pragma unroll
            for (int k = 0; k < 6; ++k) {
              const int c = 16 * (k0 + k) + cq;
              float4 rr = make_float4(0.f, 0.f, 0.f, 0.f);
              if (valid) rr = *reinterpret_cast<const float4*>(g.res + size_t(row) * g.ldr + c);
              const float rv[4] = {rr.x, rr.y, rr.z, rr.w};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                r[4 * k + e] = __float_as_uint(fmaf(float(int(r[4 * k + e])), as * s_ws[c + e], s_bias[c + e] + rv[e]));
              tmem_st4(tb + c, r + 4 * k);
            }
          }
          tmem_st_wait();
        }
        tc_fence_before();
        named_bar(1 + Q, 128);
        tc_fence_after();
        // the sequential sums of layernorm_inplace_row / l2_normalize_inplace: one warp per quadrant
        if (qq == 0 && ok) {
          float seq = 0.0f;
          for (int c = 0; c < kHidden; c += 32) {
            tmem_ld16(tb + c, r);
            tmem_ld16(tb + c + 16, r + 16);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) seq = seq + __uint_as_float(r[j]);
          }
          const float mean = seq / float(kHidden);
          seq = 0.0f;
          for (int c = 0; c < kHidden; c += 32) {
            tmem_ld16(tb + c, r);
            tmem_ld16(tb + c + 16, r + 16);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float d = __uint_as_float(r[j]) - mean;
              seq = seq + d * d;
            }
          }
          const float rstd = 1.0f / sqrtf(seq / float(kHidden) + kLnEps);
          float ss = 0.0f;
          for (int c = 0; c < kHidden; c += 32) {
            tmem_ld16(tb + c, r);
            tmem_ld16(tb + c + 16, r + 16);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float y = (__uint_as_float(r[j]) - mean) * rstd * s_gamma[c + j] + s_beta[c + j];
              ss = ss + y * y;
            }
          }
          const float inv_norm = ss > 0.0f ? 1.0f / sqrtf(ss) : 1.0f;
          for (int c = 0; c < kHidden; c += 32) {
            tmem_ld16(tb + c, r);
            tmem_ld16(tb + c + 16, r + 16);
            tmem_ld_wait();
            if (valid) {
              float4* o = reinterpret_cast<float4*>(g.out_f32 + size_t(row) * g.ldo + c);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int j = 4 * q + e;
                  const float y = (__uint_as_float(r[j]) - mean) * rstd * s_gamma[c + j] + s_beta[c + j];
                  v[e] = ss > 0.0f ? y * inv_norm : y;
                }
                o[q] = make_float4(v[0], v[1], v[2], v[3]);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[b]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (EPI == EPI_GELU_QUANT) {  // no CTA leaves while a peer may still write into it
    cluster_arrive_release();
    cluster_wait_acquire();
  }
  if (warp == 1) tmem_dealloc(tmem, Ly::TCOLS);
}

// ------------------------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Tensor map of a [rows, K] row-major int8 matrix: boxes of box_rows x 128 bytes, 128-byte swizzle.
int make_tmap_i8(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
  auto enc = get_encode();
  if (!enc) return -1;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K % 16) || rows <= 0) return -2;
  cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(K)};
  cuuint32_t box[2] = {128, cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

static int num_sms() {
  static int cache[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

template <int BN, int EPI, bool RES, int STAGES>
static int set_smem() {
  return cudaFuncSetAttribute(k_gemm_i8<BN, EPI, RES, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              Layout<BN, EPI, RES, STAGES>::TOTAL) == cudaSuccess
             ? 0
             : -1;
}

template <int BN, int EPI, bool RES, int STAGES>
static cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t st) {
  using Ly = Layout<BN, EPI, RES, STAGES>;
  auto kfn = k_gemm_i8<BN, EPI, RES, STAGES>;
  const int nt = g.N / BN;
  const int mt = (g.M + BM - 1) / BM;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Ly::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int ctas;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // pdl_wait in the kernel
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  if constexpr (EPI == EPI_GELU_QUANT) {
    // nt == cluster size: the 6 CTAs of a cluster hold the 6 column slices of one 128-row tile
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = Ly::GCL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.numAttrs = 1;
    static int max_clusters[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!max_clusters[dev]) {
      cfg.gridDim = dim3(Ly::GCL * 8, 1, 1);
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess || n <= 0) n = num_sms() / Ly::GCL;
      max_clusters[dev] = n;
    }
    const int clusters = mt < max_clusters[dev] ? mt : max_clusters[dev];
    ctas = Ly::GCL * clusters;
    cfg.numAttrs = 2;
  } else {
    cfg.attrs = attr + 1;
    cfg.numAttrs = 1;
    const int per_n = num_sms() / nt > 0 ? num_sms() / nt : 1;
    ctas = nt * (mt < per_n ? mt : per_n);
  }
  cfg.gridDim = dim3(ctas, 1, 1);
  return cudaLaunchKernelEx(&cfg, kfn, ta, tb, g, nt, mt);
}

// ------------------------------------------------------------------------ int8 tensor-pipe peak
// Throughput of tcgen05.mma kind::i8 with its operands resident in shared memory: one CTA per SM,
// A (128 rows x 128 bytes) and B (256 rows x 128 bytes) filled with a fixed pseudo-random pattern,
// one thread issuing `iters` rounds of 4 MMAs (M = 128, N = 256, K = 32 each, the whole 128-byte K
// block) into two TMEM accumulators taken in turn. The roofline denominator of the GEMMs.
constexpr int kPeakN = 256;
// 160 KB of dynamic shared memory (48 KB used) keeps the launch at one CTA per SM
constexpr int kPeakSmem = 160 * 1024;
static_assert(BM * BK + kPeakN * BK + 1024 <= kPeakSmem, "peak probe operands");

__global__ void __launch_bounds__(128, 1) k_i8_peak(int iters, int* err) {
  extern __shared__ uint8_t peak_raw[];
  __shared__ uint64_t done;
  __shared__ uint32_t tmem_base;
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(peak_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x;
  for (int i = tid; i < (BM + kPeakN) * BK / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(sm)[i] = (uint32_t(i) * 2654435761u) ^ 0x5bd1e995u;
  fence_proxy_async();  // the MMA (async proxy) reads what these generic stores wrote
  if (tid < 32) {
    tmem_alloc(&tmem_base, 2 * kPeakN);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&done, 1);
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t d = tmem_base;
  if (tid == 0) {
    constexpr uint32_t idesc = idesc_i8(BM, kPeakN);
    const uint32_t a = smem_u32(sm), b = a + BM * BK;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int ks = 0; ks < BK / 32; ++ks)
        mma_i8(d + uint32_t(it & 1) * kPeakN, sdesc_sw128(a + ks * 32), sdesc_sw128(b + ks * 32), idesc,
               (it > 1 || ks > 0) ? 1u : 0u);
    }
    mma_commit(&done);
    mbar_wait(&done, 0, err, DEV_ERR_TIMEOUT_MMA);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid < 32) tmem_dealloc(d, 2 * kPeakN);
}

int i8_peak_launch(int iters, int* err, cudaStream_t st, int* ctas_out) {
  static bool attr_set[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < kMaxDevices && !attr_set[dev]) {
    if (cudaFuncSetAttribute(k_i8_peak, cudaFuncAttributeMaxDynamicSharedMemorySize, kPeakSmem) != cudaSuccess)
      return -1;
    attr_set[dev] = true;
  }
  const int ctas = num_sms();
  if (ctas_out) *ctas_out = ctas;
  k_i8_peak<<<ctas, 128, kPeakSmem, st>>>(iters, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

double i8_peak_ops(int iters, int ctas) { return 2.0 * BM * kPeakN * BK * double(iters) * double(ctas); }

// Sets the dynamic shared-memory limit of every GEMM variant on the current device (called once per
// device before any launch can be captured into a CUDA graph).
int gemm_i8_prime() {
  int r = 0;
  r |= set_smem<64, EPI_F32, true, 4>();
  r |= set_smem<64, EPI_F32, false, 8>();
  r |= set_smem<128, EPI_F32, true, 4>();
  r |= set_smem<192, EPI_F32, true, 4>();
  r |= set_smem<256, EPI_F32, true, 4>();
  r |= set_smem<128, EPI_F32, false, 4>();
  r |= set_smem<192, EPI_F32, false, 4>();
  r |= set_smem<256, EPI_F32, false, 4>();
  r |= set_smem<384, EPI_LN_QUANT, true, 3>();
  r |= set_smem<384, EPI_LN_QUANT, false, 3>();
  r |= set_smem<384, EPI_LN_FINAL, true, 3>();
  r |= set_smem<384, EPI_LN_FINAL, false, 3>();
  r |= set_smem<256, EPI_GELU_QUANT, true, 4>();
  r |= set_smem<128, EPI_GELU_QUANT, true, 4>();
  r |= set_smem<128, EPI_GELU_QUANT, false, 4>();
  // 12-CTA clusters (128-column slices, few row tiles) exceed the portable cluster size of 8
  r |= cudaFuncSetAttribute(k_gemm_i8<128, EPI_GELU_QUANT, true, 4>, cudaFuncAttributeNonPortableClusterSizeAllowed,
                            1) == cudaSuccess ? 0 : -1;
  r |= cudaFuncSetAttribute(k_gemm_i8<128, EPI_GELU_QUANT, false, 4>, cudaFuncAttributeNonPortableClusterSizeAllowed,
                            1) == cudaSuccess ? 0 : -1;
  r |= set_smem<256, EPI_GELU_QUANT, false, 3>();
  return r;
}

int gemm_i8_launch(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t st) {
  if (g.M <= 0) return 0;
  if (g.K % BK || g.K <= 0) return -10;
  const bool res = g.K == kResK;
  cudaError_t e = cudaSuccess;
  switch (epi) {
    case EPI_F32: {
      // wide slices for large M; for few M tiles, narrower slices spread the work over more SMs
      const int mt = (g.M + BM - 1) / BM;
      const bool few = mt * (g.N / 128) < num_sms();
      if (few && g.N % 64 == 0 && mt * (g.N / 64) <= num_sms())
        e = res ? launch<64, EPI_F32, true, 4>(ta, tb, g, st) : launch<64, EPI_F32, false, 8>(ta, tb, g, st);
      else if (few && g.N % 128 == 0)
        e = res ? launch<128, EPI_F32, true, 4>(ta, tb, g, st) : launch<128, EPI_F32, false, 4>(ta, tb, g, st);
      else if (g.N % 256 == 0)
        e = res ? launch<256, EPI_F32, true, 4>(ta, tb, g, st) : launch<256, EPI_F32, false, 4>(ta, tb, g, st);
      else if (g.N % 192 == 0)
        e = res ? launch<192, EPI_F32, true, 4>(ta, tb, g, st) : launch<192, EPI_F32, false, 4>(ta, tb, g, st);
      else if (g.N % 128 == 0)
        e = res ? launch<128, EPI_F32, true, 4>(ta, tb, g, st) : launch<128, EPI_F32, false, 4>(ta, tb, g, st);
      else if (g.N % 64 == 0)
        e = res ? launch<64, EPI_F32, true, 4>(ta, tb, g, st) : launch<64, EPI_F32, false, 8>(ta, tb, g, st);
      else
        return -11;
      break;
    }
    case EPI_LN_QUANT:
      if (g.N != kHidden) return -11;
      e = res ? launch<384, EPI_LN_QUANT, true, 3>(ta, tb, g, st) : launch<384, EPI_LN_QUANT, false, 3>(ta, tb, g, st);
      break;
    case EPI_LN_FINAL:
      if (g.N != kHidden) return -11;
      e = res ? launch<384, EPI_LN_FINAL, true, 3>(ta, tb, g, st) : launch<384, EPI_LN_FINAL, false, 3>(ta, tb, g, st);
      break;
    case EPI_GELU_QUANT: {
      if (g.N != kInter) return -11;
      // few row tiles: 12 slices of 128 columns (half the epilogue work per SM sub-partition);
      // otherwise 6 slices of 256
      const int mt = (g.M + BM - 1) / BM;
      if (mt * (kInter / 128) <= num_sms())
        e = res ? launch<128, EPI_GELU_QUANT, true, 4>(ta, tb, g, st) : launch<128, EPI_GELU_QUANT, false, 4>(ta, tb, g, st);
      else
        e = res ? launch<256, EPI_GELU_QUANT, true, 4>(ta, tb, g, st) : launch<256, EPI_GELU_QUANT, false, 3>(ta, tb, g, st);
      break;
    }
      break;
    default:
      return -12;
  }
  return e == cudaSuccess ? 0 : -100 - int(e);
}

}  // namespace ae
