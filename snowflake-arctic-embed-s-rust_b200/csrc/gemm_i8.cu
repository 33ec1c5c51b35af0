// int8 x int8 -> int32 GEMM on the sm_100a tensor cores (tcgen05.mma kind::i8) with fused epilogues.
//
// Contract (src/gemm.rs:627-628, gemm_scalar_fused src/gemm.rs:2000-2029):
//   acc[m,n] = sum_k A[m,k] * W[n,k]                      (exact int32)
//   h[m,n]   = fma(float(acc), a_scale[m] * w_scale[n], bias[n] (+ res[m,n]))
// A is [M,K] row-major int8, W is [N,K] row-major int8 (out_features x in_features), both K-major
// operands for tcgen05. Tiles are 128 rows of A; K is consumed in 128-byte blocks staged by TMA
// (128-byte swizzle, no multicast) through a STAGES-deep mbarrier ring; one thread issues the MMAs,
// the int32 accumulator lives in TMEM, and the 128 epilogue threads each own one output row.
//
// Epilogues:
//   EPI_F32        out[m,n] = h                                   (QKV, KV-only, Q-only projections)
//   EPI_LN_QUANT   hidden = LayerNorm(h) written back as the new residual, then the SmoothQuant
//                  dynamic row quantization for the next GEMM       (attention-out and FFN-down;
//                  src/model.rs:330-353, :375-397 with layernorm_smooth_quantize_row_avx2,
//                  src/simd_math.rs:369-477)
//   EPI_GELU_QUANT g = GELU(h) * inv_smooth, row max over all 1536 columns exchanged across a
//                  3-CTA cluster through distributed shared memory, then row quantization
//                  (FFN-up; gelu_smooth_quantize_row_avx2, src/simd_math.rs:1371-1435). GELU is the
//                  reference's rational approximation (gelu_ref) or, on request, the exact erf.
//   EPI_LN_FINAL   out = l2_normalize(layernorm_inplace_row(h))  (layer-11 FFN-down of the [CLS]
//                  rows; src/model.rs:496-512, src/simd_math.rs:481-497, :2892-2903)
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>

#include "gemm_i8.h"
#include "ptx.cuh"
#include "rowmath.cuh"

namespace ae {

constexpr int BM = 128;        // rows per tile
constexpr int BK = 128;        // K bytes per stage (one 128-byte swizzle atom wide)
constexpr int A_STAGE = BM * BK;  // 16 KB

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int B_STAGE = BN * BK;
  static constexpr int STAGE = A_STAGE + B_STAGE;
  static constexpr int TILES = STAGES * STAGE;
  // per-column parameters: w_scale, bias, gamma, beta, inv_smooth
  static constexpr int PARAMS = 5 * BN * 4;
  static constexpr int ROWMAX = 3 * BM * 4;
  static constexpr int BARS = (2 * STAGES + 1) * 8 + 16;
  static constexpr int TOTAL = 1024 + TILES + PARAMS + ROWMAX + BARS;
};

__host__ __device__ constexpr uint32_t tmem_cols_for(int bn) {
  return bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : bn <= 256 ? 256 : 512;
}

template <int BN, int EPI, int STAGES>
__global__ void __launch_bounds__(128, 1)
    k_gemm_i8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs g) {
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* s_ws = reinterpret_cast<float*>(smem + S::TILES);
  float* s_bias = s_ws + BN;
  float* s_gamma = s_bias + BN;
  float* s_beta = s_gamma + BN;
  float* s_invs = s_beta + BN;
  float* s_rowmax = s_invs + BN;  // [3][BM], written by the cluster peers (EPI_GELU_QUANT)
  uint64_t* full = reinterpret_cast<uint64_t*>(s_rowmax + 3 * BM);
  uint64_t* empty = full + STAGES;
  uint64_t* accfull = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accfull + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n_tile = blockIdx.x;
  const int m0 = blockIdx.y * BM;
  const int n0 = n_tile * BN;
  const int KB = g.K / BK;
  constexpr uint32_t TCOLS = tmem_cols_for(BN);

  if constexpr (EPI == EPI_GELU_QUANT) cluster_arrive_release();  // peers must be running before DSMEM use

  if (tid == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accfull, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, TCOLS);
    tmem_relinquish();
  }
  // per-column epilogue parameters
  for (int i = tid; i < BN; i += blockDim.x) {
    const int n = n0 + i;
    s_ws[i] = g.w_scale[n];
    s_bias[i] = g.bias[n];
    if constexpr (EPI == EPI_LN_QUANT || EPI == EPI_LN_FINAL) {
      s_gamma[i] = g.gamma[i];
      s_beta[i] = g.beta[i];
    }
    if constexpr (EPI == EPI_LN_QUANT || EPI == EPI_GELU_QUANT) s_invs[i] = g.inv_smooth[n];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool ok = true;
  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    for (int kb = 0; kb < KB && ok; ++kb) {
      const int s = kb % STAGES;
      if (kb >= STAGES) ok = mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, g.err, DEV_ERR_TIMEOUT_PRODUCER);
      if (!ok) break;
      uint8_t* a_s = smem + s * S::STAGE;
      uint8_t* b_s = a_s + A_STAGE;
      mbar_arrive_expect_tx(&full[s], S::STAGE);
      tma_load_2d(a_s, &tmA, &full[s], kb * BK, m0);
#pragma unroll
      for (int j = 0; j < BN / 128; ++j) tma_load_2d(b_s + j * 128 * BK, &tmB, &full[s], kb * BK, n0 + j * 128);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = idesc_i8(128, 128);
    for (int kb = 0; kb < KB && ok; ++kb) {
      const int s = kb % STAGES;
      ok = mbar_wait(&full[s], (kb / STAGES) & 1, g.err, DEV_ERR_TIMEOUT_MMA);
      if (!ok) break;
      tc_fence_after();
      const uint32_t a_addr = smem_u32(smem + s * S::STAGE);
      const uint32_t b_addr = a_addr + A_STAGE;
#pragma unroll
      for (int ks = 0; ks < BK / 32; ++ks) {
        const uint64_t ad = sdesc_sw128(a_addr + ks * 32);
#pragma unroll
        for (int j = 0; j < BN / 128; ++j) {
          const uint64_t bd = sdesc_sw128(b_addr + j * 128 * BK + ks * 32);
          mma_i8(tmem + j * 128, ad, bd, idesc, (kb | ks) != 0);
        }
      }
      mma_commit(&empty[s]);
    }
    if (ok) mma_commit(accfull);
  }
  __syncwarp();

  // ---------------- epilogue: thread = row
  ok = mbar_wait(accfull, 0, g.err, DEV_ERR_TIMEOUT_EPILOGUE);
  ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld/st are warp-collective: keep the warp uniform
  tc_fence_after();
  const int row = m0 + warp * 32 + lane;
  const bool valid = ok && row < g.M;
  const uint32_t trow = tmem + (uint32_t(warp * 32) << 16);
  const float as = valid ? g.a_scale[row] : 0.0f;
  uint32_t r[32];

  if constexpr (EPI == EPI_F32) {
    if (ok) {
      for (int c = 0; c < BN / 32; ++c) {
        tmem_ld32(trow + c * 32, r);
        tmem_ld_wait();
        if (valid) {
          float* o = g.out_f32 + size_t(row) * g.ldo + n0 + c * 32;
          const float* rs = g.res ? g.res + size_t(row) * g.ldr + n0 + c * 32 : nullptr;
          if (g.acc_dbg) {
            int4* ad = reinterpret_cast<int4*>(g.acc_dbg + size_t(row) * g.N + n0 + c * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              ad[q] = make_int4(int(r[4 * q]), int(r[4 * q + 1]), int(r[4 * q + 2]), int(r[4 * q + 3]));
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float v[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = 4 * q + e;
              const int n = c * 32 + j;
              float b = s_bias[n];
              if (rs) b = b + rs[j];
              v[e] = fmaf(float(int(r[j])), as * s_ws[n], b);
            }
            reinterpret_cast<float4*>(o)[q] = make_float4(v[0], v[1], v[2], v[3]);
          }
        }
      }
    }
  } else if constexpr (EPI == EPI_LN_QUANT || EPI == EPI_LN_FINAL) {
    static_assert(BN == kHidden, "row-LayerNorm epilogue needs the full 384-wide row");
    if (ok) {
      // pass 1: h = fma(acc, as*ws, bias + res); partial sums; h -> TMEM
      float p[16];
      float seq = 0.0f;
#pragma unroll
      for (int l = 0; l < 16; ++l) p[l] = 0.0f;
      for (int c = 0; c < BN / 32; ++c) {
        tmem_ld32(trow + c * 32, r);
        tmem_ld_wait();
        float h[32];
        if (valid) {
          const float* rs = g.res + size_t(row) * g.ldr + c * 32;
          if (g.acc_dbg) {
            int4* ad = reinterpret_cast<int4*>(g.acc_dbg + size_t(row) * g.N + c * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              ad[q] = make_int4(int(r[4 * q]), int(r[4 * q + 1]), int(r[4 * q + 2]), int(r[4 * q + 3]));
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 rv = reinterpret_cast<const float4*>(rs)[q];
            const float rr[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = 4 * q + e;
              const int n = c * 32 + j;
              h[j] = fmaf(float(int(r[j])), as * s_ws[n], s_bias[n] + rr[e]);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) h[j] = 0.0f;
        }
        if constexpr (EPI == EPI_LN_QUANT) {
#pragma unroll
          for (int j = 0; j < 16; ++j) p[j] = p[j] + h[j];
#pragma unroll
          for (int j = 0; j < 16; ++j) p[j] = p[j] + h[16 + j];
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) seq = seq + h[j];
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(h[j]);
        tmem_st32(trow + c * 32, r);
      }
      tmem_st_wait();
      const float mean = (EPI == EPI_LN_QUANT ? tree16(p) : seq) / float(kHidden);
      // pass 2: variance
#pragma unroll
      for (int l = 0; l < 16; ++l) p[l] = 0.0f;
      seq = 0.0f;
      for (int c = 0; c < BN / 32; ++c) {
        tmem_ld32(trow + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float d = __uint_as_float(r[j]) - mean;
          if constexpr (EPI == EPI_LN_QUANT) p[j & 15] = fmaf(d, d, p[j & 15]);
          else seq = seq + d * d;
        }
      }
      const float var = (EPI == EPI_LN_QUANT ? tree16(p) : seq) / float(kHidden);
      const float rstd = 1.0f / sqrtf(var + kLnEps);
      if constexpr (EPI == EPI_LN_QUANT) {
        // pass 3: y = LN(h) -> residual out and TMEM; row max of |y * inv_smooth|
        float vmax = 1e-8f;
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(trow + c * 32, r);
          tmem_ld_wait();
          float y[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = c * 32 + j;
            y[j] = fmaf((__uint_as_float(r[j]) - mean) * rstd, s_gamma[n], s_beta[n]);
            vmax = fmaxf(vmax, fabsf(y[j] * s_invs[n]));
            r[j] = __float_as_uint(y[j]);
          }
          if (valid) {
            float4* o = reinterpret_cast<float4*>(g.out_f32 + size_t(row) * g.ldo + c * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) o[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
          }
          tmem_st32(trow + c * 32, r);
        }
        tmem_st_wait();
        // pass 4: quantize
        const float max_abs = vmax;
        const float inv_scale = 127.0f / max_abs;
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(trow + c * 32, r);
          tmem_ld_wait();
          uint32_t pk[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint32_t w = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int n = c * 32 + 4 * q + e;
              const int qi = quant_i8(__uint_as_float(r[4 * q + e]) * (s_invs[n] * inv_scale));
              w |= (uint32_t(qi) & 0xFFu) << (8 * e);
            }
            pk[q] = w;
          }
          if (valid) {
            uint4* qo = reinterpret_cast<uint4*>(g.out_q + size_t(row) * kHidden + c * 32);
            qo[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            qo[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
        if (valid) g.out_scale[row] = max_abs / 127.0f;
      } else {
        // EPI_LN_FINAL: y = (h - mean) * rstd * gamma + beta (unfused), then L2 normalize
        float ss = 0.0f;
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(trow + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = c * 32 + j;
            const float y = (__uint_as_float(r[j]) - mean) * rstd * s_gamma[n] + s_beta[n];
            ss = ss + y * y;
            r[j] = __float_as_uint(y);
          }
          tmem_st32(trow + c * 32, r);
        }
        tmem_st_wait();
        const float inv_norm = ss > 0.0f ? 1.0f / sqrtf(ss) : 1.0f;
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(trow + c * 32, r);
          tmem_ld_wait();
          if (valid) {
            float4* o = reinterpret_cast<float4*>(g.out_f32 + size_t(row) * g.ldo + c * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float v[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float y = __uint_as_float(r[4 * q + e]);
                v[e] = ss > 0.0f ? y * inv_norm : y;
              }
              o[q] = make_float4(v[0], v[1], v[2], v[3]);
            }
          }
        }
      }
    }
  } else if constexpr (EPI == EPI_GELU_QUANT) {
    // 3 CTAs of a cluster hold columns [512 r, 512 r + 512) of the same 128 rows.
    const uint32_t rank = cluster_ctarank();
    float vmax = 1e-8f;
    if (ok) {
      for (int c = 0; c < BN / 32; ++c) {
        tmem_ld32(trow + c * 32, r);
        tmem_ld_wait();
        if (valid && g.acc_dbg) {
          int4* ad = reinterpret_cast<int4*>(g.acc_dbg + size_t(row) * g.N + n0 + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            ad[q] = make_int4(int(r[4 * q]), int(r[4 * q + 1]), int(r[4 * q + 2]), int(r[4 * q + 3]));
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int n = c * 32 + j;
          const float h = fmaf(float(int(r[j])), as * s_ws[n], s_bias[n]);
          const float gv = (g.gelu_erf ? gelu_erf(h) : gelu_ref(h)) * s_invs[n];
          vmax = fmaxf(vmax, fabsf(gv));
          r[j] = __float_as_uint(gv);
        }
        tmem_st32(trow + c * 32, r);
      }
      tmem_st_wait();
    }
    // exchange the partial row maxima across the cluster (every thread takes part, error or not)
    cluster_wait_acquire();  // all peers have started
#pragma unroll
    for (uint32_t q = 0; q < 3; ++q) st_cluster_f32(map_peer(&s_rowmax[rank * BM + tid], q), vmax);
    cluster_arrive_release();
    cluster_wait_acquire();
    const float max_abs = fmaxf(fmaxf(s_rowmax[tid], s_rowmax[BM + tid]), s_rowmax[2 * BM + tid]);
    const float inv_scale = 127.0f / max_abs;
    if (ok) {
      for (int c = 0; c < BN / 32; ++c) {
        tmem_ld32(trow + c * 32, r);
        tmem_ld_wait();
        uint32_t pk[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint32_t w = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w |= (uint32_t(quant_i8(__uint_as_float(r[4 * q + e]) * inv_scale)) & 0xFFu) << (8 * e);
          pk[q] = w;
        }
        if (valid) {
          uint4* qo = reinterpret_cast<uint4*>(g.out_q + size_t(row) * g.N + n0 + c * 32);
          qo[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          qo[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      if (valid && rank == 0) g.out_scale[row] = max_abs / 127.0f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TCOLS);
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

// Tensor map of a [rows, K] row-major int8 matrix, 128 x 128-byte boxes, 128-byte swizzle.
int make_tmap_i8(CUtensorMap* map, const void* base, int rows, int K) {
  auto enc = get_encode();
  if (!enc) return -1;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K % 16)) return -2;
  cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(K)};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

template <int BN, int EPI, int STAGES>
static cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t st,
                          int cluster_x) {
  using S = GemmSmem<BN, STAGES>;
  auto kfn = k_gemm_i8<BN, EPI, STAGES>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.N / BN, (g.M + BM - 1) / BM, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = S::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  cfg.numAttrs = 0;
  if (cluster_x > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kfn, ta, tb, g);
}

// Sets the dynamic shared-memory limit of every GEMM variant on the current device (called once per
// device before any launch can be captured into a CUDA graph).
int gemm_i8_prime() {
  int dev = 0;
  cudaGetDevice(&dev);
  (void)dev;
  const cudaError_t e[4] = {
      cudaFuncSetAttribute(k_gemm_i8<128, EPI_F32, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           GemmSmem<128, 4>::TOTAL),
      cudaFuncSetAttribute(k_gemm_i8<384, EPI_LN_QUANT, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           GemmSmem<384, 3>::TOTAL),
      cudaFuncSetAttribute(k_gemm_i8<384, EPI_LN_FINAL, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           GemmSmem<384, 3>::TOTAL),
      cudaFuncSetAttribute(k_gemm_i8<512, EPI_GELU_QUANT, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           GemmSmem<512, 2>::TOTAL)};
  for (auto x : e)
    if (x != cudaSuccess) return -1;
  return 0;
}

int gemm_i8_launch(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t st) {
  if (g.M <= 0) return 0;
  if (g.K % BK) return -10;
  cudaError_t e = cudaSuccess;
  switch (epi) {
    case EPI_F32:
      if (g.N % 128) return -11;
      e = launch<128, EPI_F32, 4>(ta, tb, g, st, 1);
      break;
    case EPI_LN_QUANT:
      if (g.N != kHidden) return -11;
      e = launch<384, EPI_LN_QUANT, 3>(ta, tb, g, st, 1);
      break;
    case EPI_LN_FINAL:
      if (g.N != kHidden) return -11;
      e = launch<384, EPI_LN_FINAL, 3>(ta, tb, g, st, 1);
      break;
    case EPI_GELU_QUANT:
      if (g.N != 3 * 512) return -11;
      e = launch<512, EPI_GELU_QUANT, 2>(ta, tb, g, st, 3);
      break;
    default:
      return -12;
  }
  return e == cudaSuccess ? 0 : -100 - int(e);
}

}  // namespace ae
