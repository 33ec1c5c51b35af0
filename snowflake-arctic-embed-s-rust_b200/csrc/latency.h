// Host interface of the single-sequence cluster forward (latency.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "rowmath.cuh"

namespace ae {

// Longest sequence the cluster forward takes (one 32-row slab per CTA).
constexpr int kLatMaxTokens = 32;

// Per-linear parameters the kernel reads (device pointers into the model arena).
struct LatLinear {
  const float* ws;    // [n_out] per-output-channel weight scales
  const float* bias;  // [n_out]
  const float* invs;  // [k_in] inverse smoothing factors of this linear's input
};

struct LatLayer {
  LatLinear qkv, q_only, kv_only, ao, fi, fo;
  const float *ln1w, *ln1b, *ln2w, *ln2b;
};

// Tensor maps of the weights with 32-row x 128-byte boxes (128-byte swizzle), per layer.
enum { LAT_QKV = 0, LAT_Q = 1, LAT_KV = 2, LAT_AO = 3, LAT_FI = 4, LAT_FO = 5, LAT_MAPS = 6 };

// Everything the kernel reads of the model, in device memory (the tensor maps 64-byte aligned).
struct alignas(64) LatModel {
  CUtensorMap tm[kLayers][LAT_MAPS];
  LatLayer layer[kLayers];
  const int8_t* word_q;
  const float* word_s;
  const int8_t* pos_q;
  const float* pos_s;
  const float* type0;
  const float* emb_lnw;
  const float* emb_lnb;
};

// Sets the kernel's shared-memory and cluster attributes on the current device; false when the
// device cannot run a 12-CTA cluster of this kernel (the caller then keeps the multi-kernel path).
bool lat_prime();
// One sequence of 1..kLatMaxTokens ids (device) -> its L2-normalised embedding out[384] (device).
int launch_forward_lat(const LatModel* d_model, const uint16_t* d_ids, int L, float* d_out, int* err, int gelu_erf,
                       cudaStream_t st);

}  // namespace ae
