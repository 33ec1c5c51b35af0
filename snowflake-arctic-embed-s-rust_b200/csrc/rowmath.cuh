// Per-row arithmetic in the exact operation order of the reference CPU path (x86_64 AVX2 kernels),
// so that a GPU thread that owns one row rounds exactly as the reference does. The library is
// compiled with --fmad=false: every fused multiply-add below is an explicit fmaf, every other
// product/sum rounds separately, as in the reference.
#pragma once
#include <cstdint>

namespace ae {

constexpr int kHidden = 384;
constexpr int kInter = 1536;
constexpr int kHeads = 12;
constexpr int kHeadDim = 32;
constexpr int kLayers = 12;
constexpr int kVocab = 30522;
constexpr int kMaxPos = 512;
constexpr float kLnEps = 1e-12f;
constexpr int kMaxDevices = 64;

// Tile-transposed layout of the large fp32 activations ([T, C] matrices such as the QKV output and
// the hidden state): element (t, c) is stored at ((t / 128) * C + c) * 128 + t % 128, so the 32
// consecutive rows a warp's epilogue threads own write one contiguous 128-byte line per column.
__host__ __device__ __forceinline__ size_t tt_index(int t, int c, int C) {
  return ((size_t(t >> 7) * size_t(C) + size_t(c)) << 7) + size_t(t & 127);
}

// hsum256_ps(sum0 + sum1) of src/simd_math.rs:3075-3084 applied to 16 partial lanes p[0..16)
// (p[l] accumulates elements with index % 16 == l, as the two AVX2 accumulators do).
__device__ __forceinline__ float tree16(const float (&p)[16]) {
  float v[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) v[l] = p[l] + p[8 + l];
  return ((v[0] + v[4]) + (v[1] + v[5])) + ((v[2] + v[6]) + (v[3] + v[7]));
}

// hsum256_ps of one 8-lane vector.
__device__ __forceinline__ float tree8(const float (&v)[8]) {
  return ((v[0] + v[4]) + (v[1] + v[5])) + ((v[2] + v[6]) + (v[3] + v[7]));
}

// Round-to-nearest-even of |x| < 2^22 on the FP32 pipe: adding 1.5 * 2^23 leaves the rounded
// integer in the low mantissa bits (the add itself rounds half to even), subtracting it back gives
// the rounded value exactly. Same result as rintf / cvt.rni without the conversion pipe.
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
constexpr int kRoundMagicBits = 0x4B400000;

// Clamp-and-round of the AVX2 quantizers: min(max(v, -127), 127) then cvtps_epi32 (half-even).
__device__ __forceinline__ int quant_i8(float v) {
  v = fminf(fmaxf(v, -127.0f), 127.0f);
  return __float_as_int(v + kRoundMagic) - kRoundMagicBits;
}

// quant_i8 for a value already scaled by 127 / max|x| of its row: |v| <= 127 (1 + 3 * 2^-24) < 127.5
// for finite inputs, so the clamp to [-127, 127] never changes the rounded result. Returns the bits
// of v + 1.5 * 2^23, whose low byte is the int8 (the magic constant's low 22 bits are zero).
__device__ __forceinline__ uint32_t quant_bits_scaled(float v) { return __float_as_uint(v + kRoundMagic); }

// Four quant_bits_scaled results -> four int8 bytes (element 0 in the lowest byte).
__device__ __forceinline__ uint32_t pack_i8x4(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

// avx2_exp_f32, src/simd_math.rs:113-143 (Cody-Waite range reduction + degree-5 polynomial).
__device__ __forceinline__ float cw_exp(float x) {
  const float y = fmaxf(fminf(x, 88.0f), -87.3f);
  const float big = y * 1.44269504088896341f + kRoundMagic;  // LOG2_E rounded to f32; two roundings
  const float n = big - kRoundMagic;                          // round(y * log2e), half to even
  const float r = fmaf(-n, 1.428606765330187e-6f, fmaf(-n, 0.693145751953125f, y));
  float p = fmaf(r, 0.008333334f, 0.041666668f);
  p = fmaf(r, p, 0.16666667f);
  p = fmaf(r, p, 0.5f);
  p = fmaf(r, p, 1.0f);
  p = fmaf(r, p, 1.0f);
  const int ni = (__float_as_int(big) - kRoundMagicBits) + 127;
  return p * __int_as_float(ni << 23);
}

// Scalar `f32::exp` used by the reference for softmax tail elements. Evaluated in double and
// rounded once, which is the correctly rounded result except in rare double-rounding cases.
__device__ __forceinline__ float scalar_expf(float x) { return static_cast<float>(exp(static_cast<double>(x))); }

// Hardware reciprocal approximation (MUFU, within one ulp), the estimate GELU refines.
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// avx2_gelu_f32, src/simd_math.rs:152-175: rational erf approximation on x clamped to [-4.8, 4.8],
// with a reciprocal estimate refined by one Newton step, as the reference does. The reference's
// estimate comes from `rcp_ps` (12-bit, implementation defined); here it is the hardware
// reciprocal (about 23-bit), so after the Newton step the two agree to about one ulp.
__device__ __forceinline__ float gelu_ref(float x) {
  const float xc = fminf(fmaxf(x, -4.8f), 4.8f);
  const float u = xc * xc;
  float num = fmaf(u, 6.4292e-5f, 0.007572631f);
  num = fmaf(u, num, 0.055282866f);
  num = fmaf(u, num, 0.797882463f);
  float den = fmaf(u, 0.001139532f, 0.02381135f);
  den = fmaf(u, den, 0.235943093f);
  den = fmaf(u, den, 1.0f);
  const float est = rcp_approx(den);
  const float inv_den = est * fmaf(-den, est, 2.0f);
  const float erf_a = fminf(fmaxf(xc * (num * inv_den), -1.0f), 1.0f);
  return (x * 0.5f) * (1.0f + erf_a);
}

// gelu_ref on two lanes with the packed f32x2 arithmetic of sm_100 (each lane rounds exactly as
// the scalar sequence does).
__device__ __forceinline__ float2 gelu_ref2(float2 x) {
  const float2 xc = make_float2(fminf(fmaxf(x.x, -4.8f), 4.8f), fminf(fmaxf(x.y, -4.8f), 4.8f));
  const float2 u = __fmul2_rn(xc, xc);
  float2 num = __ffma2_rn(u, make_float2(6.4292e-5f, 6.4292e-5f), make_float2(0.007572631f, 0.007572631f));
  num = __ffma2_rn(u, num, make_float2(0.055282866f, 0.055282866f));
  num = __ffma2_rn(u, num, make_float2(0.797882463f, 0.797882463f));
  float2 den = __ffma2_rn(u, make_float2(0.001139532f, 0.001139532f), make_float2(0.02381135f, 0.02381135f));
  den = __ffma2_rn(u, den, make_float2(0.235943093f, 0.235943093f));
  den = __ffma2_rn(u, den, make_float2(1.0f, 1.0f));
  const float2 est = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  const float2 inv_den = __fmul2_rn(est, __ffma2_rn(make_float2(-den.x, -den.y), est, make_float2(2.0f, 2.0f)));
  const float2 t = __fmul2_rn(xc, __fmul2_rn(num, inv_den));
  // (x * 0.5) * (1 + clamp(t, -1, 1)): 1 + clamp(t, -1, 1) = clamp(RN(1 + t), 0, 2) = 2 v with
  // v = sat(RN(0.5 t + 0.5)) (halving is exact), and RN(RN(x * 0.5) * 2v) = RN(x * v) because
  // x * 0.5 is exact for |x| >= 2^-125 (below that the result is far under the quantization step).
  const float2 v = make_float2(__saturatef(fmaf(t.x, 0.5f, 0.5f)), __saturatef(fmaf(t.y, 0.5f, 0.5f)));
  return __fmul2_rn(x, v);
}

// GELU with the exact error function (0.5 x (1 + erf(x / sqrt 2))).
__device__ __forceinline__ float gelu_erf(float x) {
  return (0.5f * x) * (1.0f + erff(x * 0.70710678118654752f));
}

}  // namespace ae
