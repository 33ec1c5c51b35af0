// CPU oracle: C++ restatement of the reference crate's x86_64 forward path.
// TEST INFRASTRUCTURE ONLY (checker and CPU baseline); never linked into the product library.
//
// Each function names the reference item it restates (file:line inside the reference crate).
// Operation order, intrinsics and rounding follow the reference so that this program computes
// what the Rust crate computes on the same x86_64 host. Parity against the Rust binary itself is
// unpinned (no Rust toolchain here and no real weights); see oracle.h.
#include "oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <thread>
#include <vector>

namespace {

constexpr size_t H = 384, INTER = 1536, NH = 12, HD = 32, NL = 12, VOCAB = 30522, MAXPOS = 512;
constexpr float EPS = 1e-12f;

// ------------------------------------------------------------------------------------------ CPU features
bool cpu_avx2_fma() {
  __builtin_cpu_init();
  return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma");
}
bool cpu_avxvnni() {
  __builtin_cpu_init();
  return cpu_avx2_fma() && __builtin_cpu_supports("avxvnni");
}
const bool g_avx2_fma = cpu_avx2_fma();

// ------------------------------------------------------------------------------------------ weights
// PackedLinearInt8, src/gemm.rs:169-247
struct Linear {
  size_t n = 0, k = 0;
  int backend = OR_BACKEND_SCALAR;
  std::vector<int8_t> w;         // row-major [n, k] as loaded
  std::vector<int8_t> packed;    // backend layout
  std::vector<float> ws, bias, inv_s;
  std::vector<int32_t> comp;     // -128 * sum_k w[n, k] (VNNI only)
};

struct Layer {
  Linear qkv;
  bool has_split = false;
  Linear q_only, kv_only;
  Linear attn_out;
  std::vector<float> ln1w, ln1b;
  Linear ffn_inter, ffn_out;
  std::vector<float> ln2w, ln2b;
};

}  // namespace

struct or_model {
  int backend;
  std::vector<int8_t> word_q, pos_q, type_q;
  std::vector<float> word_s, pos_s, type_s;
  std::vector<float> type0;  // pre-dequantized token_type_embeddings[0], src/model.rs:50-54
  std::vector<float> emb_lnw, emb_lnb;
  Layer layers[NL];
  int attn_mode = OR_ATTENTION_EXACT;  // or_model_set_attention_mode
};

namespace {

// pack_weights_x86, src/gemm.rs:456-476: [N/16][K/4][2][8][4]
std::vector<int8_t> pack_weights_x86(size_t n, size_t k, const int8_t* w) {
  std::vector<int8_t> out(n * k);
  size_t dst = 0;
  for (size_t nb = 0; nb < n / 16; ++nb)
    for (size_t ks = 0; ks < k / 4; ++ks)
      for (size_t g = 0; g < 2; ++g)
        for (size_t c = 0; c < 8; ++c) {
          const size_t col = nb * 16 + g * 8 + c;
          std::memcpy(&out[dst], w + col * k + ks * 4, 4);
          dst += 4;
        }
  return out;
}

// PackedLinearInt8::from_raw_row_major, src/gemm.rs:186-246
bool pack_linear(Linear& l, int backend, std::string& err) {
  l.backend = backend;
  if (l.n == 0) {
    l.w.clear();
    l.ws.clear();
    l.bias.clear();
    return true;
  }
  if (l.w.size() != l.n * l.k || l.ws.size() != l.n || l.bias.size() != l.n || l.inv_s.size() != l.k) {
    err = "linear: inconsistent vector lengths";
    return false;
  }
  if (l.n % 16 || l.k % 16) {
    err = "linear: n_out and k_in must be multiples of 16";
    return false;
  }
  if (backend == OR_BACKEND_AVX_VNNI) {
    l.comp.resize(l.n);
    for (size_t n = 0; n < l.n; ++n) {
      int32_t s = 0;
      for (size_t k = 0; k < l.k; ++k) s += l.w[n * l.k + k];
      l.comp[n] = -128 * s;
    }
  }
  if (backend == OR_BACKEND_AVX_VNNI || backend == OR_BACKEND_AVX2)
    l.packed = pack_weights_x86(l.n, l.k, l.w.data());
  else
    l.packed = l.w;
  return true;
}

// ------------------------------------------------------------------------------------------ GEMMs
#define AVX2_FN __attribute__((target("avx2,fma")))
#define VNNI_FN __attribute__((target("avx2,fma,avxvnni")))

// gemm_x86_avx2_fused, src/gemm.rs:1718-1908 (vpsignb + vpmaddubsw + vpmaddwd, saturation-free)
AVX2_FN inline __m256i dot_avx2(__m256i va, __m256i b) {
  return _mm256_madd_epi16(_mm256_maddubs_epi16(_mm256_abs_epi8(va), _mm256_sign_epi8(b, va)),
                           _mm256_set1_epi16(1));
}
AVX2_FN inline void store_avx2(const float* a_scale, const Linear& W, const float* res, float* out, int32_t* acc_out,
                               size_t r, size_t col, __m256i c_lo, __m256i c_hi) {
  const __m256 s_row = _mm256_set1_ps(a_scale[r]);
  const size_t off = r * W.n + col;
  __m256 b0 = _mm256_loadu_ps(W.bias.data() + col), b1 = _mm256_loadu_ps(W.bias.data() + col + 8);
  if (res) {
    b0 = _mm256_add_ps(b0, _mm256_loadu_ps(res + off));
    b1 = _mm256_add_ps(b1, _mm256_loadu_ps(res + off + 8));
  }
  if (acc_out) {
    _mm256_storeu_si256(reinterpret_cast<__m256i*>(acc_out + off), c_lo);
    _mm256_storeu_si256(reinterpret_cast<__m256i*>(acc_out + off + 8), c_hi);
  }
  const __m256 ws0 = _mm256_loadu_ps(W.ws.data() + col), ws1 = _mm256_loadu_ps(W.ws.data() + col + 8);
  _mm256_storeu_ps(out + off, _mm256_fmadd_ps(_mm256_cvtepi32_ps(c_lo), _mm256_mul_ps(s_row, ws0), b0));
  _mm256_storeu_ps(out + off + 8, _mm256_fmadd_ps(_mm256_cvtepi32_ps(c_hi), _mm256_mul_ps(s_row, ws1), b1));
}
AVX2_FN void gemm_avx2(size_t m, const int8_t* a_q, const float* a_scale, const Linear& W, const float* res,
                       float* out, int32_t* acc_out) {
  const size_t k_in = W.k, k_steps = k_in / 4, n_panels = W.n / 16;
  for (size_t nb = 0; nb < n_panels; ++nb) {
    const size_t col = nb * 16;
    const int8_t* pb_panel = W.packed.data() + nb * k_steps * 64;
    size_t r = 0;
    for (; r + 4 <= m; r += 4) {
      __m256i c[4][2];
      for (int i = 0; i < 4; ++i) c[i][0] = c[i][1] = _mm256_setzero_si256();
      const int8_t* pb = pb_panel;
      for (size_t ks = 0; ks < k_steps; ++ks) {
        const __m256i b0 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(pb));
        const __m256i b1 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(pb + 32));
        pb += 64;
        for (int i = 0; i < 4; ++i) {
          int32_t av;
          std::memcpy(&av, a_q + (r + i) * k_in + ks * 4, 4);
          const __m256i va = _mm256_set1_epi32(av);
          c[i][0] = _mm256_add_epi32(c[i][0], dot_avx2(va, b0));
          c[i][1] = _mm256_add_epi32(c[i][1], dot_avx2(va, b1));
        }
      }
      for (int i = 0; i < 4; ++i) store_avx2(a_scale, W, res, out, acc_out, r + i, col, c[i][0], c[i][1]);
    }
    for (; r < m; ++r) {
      __m256i c0 = _mm256_setzero_si256(), c1 = _mm256_setzero_si256();
      const int8_t* pb = pb_panel;
      for (size_t ks = 0; ks < k_steps; ++ks) {
        int32_t av;
        std::memcpy(&av, a_q + r * k_in + ks * 4, 4);
        const __m256i va = _mm256_set1_epi32(av);
        const __m256i b0 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(pb));
        const __m256i b1 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(pb + 32));
        pb += 64;
        c0 = _mm256_add_epi32(c0, dot_avx2(va, b0));
        c1 = _mm256_add_epi32(c1, dot_avx2(va, b1));
      }
      store_avx2(a_scale, W, res, out, acc_out, r, col, c0, c1);
    }
  }
}

// gemm_x86_avx_vnni_fused, src/gemm.rs:1912-1998 (A shifted to u8 by ^0x80, -128*sum(w) compensation)
VNNI_FN void gemm_vnni(size_t m, const int8_t* a_q, const float* a_scale, const Linear& W, const float* res,
                       float* out, int32_t* acc_out, std::vector<int8_t>& a_u8) {
  const size_t n_out = W.n, k_in = W.k, k_steps = k_in / 4, n_panels = n_out / 16;
  const size_t total = m * k_in;
  if (a_u8.size() < total) a_u8.resize(total);
  const __m256i bias128 = _mm256_set1_epi8(-128);
  size_t idx = 0;
  for (; idx + 32 <= total; idx += 32)
    _mm256_storeu_si256(reinterpret_cast<__m256i*>(a_u8.data() + idx),
                        _mm256_xor_si256(_mm256_loadu_si256(reinterpret_cast<const __m256i*>(a_q + idx)), bias128));
  for (; idx < total; ++idx) a_u8[idx] = int8_t(uint8_t(a_q[idx]) ^ 0x80);
  for (size_t r = 0; r < m; ++r) {
    const int32_t* a_row = reinterpret_cast<const int32_t*>(a_u8.data() + r * k_in);
    const __m256 s_row = _mm256_set1_ps(a_scale[r]);
    const size_t row_off = r * n_out;
    for (size_t nb = 0; nb < n_panels; ++nb) {
      const size_t col = nb * 16;
      const int8_t* pb = W.packed.data() + nb * k_steps * 64;
      __m256i c0 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(W.comp.data() + col));
      __m256i c1 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(W.comp.data() + col + 8));
      for (size_t ks = 0; ks < k_steps; ++ks) {
        int32_t av;
        std::memcpy(&av, a_row + ks, 4);
        const __m256i va = _mm256_set1_epi32(av);
        const __m256i b0 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(pb));
        const __m256i b1 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(pb + 32));
        pb += 64;
        c0 = _mm256_dpbusd_avx_epi32(c0, va, b0);
        c1 = _mm256_dpbusd_avx_epi32(c1, va, b1);
      }
      const __m256 ws0 = _mm256_mul_ps(s_row, _mm256_loadu_ps(W.ws.data() + col));
      const __m256 ws1 = _mm256_mul_ps(s_row, _mm256_loadu_ps(W.ws.data() + col + 8));
      __m256 b0 = _mm256_loadu_ps(W.bias.data() + col), b1 = _mm256_loadu_ps(W.bias.data() + col + 8);
      if (res) {
        b0 = _mm256_add_ps(b0, _mm256_loadu_ps(res + row_off + col));
        b1 = _mm256_add_ps(b1, _mm256_loadu_ps(res + row_off + col + 8));
      }
      if (acc_out) {
        _mm256_storeu_si256(reinterpret_cast<__m256i*>(acc_out + row_off + col), c0);
        _mm256_storeu_si256(reinterpret_cast<__m256i*>(acc_out + row_off + col + 8), c1);
      }
      _mm256_storeu_ps(out + row_off + col, _mm256_fmadd_ps(_mm256_cvtepi32_ps(c0), ws0, b0));
      _mm256_storeu_ps(out + row_off + col + 8, _mm256_fmadd_ps(_mm256_cvtepi32_ps(c1), ws1, b1));
    }
  }
}

// gemm_scalar_fused, src/gemm.rs:2000-2029
void gemm_scalar(size_t m, const int8_t* a_q, const float* a_scale, const Linear& W, const float* res, float* out,
                 int32_t* acc_out) {
  for (size_t r = 0; r < m; ++r) {
    const int8_t* a_row = a_q + r * W.k;
    const float s_r = a_scale[r];
    for (size_t n = 0; n < W.n; ++n) {
      const int8_t* w_row = W.packed.data() + n * W.k;
      int32_t acc = 0;
      for (size_t k = 0; k < W.k; ++k) acc += int32_t(a_row[k]) * int32_t(w_row[k]);
      float b = W.bias[n];
      if (res) b += res[r * W.n + n];
      if (acc_out) acc_out[r * W.n + n] = acc;
      out[r * W.n + n] = std::fma(float(acc), s_r * W.ws[n], b);
    }
  }
}

// gemm_int8_fused dispatch, src/gemm.rs:630-671
void gemm(size_t m, const int8_t* a_q, std::vector<int8_t>& scratch, const float* a_scale, const Linear& W,
          const float* res, float* out, int32_t* acc_out = nullptr) {
  if (m == 0) return;
  switch (W.backend) {
    case OR_BACKEND_AVX_VNNI: gemm_vnni(m, a_q, a_scale, W, res, out, acc_out, scratch); break;
    case OR_BACKEND_AVX2: gemm_avx2(m, a_q, a_scale, W, res, out, acc_out); break;
    default: gemm_scalar(m, a_q, a_scale, W, res, out, acc_out); break;
  }
}

// ------------------------------------------------------------------------------------------ simd_math
// hsum256_ps / hmax256_ps, src/simd_math.rs:3075-3096
AVX2_FN inline float hsum256(__m256 v) {
  __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  __m128 sums = _mm_add_ps(s, _mm_movehdup_ps(s));
  return _mm_cvtss_f32(_mm_add_ss(sums, _mm_movehl_ps(sums, sums)));
}
AVX2_FN inline float hmax256(__m256 v) {
  __m128 m = _mm_max_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
  __m128 m64 = _mm_max_ps(m, _mm_movehdup_ps(m));
  return _mm_cvtss_f32(_mm_max_ss(m64, _mm_movehl_ps(m64, m64)));
}

// avx2_exp_f32, src/simd_math.rs:113-143
AVX2_FN inline __m256 avx2_exp(__m256 y_in) {
  __m256 y = _mm256_max_ps(_mm256_min_ps(y_in, _mm256_set1_ps(88.0f)), _mm256_set1_ps(-87.3f));
  __m256 n = _mm256_round_ps(_mm256_mul_ps(y, _mm256_set1_ps(1.44269504088896341f)),
                             _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
  __m256 r = _mm256_fnmadd_ps(n, _mm256_set1_ps(1.428606765330187e-6f),
                              _mm256_fnmadd_ps(n, _mm256_set1_ps(0.693145751953125f), y));
  __m256 p = _mm256_fmadd_ps(r, _mm256_set1_ps(0.008333334f), _mm256_set1_ps(0.041666668f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(0.16666667f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(0.5f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(1.0f));
  p = _mm256_fmadd_ps(r, p, _mm256_set1_ps(1.0f));
  __m256i ni = _mm256_add_epi32(_mm256_cvtps_epi32(n), _mm256_set1_epi32(127));
  return _mm256_mul_ps(p, _mm256_castsi256_ps(_mm256_slli_epi32(ni, 23)));
}

// avx2_gelu_f32, src/simd_math.rs:152-175 (rational approximation, clamped to [-4.8, 4.8])
AVX2_FN inline __m256 avx2_gelu(__m256 x) {
  __m256 xc = _mm256_min_ps(_mm256_max_ps(x, _mm256_set1_ps(-4.8f)), _mm256_set1_ps(4.8f));
  __m256 u = _mm256_mul_ps(xc, xc);
  __m256 num = _mm256_fmadd_ps(u, _mm256_set1_ps(6.4292e-5f), _mm256_set1_ps(0.007572631f));
  num = _mm256_fmadd_ps(u, num, _mm256_set1_ps(0.055282866f));
  num = _mm256_fmadd_ps(u, num, _mm256_set1_ps(0.797882463f));
  __m256 den = _mm256_fmadd_ps(u, _mm256_set1_ps(0.001139532f), _mm256_set1_ps(0.02381135f));
  den = _mm256_fmadd_ps(u, den, _mm256_set1_ps(0.235943093f));
  den = _mm256_fmadd_ps(u, den, _mm256_set1_ps(1.0f));
  __m256 est = _mm256_rcp_ps(den);
  __m256 inv_den = _mm256_mul_ps(est, _mm256_fnmadd_ps(den, est, _mm256_set1_ps(2.0f)));
  __m256 erf_a = _mm256_min_ps(_mm256_max_ps(_mm256_mul_ps(xc, _mm256_mul_ps(num, inv_den)), _mm256_set1_ps(-1.0f)),
                               _mm256_set1_ps(1.0f));
  return _mm256_mul_ps(_mm256_mul_ps(x, _mm256_set1_ps(0.5f)), _mm256_add_ps(_mm256_set1_ps(1.0f), erf_a));
}

// One lane through avx2_gelu (test helper).
AVX2_FN float gelu_lane(float x) { return _mm256_cvtss_f32(avx2_gelu(_mm256_set1_ps(x))); }

// scalar_gelu, src/simd_math.rs:14-23 (Abramowitz-Stegun erf)
float scalar_gelu(float x) {
  const float z = std::fabs(x) * 0.70710678118654752f;
  const float t = 1.0f / (1.0f + 0.3275911f * z);
  const float poly =
      t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
  const float erf_val = std::copysign(1.0f - poly * std::exp(-z * z), x);
  return 0.5f * x * (1.0f + erf_val);
}

// Quantize 16 lanes (clamp, cvtps_epi32, saturating packs) as the AVX2 kernels do.
AVX2_FN inline void quant16(__m256 v0, __m256 v1, int8_t* q) {
  const __m256 lo = _mm256_set1_ps(-127.0f), hi = _mm256_set1_ps(127.0f);
  __m256i q0 = _mm256_cvtps_epi32(_mm256_min_ps(_mm256_max_ps(v0, lo), hi));
  __m256i q1 = _mm256_cvtps_epi32(_mm256_min_ps(_mm256_max_ps(v1, lo), hi));
  __m256i q16 = _mm256_permute4x64_epi64(_mm256_packs_epi32(q0, q1), 0xD8);
  __m128i q8 = _mm_packs_epi16(_mm256_castsi256_si128(q16), _mm256_extracti128_si256(q16, 1));
  _mm_storeu_si128(reinterpret_cast<__m128i*>(q), q8);
}

// layernorm_smooth_quantize_row_avx2, src/simd_math.rs:369-477
AVX2_FN float ln_sq_avx2(float* x, const float* g, const float* b, const float* s, int8_t* q, size_t n) {
  __m256 sum0 = _mm256_setzero_ps(), sum1 = _mm256_setzero_ps();
  for (size_t i = 0; i < n; i += 16) {
    sum0 = _mm256_add_ps(sum0, _mm256_loadu_ps(x + i));
    sum1 = _mm256_add_ps(sum1, _mm256_loadu_ps(x + i + 8));
  }
  const float mean = hsum256(_mm256_add_ps(sum0, sum1)) / float(n);
  const __m256 vmean = _mm256_set1_ps(mean);
  __m256 v0 = _mm256_setzero_ps(), v1 = _mm256_setzero_ps();
  for (size_t i = 0; i < n; i += 16) {
    __m256 d0 = _mm256_sub_ps(_mm256_loadu_ps(x + i), vmean), d1 = _mm256_sub_ps(_mm256_loadu_ps(x + i + 8), vmean);
    v0 = _mm256_fmadd_ps(d0, d0, v0);
    v1 = _mm256_fmadd_ps(d1, d1, v1);
  }
  const float var = hsum256(_mm256_add_ps(v0, v1)) / float(n);
  const __m256 vrstd = _mm256_set1_ps(1.0f / std::sqrt(var + EPS));
  const __m256 sign = _mm256_set1_ps(-0.0f);
  __m256 vmax = _mm256_set1_ps(1e-8f);
  for (size_t i = 0; i < n; i += 16) {
    __m256 y0 = _mm256_fmadd_ps(_mm256_mul_ps(_mm256_sub_ps(_mm256_loadu_ps(x + i), vmean), vrstd),
                                _mm256_loadu_ps(g + i), _mm256_loadu_ps(b + i));
    __m256 y1 = _mm256_fmadd_ps(_mm256_mul_ps(_mm256_sub_ps(_mm256_loadu_ps(x + i + 8), vmean), vrstd),
                                _mm256_loadu_ps(g + i + 8), _mm256_loadu_ps(b + i + 8));
    _mm256_storeu_ps(x + i, y0);
    _mm256_storeu_ps(x + i + 8, y1);
    __m256 a0 = _mm256_andnot_ps(sign, _mm256_mul_ps(y0, _mm256_loadu_ps(s + i)));
    __m256 a1 = _mm256_andnot_ps(sign, _mm256_mul_ps(y1, _mm256_loadu_ps(s + i + 8)));
    vmax = _mm256_max_ps(vmax, _mm256_max_ps(a0, a1));
  }
  const float max_abs = hmax256(vmax);
  const float scale = max_abs / 127.0f;
  const __m256 vinv = _mm256_set1_ps(127.0f / max_abs);
  for (size_t i = 0; i < n; i += 16)
    quant16(_mm256_mul_ps(_mm256_loadu_ps(x + i), _mm256_mul_ps(_mm256_loadu_ps(s + i), vinv)),
            _mm256_mul_ps(_mm256_loadu_ps(x + i + 8), _mm256_mul_ps(_mm256_loadu_ps(s + i + 8), vinv)), q + i);
  return scale;
}

// layernorm_smooth_quantize_row_scalar, src/simd_math.rs:203-247
float ln_sq_scalar(float* x, const float* g, const float* b, const float* s, int8_t* q, size_t n) {
  float sum = 0.0f;
  for (size_t j = 0; j < n; ++j) sum += x[j];
  const float mean = sum / float(n);
  float var_sum = 0.0f;
  for (size_t j = 0; j < n; ++j) {
    const float d = x[j] - mean;
    var_sum += d * d;
  }
  const float rstd = 1.0f / std::sqrt(var_sum / float(n) + EPS);
  float max_abs = 1e-8f;
  for (size_t j = 0; j < n; ++j) {
    const float y = (x[j] - mean) * rstd * g[j] + b[j];
    x[j] = y;
    const float a = std::fabs(y * s[j]);
    if (a > max_abs) max_abs = a;
  }
  const float scale = max_abs / 127.0f, inv = 127.0f / max_abs;
  for (size_t j = 0; j < n; ++j) {
    const float v = std::round(x[j] * s[j] * inv);  // f32::round: half away from zero
    q[j] = int8_t(std::fmin(std::fmax(v, -127.0f), 127.0f));
  }
  return scale;
}

// layernorm_smooth_quantize_row dispatch, src/simd_math.rs:181-201
float ln_sq(float* x, const float* g, const float* b, const float* s, int8_t* q, size_t n) {
  return g_avx2_fma ? ln_sq_avx2(x, g, b, s, q, n) : ln_sq_scalar(x, g, b, s, q, n);
}

// smooth_quantize_row_avx2, src/simd_math.rs:584-649 (and the scalar fallback :501-531)
AVX2_FN float sq_avx2(const float* x, const float* s, int8_t* q, size_t n) {
  const __m256 sign = _mm256_set1_ps(-0.0f);
  __m256 vmax = _mm256_set1_ps(1e-8f);
  for (size_t i = 0; i < n; i += 16) {
    __m256 a0 = _mm256_andnot_ps(sign, _mm256_mul_ps(_mm256_loadu_ps(x + i), _mm256_loadu_ps(s + i)));
    __m256 a1 = _mm256_andnot_ps(sign, _mm256_mul_ps(_mm256_loadu_ps(x + i + 8), _mm256_loadu_ps(s + i + 8)));
    vmax = _mm256_max_ps(vmax, _mm256_max_ps(a0, a1));
  }
  const float max_abs = hmax256(vmax);
  const __m256 vinv = _mm256_set1_ps(127.0f / max_abs);
  for (size_t i = 0; i < n; i += 16)
    quant16(_mm256_mul_ps(_mm256_loadu_ps(x + i), _mm256_mul_ps(_mm256_loadu_ps(s + i), vinv)),
            _mm256_mul_ps(_mm256_loadu_ps(x + i + 8), _mm256_mul_ps(_mm256_loadu_ps(s + i + 8), vinv)), q + i);
  return max_abs / 127.0f;
}
float sq_scalar(const float* x, const float* s, int8_t* q, size_t n) {
  float max_abs = 1e-8f;
  for (size_t j = 0; j < n; ++j) {
    const float a = std::fabs(x[j] * s[j]);
    if (a > max_abs) max_abs = a;
  }
  const float inv = 127.0f / max_abs;
  for (size_t j = 0; j < n; ++j) q[j] = int8_t(std::fmin(std::fmax(std::round(x[j] * s[j] * inv), -127.0f), 127.0f));
  return max_abs / 127.0f;
}
float smooth_quant(const float* x, const float* s, int8_t* q, size_t n) {
  return g_avx2_fma ? sq_avx2(x, s, q, n) : sq_scalar(x, s, q, n);
}

// gelu_smooth_quantize_row_avx2, src/simd_math.rs:1371-1435 (scalar fallback :1295-1312)
AVX2_FN float gq_avx2(float* x, const float* s, int8_t* q, size_t n) {
  const __m256 sign = _mm256_set1_ps(-0.0f);
  __m256 vmax = _mm256_set1_ps(1e-8f);
  for (size_t i = 0; i < n; i += 16) {
    __m256 g0 = _mm256_mul_ps(avx2_gelu(_mm256_loadu_ps(x + i)), _mm256_loadu_ps(s + i));
    __m256 g1 = _mm256_mul_ps(avx2_gelu(_mm256_loadu_ps(x + i + 8)), _mm256_loadu_ps(s + i + 8));
    _mm256_storeu_ps(x + i, g0);
    _mm256_storeu_ps(x + i + 8, g1);
    vmax = _mm256_max_ps(vmax, _mm256_max_ps(_mm256_andnot_ps(sign, g0), _mm256_andnot_ps(sign, g1)));
  }
  const float max_abs = hmax256(vmax);
  const __m256 vinv = _mm256_set1_ps(127.0f / max_abs);
  for (size_t i = 0; i < n; i += 16)
    quant16(_mm256_mul_ps(_mm256_loadu_ps(x + i), vinv), _mm256_mul_ps(_mm256_loadu_ps(x + i + 8), vinv), q + i);
  return max_abs / 127.0f;
}
float gq_scalar(float* x, const float* s, int8_t* q, size_t n) {
  float max_abs = 1e-8f;
  for (size_t j = 0; j < n; ++j) {
    const float g = scalar_gelu(x[j]) * s[j];
    x[j] = g;
    if (std::fabs(g) > max_abs) max_abs = std::fabs(g);
  }
  const float inv = 127.0f / max_abs;
  for (size_t j = 0; j < n; ++j) q[j] = int8_t(std::fmin(std::fmax(std::round(x[j] * inv), -127.0f), 127.0f));
  return max_abs / 127.0f;
}
float gelu_quant(float* x, const float* s, int8_t* q, size_t n) {
  return g_avx2_fma ? gq_avx2(x, s, q, n) : gq_scalar(x, s, q, n);
}

// layernorm_inplace_row, src/simd_math.rs:481-497
void ln_inplace(float* x, const float* g, const float* b, size_t n) {
  float sum = 0.0f;
  for (size_t j = 0; j < n; ++j) sum += x[j];
  const float mean = sum / float(n);
  float var_sum = 0.0f;
  for (size_t j = 0; j < n; ++j) {
    const float d = x[j] - mean;
    var_sum += d * d;
  }
  const float rstd = 1.0f / std::sqrt(var_sum / float(n) + EPS);
  for (size_t j = 0; j < n; ++j) x[j] = (x[j] - mean) * rstd * g[j] + b[j];
}

// l2_normalize_inplace, src/simd_math.rs:2892-2903
void l2_normalize(float* v, size_t n) {
  float sum_sq = 0.0f;
  for (size_t j = 0; j < n; ++j) sum_sq += v[j] * v[j];
  if (sum_sq > 0.0f) {
    const float inv = 1.0f / std::sqrt(sum_sq);
    for (size_t j = 0; j < n; ++j) v[j] *= inv;
  }
}

// dequant_add_embeddings_row, src/simd_math.rs:1827-1881 (generic path taken on x86_64)
void dequant_add_emb(const int8_t* w, float w_s, const int8_t* p, float p_s, const float* t, float* h, size_t n) {
  for (size_t j = 0; j < n; ++j) h[j] = float(w[j]) * w_s + float(p[j]) * p_s + t[j];
}

// compute_scores_head32_avx2, src/simd_math.rs:2953-2984 (dot32x4_avx2 :2937-2950)
AVX2_FN inline __m256 dot32x4(__m256 q0, __m256 q1, __m256 q2, __m256 q3, const float* kp) {
  __m256 a = _mm256_fmadd_ps(q1, _mm256_loadu_ps(kp + 8), _mm256_mul_ps(q0, _mm256_loadu_ps(kp)));
  __m256 b = _mm256_fmadd_ps(q3, _mm256_loadu_ps(kp + 24), _mm256_mul_ps(q2, _mm256_loadu_ps(kp + 16)));
  return _mm256_add_ps(a, b);
}
AVX2_FN void scores_avx2(const float* q, const float* k, float scale, float* sp, size_t L) {
  const __m256 vs = _mm256_set1_ps(scale);
  const __m256 q0 = _mm256_mul_ps(_mm256_loadu_ps(q), vs), q1 = _mm256_mul_ps(_mm256_loadu_ps(q + 8), vs);
  const __m256 q2 = _mm256_mul_ps(_mm256_loadu_ps(q + 16), vs), q3 = _mm256_mul_ps(_mm256_loadu_ps(q + 24), vs);
  size_t tk = 0;
  for (; tk + 4 <= L; tk += 4) {
    const float* k0 = k + tk * 32;
    __m256 s0 = dot32x4(q0, q1, q2, q3, k0), s1 = dot32x4(q0, q1, q2, q3, k0 + 32);
    __m256 s2 = dot32x4(q0, q1, q2, q3, k0 + 64), s3 = dot32x4(q0, q1, q2, q3, k0 + 96);
    __m256 t = _mm256_hadd_ps(_mm256_hadd_ps(s0, s1), _mm256_hadd_ps(s2, s3));
    _mm_storeu_ps(sp + tk, _mm_add_ps(_mm256_castps256_ps128(t), _mm256_extractf128_ps(t, 1)));
  }
  for (; tk < L; ++tk) sp[tk] = hsum256(dot32x4(q0, q1, q2, q3, k + tk * 32));
}
void scores_scalar(const float* q, const float* k, float scale, float* sp, size_t L) {
  for (size_t tk = 0; tk < L; ++tk) {
    float sum = 0.0f;
    for (size_t i = 0; i < 32; ++i) sum += q[i] * k[tk * 32 + i];
    sp[tk] = sum * scale;
  }
}

// softmax_inplace_avx2, src/simd_math.rs:2989-3042 (scalar fallback :1681-1702)
AVX2_FN void softmax_avx2(float* p, size_t len) {
  size_t i = 0;
  __m256 vmax = _mm256_set1_ps(-INFINITY);
  for (; i + 8 <= len; i += 8) vmax = _mm256_max_ps(vmax, _mm256_loadu_ps(p + i));
  float max_val = hmax256(vmax);
  for (; i < len; ++i) max_val = std::fmax(max_val, p[i]);
  const __m256 vm = _mm256_set1_ps(max_val);
  __m256 vs0 = _mm256_setzero_ps(), vs1 = _mm256_setzero_ps();
  i = 0;
  for (; i + 16 <= len; i += 16) {
    __m256 e0 = avx2_exp(_mm256_sub_ps(_mm256_loadu_ps(p + i), vm));
    __m256 e1 = avx2_exp(_mm256_sub_ps(_mm256_loadu_ps(p + i + 8), vm));
    _mm256_storeu_ps(p + i, e0);
    _mm256_storeu_ps(p + i + 8, e1);
    vs0 = _mm256_add_ps(vs0, e0);
    vs1 = _mm256_add_ps(vs1, e1);
  }
  for (; i + 8 <= len; i += 8) {
    __m256 e = avx2_exp(_mm256_sub_ps(_mm256_loadu_ps(p + i), vm));
    _mm256_storeu_ps(p + i, e);
    vs0 = _mm256_add_ps(vs0, e);
  }
  float sum = hsum256(_mm256_add_ps(vs0, vs1));
  for (; i < len; ++i) {
    const float e = std::exp(p[i] - max_val);
    p[i] = e;
    sum += e;
  }
  const float inv = 1.0f / sum;
  const __m256 vinv = _mm256_set1_ps(inv);
  i = 0;
  for (; i + 8 <= len; i += 8) _mm256_storeu_ps(p + i, _mm256_mul_ps(_mm256_loadu_ps(p + i), vinv));
  for (; i < len; ++i) p[i] *= inv;
}
void softmax_scalar(float* p, size_t len) {
  float max_val = -INFINITY;
  for (size_t i = 0; i < len; ++i)
    if (p[i] > max_val) max_val = p[i];
  float sum = 0.0f;
  for (size_t i = 0; i < len; ++i) {
    const float e = std::exp(p[i] - max_val);
    p[i] = e;
    sum += e;
  }
  const float inv = 1.0f / sum;
  for (size_t i = 0; i < len; ++i) p[i] *= inv;
}

// weighted_sum_head32_avx2, src/simd_math.rs:3047-3070 (scalar fallback :1811-1821)
AVX2_FN void wsum_avx2(const float* p, const float* v, size_t L, float* out) {
  __m256 a[4], b[4];
  for (int j = 0; j < 4; ++j) a[j] = b[j] = _mm256_setzero_ps();
  size_t t = 0;
  for (; t + 2 <= L; t += 2) {
    const __m256 pa = _mm256_set1_ps(p[t]), pb = _mm256_set1_ps(p[t + 1]);
    const float *ra = v + t * 32, *rb = v + t * 32 + 32;
    for (int j = 0; j < 4; ++j) {
      a[j] = _mm256_fmadd_ps(_mm256_loadu_ps(ra + 8 * j), pa, a[j]);
      b[j] = _mm256_fmadd_ps(_mm256_loadu_ps(rb + 8 * j), pb, b[j]);
    }
  }
  if (t < L) {
    const __m256 pa = _mm256_set1_ps(p[t]);
    for (int j = 0; j < 4; ++j) a[j] = _mm256_fmadd_ps(_mm256_loadu_ps(v + t * 32 + 8 * j), pa, a[j]);
  }
  for (int j = 0; j < 4; ++j) _mm256_storeu_ps(out + 8 * j, _mm256_add_ps(a[j], b[j]));
}
void wsum_scalar(const float* p, const float* v, size_t L, float* out) {
  for (int d = 0; d < 32; ++d) out[d] = 0.0f;
  for (size_t t = 0; t < L; ++t)
    for (int d = 0; d < 32; ++d) out[d] += p[t] * v[t * 32 + d];
}

// One (head, query): compute_scores_head32 + softmax_inplace + weighted_sum_head32,
// as in the per-head loops of src/model.rs:306-320.
void attend(const float* q, const float* k_head, const float* v_head, size_t L, float* scores, float* out) {
  const float inv_sqrt_d = 1.0f / std::sqrt(32.0f);
  if (g_avx2_fma) {
    scores_avx2(q, k_head, inv_sqrt_d, scores, L);
    softmax_avx2(scores, L);
    wsum_avx2(scores, v_head, L, out);
  } else {
    scores_scalar(q, k_head, inv_sqrt_d, scores, L);
    softmax_scalar(scores, L);
    wsum_scalar(scores, v_head, L, out);
  }
}

// ------------------------------------------------------------------------------------------ int8 attention
// The reference's int8 attention scheme, attention_heads_sme (src/simd_math.rs:1933-2186), which
// the crate runs on its SME backend for layers 0-10 (src/model.rs:245, :608):
//   pack_qkv_head_int8_neon (:2564-2800): Q and K rows of a head quantized per token with
//     quantize_head32_row_neon (:2482-2527), the K scale carrying 1/sqrt(32) * log2(e) so that the
//     softmax runs in base 2; V quantized per column (:2598-2640, quantize_v_row_neon :2530-2561);
//   Q.K^T as int32 dot products, dequantized as (acc * k_scale) * q_scale
//     (softmax_quantize_i16_from_acc_neon :2291-2336);
//   softmax_exp2_quantize_pass_i16_neon (:2379-2410): q = round(16383 * 2^(s - max)) through
//     exp2_q_neon (:2353-2366) for the row's complete 8-key blocks and through exp2 + round for
//     the last len % 8 keys, p_scale = 1 / sum(q);
//   P.V as int32 dot products of the 14-bit q with the int8 V, ctx = acc * (v_scale * p_scale).
// Every step is elementwise or an integer sum, so this scalar restatement gives the NEON lanes'
// values whatever the order. Scales are taken over one sequence's keys: what forward_cls computes
// for that sequence on its own.
inline int8_t sat_i8(int32_t v) { return int8_t(v < -128 ? -128 : v > 127 ? 127 : v); }
inline int32_t rn_even(float x) { return int32_t(std::nearbyint(x)); }  // vcvtnq_s32_f32

// quantize_head32_row_neon: q = sat(rn(x * (127 / m))), m = max(1e-8, max |x|); returns (m / 127) * mul
float quant_head_row(const float* x, float mul, int8_t* q) {
  float m = 0.0f;
  for (size_t d = 0; d < HD; ++d) m = std::max(m, std::fabs(x[d]));
  m = std::max(m, 1e-8f);
  const float inv = 127.0f / m;
  for (size_t d = 0; d < HD; ++d) q[d] = sat_i8(rn_even(x[d] * inv));
  return (m / 127.0f) * mul;
}

// exp2_q_neon(x, 16383, -16): round(16383 * 2^x) for x <= 0, degree-3 polynomial for 2^f on
// [0, 1) and the integer part added to the exponent field.
int32_t exp2_q16383(float x) {
  const float scale = 16383.0f;
  x = std::max(x, -16.0f);
  const int32_t n = int32_t(std::floor(x));
  const float f = x - float(n);
  float p = std::fma(f, 0.07842169f * scale, 0.22511937f * scale);
  p = std::fma(f, p, 0.6963853f * scale);
  p = std::fma(f, p, 0.999857f * scale);
  uint32_t b;
  std::memcpy(&b, &p, 4);
  b += uint32_t(n) << 23;
  std::memcpy(&p, &b, 4);
  return rn_even(p);
}

// One sequence of L keys: qkv rows (stride 3 * 384: Q | K | V) -> ctx rows (stride 384).
void attention_i8_seq(const float* qkv, size_t L, float* ctx) {
  const float k_mul = (1.0f / std::sqrt(32.0f)) * 1.44269504088896341f;  // inv_sqrt_d * LOG2_E
  std::vector<int8_t> qq(L * HD), kq(L * HD), vq(L * HD);
  std::vector<float> qs(L), ks(L), s(L);
  std::vector<int32_t> p(L);
  for (size_t h = 0; h < NH; ++h) {
    const size_t ho = h * HD;
    float vm[HD], v_scale[HD], v_inv[HD];
    for (size_t c = 0; c < HD; ++c) vm[c] = 1e-8f;
    for (size_t t = 0; t < L; ++t)
      for (size_t c = 0; c < HD; ++c) vm[c] = std::max(vm[c], std::fabs(qkv[t * 3 * H + 2 * H + ho + c]));
    for (size_t c = 0; c < HD; ++c) {
      v_scale[c] = vm[c] * (1.0f / 127.0f);
      v_inv[c] = 127.0f / vm[c];
    }
    for (size_t t = 0; t < L; ++t) {
      const float* row = qkv + t * 3 * H;
      for (size_t c = 0; c < HD; ++c) vq[t * HD + c] = sat_i8(rn_even(row[2 * H + ho + c] * v_inv[c]));
      qs[t] = quant_head_row(row + ho, 1.0f, &qq[t * HD]);
      ks[t] = quant_head_row(row + H + ho, k_mul, &kq[t * HD]);
    }
    const size_t vec_end = L - L % 8;
    for (size_t i = 0; i < L; ++i) {
      float mx = -INFINITY;
      for (size_t j = 0; j < L; ++j) {
        int32_t acc = 0;
        for (size_t d = 0; d < HD; ++d) acc += int32_t(qq[i * HD + d]) * int32_t(kq[j * HD + d]);
        s[j] = (float(acc) * ks[j]) * qs[i];
        mx = std::max(mx, s[j]);
      }
      int32_t isum = 0;
      for (size_t j = 0; j < L; ++j) {
        int32_t q;
        if (j < vec_end) {
          q = exp2_q16383(s[j] - mx);
        } else {
          const int32_t e = int32_t(std::round(std::exp2(s[j] - mx) * 16383.0f));
          q = e < 0 ? 0 : e > 16383 ? 16383 : e;
        }
        p[j] = q;
        isum += q;
      }
      const float p_scale = 1.0f / float(std::max(isum, 1));
      for (size_t c = 0; c < HD; ++c) {
        int32_t acc = 0;
        for (size_t j = 0; j < L; ++j) acc += p[j] * int32_t(vq[j * HD + c]);
        ctx[i * H + ho + c] = float(acc) * (v_scale[c] * p_scale);
      }
    }
  }
}

// ------------------------------------------------------------------------------------------ forward
// Workspace, src/model.rs:123-173
struct Workspace {
  std::vector<float> hidden, tmp_hidden, qkv, q_cls, ctx, k_head, v_head, scores, inter;
  std::vector<int8_t> act_q, inter_q, scratch;
  std::vector<float> act_scale;
  Workspace()
      : hidden(MAXPOS * H), tmp_hidden(MAXPOS * H), qkv(MAXPOS * 3 * H), q_cls(MAXPOS * H), ctx(MAXPOS * H),
        k_head(MAXPOS * HD), v_head(MAXPOS * HD), scores(MAXPOS), inter(MAXPOS * INTER), act_q(MAXPOS * H),
        inter_q(MAXPOS * INTER), act_scale(MAXPOS) {}
};

struct Trace {
  int8_t* gemm_in_q = nullptr;
  float* gemm_in_s = nullptr;
  float* qkv_out = nullptr;
  float* ctx = nullptr;
  float* hidden = nullptr;
  int8_t* down_in_q = nullptr;
  float* down_in_s = nullptr;
};

void embed_rows(const or_model& m, const uint16_t* ids, size_t len, size_t dst0, Workspace& ws) {
  const float* first_inv = m.layers[0].qkv.inv_s.data();
  for (size_t t = 0; t < len; ++t) {
    const size_t tok = ids[t], dst = (dst0 + t) * H;
    float* h = ws.hidden.data() + dst;
    dequant_add_emb(m.word_q.data() + tok * H, m.word_s[tok], m.pos_q.data() + t * H, m.pos_s[t], m.type0.data(), h, H);
    ws.act_scale[dst0 + t] =
        ln_sq(h, m.emb_lnw.data(), m.emb_lnb.data(), first_inv, ws.act_q.data() + dst, H);
  }
}

// Attention of one segment [s0, s0+L) of the fused QKV buffer (src/model.rs:294-321, :663-694).
void attention_segment(Workspace& ws, size_t s0, size_t L) {
  for (size_t h = 0; h < NH; ++h) {
    const size_t ho = h * HD;
    for (size_t t = 0; t < L; ++t) {
      const float* row = ws.qkv.data() + (s0 + t) * 3 * H;
      std::memcpy(ws.k_head.data() + t * HD, row + H + ho, HD * 4);
      std::memcpy(ws.v_head.data() + t * HD, row + 2 * H + ho, HD * 4);
    }
    for (size_t tq = 0; tq < L; ++tq)
      attend(ws.qkv.data() + (s0 + tq) * 3 * H + ho, ws.k_head.data(), ws.v_head.data(), L, ws.scores.data(),
             ws.ctx.data() + (s0 + tq) * H + ho);
  }
}

// Layers 0..10 over `total` rows with segment bounds (src/model.rs:224-398, :593-768).
void layers_0_10(const or_model& m, Workspace& ws, size_t total, const std::vector<std::pair<size_t, size_t>>& segs,
                 const Trace* tr) {
  for (size_t l = 0; l + 1 < NL; ++l) {
    const Layer& ly = m.layers[l];
    const float* next_inv = m.layers[l + 1].qkv.inv_s.data();
    if (tr && tr->gemm_in_q) std::memcpy(tr->gemm_in_q + l * total * H, ws.act_q.data(), total * H);
    if (tr && tr->gemm_in_s) std::memcpy(tr->gemm_in_s + l * total, ws.act_scale.data(), total * 4);
    gemm(total, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.qkv, nullptr, ws.qkv.data());
    if (tr && tr->qkv_out) std::memcpy(tr->qkv_out + l * total * 3 * H, ws.qkv.data(), total * 3 * H * 4);
    for (auto& sg : segs) {
      const size_t L = sg.second - sg.first;
      // int8 mode: the reference's crossover for one sequence (src/model.rs:245), per sequence
      if (m.attn_mode == OR_ATTENTION_INT8 && L >= 16)
        attention_i8_seq(ws.qkv.data() + sg.first * 3 * H, L, ws.ctx.data() + sg.first * H);
      else
        attention_segment(ws, sg.first, L);
    }
    if (tr && tr->ctx) std::memcpy(tr->ctx + l * total * H, ws.ctx.data(), total * H * 4);
    for (size_t t = 0; t < total; ++t)
      ws.act_scale[t] = smooth_quant(ws.ctx.data() + t * H, ly.attn_out.inv_s.data(), ws.act_q.data() + t * H, H);
    gemm(total, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.attn_out, ws.hidden.data(), ws.tmp_hidden.data());
    std::swap(ws.hidden, ws.tmp_hidden);
    for (size_t t = 0; t < total; ++t)
      ws.act_scale[t] = ln_sq(ws.hidden.data() + t * H, ly.ln1w.data(), ly.ln1b.data(), ly.ffn_inter.inv_s.data(),
                              ws.act_q.data() + t * H, H);
    gemm(total, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.ffn_inter, nullptr, ws.inter.data());
    for (size_t t = 0; t < total; ++t)
      ws.act_scale[t] = gelu_quant(ws.inter.data() + t * INTER, ly.ffn_out.inv_s.data(), ws.inter_q.data() + t * INTER,
                                   INTER);
    if (tr && tr->down_in_q) std::memcpy(tr->down_in_q + l * total * INTER, ws.inter_q.data(), total * INTER);
    if (tr && tr->down_in_s) std::memcpy(tr->down_in_s + l * total, ws.act_scale.data(), total * 4);
    gemm(total, ws.inter_q.data(), ws.scratch, ws.act_scale.data(), ly.ffn_out, ws.hidden.data(), ws.tmp_hidden.data());
    std::swap(ws.hidden, ws.tmp_hidden);
    for (size_t t = 0; t < total; ++t)
      ws.act_scale[t] = ln_sq(ws.hidden.data() + t * H, ly.ln2w.data(), ly.ln2b.data(), next_inv,
                              ws.act_q.data() + t * H, H);
    if (tr && tr->hidden) std::memcpy(tr->hidden + l * total * H, ws.hidden.data(), total * H * 4);
  }
}

// Batched [CLS] tail of layer 11 over b rows already compacted to rows 0..b (src/model.rs:845-913).
void cls_tail(const or_model& m, Workspace& ws, size_t b, float* out) {
  const Layer& ly = m.layers[NL - 1];
  for (size_t i = 0; i < b; ++i)
    ws.act_scale[i] = smooth_quant(ws.ctx.data() + i * H, ly.attn_out.inv_s.data(), ws.act_q.data() + i * H, H);
  gemm(b, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.attn_out, ws.hidden.data(), ws.tmp_hidden.data());
  for (size_t i = 0; i < b; ++i)
    ws.act_scale[i] = ln_sq(ws.tmp_hidden.data() + i * H, ly.ln1w.data(), ly.ln1b.data(), ly.ffn_inter.inv_s.data(),
                            ws.act_q.data() + i * H, H);
  gemm(b, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.ffn_inter, nullptr, ws.inter.data());
  for (size_t i = 0; i < b; ++i)
    ws.act_scale[i] =
        gelu_quant(ws.inter.data() + i * INTER, ly.ffn_out.inv_s.data(), ws.inter_q.data() + i * INTER, INTER);
  gemm(b, ws.inter_q.data(), ws.scratch, ws.act_scale.data(), ly.ffn_out, ws.tmp_hidden.data(), ws.hidden.data());
  for (size_t i = 0; i < b; ++i) {
    float* row = ws.hidden.data() + i * H;
    ln_inplace(row, ly.ln2w.data(), ly.ln2b.data(), H);
    l2_normalize(row, H);
    std::memcpy(out + i * H, row, H * 4);
  }
}

// PackedModel::forward_cls, src/model.rs:185-513
void forward_cls(const or_model& m, const uint16_t* ids, size_t n_ids, Workspace& ws, float* out, const Trace* tr) {
  const size_t L = n_ids < MAXPOS ? n_ids : MAXPOS;
  if (L < 1) return;
  embed_rows(m, ids, L, 0, ws);
  std::vector<std::pair<size_t, size_t>> segs{{0, L}};
  layers_0_10(m, ws, L, segs, tr);

  const Layer& ly = m.layers[NL - 1];
  if (tr && tr->gemm_in_q) std::memcpy(tr->gemm_in_q + 11 * L * H, ws.act_q.data(), L * H);
  if (tr && tr->gemm_in_s) std::memcpy(tr->gemm_in_s + 11 * L, ws.act_scale.data(), L * 4);
  gemm(1, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.q_only, nullptr, ws.q_cls.data());
  gemm(L, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.kv_only, nullptr, ws.qkv.data());
  for (size_t h = 0; h < NH; ++h) {
    const size_t ho = h * HD;
    for (size_t t = 0; t < L; ++t) {
      const float* row = ws.qkv.data() + t * 2 * H;
      std::memcpy(ws.k_head.data() + t * HD, row + ho, HD * 4);
      std::memcpy(ws.v_head.data() + t * HD, row + H + ho, HD * 4);
    }
    attend(ws.q_cls.data() + ho, ws.k_head.data(), ws.v_head.data(), L, ws.scores.data(), ws.ctx.data() + ho);
  }
  cls_tail(m, ws, 1, out);
}

// PackedModel::forward_ragged_cls, src/model.rs:521-914 (<= 64 sequences, <= 512 packed rows)
void forward_ragged(const or_model& m, const uint16_t* const* seqs, const size_t* lens, size_t b, Workspace& ws,
                    float* out) {
  if (b == 0) return;
  if (b == 1) {
    forward_cls(m, seqs[0], lens[0], ws, out, nullptr);
    return;
  }
  std::vector<std::pair<size_t, size_t>> segs;
  size_t cursor = 0;
  for (size_t i = 0; i < b; ++i) {
    const size_t s_len = lens[i] < MAXPOS - cursor ? lens[i] : MAXPOS - cursor;
    if (s_len < 1) return;  // the reference asserts here
    embed_rows(m, seqs[i], s_len, cursor, ws);
    segs.push_back({cursor, cursor + s_len});
    cursor += s_len;
  }
  const size_t total = cursor;
  layers_0_10(m, ws, total, segs, nullptr);

  const Layer& ly = m.layers[NL - 1];
  gemm(total, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.kv_only, nullptr, ws.qkv.data());
  for (size_t i = 0; i < b; ++i) {
    const size_t c = segs[i].first;
    if (c != i) {
      std::memmove(ws.act_q.data() + i * H, ws.act_q.data() + c * H, H);
      ws.act_scale[i] = ws.act_scale[c];
      std::memmove(ws.hidden.data() + i * H, ws.hidden.data() + c * H, H * 4);
    }
  }
  gemm(b, ws.act_q.data(), ws.scratch, ws.act_scale.data(), ly.q_only, nullptr, ws.q_cls.data());
  for (size_t i = 0; i < b; ++i) {
    const size_t s0 = segs[i].first, L = segs[i].second - s0;
    for (size_t h = 0; h < NH; ++h) {
      const size_t ho = h * HD;
      for (size_t t = 0; t < L; ++t) {
        const float* row = ws.qkv.data() + (s0 + t) * 2 * H;
        std::memcpy(ws.k_head.data() + t * HD, row + ho, HD * 4);
        std::memcpy(ws.v_head.data() + t * HD, row + H + ho, HD * 4);
      }
      attend(ws.q_cls.data() + i * H + ho, ws.k_head.data(), ws.v_head.data(), L, ws.scores.data(),
             ws.ctx.data() + i * H + ho);
    }
  }
  cls_tail(m, ws, b, out);
}

// ------------------------------------------------------------------------------------------ loader
struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  bool take(void* dst, size_t n) {
    if (!ok || size_t(end - p) < n) return ok = false;
    std::memcpy(dst, p, n);
    p += n;
    return true;
  }
  uint64_t u64() {
    uint64_t v = 0;
    take(&v, 8);
    return v;
  }
  std::vector<int8_t> i8vec() {
    const uint64_t n = u64();
    std::vector<int8_t> v;
    if (!ok || n > uint64_t(end - p)) {
      ok = false;
      return v;
    }
    v.resize(n);
    take(v.data(), n);
    return v;
  }
  std::vector<float> f32vec() {
    const uint64_t n = u64();
    std::vector<float> v;
    if (!ok || n > uint64_t(end - p) / 4) {
      ok = false;
      return v;
    }
    v.resize(n);
    take(v.data(), n * 4);
    return v;
  }
  Linear linear() {
    Linear l;
    l.n = u64();
    l.k = u64();
    l.w = i8vec();
    l.ws = f32vec();
    l.bias = f32vec();
    l.inv_s = f32vec();
    return l;
  }
};

thread_local std::string g_err;

// QuantizedModelRaw::load_ae8, src/quantize.rs:76-137
or_model* load_mem(const uint8_t* buf, uint64_t len, int backend) {
  if (len < 8 || std::memcmp(buf, "ARCTIC8\x01", 8) != 0) {
    g_err = "invalid .ae8 magic header";
    return nullptr;
  }
  Reader rd{buf + 8, buf + len};
  auto* m = new or_model();
  m->backend = backend;
  m->word_q = rd.i8vec();
  m->word_s = rd.f32vec();
  m->pos_q = rd.i8vec();
  m->pos_s = rd.f32vec();
  m->type_q = rd.i8vec();
  m->type_s = rd.f32vec();
  m->emb_lnw = rd.f32vec();
  m->emb_lnb = rd.f32vec();
  for (size_t l = 0; l < NL && rd.ok; ++l) {
    Layer& ly = m->layers[l];
    ly.qkv = rd.linear();
    uint8_t split = 0;
    rd.take(&split, 1);
    ly.has_split = split == 1;
    if (ly.has_split) {
      ly.q_only = rd.linear();
      ly.kv_only = rd.linear();
    }
    ly.attn_out = rd.linear();
    ly.ln1w = rd.f32vec();
    ly.ln1b = rd.f32vec();
    ly.ffn_inter = rd.linear();
    ly.ffn_out = rd.linear();
    ly.ln2w = rd.f32vec();
    ly.ln2b = rd.f32vec();
  }
  std::string err;
  bool ok = rd.ok;
  if (!ok) err = "truncated .ae8 pack";
  if (ok && (m->word_q.size() != VOCAB * H || m->word_s.size() != VOCAB || m->pos_q.size() != MAXPOS * H ||
             m->pos_s.size() != MAXPOS || m->type_q.size() < H || m->type_s.empty() || m->emb_lnw.size() != H ||
             m->emb_lnb.size() != H)) {
    ok = false;
    err = "embedding tables have unexpected sizes";
  }
  for (size_t l = 0; ok && l < NL; ++l) {
    Layer& ly = m->layers[l];
    const bool last = l + 1 == NL;
    if (last != ly.has_split) {
      ok = false;
      err = "has_split must be set on layer 11 only";
      break;
    }
    if (ly.qkv.k != H || ly.qkv.inv_s.size() != H) {
      ok = false;
      err = "qkv input smoothing must have 384 entries";
      break;
    }
    ok = pack_linear(ly.qkv, backend, err) && pack_linear(ly.attn_out, backend, err) &&
         pack_linear(ly.ffn_inter, backend, err) && pack_linear(ly.ffn_out, backend, err) &&
         (!ly.has_split || (pack_linear(ly.q_only, backend, err) && pack_linear(ly.kv_only, backend, err)));
  }
  if (!ok) {
    g_err = err;
    delete m;
    return nullptr;
  }
  m->type0.resize(H);
  for (size_t j = 0; j < H; ++j) m->type0[j] = float(m->type_q[j]) * m->type_s[0];
  return m;
}

}  // namespace

// ------------------------------------------------------------------------------------------ C ABI
extern "C" {

int or_detect_backend(void) {
  if (cpu_avxvnni()) return OR_BACKEND_AVX_VNNI;
  if (cpu_avx2_fma()) return OR_BACKEND_AVX2;
  return OR_BACKEND_SCALAR;
}
int or_has_avx2_fma(void) { return g_avx2_fma ? 1 : 0; }

or_model* or_model_load_mem(const uint8_t* buf, uint64_t len, int backend, const char** err) {
  if (backend == OR_BACKEND_AVX_VNNI && !cpu_avxvnni()) backend = -1;
  if (backend == OR_BACKEND_AVX2 && !cpu_avx2_fma()) backend = -1;
  if (backend != OR_BACKEND_AVX_VNNI && backend != OR_BACKEND_AVX2 && backend != OR_BACKEND_SCALAR) {
    g_err = "SIMD backend is not supported by this CPU";
    if (err) *err = g_err.c_str();
    return nullptr;
  }
  or_model* m = load_mem(buf, len, backend);
  if (!m && err) *err = g_err.c_str();
  return m;
}

or_model* or_model_load(const char* path, int backend, const char** err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    g_err = std::string("cannot open ") + path;
    if (err) *err = g_err.c_str();
    return nullptr;
  }
  std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  return or_model_load_mem(bytes.data(), bytes.size(), backend, err);
}

void or_model_free(or_model* m) { delete m; }
int or_model_backend(const or_model* m) { return m->backend; }

void or_forward_cls(const or_model* m, const uint16_t* ids, uint32_t len, float* out) {
  thread_local Workspace ws;
  forward_cls(*m, ids, len, ws, out, nullptr);
}

void or_forward_trace(const or_model* m, const uint16_t* ids, uint32_t len, int8_t* gemm_in_q, float* gemm_in_s,
                      float* qkv_out, float* ctx, float* hidden, int8_t* down_in_q, float* down_in_s) {
  Workspace ws;
  Trace tr{gemm_in_q, gemm_in_s, qkv_out, ctx, hidden, down_in_q, down_in_s};
  float out[H];
  forward_cls(*m, ids, len, ws, out, &tr);
}

// The embedding rows of one sequence (dequant_add_embeddings_row, src/simd_math.rs:1827-1881, then
// the first layernorm_smooth_quantize_row with layers[0].qkv.inv_smooth, src/model.rs:196-219).
void or_embed_rows(const or_model* m, const uint16_t* ids, uint32_t len, float* hidden, int8_t* q, float* scale) {
  Workspace ws;
  const size_t L = len < MAXPOS ? len : MAXPOS;
  embed_rows(*m, ids, L, 0, ws);
  std::memcpy(hidden, ws.hidden.data(), L * H * 4);
  std::memcpy(q, ws.act_q.data(), L * H);
  std::memcpy(scale, ws.act_scale.data(), L * 4);
}

void or_forward_ragged(const or_model* m, const uint16_t* ids, const uint32_t* cu, uint32_t n, float* out) {
  thread_local Workspace ws;
  std::vector<const uint16_t*> seqs(n);
  std::vector<size_t> lens(n);
  for (uint32_t i = 0; i < n; ++i) {
    seqs[i] = ids + cu[i];
    lens[i] = cu[i + 1] - cu[i];
  }
  forward_ragged(*m, seqs.data(), lens.data(), n, ws, out);
}

// embed_batch, src/lib.rs:138-260, over pre-tokenised sequences.
void or_embed_batch(const or_model* m, const uint16_t* ids, const uint32_t* cu, uint32_t n, uint32_t threads,
                    float* out) {
  if (n == 0) return;
  threads = threads < 1 ? 1 : (threads > n ? n : threads);
  std::atomic<size_t> next{0};
  auto worker = [&]() {
    Workspace ws;
    const size_t MAX_PACK_TOKENS = 32;
    while (true) {
      const size_t i0 = next.fetch_add(1, std::memory_order_relaxed);
      if (i0 >= n) break;
      const uint16_t* s0 = ids + cu[i0];
      const size_t l0 = cu[i0 + 1] - cu[i0];
      if (l0 >= 16) {
        forward_cls(*m, s0, l0, ws, out + i0 * H, nullptr);
        continue;
      }
      size_t idx[4] = {i0, 0, 0, 0};
      const uint16_t* sp[4] = {s0, nullptr, nullptr, nullptr};
      size_t ln[4] = {l0, 0, 0, 0};
      size_t cnt = 1, tokens = l0;
      while (cnt < 4 && tokens + 12 <= MAX_PACK_TOKENS) {
        const size_t ni = next.fetch_add(1, std::memory_order_relaxed);
        if (ni >= n) break;
        const size_t nl = cu[ni + 1] - cu[ni];
        if (tokens + nl <= MAX_PACK_TOKENS) {
          idx[cnt] = ni;
          sp[cnt] = ids + cu[ni];
          ln[cnt] = nl;
          tokens += nl;
          ++cnt;
        } else {
          forward_cls(*m, ids + cu[ni], nl, ws, out + ni * H, nullptr);
          break;
        }
      }
      if (cnt == 1) {
        forward_cls(*m, s0, l0, ws, out + i0 * H, nullptr);
      } else {
        float staging[4 * H];
        forward_ragged(*m, sp, ln, cnt, ws, staging);
        for (size_t k = 0; k < cnt; ++k) std::memcpy(out + idx[k] * H, staging + k * H, H * 4);
      }
    }
  };
  if (threads == 1) {
    worker();
    return;
  }
  std::vector<std::thread> pool;
  for (uint32_t t = 0; t < threads; ++t) pool.emplace_back(worker);
  for (auto& th : pool) th.join();
}

void or_gemm(int backend, uint32_t M, uint32_t K, uint32_t N, const int8_t* a_q, const float* a_scale,
             const int8_t* w, const float* w_scale, const float* bias, const float* res, float* out,
             int32_t* acc_out) {
  Linear l;
  l.n = N;
  l.k = K;
  l.w.assign(w, w + size_t(N) * K);
  l.ws.assign(w_scale, w_scale + N);
  l.bias.assign(bias, bias + N);
  l.inv_s.assign(K, 1.0f);
  std::string err;
  if (!pack_linear(l, backend, err)) return;
  std::vector<int8_t> scratch;
  gemm(M, a_q, scratch, a_scale, l, res, out, acc_out);
}

float or_layernorm_smooth_quantize_row(float* x, const float* g, const float* b, const float* s, int8_t* q,
                                       uint32_t n) {
  return ln_sq(x, g, b, s, q, n);
}
float or_smooth_quantize_row(const float* x, const float* s, int8_t* q, uint32_t n) { return smooth_quant(x, s, q, n); }
float or_gelu_smooth_quantize_row(float* x, const float* s, int8_t* q, uint32_t n) { return gelu_quant(x, s, q, n); }
void or_layernorm_inplace_row(float* x, const float* g, const float* b, uint32_t n) { ln_inplace(x, g, b, n); }
void or_l2_normalize(float* x, uint32_t n) { l2_normalize(x, n); }
void or_attention_query(const float* q32, const float* k, const float* v, uint32_t L, float* out32) {
  std::vector<float> scores(L > 0 ? L : 1);
  attend(q32, k, v, L, scores.data(), out32);
}
int or_model_set_attention_mode(or_model* m, int mode) {
  if (mode != OR_ATTENTION_EXACT && mode != OR_ATTENTION_INT8) return -1;
  m->attn_mode = mode;
  return 0;
}
void or_attention_i8(const float* qkv, uint32_t L, float* ctx) {
  if (L > 0) attention_i8_seq(qkv, L, ctx);
}
void or_gelu_ref(const float* x, float* y, uint32_t n) {
  for (uint32_t i = 0; i < n; ++i) y[i] = g_avx2_fma ? gelu_lane(x[i]) : scalar_gelu(x[i]);
}

}  // extern "C"
