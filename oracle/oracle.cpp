// CPU oracle: restatement of the reference's CPU decode path. TEST INFRASTRUCTURE
// ONLY (parity checker and timed CPU baseline); the product never links it.
// Each function cites the reference file:line it restates (paths relative to the
// Querent-ai/realm project root).
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <vector>
#if defined(__AVX2__) && defined(__FMA__)
#include <immintrin.h>
#define OR_HAVE_AVX2 1
#endif
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

inline float bits_f32(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline uint32_t f32_bits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }

}  // namespace

extern "C" {

// half 2.7.1 f16::to_f32: exact IEEE binary16 -> binary32 widening.
float or_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  if (exp == 0) {
    if (man == 0) return bits_f32(sign);
    // subnormal: value = man * 2^-24, exact in fp32
    float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (exp == 31) return bits_f32(sign | 0x7f800000u | (man << 13));
  return bits_f32(sign | ((exp + 112) << 23) | (man << 13));
}

// IEEE binary32 -> binary16, round to nearest even (half::f16::from_f32).
uint16_t or_f32_to_f16(float f) {
  uint32_t x = f32_bits(f);
  uint32_t sign = (x >> 16) & 0x8000;
  uint32_t exp = (x >> 23) & 0xff;
  uint32_t man = x & 0x7fffff;
  if (exp == 0xff) return (uint16_t)(sign | 0x7c00 | (man ? 0x200 | (man >> 13) : 0));
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    uint32_t m = man | 0x800000;
    int shift = 14 - e;  // bits dropped
    uint32_t half_v = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (half_v & 1))) half_v++;
    return (uint16_t)(sign | half_v);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;  // may carry into exponent: correct
  return (uint16_t)h;
}

// crates/realm-core/src/quant.rs:108-122 get_scale_min_k4
void or_get_scale_min_k4(int j, const uint8_t* s, uint8_t* sc, uint8_t* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (uint8_t)((s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4));
    *m = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
}

size_t or_block_bytes(int dtype) {
  switch (dtype) {
    case OR_Q4K: return 144;
    case OR_Q6K: return 210;
    case OR_Q80: return 34;
    case OR_F32: return 4;
    case OR_F16: return 2;
  }
  return 0;
}
size_t or_block_elems(int dtype) {
  switch (dtype) {
    case OR_Q4K: case OR_Q6K: return 256;
    case OR_Q80: return 32;
    case OR_F32: case OR_F16: return 1;
  }
  return 0;
}

}  // extern "C"

namespace {

// crates/realm-core/src/quant.rs:127-187 dequantize_q4_k. Two roundings per
// element (d1*q then -m1); compiled with -ffp-contract=off so nothing fuses.
void dequant_q4k_block(const OrBlockQ4K& b, float* y) {
  const float d = or_f16_to_f32(b.d);
  const float mn = or_f16_to_f32(b.dmin);
  for (int i = 0; i < 4; ++i) {
    uint8_t sc, m;
    or_get_scale_min_k4(2 * i, b.scales, &sc, &m);
    const float d1 = d * (float)sc, m1 = mn * (float)m;
    or_get_scale_min_k4(2 * i + 1, b.scales, &sc, &m);
    const float d2 = d * (float)sc, m2 = mn * (float)m;
    for (int j = 0; j < 32; ++j) {
      const uint8_t q = b.qs[32 * i + j];
      y[64 * i + j] = d1 * (float)(q & 0xF) - m1;
      y[64 * i + 32 + j] = d2 * (float)(q >> 4) - m2;
    }
  }
}

// crates/realm-core/src/quant.rs:393-451 dequantize_q6_k: (d*sc)*q, left to right.
void dequant_q6k_block(const OrBlockQ6K& b, float* y) {
  const float d = or_f16_to_f32(b.d);
  for (int h = 0; h < 2; ++h) {
    const uint8_t* ql = b.ql + 64 * h;
    const uint8_t* qh = b.qh + 32 * h;
    const int8_t* sc = b.scales + 8 * h;
    float* out = y + 128 * h;
    for (int l = 0; l < 32; ++l) {
      const int is = l / 16;
      const int q1 = (int)((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
      const int q2 = (int)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
      const int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
      const int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
      out[l] = d * (float)sc[is] * (float)q1;
      out[l + 32] = d * (float)sc[is + 2] * (float)q2;
      out[l + 64] = d * (float)sc[is + 4] * (float)q3;
      out[l + 96] = d * (float)sc[is + 6] * (float)q4;
    }
  }
}

// crates/realm-core/src/quant.rs:371-387 dequantize_q8_0: q * d.
void dequant_q80_block(const OrBlockQ80& b, float* y) {
  const float d = or_f16_to_f32(b.d);
  for (int i = 0; i < 32; ++i) y[i] = (float)b.qs[i] * d;
}

inline float rne(float v) { return std::nearbyint(v); }  // default rounding mode: to nearest even
inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Q4_K quantiser (own design from the block definition; the reference ships
// none). Per 32-element sub-block: scale=(max-min)/15 with min<=0 clamped,
// 6-bit sub-scales relative to fp16 super-scales d=max(scale)/63,
// dmin=max(-min)/63. Every step is an IEEE op so the CUDA quantiser matches.
void quant_q4k_block(const float* x, OrBlockQ4K& b) {
  float scale[8], minv[8];
  float max_scale = 0.f, max_min = 0.f;
  for (int j = 0; j < 8; ++j) {
    float mn = x[32 * j], mx = x[32 * j];
    for (int i = 1; i < 32; ++i) {
      mn = std::min(mn, x[32 * j + i]);
      mx = std::max(mx, x[32 * j + i]);
    }
    if (mn > 0.f) mn = 0.f;
    scale[j] = (mx - mn) / 15.0f;
    minv[j] = -mn;
    max_scale = std::max(max_scale, scale[j]);
    max_min = std::max(max_min, minv[j]);
  }
  b.d = or_f32_to_f16(max_scale / 63.0f);
  b.dmin = or_f32_to_f16(max_min / 63.0f);
  const float df = or_f16_to_f32(b.d), dmf = or_f16_to_f32(b.dmin);
  uint8_t sc[8], m[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = (uint8_t)(df > 0.f ? clampi((int)rne(scale[j] / df), 0, 63) : 0);
    m[j] = (uint8_t)(dmf > 0.f ? clampi((int)rne(minv[j] / dmf), 0, 63) : 0);
  }
  for (int j = 0; j < 4; ++j) {
    b.scales[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
    b.scales[j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
    b.scales[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
  }
  uint8_t q[256];
  for (int j = 0; j < 8; ++j) {
    const float dd = df * (float)sc[j], mm = dmf * (float)m[j];
    for (int i = 0; i < 32; ++i)
      q[32 * j + i] = (uint8_t)(dd > 0.f ? clampi((int)rne((x[32 * j + i] + mm) / dd), 0, 15) : 0);
  }
  for (int i = 0; i < 4; ++i)
    for (int l = 0; l < 32; ++l)
      b.qs[32 * i + l] = (uint8_t)(q[64 * i + l] | (q[64 * i + 32 + l] << 4));
}

// Q6_K quantiser: 16 groups of 16 with signed 8-bit group scales relative to
// an fp16 super-scale d=max(amax/31)/127; values in [-32,31].
void quant_q6k_block(const float* x, OrBlockQ6K& b) {
  float s[16];
  float smax = 0.f;
  for (int g = 0; g < 16; ++g) {
    float amax = 0.f;
    for (int i = 0; i < 16; ++i) amax = std::max(amax, std::fabs(x[16 * g + i]));
    s[g] = amax / 31.0f;
    smax = std::max(smax, s[g]);
  }
  b.d = or_f32_to_f16(smax / 127.0f);
  const float df = or_f16_to_f32(b.d);
  for (int g = 0; g < 16; ++g)
    b.scales[g] = (int8_t)(df > 0.f ? clampi((int)rne(s[g] / df), -128, 127) : 0);
  uint8_t q[256];
  for (int i = 0; i < 256; ++i) {
    const float dd = df * (float)b.scales[i / 16];
    const int v = dd != 0.f ? clampi((int)rne(x[i] / dd), -32, 31) : 0;
    q[i] = (uint8_t)(v + 32);
  }
  for (int h = 0; h < 2; ++h)
    for (int l = 0; l < 32; ++l) {
      const uint8_t* qq = q + 128 * h;
      const uint8_t q1 = qq[l], q2 = qq[l + 32], q3 = qq[l + 64], q4 = qq[l + 96];
      b.ql[64 * h + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      b.ql[64 * h + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      b.qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
}

// Q8_0 quantiser: d = amax/127 (fp16), q = rne(x/d).
void quant_q80_block(const float* x, OrBlockQ80& b) {
  float amax = 0.f;
  for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[i]));
  b.d = or_f32_to_f16(amax / 127.0f);
  const float df = or_f16_to_f32(b.d);
  for (int i = 0; i < 32; ++i)
    b.qs[i] = (int8_t)(df > 0.f ? clampi((int)rne(x[i] / df), -128, 127) : 0);
}

void dequant_row(int dtype, const void* blocks, size_t row, size_t k, float* out) {
  if (dtype == OR_Q4K) {
    const OrBlockQ4K* b = (const OrBlockQ4K*)blocks + row * (k / 256);
    for (size_t i = 0; i < k / 256; ++i) dequant_q4k_block(b[i], out + 256 * i);
  } else if (dtype == OR_Q6K) {
    const OrBlockQ6K* b = (const OrBlockQ6K*)blocks + row * (k / 256);
    for (size_t i = 0; i < k / 256; ++i) dequant_q6k_block(b[i], out + 256 * i);
  } else if (dtype == OR_Q80) {
    const OrBlockQ80* b = (const OrBlockQ80*)blocks + row * (k / 32);
    for (size_t i = 0; i < k / 32; ++i) dequant_q80_block(b[i], out + 32 * i);
  } else if (dtype == OR_F32) {
    std::memcpy(out, (const float*)blocks + row * k, k * 4);
  } else if (dtype == OR_F16) {
    const uint16_t* h = (const uint16_t*)blocks + row * k;
    for (size_t i = 0; i < k; ++i) out[i] = or_f16_to_f32(h[i]);
  }
}

// ---- fused kernels, faithful lane/reduction order -------------------------

// fused.rs:35-88 q4k_accumulate_avx2 for one 8-byte chunk: lanes
// a_i = fma(fmsub(d2,qh_i,m2), xh_i, fmsub(d1,ql_i,m1)*xl_i), then
// ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)) added into the scalar accumulator.
inline void q4k_chunk(float& acc, const uint8_t* p, const float* x, float d1, float m1, float d2,
                      float m2) {
#ifdef OR_HAVE_AVX2
  const __m128i bytes = _mm_loadl_epi64((const __m128i*)p);
  const __m256i w = _mm256_cvtepu8_epi32(bytes);
  const __m256 lo = _mm256_cvtepi32_ps(_mm256_and_si256(w, _mm256_set1_epi32(0xF)));
  const __m256 hi = _mm256_cvtepi32_ps(_mm256_srli_epi32(w, 4));
  __m256 vacc = _mm256_setzero_ps();
  const __m256 dql = _mm256_fmsub_ps(_mm256_set1_ps(d1), lo, _mm256_set1_ps(m1));
  vacc = _mm256_fmadd_ps(dql, _mm256_loadu_ps(x), vacc);
  const __m256 dqh = _mm256_fmsub_ps(_mm256_set1_ps(d2), hi, _mm256_set1_ps(m2));
  vacc = _mm256_fmadd_ps(dqh, _mm256_loadu_ps(x + 32), vacc);
  const __m128 s128 = _mm_add_ps(_mm256_castps256_ps128(vacc), _mm256_extractf128_ps(vacc, 1));
  const __m128 s64 = _mm_add_ps(s128, _mm_movehl_ps(s128, s128));
  const __m128 s32 = _mm_add_ss(s64, _mm_shuffle_ps(s64, s64, 0x1));
  acc += _mm_cvtss_f32(s32);
#else
  float a[8];
  for (int i = 0; i < 8; ++i) {
    const float ql = (float)(p[i] & 0xF), qh = (float)(p[i] >> 4);
    a[i] = std::fma(std::fma(d1, ql, -m1), x[i], 0.0f);
    a[i] = std::fma(std::fma(d2, qh, -m2), x[32 + i], a[i]);
  }
  float s[4];
  for (int i = 0; i < 4; ++i) s[i] = a[i] + a[i + 4];
  acc += (s[0] + s[2]) + (s[1] + s[3]);
#endif
}

// fused.rs:229-374 fused_dequant_matmul_q4k: one output element.
float fused_q4k_elem(const OrBlockQ4K* row_blocks, size_t nb, const float* x) {
  float acc = 0.f;
  for (size_t bi = 0; bi < nb; ++bi) {
    const OrBlockQ4K& b = row_blocks[bi];
    float d = or_f16_to_f32(b.d), mn = or_f16_to_f32(b.dmin);
    if (std::isnan(d) || std::isinf(d)) d = 0.00000006f;     // fused.rs:276-280
    if (std::isnan(mn) || std::isinf(mn)) mn = 0.00000024f;  // fused.rs:281-285
    for (int g = 0; g < 4; ++g) {
      uint8_t sc, m;
      or_get_scale_min_k4(2 * g, b.scales, &sc, &m);
      const float d1 = d * (float)sc, m1 = mn * (float)m;
      or_get_scale_min_k4(2 * g + 1, b.scales, &sc, &m);
      const float d2 = d * (float)sc, m2 = mn * (float)m;
      const float* xi = x + bi * 256 + 64 * g;
      for (int c = 0; c < 4; ++c) q4k_chunk(acc, b.qs + 32 * g + 8 * c, xi + 8 * c, d1, m1, d2, m2);
    }
  }
  return acc;
}

// fused.rs:977-1022 q6k_accumulate_avx2 (4-wide): ((d*sc)*q)*x, hsum (p0+p2)+(p1+p3).
float fused_q6k_elem(const OrBlockQ6K* row_blocks, size_t nb, const float* x) {
  float acc = 0.f;
  for (size_t bi = 0; bi < nb; ++bi) {
    const OrBlockQ6K& b = row_blocks[bi];
    float d = or_f16_to_f32(b.d);
    if (std::isnan(d) || std::isinf(d)) d = 0.00000006f;  // fused.rs:1171-1175
    for (int h = 0; h < 2; ++h) {
      for (int l = 0; l < 32; ++l) {
        const int sb = 8 * h + l / 16;
        const uint8_t ql1 = b.ql[64 * h + l], ql2 = b.ql[64 * h + l + 32], qh = b.qh[32 * h + l];
        const int q[4] = {(int)((ql1 & 0x0F) | ((qh & 3) << 4)) - 32,
                          (int)((ql2 & 0x0F) | (((qh >> 2) & 3) << 4)) - 32,
                          (int)((ql1 >> 4) | (((qh >> 4) & 3) << 4)) - 32,
                          (int)((ql2 >> 4) | (((qh >> 6) & 3) << 4)) - 32};
        const float* xi = x + bi * 256 + 128 * h + l;
        float p[4];
        for (int t = 0; t < 4; ++t)
          p[t] = ((d * (float)b.scales[sb + 2 * t]) * (float)q[t]) * xi[32 * t];
        acc += (p[0] + p[2]) + (p[1] + p[3]);
      }
    }
  }
  return acc;
}

// fused.rs:1768-1804 q80_accumulate_avx2: (d*q)*x, hsum ((p0+p4)+(p2+p6))+((p1+p5)+(p3+p7)).
float fused_q80_elem(const OrBlockQ80* row_blocks, size_t nb, const float* x, size_t k) {
  float acc = 0.f;
  for (size_t bi = 0; bi < nb; ++bi) {
    const OrBlockQ80& b = row_blocks[bi];
    const float d = or_f16_to_f32(b.d);  // no NaN guard in this kernel (fused.rs:2497-2499)
    const size_t k0 = bi * 32;
    const size_t bs = std::min<size_t>(32, k - k0);
    size_t i = 0;
    for (; i + 8 <= bs; i += 8) {
      float p[8];
      for (int t = 0; t < 8; ++t) p[t] = (d * (float)b.qs[i + t]) * x[k0 + i + t];
      acc += ((p[0] + p[4]) + (p[2] + p[6])) + ((p[1] + p[5]) + (p[3] + p[7]));
    }
    for (; i < bs; ++i) acc += ((float)b.qs[i] * d) * x[k0 + i];
  }
  return acc;
}

int set_threads(int threads) {
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
  return threads;
#else
  (void)threads;
  return 1;
#endif
}

}  // namespace

extern "C" {

int or_dequant(int dtype, const void* blocks, size_t nblocks, float* out) {
  for (size_t i = 0; i < nblocks; ++i) {
    if (dtype == OR_Q4K) dequant_q4k_block(((const OrBlockQ4K*)blocks)[i], out + 256 * i);
    else if (dtype == OR_Q6K) dequant_q6k_block(((const OrBlockQ6K*)blocks)[i], out + 256 * i);
    else if (dtype == OR_Q80) dequant_q80_block(((const OrBlockQ80*)blocks)[i], out + 32 * i);
    else return -23;
  }
  return (int)0;
}

int or_quantize(int dtype, const float* x, size_t n, void* out) {
  const size_t be = or_block_elems(dtype);
  if (be == 0 || n % be) return -23;
  const long nb = (long)(n / be);
#pragma omp parallel for schedule(static)
  for (long i = 0; i < nb; ++i) {
    if (dtype == OR_Q4K) quant_q4k_block(x + 256 * i, ((OrBlockQ4K*)out)[i]);
    else if (dtype == OR_Q6K) quant_q6k_block(x + 256 * i, ((OrBlockQ6K*)out)[i]);
    else if (dtype == OR_Q80) quant_q80_block(x + 32 * i, ((OrBlockQ80*)out)[i]);
  }
  return 0;
}

// Validation mirrors fused.rs:238-254 (Q4_K), the same lines for Q6_K, and
// fused.rs:2459-2482 (Q8_0: block count (n*k).div_ceil(32), input and output sizes).
int or_fused_matmul(int dtype, const void* blocks, size_t nblocks, const float* x, float* y,
                    size_t m, size_t n, size_t k, int threads) {
  if (dtype == OR_Q4K || dtype == OR_Q6K) {
    if (k % 256) return -23;
    if (nblocks != n * (k / 256)) return -3;
  } else if (dtype == OR_Q80) {
    if (nblocks != (n * k + 31) / 32) return -3;
  } else {
    return -23;
  }
  threads = set_threads(threads);
  const long N = (long)n;
#pragma omp parallel for schedule(static) num_threads(threads) if (threads > 1)
  for (long o = 0; o < N; ++o) {
    for (size_t b = 0; b < m; ++b) {
      const float* xr = x + b * k;
      float v;
      if (dtype == OR_Q4K) v = fused_q4k_elem((const OrBlockQ4K*)blocks + o * (k / 256), k / 256, xr);
      else if (dtype == OR_Q6K) v = fused_q6k_elem((const OrBlockQ6K*)blocks + o * (k / 256), k / 256, xr);
      else v = fused_q80_elem((const OrBlockQ80*)blocks + o * ((k + 31) / 32), (k + 31) / 32, xr, k);
      y[b * n + o] = v;
    }
  }
  return (int)(m * n);
}

int or_dequant_matmul(int dtype, const void* blocks, size_t nblocks, const float* x, float* y,
                      size_t m, size_t n, size_t k, int threads) {
  const size_t be = or_block_elems(dtype);
  if (be == 0 || k % be || nblocks != n * (k / be)) return -3;
  threads = set_threads(threads);
  // Each y[b, o] is the sequential sum s += w[i] * x[i] over i = 0..k-1 (product
  // and sum rounded separately). Eight output rows are carried side by side in
  // one vector (w transposed to [k][8]) and four tokens at a time, which only
  // interleaves independent sums: every element gets exactly the scalar result.
  const long NG = (long)((n + 7) / 8);
#pragma omp parallel num_threads(threads) if (threads > 1)
  {
    std::vector<float> w(8 * k), wt(8 * k);
#pragma omp for schedule(static)
    for (long gi = 0; gi < NG; ++gi) {
      const size_t o0 = (size_t)gi * 8, nr = std::min<size_t>(8, n - o0);
      for (size_t r = 0; r < 8; ++r) {
        if (r < nr) dequant_row(dtype, blocks, o0 + r, k, w.data() + r * k);
        else std::fill(w.begin() + r * k, w.begin() + (r + 1) * k, 0.f);
      }
      for (size_t i = 0; i < k; ++i)
        for (size_t r = 0; r < 8; ++r) wt[i * 8 + r] = w[r * k + i];
      size_t b = 0;
#ifdef OR_HAVE_AVX2
      for (; b + 4 <= m; b += 4) {
        __m256 s0 = _mm256_setzero_ps(), s1 = s0, s2 = s0, s3 = s0;
        const float *x0 = x + b * k, *x1 = x0 + k, *x2 = x1 + k, *x3 = x2 + k;
        for (size_t i = 0; i < k; ++i) {
          const __m256 wv = _mm256_loadu_ps(wt.data() + i * 8);
          s0 = _mm256_add_ps(s0, _mm256_mul_ps(wv, _mm256_set1_ps(x0[i])));
          s1 = _mm256_add_ps(s1, _mm256_mul_ps(wv, _mm256_set1_ps(x1[i])));
          s2 = _mm256_add_ps(s2, _mm256_mul_ps(wv, _mm256_set1_ps(x2[i])));
          s3 = _mm256_add_ps(s3, _mm256_mul_ps(wv, _mm256_set1_ps(x3[i])));
        }
        float o[4][8];
        _mm256_storeu_ps(o[0], s0);
        _mm256_storeu_ps(o[1], s1);
        _mm256_storeu_ps(o[2], s2);
        _mm256_storeu_ps(o[3], s3);
        for (size_t t = 0; t < 4; ++t)
          for (size_t r = 0; r < nr; ++r) y[(b + t) * n + o0 + r] = o[t][r];
      }
      for (; b < m; ++b) {
        __m256 s = _mm256_setzero_ps();
        const float* xr = x + b * k;
        for (size_t i = 0; i < k; ++i)
          s = _mm256_add_ps(s, _mm256_mul_ps(_mm256_loadu_ps(wt.data() + i * 8), _mm256_set1_ps(xr[i])));
        float o[8];
        _mm256_storeu_ps(o, s);
        for (size_t r = 0; r < nr; ++r) y[b * n + o0 + r] = o[r];
      }
#else
      for (; b < m; ++b) {
        const float* xr = x + b * k;
        for (size_t r = 0; r < nr; ++r) {
          float s = 0.f;
          for (size_t i = 0; i < k; ++i) s += wt[i * 8 + r] * xr[i];
          y[b * n + o0 + r] = s;
        }
      }
#endif
    }
  }
  return (int)(m * n);
}

// The plain row-at-a-time form of or_dequant_matmul (one sequential sum per
// output element); kept to check that the vectorised form gives the same bits.
int or_dequant_matmul_scalar(int dtype, const void* blocks, size_t nblocks, const float* x, float* y,
                             size_t m, size_t n, size_t k, int threads) {
  const size_t be = or_block_elems(dtype);
  if (be == 0 || k % be || nblocks != n * (k / be)) return -3;
  threads = set_threads(threads);
  const long N = (long)n;
#pragma omp parallel num_threads(threads) if (threads > 1)
  {
    std::vector<float> w(k);
#pragma omp for schedule(static)
    for (long o = 0; o < N; ++o) {
      dequant_row(dtype, blocks, (size_t)o, k, w.data());
      for (size_t b = 0; b < m; ++b) {
        const float* xr = x + b * k;
        float s = 0.f;
        for (size_t i = 0; i < k; ++i) s += w[i] * xr[i];
        y[b * n + o] = s;
      }
    }
  }
  return (int)(m * n);
}

int or_dequant_matmul_f64(int dtype, const void* blocks, size_t nblocks, const float* x, double* y,
                          size_t m, size_t n, size_t k, int threads) {
  const size_t be = or_block_elems(dtype);
  if (be == 0 || k % be || nblocks != n * (k / be)) return -3;
  threads = set_threads(threads);
  const long N = (long)n;
#pragma omp parallel num_threads(threads) if (threads > 1)
  {
    std::vector<float> w(k);
#pragma omp for schedule(static)
    for (long o = 0; o < N; ++o) {
      dequant_row(dtype, blocks, (size_t)o, k, w.data());
      for (size_t b = 0; b < m; ++b) {
        const float* xr = x + b * k;
        double s = 0.0;
        for (size_t i = 0; i < k; ++i) s += (double)w[i] * (double)xr[i];
        y[b * n + o] = s;
      }
    }
  }
  return (int)(m * n);
}

// candle-nn 0.9.1 ops::rms_norm as called from
// crates/realm-compute-cpu/src/candle_neural_ops_backend.rs:32-59:
// y = x / sqrt(mean(x^2) + eps) * w, fp32, sequential sum.
void or_rms_norm(const float* x, const float* w, float eps, size_t rows, size_t h, float* y) {
  for (size_t r = 0; r < rows; ++r) {
    const float* xr = x + r * h;
    float s = 0.f;
    for (size_t i = 0; i < h; ++i) s += xr[i] * xr[i];
    const float m = std::sqrt(s / (float)h + eps);
    for (size_t i = 0; i < h; ++i) y[r * h + i] = xr[i] / m * w[i];
  }
}

// crates/realm-models/src/attention.rs:171-240 apply_rope: adjacent pairs,
// freq = 1/theta^(i/hd) for even i, angle = pos*freq.
void or_rope(float* t, size_t start_pos, size_t seq_len, size_t n_heads, size_t hd, float theta) {
  for (size_t s = 0; s < seq_len; ++s) {
    const float pos = (float)(start_pos + s);
    for (size_t h = 0; h < n_heads; ++h) {
      float* base = t + (s * n_heads + h) * hd;
      for (size_t i = 0; i < hd; i += 2) {
        const float freq = 1.0f / std::pow(theta, (float)i / (float)hd);
        const float angle = pos * freq;
        const float c = std::cos(angle), sn = std::sin(angle);
        const float x0 = base[i], x1 = base[i + 1];
        base[i] = x0 * c - x1 * sn;
        base[i + 1] = x0 * sn + x1 * c;
      }
    }
  }
}

// attention.rs:310-380 (repeat_kv, causal mask j > position+i) and
// attention_stub/mod.rs:42-158 (StandardAttention). Layouts [S, heads, hd].
void or_attention(const float* q, const float* k, const float* v, size_t seq_len, size_t kv_len,
                  size_t position, size_t n_heads, size_t n_kv, size_t hd, float* out) {
  const size_t n_rep = n_heads / n_kv;
  const float scale = 1.0f / std::sqrt((float)hd);
  std::vector<float> sc(kv_len);
  for (size_t h = 0; h < n_heads; ++h) {
    const size_t kh = h / n_rep;
    for (size_t i = 0; i < seq_len; ++i) {
      const float* qi = q + (i * n_heads + h) * hd;
      for (size_t j = 0; j < kv_len; ++j) {
        const float* kj = k + (j * n_kv + kh) * hd;
        float dot = 0.f;
        for (size_t d = 0; d < hd; ++d) dot += qi[d] * kj[d];
        sc[j] = dot * scale;
        if (j > position + i) sc[j] = -std::numeric_limits<float>::infinity();
      }
      float mx = -std::numeric_limits<float>::infinity();
      for (size_t j = 0; j < kv_len; ++j) mx = std::max(mx, sc[j]);
      float sum = 0.f;
      for (size_t j = 0; j < kv_len; ++j) {
        if (std::isfinite(sc[j])) {
          sc[j] = std::exp(sc[j] - mx);
          sum += sc[j];
        } else {
          sc[j] = 0.f;
        }
      }
      if (sum > 0.f)
        for (size_t j = 0; j < kv_len; ++j) sc[j] /= sum;
      float* o = out + (i * n_heads + h) * hd;
      for (size_t d = 0; d < hd; ++d) {
        float s = 0.f;
        for (size_t j = 0; j < kv_len; ++j) s += sc[j] * v[(j * n_kv + kh) * hd + d];
        o[d] = s;
      }
    }
  }
}

}  // extern "C"

namespace {

// crates/realm-models/src/kv_cache.rs:7-80
struct KV {
  size_t max_seq, n_kv, hd, cur = 0;
  bool fp16;
  std::vector<float> k, v;
  KV(size_t ms, size_t nk, size_t h, bool f) : max_seq(ms), n_kv(nk), hd(h), fp16(f), k(ms * nk * h), v(ms * nk * h) {}
  int append(const float* kk, const float* vv, size_t nf) {
    const size_t row = n_kv * hd;
    const size_t s = nf / row;
    if (cur + s > max_seq) return -22;  // kv_cache.rs:48-53 overflow
    for (size_t i = 0; i < nf; ++i) {
      float a = kk[i], b = vv[i];
      if (fp16) { a = or_f16_to_f32(or_f32_to_f16(a)); b = or_f16_to_f32(or_f32_to_f16(b)); }
      k[cur * row + i] = a;
      v[cur * row + i] = b;
    }
    cur += s;
    return (int)s;
  }
};

struct Tensor {
  int dtype = OR_F32;
  std::vector<uint8_t> data;
};

struct Layer {
  Tensor attn_norm, wq, wk, wv, wo, ffn_norm, gate, up, down;
};

struct Model {
  OrModelConfig cfg;
  Tensor embd, out_norm, out;
  std::vector<Layer> layers;
  std::vector<KV> kv;
  std::vector<float> last_hidden;
};

// y[s, n] = x[s, :] . W[n, :] with W dequantised row by row (CandleCpuBackend
// fused_* semantics, candle_cpu_backend.rs:92-114; the host path reaches it via
// dispatch_matmul, matmul_dispatch.rs:47-283).
void mm(const Tensor& w, const float* x, size_t s, size_t k, size_t n, float* y, int threads) {
  const size_t be = or_block_elems(w.dtype);
  const size_t nb = n * k / be;
  or_dequant_matmul(w.dtype, w.data.data(), nb, x, y, s, n, k, threads);
}

const float* fptr(const Tensor& t) { return (const float*)t.data.data(); }

// crates/realm-models/src/layer.rs:37-94 with the host path's config eps
// (crates/realm-runtime/src/memory64_host.rs:2069, 2337), attention.rs:79-162, ffn.rs:57-115.
std::vector<float> layer_forward(Model& M, size_t l, const std::vector<float>& x, size_t S, size_t pos) {
  const OrModelConfig& c = M.cfg;
  const size_t H = c.hidden, hd = c.head_dim, nh = c.n_heads, nk = c.n_kv_heads, F = c.ffn;
  Layer& L = M.layers[l];
  std::vector<float> normed(S * H), q(S * nh * hd), k(S * nk * hd), v(S * nk * hd);
  or_rms_norm(x.data(), fptr(L.attn_norm), c.layer_eps, S, H, normed.data());
  mm(L.wq, normed.data(), S, H, nh * hd, q.data(), c.threads);
  mm(L.wk, normed.data(), S, H, nk * hd, k.data(), c.threads);
  mm(L.wv, normed.data(), S, H, nk * hd, v.data(), c.threads);
  or_rope(q.data(), pos, S, nh, hd, c.rope_theta);
  or_rope(k.data(), pos, S, nk, hd, c.rope_theta);
  M.kv[l].append(k.data(), v.data(), k.size());
  const size_t kvl = M.kv[l].cur;
  std::vector<float> att(S * nh * hd), o(S * H);
  or_attention(q.data(), M.kv[l].k.data(), M.kv[l].v.data(), S, kvl, pos, nh, nk, hd, att.data());
  mm(L.wo, att.data(), S, nh * hd, H, o.data(), c.threads);
  std::vector<float> h(S * H);
  for (size_t i = 0; i < S * H; ++i) h[i] = x[i] + o[i];
  or_rms_norm(h.data(), fptr(L.ffn_norm), c.layer_eps, S, H, normed.data());
  std::vector<float> g(S * F), u(S * F), dn(S * H);
  mm(L.gate, normed.data(), S, H, F, g.data(), c.threads);
  mm(L.up, normed.data(), S, H, F, u.data(), c.threads);
  for (size_t i = 0; i < S * F; ++i) {
    const float sig = 1.0f / (1.0f + std::exp(-g[i]));
    const float silu = g[i] * sig;
    g[i] = silu * u[i];
  }
  mm(L.down, g.data(), S, F, H, dn.data(), c.threads);
  std::vector<float> out(S * H);
  for (size_t i = 0; i < S * H; ++i) out[i] = h[i] + dn[i];
  return out;
}

}  // namespace

extern "C" {

void* or_kv_new(size_t max_seq, size_t n_kv, size_t hd, int kv_fp16) { return new KV(max_seq, n_kv, hd, kv_fp16 != 0); }
void or_kv_free(void* kv) { delete (KV*)kv; }
int or_kv_append(void* kv, const float* k, const float* v, size_t n) { return ((KV*)kv)->append(k, v, n); }
size_t or_kv_len(void* kv) { return ((KV*)kv)->cur; }
void or_kv_data(void* kv, float* ko, float* vo) {
  KV* p = (KV*)kv;
  const size_t n = p->cur * p->n_kv * p->hd;
  std::memcpy(ko, p->k.data(), n * 4);
  std::memcpy(vo, p->v.data(), n * 4);
}
// kv_cache.rs:36-40 clear
void or_kv_clear(void* kv) {
  KV* p = (KV*)kv;
  std::fill(p->k.begin(), p->k.end(), 0.f);
  std::fill(p->v.begin(), p->v.end(), 0.f);
  p->cur = 0;
}

void* or_model_new(const OrModelConfig* cfg) {
  Model* m = new Model();
  m->cfg = *cfg;
  m->layers.resize(cfg->n_layers);
  for (int i = 0; i < cfg->n_layers; ++i) m->kv.emplace_back(cfg->max_seq, cfg->n_kv_heads, cfg->head_dim, cfg->kv_fp16 != 0);
  return m;
}
void or_model_free(void* model) { delete (Model*)model; }

int or_model_set_weight(void* model, int which, int layer, int dtype, const void* data, size_t nbytes) {
  Model* m = (Model*)model;
  Tensor* t = nullptr;
  if (which == OR_W_TOKEN_EMBD) t = &m->embd;
  else if (which == OR_W_OUTPUT_NORM) t = &m->out_norm;
  else if (which == OR_W_OUTPUT) t = &m->out;
  else {
    if (layer < 0 || layer >= m->cfg.n_layers) return -2;
    Layer& L = m->layers[layer];
    switch (which) {
      case OR_W_ATTN_NORM: t = &L.attn_norm; break;
      case OR_W_Q: t = &L.wq; break;
      case OR_W_K: t = &L.wk; break;
      case OR_W_V: t = &L.wv; break;
      case OR_W_O: t = &L.wo; break;
      case OR_W_FFN_NORM: t = &L.ffn_norm; break;
      case OR_W_GATE: t = &L.gate; break;
      case OR_W_UP: t = &L.up; break;
      case OR_W_DOWN: t = &L.down; break;
      default: return -2;
    }
  }
  t->dtype = dtype;
  t->data.assign((const uint8_t*)data, (const uint8_t*)data + nbytes);
  return (int)nbytes;
}

// crates/realm-models/src/model.rs:572-625
int or_model_forward(void* model, const uint32_t* tokens, size_t n, size_t position, float* logits) {
  Model& M = *(Model*)model;
  const OrModelConfig& c = M.cfg;
  const size_t H = c.hidden;
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] >= (uint32_t)c.vocab) return -3;
  if (M.kv[0].cur + n > (size_t)c.max_seq) return -22;
  std::vector<float> x(n * H);
  for (size_t i = 0; i < n; ++i) dequant_row(M.embd.dtype, M.embd.data.data(), tokens[i], H, x.data() + i * H);
  for (int l = 0; l < c.n_layers; ++l) x = layer_forward(M, (size_t)l, x, n, position);
  std::vector<float> xn(n * H);
  or_rms_norm(x.data(), fptr(M.out_norm), c.rms_eps, n, H, xn.data());
  M.last_hidden.assign(xn.end() - H, xn.end());
  mm(M.out, M.last_hidden.data(), 1, H, c.vocab, logits, c.threads);
  return c.vocab;
}

int or_model_last_hidden(void* model, float* out) {
  Model& M = *(Model*)model;
  std::copy(M.last_hidden.begin(), M.last_hidden.end(), out);
  return (int)M.last_hidden.size();
}

void or_model_clear_kv(void* model) {
  Model& M = *(Model*)model;
  for (auto& k : M.kv) or_kv_clear(&k);
}
// Benchmark helper: reset every layer's cache to n rows of N(0,1) K/V so a
// decode step can be timed at a given context length without a prefill.
int or_model_kv_fill(void* model, size_t n, uint64_t seed) {
  Model& M = *(Model*)model;
  const size_t row = (size_t)M.cfg.n_kv_heads * M.cfg.head_dim;
  if (n > (size_t)M.cfg.max_seq) return -22;
  std::vector<float> k(n * row), v(n * row);
  uint64_t s = seed * 0x9E3779B97F4A7C15ull + 1;
  auto uni = [&]() { s ^= s << 13; s ^= s >> 7; s ^= s << 17; return (float)((s >> 11) * (1.0 / 9007199254740992.0)); };
  for (auto& kv : M.kv) {
    or_kv_clear(&kv);
    for (size_t i = 0; i < n * row; ++i) {
      k[i] = uni() * 2.f - 1.f;
      v[i] = uni() * 2.f - 1.f;
    }
    kv.append(k.data(), v.data(), n * row);
  }
  return (int)n;
}

size_t or_model_kv_len(void* model, int layer) { return ((Model*)model)->kv[layer].cur; }
void or_model_kv_data(void* model, int layer, float* ko, float* vo) { or_kv_data(&((Model*)model)->kv[layer], ko, vo); }

uint32_t or_argmax(const float* x, size_t n) {
  size_t best = 0;
  for (size_t i = 1; i < n; ++i)
    if (!(x[i] < x[best])) best = i;  // ties go to the later index
  return (uint32_t)best;
}

// model.rs:749-847 (greedy, repetition_penalty 1.0, 8-token prefill chunks).
int or_model_generate(void* model, const uint32_t* prompt, size_t n_prompt, size_t n_gen,
                      uint32_t* out_tokens, float* step_logits) {
  Model& M = *(Model*)model;
  const size_t V = M.cfg.vocab;
  or_model_clear_kv(model);
  std::vector<float> logits(V);
  for (size_t cs = 0; cs < n_prompt; cs += 8) {
    const size_t ce = std::min(n_prompt, cs + 8);
    int r = or_model_forward(model, prompt + cs, ce - cs, cs, logits.data());
    if (r < 0) return r;
  }
  for (size_t g = 0; g < n_gen; ++g) {
    if (g > 0) {
      const uint32_t last = out_tokens[g - 1];
      int r = or_model_forward(model, &last, 1, M.kv[0].cur, logits.data());
      if (r < 0) return r;
    }
    if (step_logits) std::copy(logits.begin(), logits.end(), step_logits + g * V);
    out_tokens[g] = or_argmax(logits.data(), V);
  }
  return (int)n_gen;
}

}  // extern "C"
// ---- sampling (crates/realm-models/src/sampling.rs) ----
namespace {

// rand 0.8.5 WeightedIndex<f32>::new + sample with the uniform draw supplied:
// cumulative weights w0, w0+w1, ... (sequential f32 sums, the last excluded),
// total = the full sum; Uniform<f32>::new(0, total) shrinks its scale until
// scale * (1 - 2^-23) < total; chosen = u * scale; the index is the number of
// cumulative weights <= chosen. Err on a negative / NaN weight or a zero total.
int weighted_index(const std::vector<float>& w, float u, uint32_t* out) {
  if (w.empty() || !(w[0] >= 0.f)) return -1;
  std::vector<float> cum;
  cum.reserve(w.size());
  float total = w[0];
  for (size_t i = 1; i < w.size(); ++i) {
    if (!(w[i] >= 0.f)) return -1;
    cum.push_back(total);
    total += w[i];
  }
  if (!(total > 0.f) || !std::isfinite(total)) return -1;
  const float max_rand = 1.0f - 1.1920928955078125e-07f;
  float scale = total;
  while (scale * max_rand >= total) scale = std::nextafter(scale, 0.0f);
  const float chosen = u * scale;
  *out = (uint32_t)(std::partition_point(cum.begin(), cum.end(), [&](float c) { return c <= chosen; }) - cum.begin());
  return 0;
}

// compute_probabilities (sampling.rs:125-137): x / (temperature as f32), then a
// softmax with sequential f32 sums.
std::vector<float> probabilities(const float* logits, size_t n, double temperature) {
  const float t = (float)temperature;
  std::vector<float> s(n);
  float mx = -std::numeric_limits<float>::infinity();
  for (size_t i = 0; i < n; ++i) {
    s[i] = logits[i] / t;
    mx = std::max(mx, s[i]);
  }
  float sum = 0.f;
  for (size_t i = 0; i < n; ++i) sum += std::exp(s[i] - mx);
  for (size_t i = 0; i < n; ++i) s[i] = std::exp(s[i] - mx) / sum;
  return s;
}

void renormalize(std::vector<float>& p) {
  float sum = 0.f;
  for (float v : p) sum += v;
  if (sum > 0.f)
    for (float& v : p) v /= sum;
}

// top-k (sampling.rs:194-216): keep the k largest (ties go to the lower index;
// the reference's unstable selection leaves them unspecified), zero the rest.
void keep_top_k(std::vector<float>& p, size_t k) {
  std::vector<uint32_t> idx(p.size());
  for (size_t i = 0; i < p.size(); ++i) idx[i] = (uint32_t)i;
  std::stable_sort(idx.begin(), idx.end(), [&](uint32_t a, uint32_t b) { return p[a] > p[b]; });
  for (size_t r = k; r < idx.size(); ++r) p[idx[r]] = 0.f;
  renormalize(p);
}

// top-p (sampling.rs:162-188): stable descending sort; a token is zeroed once the
// running f32 sum of the tokens before it has reached top_p.
void keep_top_p(std::vector<float>& p, float top_p) {
  std::vector<uint32_t> idx(p.size());
  for (size_t i = 0; i < p.size(); ++i) idx[i] = (uint32_t)i;
  std::stable_sort(idx.begin(), idx.end(), [&](uint32_t a, uint32_t b) { return p[a] > p[b]; });
  float cum = 0.f;
  for (uint32_t i : idx) {
    if (cum >= top_p) p[i] = 0.f;
    else cum += p[i];
  }
  renormalize(p);
}

}  // namespace

extern "C" {

int or_sample(float* logits, size_t n, double temperature, double top_p, size_t top_k, float penalty,
              const uint32_t* prev, size_t n_prev, float u, uint32_t* out) {
  // apply_repetition_penalty (sampling.rs:107-122): once per occurrence
  if (penalty != 1.0f)
    for (size_t j = 0; j < n_prev; ++j) {
      const size_t i = prev[j];
      if (i < n) logits[i] = logits[i] > 0.f ? logits[i] / penalty : logits[i] * penalty;
    }
  // with_params (sampling.rs:63-100) picks the strategy; sample (:250-290) runs it
  if (temperature < 1e-7) {
    *out = or_argmax(logits, n);
    return 0;
  }
  std::vector<float> p = probabilities(logits, n, temperature);
  if (top_k > 0 && top_k < n) keep_top_k(p, top_k);
  if (top_p > 0.0 && top_p < 1.0) keep_top_p(p, (float)top_p);
  return weighted_index(p, u, out);
}

}  // extern "C"
