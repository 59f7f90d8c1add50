// Activation fragments: the form in which every GEMV reads its input.
//
// A GEMV input x[M][K] (fp32, already multiplied by the consumer's RMSNorm
// weight when one is fused) is stored pre-arranged in tensor-core B-fragment
// order, so the GEMV copies it with the bulk-copy engine and feeds the tensor
// cores without conversion work. Producers (embedding, the residual / SwiGLU
// epilogues, the attention kernel, or xfrag_launch for plain inputs) write it
// once. Two encodings are kept side by side:
//
//  fp16 hi/lo (m16n8k16 .f16, read by the Q6_K and Q8_0 GEMVs and the tcgen05
//   GEMM): x ~= 256 * hi + lo with hi = fp16(x / 256), lo = fp16(x - 256 hi),
//   ~22 significant bits for |x| >= 2^-3 (lo stays a normal fp16 number) and
//   no overflow below |x| ~ 1.6e7 (SwiGLU outputs of outlier channels exceed the
//   fp16 range). Consumers weight the hi products by 256.
//   XF: uint4 [K/256][NT][16 k-steps][32 lanes]   (NT = ceil(M/8) n-tiles)
//       lane l: token 8*nt + l/4, columns c = 16*ks + 2*(l%4) (+1, +8, +9):
//       {hi(c, c+1), hi(c+8, c+9), lo(c, c+1), lo(c+8, c+9)} as half2.
//
//  int8 three-limb (m16n8k32 .s8, read by the Q4_K GEMV): per token and 64-column
//   group, s = max|x| / 127, x ~= s * (x1 + x2 / 256 + x3 / 65536) with x1, x2, x3
//   in [-127, 127] (error <= s / 131072, i.e. 2^-24 of the group maximum; two
//   limbs alone leave 2^-16, too coarse for the logits bound at 4096-wide layers).
//   XI: uint4 [K/256][NT][8 sub-blocks][32 lanes]: lane l: token 8*nt + l/4,
//       columns c = 32*j + 4*(l%4) + 0..3 and c + 16 + 0..3:
//       {x1[c..c+3], x1[c+16..c+19], x2[c..c+3], x2[c+16..c+19]} as int8x4.
//   X3: uint2 [K/256][NT][8 sub-blocks][32 lanes]: {x3[c..c+3], x3[c+16..c+19]}.
//   XC: float [K/256][NT][4 groups][8 tokens]  the scale s.
//
//  XS: uint32 [K/256][NT][8 tokens][8 sub-blocks] half2(hi, lo) of the sum of
//      the 32 values of each 32-column sub-block (the Q4_K min term), split as
//      the XF values are (sum ~= 256 hi + lo).
#pragma once
#include "common.cuh"

namespace rb {

constexpr int kXfSbBytes = 16 * 32 * 16;  // fp16 hi/lo: one n-tile of one 256-column super-block
constexpr float kXfHiScale = 1.0f / 256.0f;  // hi parts hold x / 256 (consumers weight them by 256)
constexpr int kXiSbBytes = 8 * 32 * 16;   // int8 limbs 1 and 2
constexpr int kX3SbBytes = 8 * 32 * 8;    // int8 limb 3
constexpr int kXcSbBytes = 8 * 4 * 4;     // limb scales
constexpr int kXsSbBytes = 8 * 8 * 4;     // sub-block sums

__host__ __device__ inline size_t xf_bytes(int k, int nt) { return (size_t)(k / 256) * nt * kXfSbBytes; }
__host__ __device__ inline size_t xi_bytes(int k, int nt) { return (size_t)(k / 256) * nt * kXiSbBytes; }
__host__ __device__ inline size_t x3_bytes(int k, int nt) { return (size_t)(k / 256) * nt * kX3SbBytes; }
__host__ __device__ inline size_t xc_bytes(int k, int nt) { return (size_t)(k / 256) * nt * kXcSbBytes; }
__host__ __device__ inline size_t xs_bytes(int k, int nt) { return (size_t)(k / 256) * nt * kXsSbBytes; }

// One buffer set for a GEMV input (every encoding).
struct XFrags {
  uint4* xf = nullptr;
  uint4* xi = nullptr;
  uint2* x3 = nullptr;  // third limb (written whenever xi is)
  float* xc = nullptr;
  uint32_t* xs = nullptr;
};

__device__ __forceinline__ uint32_t pack2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Four values of token t at columns k, k+1, k+8, k+9 (k = 16*ks + 2*c, ks/c local
// to the super-block `sb`) -> one fp16 B-fragment entry.
// x ~= 256 * hi + lo (see above), two values at a time
__device__ __forceinline__ void split_hi256(float x0, float x1, __half2& hi, __half2& lo) {
  hi = __floats2half2_rn(x0 * kXfHiScale, x1 * kXfHiScale);
  const float2 f = __half22float2(hi);
  lo = __floats2half2_rn(fmaf(-256.0f, f.x, x0), fmaf(-256.0f, f.y, x1));
}

// Four values of token t at columns k, k+1, k+8, k+9 (k = 16*ks + 2*c, ks/c local
// to the super-block `sb`) -> one fp16 B-fragment entry.
__device__ __forceinline__ void xf_put(uint4* xf, int nt_total, int t, int sb, int ks, int c, float v0, float v1,
                                       float v2, float v3) {
  __half2 h01, h23, l01, l23;
  split_hi256(v0, v1, h01, l01);
  split_hi256(v2, v3, h23, l23);
  uint4 o;
  o.x = *reinterpret_cast<const uint32_t*>(&h01);
  o.y = *reinterpret_cast<const uint32_t*>(&h23);
  o.z = *reinterpret_cast<const uint32_t*>(&l01);
  o.w = *reinterpret_cast<const uint32_t*>(&l23);
  xf[(((size_t)sb * nt_total + (t >> 3)) * 16 + ks) * 32 + (t & 7) * 4 + c] = o;
}

// Sum of the 32 values of sub-block j (0..7) of super-block sb for token t.
__device__ __forceinline__ void xs_put(uint32_t* xs, int nt_total, int t, int sb, int j, float s) {
  const __half hi = __float2half_rn(s * kXfHiScale);
  const __half lo = __float2half_rn(fmaf(-256.0f, __half2float(hi), s));
  xs[(((size_t)sb * nt_total + (t >> 3)) * 8 + (t & 7)) * 8 + j] = pack2(hi, lo);
}

// int8 limbs of 8 values (columns c..c+3 and c+16..c+19 of sub-block j) with scale s:
// x1 = rn(x / s), x2 = rn(256 r1 / s), x3 = rn(65536 r2 / s) with the residuals
// r1 = x - s x1 and r2 = r1 - (s / 256) x2 taken by fused multiply-add.
__device__ __forceinline__ void xi_put(uint4* xi, uint2* x3, int nt_total, int t, int sb, int j, int c,
                                       const float v[8], float s) {
  uint32_t w1[2] = {0u, 0u}, w2[2] = {0u, 0u}, w3[2] = {0u, 0u};
  if (s > 0.f) {
    const float inv = 1.0f / s, s2 = s * (1.0f / 256.0f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float q1 = fminf(fmaxf(rintf(v[i] * inv), -127.f), 127.f);
      const float r1 = fmaf(-q1, s, v[i]);
      const float q2 = fminf(fmaxf(rintf(r1 * inv * 256.0f), -127.f), 127.f);
      const float r2 = fmaf(-q2, s2, r1);
      const float q3 = fminf(fmaxf(rintf(r2 * inv * 65536.0f), -127.f), 127.f);
      w1[i >> 2] |= ((uint32_t)(int)q1 & 0xffu) << (8 * (i & 3));
      w2[i >> 2] |= ((uint32_t)(int)q2 & 0xffu) << (8 * (i & 3));
      w3[i >> 2] |= ((uint32_t)(int)q3 & 0xffu) << (8 * (i & 3));
    }
  }
  const size_t idx = (((size_t)sb * nt_total + (t >> 3)) * 8 + j) * 32 + (t & 7) * 4 + c;
  xi[idx] = make_uint4(w1[0], w1[1], w2[0], w2[1]);
  x3[idx] = make_uint2(w3[0], w3[1]);
}

__device__ __forceinline__ void xc_put(float* xc, int nt_total, int t, int sb, int grp, float s) {
  xc[(((size_t)sb * nt_total + (t >> 3)) * 4 + grp) * 8 + (t & 7)] = s;
}

// Writes every encoding of the block of values val(k, t) = T[k*sk + t*st] * (w ? w[k_base+k] : 1)
// for local columns k in [0, nk) (global column k_base + k; nk and k_base
// multiples of 64) and local tokens t in [0, ntok) (global token t_base + t).
// Every thread of the calling group (ids tid < nthreads, whole warps) must
// call it; `sync()` is a barrier among them; scratch holds >= ntok * nk / 64
// floats of shared memory. Group maxima and sub-block sums are reduced one
// warp per (group, token) with shuffles in a fixed order (deterministic).
template <class Sync>
__device__ void frags_write(const float* T, int sk, int st, int nk, int ntok, int k_base, int t_base,
                            const float* w, const XFrags& out, int nt_total, float* scratch, int tid, int nthreads,
                            Sync sync) {
  auto val = [&](int k, int t) { return T[(size_t)k * sk + (size_t)t * st] * (w ? w[k_base + k] : 1.f); };
  const int lane = tid & 31, wid = tid >> 5, nwarps = nthreads >> 5;
  if (out.xi) {
    const int ngrp = nk / 64;
    for (int e = wid; e < ngrp * ntok; e += nwarps) {
      const int gq = e / ntok, t = e % ntok;
      float amax = fmaxf(fabsf(val(gq * 64 + lane, t)), fabsf(val(gq * 64 + 32 + lane, t)));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = amax / 127.0f;
      if (lane == 0) {
        scratch[e] = s;
        const int kg = k_base + gq * 64;
        xc_put(out.xc, nt_total, t_base + t, kg >> 8, (kg & 255) >> 6, s);
      }
    }
    sync();
    const int n_e = (nk / 32) * ntok * 4;
    for (int e = tid; e < n_e; e += nthreads) {
      const int jl = e / (ntok * 4), rem = e % (ntok * 4), t = rem >> 2, c = rem & 3;
      float v[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[i] = val(jl * 32 + 4 * c + i, t);
        v[4 + i] = val(jl * 32 + 16 + 4 * c + i, t);
      }
      const int kg = k_base + jl * 32;
      xi_put(out.xi, out.x3, nt_total, t_base + t, kg >> 8, (kg & 255) >> 5, c, v, scratch[(jl >> 1) * ntok + t]);
    }
  }
  if (out.xf) {
    const int n_e = (nk / 16) * ntok * 4;
    for (int e = tid; e < n_e; e += nthreads) {
      const int ksl = e / (ntok * 4), rem = e % (ntok * 4), t = rem >> 2, c = rem & 3;
      const int r0 = ksl * 16 + 2 * c;
      const int kg = k_base + ksl * 16;
      xf_put(out.xf, nt_total, t_base + t, kg >> 8, (kg & 255) >> 4, c, val(r0, t), val(r0 + 1, t), val(r0 + 8, t),
             val(r0 + 9, t));
    }
  }
  if (out.xs) {
    const int n_s = (nk / 32) * ntok;
    for (int e = wid; e < n_s; e += nwarps) {
      const int jl = e / ntok, t = e % ntok;
      float s = val(jl * 32 + lane, t);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) {
        const int kg = k_base + jl * 32;
        xs_put(out.xs, nt_total, t_base + t, kg >> 8, (kg & 255) >> 5, s);
      }
    }
  }
  sync();
}

// Plain fp32 rows -> fragments (+ optional elementwise weight), plus the
// per-128-column sums of squares of the unweighted rows (RMSNorm statistics).
cudaError_t xfrag_launch(const float* x, int ldx, const float* w, int m, int k, int nt, const XFrags& out, float* ss,
                         int ld_ss, cudaStream_t s);

}  // namespace rb
