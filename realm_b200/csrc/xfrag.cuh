// Activation fragments: the form in which every GEMV reads its input.
//
// A GEMV input x[M][K] (fp32, already multiplied by the consumer's RMSNorm
// weight when one is fused) is stored as fp16 hi/lo pairs (x ~= hi + lo to
// ~22 significant bits) pre-arranged in the m16n8k16 B-fragment order, so the
// GEMV copies it with the bulk-copy engine and feeds the tensor cores without
// any conversion work. Producers (embedding, the residual / SwiGLU epilogues,
// the attention kernel, or xfrag_launch for plain inputs) write it once.
//
//  XF: uint4 [K/256][NT][16 k-steps][32 lanes]   (NT = ceil(M/8) n-tiles)
//      lane l holds token 8*nt + l/4 at columns c = 16*ks + 2*(l%4) (+1, +8, +9):
//      {hi(c, c+1), hi(c+8, c+9), lo(c, c+1), lo(c+8, c+9)} as half2.
//  XS: uint32 [K/256][NT][8 tokens][8 sub-blocks]  half2(hi, lo) of the sum of
//      the 32 values of each 32-column sub-block (the Q4_K min term).
#pragma once
#include "common.cuh"

namespace rb {

constexpr int kXfSbBytes = 16 * 32 * 16;  // one n-tile of one 256-column super-block
constexpr int kXsSbBytes = 8 * 8 * 4;

__host__ __device__ inline size_t xf_bytes(int k, int nt) { return (size_t)(k / 256) * nt * kXfSbBytes; }
__host__ __device__ inline size_t xs_bytes(int k, int nt) { return (size_t)(k / 256) * nt * kXsSbBytes; }

// One buffer set for a GEMV input.
struct XFrags {
  uint4* xf = nullptr;
  uint32_t* xs = nullptr;
};

__device__ __forceinline__ uint32_t pack2(__half lo, __half hi) {
  return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// Four values of token t at columns k, k+1, k+8, k+9 (k = 16*ks + 2*c, ks/c local
// to the super-block `sb`) -> one B-fragment entry.
__device__ __forceinline__ void xf_put(uint4* xf, int nt_total, int t, int sb, int ks, int c, float v0, float v1,
                                       float v2, float v3) {
  const __half2 h01 = __floats2half2_rn(v0, v1), h23 = __floats2half2_rn(v2, v3);
  const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
  const __half2 l01 = __floats2half2_rn(v0 - f01.x, v1 - f01.y), l23 = __floats2half2_rn(v2 - f23.x, v3 - f23.y);
  uint4 o;
  o.x = *reinterpret_cast<const uint32_t*>(&h01);
  o.y = *reinterpret_cast<const uint32_t*>(&h23);
  o.z = *reinterpret_cast<const uint32_t*>(&l01);
  o.w = *reinterpret_cast<const uint32_t*>(&l23);
  xf[(((size_t)sb * nt_total + (t >> 3)) * 16 + ks) * 32 + (t & 7) * 4 + c] = o;
}

// Sum of the 32 values of sub-block j (0..7) of super-block sb for token t.
__device__ __forceinline__ void xs_put(uint32_t* xs, int nt_total, int t, int sb, int j, float s) {
  const __half hi = __float2half_rn(s);
  const __half lo = __float2half_rn(s - __half2float(hi));
  xs[(((size_t)sb * nt_total + (t >> 3)) * 8 + (t & 7)) * 8 + j] = pack2(hi, lo);
}

// Writes the fragments of the block of values val(k, t) = T[k*sk + t*st] * (w ? w[k_base+k] : 1)
// for local columns k in [0, nk) (global column k_base + k; nk and k_base multiples
// of 32) and local tokens t in [0, ntok) (global token t_base + t). Every thread
// of the calling group (ids tid < nthreads) must call it.
__device__ inline void frags_write(const float* T, int sk, int st, int nk, int ntok, int k_base, int t_base,
                                   const float* w, const XFrags& out, int nt_total, int tid, int nthreads) {
  auto val = [&](int k, int t) { return T[(size_t)k * sk + (size_t)t * st] * (w ? w[k_base + k] : 1.f); };
  const int n_e = (nk / 16) * ntok * 4;
  for (int e = tid; e < n_e; e += nthreads) {
    const int ksl = e / (ntok * 4), rem = e % (ntok * 4), t = rem >> 2, c = rem & 3;
    const int r0 = ksl * 16 + 2 * c;
    const int kg = k_base + ksl * 16;
    xf_put(out.xf, nt_total, t_base + t, kg >> 8, (kg & 255) >> 4, c, val(r0, t), val(r0 + 1, t), val(r0 + 8, t),
           val(r0 + 9, t));
  }
  const int n_s = (nk / 32) * ntok;
  for (int e = tid; e < n_s; e += nthreads) {
    const int jl = e / ntok, t = e % ntok;
    float s = 0.f;
#pragma unroll 8
    for (int i = 0; i < 32; ++i) s += val(jl * 32 + i, t);
    const int kg = k_base + jl * 32;
    xs_put(out.xs, nt_total, t_base + t, kg >> 8, (kg & 255) >> 5, s);
  }
}

// Plain fp32 rows -> fragments (+ optional elementwise weight), plus the
// per-128-column sums of squares of the unweighted rows (RMSNorm statistics).
cudaError_t xfrag_launch(const float* x, int ldx, const float* w, int m, int k, int nt, const XFrags& out, float* ss,
                         int ld_ss, cudaStream_t s);

}  // namespace rb
