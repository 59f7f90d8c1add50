// Fused GGUF dequant GEMV/GEMM for decode: y[t, n] = sum_k x[t, k] * W[n, k].
//
// Replaces the reference's fused_dequant_matmul_{q4k,q6k,q80}
// (crates/realm-compute-cpu/src/fused.rs:229-374, 1128-1259, 2451-2554) and the
// CandleCpuBackend dequant+GEMM (candle_cpu_backend.rs:92-114) on the decode path.
//
// Design (B200, HBM-bound for M <= 64 tokens):
//  * Persistent CTAs (one per SM) split the (row-group, super-block) unit space
//    evenly (stream-K), so every SM streams the same number of weight bytes.
//  * One producer lane streams 256-row x 256-column units (37-70 KB) with the
//    bulk-copy engine (cp.async.bulk, no multicast) into a shared-memory ring.
//  * The activations arrive as pre-built B fragments (xfrag.cuh, written once
//    by the producing kernel): int8 three-limb for Q4_K, fp16 hi/lo (~22 bits)
//    for Q6_K and Q8_0. They are bulk-copied next to each weight unit, so the
//    tensor cores see exact integer weights and no conversion work happens here.
//  * Sixteen consumer warps (one 16-row tile each) turn the quantised values
//    into exact A fragments: 4-bit quants as int8 for Q4_K (mma.sync m16n8k32
//    s8, int32 accumulate), q-32 (Q6_K) and q (Q8_0) as fp16 (m16n8k16, fp32
//    accumulate). Per-32/16-column scales need register accumulators, which is
//    why this decode path uses mma.sync rather than TMEM-resident tcgen05 tiles.
//  * Row groups split across CTAs are reduced by the last-arriving CTA in a
//    fixed order (deterministic; no spin waits), then the fused epilogue runs.
#include "gemv.cuh"

#include <mutex>
#include <set>
#include <utility>
#include "quant.cuh"
#include "xfrag.cuh"

namespace rb {

namespace {

constexpr int kConsumerWarps = kUnitTiles;  // one per 16-row tile (256-row units)
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kThreads = 32 * (kConsumerWarps + 1);
constexpr int kMaxTokens = 64;
constexpr int kSmemBudget = 200 * 1024;

// activation bytes staged per unit: Q4_K reads int8 limbs + scales + sums, the
// others fp16 hi/lo fragments + sums
__host__ __device__ constexpr int x_stage_bytes(int dtype, int nt) {
  return dtype == DT_Q4_K ? nt * (kXiSbBytes + kX3SbBytes + kXcSbBytes + kXsSbBytes) : nt * (kXfSbBytes + kXsSbBytes);
}
__host__ __device__ constexpr int stage_bytes(int dtype, int nt) { return unit_bytes(dtype) + x_stage_bytes(dtype, nt); }
// epilogue tile: token-major, a row of kRowGroup + 1 floats per token (the
// padding spreads the fragment writer's column reads over all banks)
constexpr int kTLd = kRowGroup + 1;
__host__ __device__ constexpr int tile_floats(int nt) { return kTLd * 8 * nt; }
constexpr int kMaxStages = 6;
constexpr int kChainMinSmem = 120 * 1024;  // > half the SM's shared memory: one CTA per SM

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }

__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// measurement stamps (dbg bit 1): [cta][phase][kStampSlots] %globaltimer values
#define RB_TS(p, slot)                                                                                    \
  do {                                                                                                    \
    if ((a.dbg & 2) && a.dbg_ts) a.dbg_ts[((size_t)blockIdx.x * kMaxPhases + (p)) * kStampSlots + (slot)] = gtimer(); \
  } while (0)

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }
// L2 loads issued where they stand in the program (volatile): the tail of a
// split row group requests the residual rows before the partial sums, so both
// round trips overlap
__device__ __forceinline__ float ldcg_issue(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float4 ldcg4_issue(const float* p) {
  float4 v;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ float guard_scale(float v, float repl) {
  // fused.rs:276-285 / 1171-1175: NaN or Inf super-scales are replaced
  return (isnan(v) || isinf(v)) ? repl : v;
}

// ---------------------------------------------------------------------------
// Consumers: one 16-row tile x one super-block, accumulated into acc[NT][4]
// (C fragment: [0]=(g, 2c) [1]=(g, 2c+1) [2]=(g+8, 2c) [3]=(g+8, 2c+1)).
// xb: the super-block's B fragments, xsb: its sub-block sums.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_s8_16832(int d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// Q4_K on the int8 tensor path. Per 32-column sub-block j the MMA gives exact
// integer dot products C1, C2, C3 of the 4-bit quants with the three activation
// limbs; sc_j * (256*C1 + C2) accumulates exactly in int32 over a 64-column
// group (|.| < 2^31 by construction), sc_j * C3 in a second int32, and the pair
// is scaled by the group's activation scale: s * (S12 + S3 / 256) / 256.
// Per row: y = d/256 * sum_g s_g * (S12_g + S3_g / 256) - dmin * sum_j m_j * xsum_j
// (dequantize_q4_k, quant.rs:160-182: q*d*sc - dmin*m, regrouped).
template <int NT>
__device__ __forceinline__ void tile_q4k(const uint8_t* tile, const uint8_t* xi, const uint8_t* x3, const uint8_t* xc,
                                         const uint8_t* xsb, int lane, float acc[NT][4]) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 hA = lds128(tile + g * 16);
  const uint4 hB = lds128(tile + (g + 8) * 16);
  const float dA = guard_scale(half_bits_to_float(hA.x), 0.00000006f);
  const float mA = guard_scale(half_bits_to_float(hA.x >> 16), 0.00000024f);
  const float dB = guard_scale(half_bits_to_float(hB.x), 0.00000006f);
  const float mB = guard_scale(half_bits_to_float(hB.x >> 16), 0.00000024f);
  // 6-bit sub-scales and mins (get_scale_min_k4, quant.rs:108-122), 4 per word
  const uint32_t scA_lo = hA.y & 0x3F3F3F3Fu, scA_hi = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
  const uint32_t mnA_lo = hA.z & 0x3F3F3F3Fu, mnA_hi = ((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u);
  const uint32_t scB_lo = hB.y & 0x3F3F3F3Fu, scB_hi = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
  const uint32_t mnB_lo = hB.z & 0x3F3F3F3Fu, mnB_hi = ((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u);
  const uint32_t mwA = (c < 2) ? mnA_lo : mnA_hi, mwB = (c < 2) ? mnB_lo : mnB_hi;
  const uint32_t jb = (uint32_t)((2 * c) & 3);
  const uint32_t sel = jb | (4u << 4) | ((jb + 1) << 8) | (4u << 12);
  const uint32_t am0 = hsub2_u(prmt(mwA, 0x64646464u, sel), 0x64006400u);
  const uint32_t am1 = hsub2_u(prmt(mwB, 0x64646464u, sel), 0x64006400u);

  float u[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) u[nt][0] = u[nt][1] = u[nt][2] = u[nt][3] = 0.f;
  const uint8_t* qs = tile + 256;
#pragma unroll
  for (int grp = 0; grp < 4; ++grp) {  // 64-column group = sub-blocks 2grp, 2grp+1
    const uint4 q = lds128(qs + grp * 512 + lane * 16);
    int S[NT][4], S3[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) S[nt][r] = S3[nt][r] = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 2 * grp + h;
      const uint32_t w0 = h ? q.z : q.x, w1 = h ? q.w : q.y;
      uint32_t af[4];
      af[0] = w0 & 0x0F0F0F0Fu;
      af[1] = (w0 >> 4) & 0x0F0F0F0Fu;
      af[2] = w1 & 0x0F0F0F0Fu;
      af[3] = (w1 >> 4) & 0x0F0F0F0Fu;
      const int sa = (int)(((j < 4 ? scA_lo : scA_hi) >> (8 * (j & 3))) & 0xffu);
      const int sbv = (int)(((j < 4 ? scB_lo : scB_hi) >> (8 * (j & 3))) & 0xffu);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint4 b = lds128(xi + nt * kXiSbBytes + (j * 32 + lane) * 16);
        const uint2 b3 = lds64(x3 + nt * kX3SbBytes + (j * 32 + lane) * 8);
        int c1[4], c2[4], c3[4];
        mma_s8_16832(c1, af, b.x, b.y);
        mma_s8_16832(c2, af, b.z, b.w);
        mma_s8_16832(c3, af, b3.x, b3.y);
        S[nt][0] += sa * (c1[0] * 256 + c2[0]);
        S[nt][1] += sa * (c1[1] * 256 + c2[1]);
        S[nt][2] += sbv * (c1[2] * 256 + c2[2]);
        S[nt][3] += sbv * (c1[3] * 256 + c2[3]);
        S3[nt][0] += sa * c3[0];
        S3[nt][1] += sa * c3[1];
        S3[nt][2] += sbv * c3[2];
        S3[nt][3] += sbv * c3[3];
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float2 sv = *reinterpret_cast<const float2*>(xc + nt * kXcSbBytes + (grp * 8 + 2 * c) * 4);
      u[nt][0] = fmaf(sv.x, fmaf((float)S3[nt][0], 1.0f / 256.0f, (float)S[nt][0]), u[nt][0]);
      u[nt][1] = fmaf(sv.y, fmaf((float)S3[nt][1], 1.0f / 256.0f, (float)S[nt][1]), u[nt][1]);
      u[nt][2] = fmaf(sv.x, fmaf((float)S3[nt][2], 1.0f / 256.0f, (float)S[nt][2]), u[nt][2]);
      u[nt][3] = fmaf(sv.y, fmaf((float)S3[nt][3], 1.0f / 256.0f, (float)S[nt][3]), u[nt][3]);
    }
  }
  const float dA8 = dA * (1.0f / 256.0f), dB8 = dB * (1.0f / 256.0f);
  const float mA8 = mA * 256.0f, mB8 = mB * 256.0f;  // the hi parts of the sums hold sum / 256
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const uint2 sw = lds64(xsb + nt * kXsSbBytes + (g * 8 + 2 * c) * 4);
    const uint32_t bm_hi = prmt(sw.x, sw.y, 0x5410u), bm_lo = prmt(sw.x, sw.y, 0x7632u);
    float ch[4] = {0.f, 0.f, 0.f, 0.f}, cl[4] = {0.f, 0.f, 0.f, 0.f};
    mma_1688(ch, am0, am1, bm_hi);
    mma_1688(cl, am0, am1, bm_lo);
    acc[nt][0] = fmaf(-mA, cl[0], fmaf(-mA8, ch[0], fmaf(dA8, u[nt][0], acc[nt][0])));
    acc[nt][1] = fmaf(-mA, cl[1], fmaf(-mA8, ch[1], fmaf(dA8, u[nt][1], acc[nt][1])));
    acc[nt][2] = fmaf(-mB, cl[2], fmaf(-mB8, ch[2], fmaf(dB8, u[nt][2], acc[nt][2])));
    acc[nt][3] = fmaf(-mB, cl[3], fmaf(-mB8, ch[3], fmaf(dB8, u[nt][3], acc[nt][3])));
  }
}

template <int NT>
__device__ __forceinline__ void tile_q6k(const uint8_t* tile, const uint8_t* xb, int lane, float acc[NT][4]) {
  const int g = lane >> 2;
  const uint16_t* dd = reinterpret_cast<const uint16_t*>(tile);
  const float dA = guard_scale(half_bits_to_float(dd[g]), 0.00000006f);
  const float dB = guard_scale(half_bits_to_float(dd[g + 8]), 0.00000006f);
  const uint4 sAw = lds128(tile + 32 + g * 16);
  const uint4 sBw = lds128(tile + 32 + (g + 8) * 16);
  const uint32_t sAs[4] = {sAw.x, sAw.y, sAw.z, sAw.w};
  const uint32_t sBs[4] = {sBw.x, sBw.y, sBw.z, sBw.w};
  const uint8_t* lo = tile + 288;
  const uint8_t* hi = tile + 288 + 2048;
#pragma unroll
  for (int hc = 0; hc < 2; ++hc) {
    const uint4 hw = lds128(hi + hc * 512 + lane * 16);
    const uint32_t hws[4] = {hw.x, hw.y, hw.z, hw.w};
#pragma unroll
    for (int half_ch = 0; half_ch < 2; ++half_ch) {
      const int ch = hc * 2 + half_ch;
      const uint4 q = lds128(lo + ch * 512 + lane * 16);
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int ks = ch * 4 + w;      // 0..15
        const int hwi = (ks & 7) >> 1;  // word within the hi chunk
        const uint32_t H = (ks & 1) ? (hws[hwi] >> 16) : (hws[hwi] & 0xffffu);
        const uint32_t X = (H & 0xffu) | ((H & 0xff00u) << 8);
        const uint32_t word = qw[w];
        uint32_t af[4];
        af[0] = hsub2_u(lop3_and_or(word, 0x000F000Fu, 0x64006400u) | ((X << 4) & 0x00300030u), 0x64206420u);
        af[1] = hsub2_u(lop3_and_or(word >> 4, 0x000F000Fu, 0x64006400u) | ((X << 2) & 0x00300030u), 0x64206420u);
        af[2] = hsub2_u(lop3_and_or(word >> 8, 0x000F000Fu, 0x64006400u) | (X & 0x00300030u), 0x64206420u);
        af[3] = hsub2_u(lop3_and_or(word >> 12, 0x000F000Fu, 0x64006400u) | ((X >> 2) & 0x00300030u), 0x64206420u);
        const float fa = dA * (float)(int8_t)(sAs[ks >> 2] >> (8 * (ks & 3)));
        const float fb = dB * (float)(int8_t)(sBs[ks >> 2] >> (8 * (ks & 3)));
        const float fa8 = fa * 256.0f, fb8 = fb * 256.0f;  // hi activation parts hold x / 256
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint4 b = lds128(xb + nt * kXfSbBytes + (ks * 32 + lane) * 16);
          float ch_[4] = {0.f, 0.f, 0.f, 0.f}, cl_[4] = {0.f, 0.f, 0.f, 0.f};
          mma_16816(ch_, af, b.x, b.y);
          mma_16816(cl_, af, b.z, b.w);
          acc[nt][0] = fmaf(fa, cl_[0], fmaf(fa8, ch_[0], acc[nt][0]));
          acc[nt][1] = fmaf(fa, cl_[1], fmaf(fa8, ch_[1], acc[nt][1]));
          acc[nt][2] = fmaf(fb, cl_[2], fmaf(fb8, ch_[2], acc[nt][2]));
          acc[nt][3] = fmaf(fb, cl_[3], fmaf(fb8, ch_[3], acc[nt][3]));
        }
      }
    }
  }
}

template <int NT>
__device__ __forceinline__ void tile_q80(const uint8_t* tile, const uint8_t* xb, int lane, float acc[NT][4]) {
  const int g = lane >> 2;
  const uint4 dAw = lds128(tile + g * 16);
  const uint4 dBw = lds128(tile + (g + 8) * 16);
  const uint32_t dAs[4] = {dAw.x, dAw.y, dAw.z, dAw.w};
  const uint32_t dBs[4] = {dBw.x, dBw.y, dBw.z, dBw.w};
  const uint8_t* qs = tile + 256;
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {  // one 32-column block per chunk
    const uint4 q = lds128(qs + ch * 512 + lane * 16);
    const float da = half_bits_to_float(dAs[ch >> 1] >> ((ch & 1) * 16));
    const float db = half_bits_to_float(dBs[ch >> 1] >> ((ch & 1) * 16));
    const float da8 = da * 256.0f, db8 = db * 256.0f;  // hi activation parts hold x / 256
    float ct[2][NT][4];
#pragma unroll
    for (int hl = 0; hl < 2; ++hl)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) ct[hl][nt][0] = ct[hl][nt][1] = ct[hl][nt][2] = ct[hl][nt][3] = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2) {
      const int ks = ch * 2 + s2;
      const uint32_t w0 = s2 ? q.z : q.x, w1 = s2 ? q.w : q.y;
      uint32_t af[4];
      af[0] = hsub2_u(prmt(w0, 0x64646464u, 0x4140u), 0x64806480u);
      af[1] = hsub2_u(prmt(w0, 0x64646464u, 0x4342u), 0x64806480u);
      af[2] = hsub2_u(prmt(w1, 0x64646464u, 0x4140u), 0x64806480u);
      af[3] = hsub2_u(prmt(w1, 0x64646464u, 0x4342u), 0x64806480u);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const uint4 b = lds128(xb + nt * kXfSbBytes + (ks * 32 + lane) * 16);
        mma_16816(ct[0][nt], af, b.x, b.y);
        mma_16816(ct[1][nt], af, b.z, b.w);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      acc[nt][0] = fmaf(da, ct[1][nt][0], fmaf(da8, ct[0][nt][0], acc[nt][0]));
      acc[nt][1] = fmaf(da, ct[1][nt][1], fmaf(da8, ct[0][nt][1], acc[nt][1]));
      acc[nt][2] = fmaf(db, ct[1][nt][2], fmaf(db8, ct[0][nt][2], acc[nt][2]));
      acc[nt][3] = fmaf(db, ct[1][nt][3], fmaf(db8, ct[0][nt][3], acc[nt][3]));
    }
  }
}

// ---------------------------------------------------------------------------
// Epilogues (run by the 16 consumer warps; warp = tile within the row group)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void kv_store(const KvView& kv, int layer, int which, int tenant, int pos, int head,
                                         int d, float v) {
  const int page = kv.ptab[(size_t)tenant * kv.ptab_stride + (pos >> 4)];
  const size_t off = ((((size_t)page * kv.n_layers + layer) * 2 + which) * kv.n_kv + head) * 16 * (size_t)kv.hd +
                     (size_t)(pos & 15) * kv.hd + d;
  if (kv.f16) reinterpret_cast<__half*>(kv.pool)[off] = __float2half_rn(v);
  else reinterpret_cast<float*>(kv.pool)[off] = v;
}

// RESID rows x[t][row] of this thread's accumulator elements, read through L2
// (written by another CTA earlier in the launch); issued early by callers so
// the load overlaps other L2 round trips.
template <int NT>
__device__ __forceinline__ void load_resid(const GemvArgs& a, int rg, int warp, int lane, float xv[NT][4]) {
  const int g = lane >> 2, c = lane & 3;
  const int row0 = rg * kRowGroup + warp * kTileRows + g;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = nt * 8 + 2 * c + (r & 1), row = row0 + ((r & 2) ? 8 : 0);
      xv[nt][r] = (t < a.m && row < a.n) ? ldcg_issue(a.resid + (size_t)t * a.ldr + row) : 0.f;
    }
}

// rg: row group within the phase's unit space; rows of a second weight
// (rg >= a.n_rg, QKV only) are numbered from its own first row.
template <int NT>
__device__ void epilogue(const GemvArgs& a, int p, int rg_u, int warp, int lane, float acc[NT][4],
                         const float* inv_rms, float* red, float* T, const float (*xpre)[4] = nullptr) {
  constexpr int LD = 8 * NT;
  const bool part2 = rg_u >= a.n_rg;
  const int rg = part2 ? rg_u - a.n_rg : rg_u;
  const int a_n = part2 ? a.n2 : a.n;
  const int g = lane >> 2, c = lane & 3;
  const int tid = warp * 32 + lane;
  const int row0 = rg * kRowGroup + warp * kTileRows + g;  // rows row0 and row0+8
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int t0 = nt * 8 + 2 * c;
    const float s0 = inv_rms ? inv_rms[t0] : 1.f, s1 = inv_rms ? inv_rms[t0 + 1] : 1.f;
    acc[nt][0] *= s0;
    acc[nt][1] *= s1;
    acc[nt][2] *= s0;
    acc[nt][3] *= s1;
  }
  if (a.epi == EPI_STORE) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = nt * 8 + 2 * c + (r & 1), row = row0 + ((r & 2) ? 8 : 0);
        if (t < a.m && row < a_n) a.y[(size_t)t * a.ldy + row] = acc[nt][r];
      }
    }
  } else if (a.epi == EPI_SWIGLU) {
    // tile rows 0-7 gate, 8-15 up, same output index (ffn.rs:98-103 order)
    const int ol = warp * 8 + g;  // output index within the row group (0..63)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int t = nt * 8 + 2 * c + r;
        const float gt = acc[nt][r], up = acc[nt][r + 2];
        const float sig = 1.0f / (1.0f + expf(-gt));
        const float h = (gt * sig) * up;
        const bool ok = t < a.m && 2 * (rg * (kRowGroup / 2) + ol) < a_n;
        T[t * kTLd + ol] = ok ? h : 0.f;
        if (ok && a.y) a.y[(size_t)t * a.ldy + rg * (kRowGroup / 2) + ol] = h;
      }
    }
    named_bar(2, 32 * kConsumerWarps);
    frags_write(T, 1, kTLd, kRowGroup / 2, LD, rg * (kRowGroup / 2), a.xout_t0, nullptr, a.xout,
                a.xout_nt ? a.xout_nt : NT, red, tid,
                32 * kConsumerWarps, [] { named_bar(2, 32 * kConsumerWarps); });
  } else if (a.epi == EPI_RESID) {
    // x rows were written by another CTA earlier in this launch: read through
    // L2, all before the first store (one round trip), unless the caller
    // already issued the loads
    float xv[NT][4];
    if (xpre) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) xv[nt][r] = xpre[nt][r];
    } else {
      load_resid<NT>(a, rg, warp, lane, xv);
    }
    float sq[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      sq[nt][0] = sq[nt][1] = 0.f;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = nt * 8 + 2 * c + (r & 1), row = row0 + ((r & 2) ? 8 : 0);
        const int rl = row - rg * kRowGroup;
        float tv = 0.f;
        if (t < a.m && row < a_n) {
          const float v = xv[nt][r] + acc[nt][r];
          a.resid[(size_t)t * a.ldr + row] = v;
          sq[nt][r & 1] += v * v;
          tv = a.xf_norm ? v * a.xf_norm[row] : v;
        }
        T[t * kTLd + rl] = tv;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        sq[nt][h] += __shfl_xor_sync(0xffffffffu, sq[nt][h], 4);
        sq[nt][h] += __shfl_xor_sync(0xffffffffu, sq[nt][h], 8);
        sq[nt][h] += __shfl_xor_sync(0xffffffffu, sq[nt][h], 16);
      }
      if (g == 0) {
        red[warp * kMaxTokens + nt * 8 + 2 * c] = sq[nt][0];
        red[warp * kMaxTokens + nt * 8 + 2 * c + 1] = sq[nt][1];
      }
    }
    named_bar(2, 32 * kConsumerWarps);
    if (tid == 0) RB_TS(p, 13);
    // RMSNorm statistics per 128 columns: two slots per 256-row group
    for (int e = tid; e < 2 * a.m; e += 32 * kConsumerWarps) {
      const int hlf = e / a.m, t = e % a.m;
      float s = 0.f;
      for (int w = hlf * (kConsumerWarps / 2); w < (hlf + 1) * (kConsumerWarps / 2); ++w) s += red[w * kMaxTokens + t];
      a.ss_out[(size_t)(2 * rg + hlf) * a.ld_ss + t] = s;
    }
    named_bar(2, 32 * kConsumerWarps);  // red is reused as frags_write scratch below
    if (tid == 0) RB_TS(p, 14);
    if (a.xout.xs)
      frags_write(T, 1, kTLd, kRowGroup, LD, rg * kRowGroup, a.xout_t0, nullptr, a.xout, a.xout_nt ? a.xout_nt : NT,
                  red, tid, 32 * kConsumerWarps,
                  [] { named_bar(2, 32 * kConsumerWarps); });
    if (tid == 0) RB_TS(p, 15);
  } else if (a.epi == EPI_LOGITS) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      unsigned long long best[2] = {0ull, 0ull};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = nt * 8 + 2 * c + (r & 1), row = row0 + ((r & 2) ? 8 : 0);
        if (t < a.m && row < a_n) {
          if (a.y) a.y[(size_t)t * a.ldy + row] = acc[nt][r];
          const unsigned long long key =
              ((unsigned long long)float_order_key(acc[nt][r]) << 32) | (unsigned long long)row;
          best[r & 1] = key > best[r & 1] ? key : best[r & 1];
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int sh = 4; sh <= 16; sh <<= 1) {
          const unsigned long long o = __shfl_xor_sync(0xffffffffu, best[h], sh);
          best[h] = o > best[h] ? o : best[h];
        }
        const int t = nt * 8 + 2 * c + h;
        if (g == 0 && t < a.m && best[h]) atomicMax(a.argmax + t, best[h]);
      }
    }
  } else if (a.epi == EPI_QKV) {
    // RoPE on adjacent pairs (attention.rs:171-240): rows 2i and 2i+1 live in
    // lanes that differ by 4 (g and g^1).
    const int hd = a.head_dim;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int t = nt * 8 + 2 * c + (r & 1);
        const int row = row0 + ((r & 2) ? 8 : 0);
        const int grow = (part2 ? a.qkv_row0_2 : a.qkv_row0) + row;
        const bool is_v = grow >= a.n_q_rows + a.n_k_rows;
        const float partner = __shfl_xor_sync(0xffffffffu, acc[nt][r], 4);
        const bool valid = t < a.m && row < a_n;
        if (!valid) continue;
        const int pos = a.row_pos[t];
        float v = acc[nt][r];
        const int rr = grow < a.n_q_rows ? grow : (grow < a.n_q_rows + a.n_k_rows ? grow - a.n_q_rows
                                                                                   : grow - a.n_q_rows - a.n_k_rows);
        const int head = rr / hd, dim = rr % hd;
        if (!is_v) {
          const int i = dim & ~1;
          const float freq = 1.0f / powf(a.rope_theta, (float)i / (float)hd);
          const float ang = (float)pos * freq;
          float sn, cs;
          sincosf(ang, &sn, &cs);
          if ((dim & 1) == 0) v = __fsub_rn(__fmul_rn(v, cs), __fmul_rn(partner, sn));
          else v = __fadd_rn(__fmul_rn(partner, sn), __fmul_rn(v, cs));
        }
        if (grow < a.n_q_rows) {
          a.q_out[(size_t)t * a.ldq + rr] = v;
        } else {
          kv_store(a.kv, a.layer, is_v ? 1 : 0, a.row_tenant[t], pos, head, dim, v);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// The kernel: a chain of GEMV phases run by one persistent grid.
//
// ChainArgs holds 1..kMaxPhases GEMVs (e.g. o-proj -> gate|up -> down -> next
// layer's q|k -> v). Every CTA walks all phases in order; within a phase the
// units (256-row group x 256-column super-block) are split evenly over the
// CTAs as in a single GEMV. The producer lane streams the weight units of
// consecutive phases through one shared-memory ring without pausing at phase
// boundaries; only the activation copies of a phase wait for what they depend
// on: phase 0 on the previous kernel (programmatic dependent launch), a phase
// with its bit set in bar_mask on a grid barrier that every CTA passes after
// finishing the phase before it (last epilogue written). Each barrier slot is
// a monotonic 64-bit arrival counter (CTAs without units in a phase reach
// later barriers early, so slots must not share one); a CTA's ticket t gives
// the target (t / G + 1) * G. All CTAs of a multi-phase launch are resident
// at once (grid <= SM count, one CTA per SM by shared memory), and every wait
// is bounded.
// ---------------------------------------------------------------------------
struct ChainSmem {
  int ring, tile, bars, inv_rms, red, tgt, total;
};

__host__ __device__ inline ChainSmem chain_smem(int stages, int stage_bytes, int nt) {
  ChainSmem L;
  L.ring = 0;
  L.tile = stages * stage_bytes;
  L.bars = L.tile + 4 * tile_floats(nt);
  L.inv_rms = L.bars + 8 * (2 * stages);
  L.red = L.inv_rms + 4 * kMaxTokens;
  L.tgt = L.red + 4 * kConsumerWarps * kMaxTokens + 16;
  L.total = L.tgt + 8 * kMaxPhases;
  return L;
}

// This CTA's unit range [u0, u0 + n_units) of phase a; Gp = CTAs with work.
struct PhaseRange {
  long long U, u0;
  int Gp, n_units;
};
__device__ __forceinline__ PhaseRange phase_range(const GemvArgs& a) {
  PhaseRange r;
  r.U = (long long)(a.n_rg + a.n_rg2) * a.nsb;
  r.Gp = r.U < (long long)gridDim.x ? (int)r.U : (int)gridDim.x;
  if ((int)blockIdx.x < r.Gp) {
    r.u0 = r.U * blockIdx.x / r.Gp;
    r.n_units = (int)(r.U * (blockIdx.x + 1) / r.Gp - r.u0);
  } else {
    r.u0 = 0;
    r.n_units = 0;
  }
  return r;
}

// Ring position shared by producer and consumers: unit sequence number over
// all phases -> stage s, and how many times the ring has wrapped (round).
struct RingPos {
  int s = 0;
  uint32_t round = 0;
  __device__ __forceinline__ void next(int S) {
    if (++s == S) {
      s = 0;
      ++round;
    }
  }
};

// End of a row-group segment: a whole row group goes straight to the
// epilogue; a partial one is deposited, and the last of its contributors sums
// them and runs the epilogue.
template <int NT>
__device__ __forceinline__ void finish_segment(const GemvArgs& a, int p, int n_phases, const PhaseRange& pr, int rg,
                                            int sb, int first_rg, float (&acc)[NT][4], const float* inv_rms,
                                            float* red, float* T) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long U = pr.U, u0 = pr.u0;
  const int Gp = pr.Gp;
  // two partial slots per CTA and phase; chains alternate two pairs so that
  // consecutive phases never share a slot
  const int nslots = n_phases > 1 ? 4 : 2;
  const int slot_base = n_phases > 1 ? (p & 1) * 2 : 0;
  const float* irms = a.ss_part ? inv_rms : nullptr;
  const bool stamp = threadIdx.x == 0;
  if (stamp) RB_TS(p, 8);
  const long long seg_lo = (u0 > (long long)rg * a.nsb) ? u0 : (long long)rg * a.nsb;
  const bool full_seg = (seg_lo == (long long)rg * a.nsb) && (sb + 1 == a.nsb);
  if (!full_seg) {
    // deposit this CTA's partial; slot 0 if rg is this CTA's first row group
    const int slot = slot_base + ((rg == first_rg) ? 0 : 1);
    float* dst = a.partials + ((((size_t)blockIdx.x * nslots + slot) * kConsumerWarps + warp) * NT) * 128;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      __stcg(reinterpret_cast<float4*>(dst + nt * 128 + lane * 4),
             make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]));
    // the CTA's partial stores are ordered before thread 0's release (bar.sync,
    // then one cumulative fence) and after its acquire for the reads below
    named_bar(1, 32 * kConsumerWarps);
    if (stamp) RB_TS(p, 9);
    __shared__ int s_last;
    // contributors: CTAs whose unit range intersects row group rg
    const long long ua = (long long)rg * a.nsb, ub = ua + a.nsb - 1;
    long long cf = ua * Gp / U, cl = ub * Gp / U;
    while (cf + 1 < Gp && U * (cf + 1) / Gp <= ua) ++cf;
    while (cf > 0 && U * cf / Gp > ua) --cf;
    while (cl + 1 < Gp && U * (cl + 1) / Gp <= ub) ++cl;
    while (cl > 0 && U * cl / Gp > ub) --cl;
    const int ncontrib = (int)(cl - cf + 1);
    if (threadIdx.x == 0) {
      // release: every partial store of the CTA (ordered by the barrier above)
      // is visible before the ticket; acquire: the other contributors' are
      // visible to the reads below when this CTA is last
      // (one acquire-release atomic: 3 % faster per decode step than a fence,
      // a relaxed atomic and a second fence)
      s_last = (atom_add_acq_rel(a.counters + rg, 1) == ncontrib - 1);
      RB_TS(p, 10);
    }
    named_bar(1, 32 * kConsumerWarps);
    if (s_last) {
      float xv[NT][4];
      const bool resid = a.epi == EPI_RESID;
      if (resid) load_resid<NT>(a, rg, warp, lane, xv);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
      // contributor cc deposited into slot 0 iff rg is its first row group:
      // true for every cc > cf, and for cf iff its range starts at rg's start
      const int sl_cf = slot_base + ((U * cf / Gp == ua) ? 0 : 1);
      auto src_of = [&](long long cc) {
        const int sl = cc == cf ? sl_cf : slot_base;
        return a.partials + ((((size_t)cc * nslots + sl) * kConsumerWarps + warp) * NT) * 128 + lane * 4;
      };
      // summed in contributor order (deterministic); the loads of a batch of
      // contributors are all in flight before the first add
      constexpr int kB = 1;  // more batching spills registers (96 per thread at 17 warps)
      for (long long c0 = cf; c0 <= cl; c0 += kB) {
        float4 q[kB][NT];
#pragma unroll
        for (int b = 0; b < kB; ++b)
          if (c0 + b <= cl) {
            const float* src = src_of(c0 + b);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) q[b][nt] = ldcg4_issue(src + nt * 128);
          }
#pragma unroll
        for (int b = 0; b < kB; ++b)
          if (c0 + b <= cl) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              acc[nt][0] += q[b][nt].x;
              acc[nt][1] += q[b][nt].y;
              acc[nt][2] += q[b][nt].z;
              acc[nt][3] += q[b][nt].w;
            }
          }
      }
      if (stamp) RB_TS(p, 11);
      // the epilogue runs even after a timed-out wait (error already reported):
      // its named barriers must be reached by every consumer warp
      epilogue<NT>(a, p, rg, warp, lane, acc, irms, red, T, resid ? xv : nullptr);
      if (threadIdx.x == 0) a.counters[rg] = 0;
      if (stamp) RB_TS(p, 12);
    }
  } else {
    epilogue<NT>(a, p, rg, warp, lane, acc, irms, red, T);
  }
}

template <int DT, int NT>
__device__ __forceinline__ void tile_dt(const uint8_t* st, int warp, int lane, float (&acc)[NT][4]) {
  constexpr int UB = unit_bytes(DT), TB = tile_bytes(DT);
  const uint8_t* tile = st + warp * TB;
  const uint8_t* xb = st + UB;
  if (DT == DT_Q4_K)
    tile_q4k<NT>(tile, xb, xb + NT * kXiSbBytes, xb + NT * (kXiSbBytes + kX3SbBytes),
                 xb + NT * (kXiSbBytes + kX3SbBytes + kXcSbBytes), lane, acc);
  else if (DT == DT_Q6_K) tile_q6k<NT>(tile, xb, lane, acc);
  else tile_q80<NT>(tile, xb, lane, acc);
}

// DT: format of the phase's weight; DT2: of its second weight (row groups
// from a.n_rg on), DT2 == DT when there is none.
template <int DT, int DT2, int NT>
__device__ __forceinline__ void consume_phase(const GemvArgs& a, int p, int n_phases, const PhaseRange& pr, uint8_t* ring, int S,
                                              int SB, uint64_t* full, uint64_t* empty, float* inv_rms, float* red,
                                              float* T, RingPos& rp, bool& alive,
                                              const unsigned long long* gbar /* this barrier's counter */,
                                              bool wait_grid,
                                              unsigned long long bar_target, uint32_t grid_spin) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  if (tid == 0) RB_TS(p, 0);
  if (pr.n_units == 0) return;
  if (wait_grid) {  // uniform over the CTA; only thread 0 reads the target
    // everything the phases before wrote is visible once all CTAs arrived
    if (tid == 0) grid_wait(gbar, bar_target, a.err, (blockIdx.x << 8) | ((uint32_t)p << 1), grid_spin);
    named_bar(1, 32 * kConsumerWarps);
  }
  if (tid == 0) RB_TS(p, 1);
  if (a.ss_part) {
    // 1/rms per token from the partial sums of squares (written by other CTAs
    // or the previous kernel: read through L2). Thread (t, r) sums partials
    // r, r + 8, ... of token t; the eight sums are added in a fixed order.
    const int t = tid & 63, r = tid >> 6;
    if (t < a.m) {
      float ss = 0.f;
      for (int j = r; j < a.n_ss; j += 8) ss += __ldcg(a.ss_part + (size_t)j * a.ld_ss + t);
      red[r * 64 + t] = ss;
    }
    named_bar(1, 32 * kConsumerWarps);
    if (tid < a.m) {
      float ss = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) ss += red[q * 64 + tid];
      inv_rms[tid] = 1.0f / sqrtf(ss / (float)a.norm_dim + a.norm_eps);
    }
    named_bar(1, 32 * kConsumerWarps);
  }
  const long long u0 = pr.u0;
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  const int first_rg = (int)(u0 / a.nsb);
  int rg = first_rg, sb = (int)(u0 - (long long)first_rg * a.nsb);  // advanced per unit (no divisions)
  for (int i = 0; i < pr.n_units; ++i, (++sb == a.nsb) ? (sb = 0, ++rg) : 0) {
    const int s = rp.s;
    if (alive) alive = mbar_wait(&full[s], rp.round & 1, a.err, DEV_TIMEOUT_FULL);
    if (i == 0 && tid == 0) RB_TS(p, 2);
    if (alive && !(a.dbg & 1)) {
      const uint8_t* st = ring + (size_t)s * SB;
      if (DT2 != DT && rg >= a.n_rg) tile_dt<DT2, NT>(st, warp, lane, acc);
      else tile_dt<DT, NT>(st, warp, lane, acc);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    rp.next(S);
    if (i + 1 == pr.n_units && tid == 0) RB_TS(p, 3);
    const bool seg_end = (i + 1 == pr.n_units) || (sb + 1 == a.nsb);
    if (!seg_end) continue;
    finish_segment<NT>(a, p, n_phases, pr, rg, sb, first_rg, acc, inv_rms, red, T);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    if (i + 1 == pr.n_units && tid == 0) RB_TS(p, 4);
  }
}

// Index of the latest grid barrier at or before phase p (0: none in this launch).
__device__ __forceinline__ int last_barrier(uint32_t mask, int p) {
  int q = 0;
  for (int i = 1; i <= p; ++i)
    if ((mask >> i) & 1u) q = i;
  return q;
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ ChainArgs ca) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = ca.stages, SB = ca.stage_bytes;
  const ChainSmem L = chain_smem(S, SB, NT);
  uint8_t* ring = smem + L.ring;
  float* T = reinterpret_cast<float*>(smem + L.tile);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + S;
  float* inv_rms = reinterpret_cast<float*>(smem + L.inv_rms);
  float* red = reinterpret_cast<float*>(smem + L.red);
  volatile unsigned long long* s_tgt = reinterpret_cast<volatile unsigned long long*>(smem + L.tgt);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const GemvArgs& a0 = ca.ph[0];

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int p = 0; p < kMaxPhases; ++p) s_tgt[p] = 0ull;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      RingPos rp;
      uint32_t issued = 0;  // units issued over all phases
      bool ok = true, pdl_done = false;
      int passed = 0;  // highest grid barrier this producer has waited for
      int pend_s[kMaxStages], pend_sb[kMaxStages];
      for (int p = 0; p < ca.n_phases && ok; ++p) {
        const GemvArgs& a = ca.ph[p];
        const PhaseRange pr = phase_range(a);
        const long long U1 = (long long)a.n_rg * a.nsb;  // units of the first weight
        // the phase's activations depend on the latest grid barrier at or before it
        const int need = last_barrier(ca.bar_mask, p);
        bool dep = pdl_done && need <= passed;
        int npend = 0;
        int x_sb = pr.n_units ? (int)(pr.u0 % a.nsb) : 0;
        int pend_dt[kMaxStages];
        // activation bytes for super-block sb: Q4_K {int8 limbs, scales, sums}, else {fp16 hi/lo, sums}
        auto issue_x = [&](int s, int sb, int dt) {
          uint8_t* st = ring + (size_t)s * SB + unit_bytes(dt);
          uint64_t* bar = &full[s];
          if (dt == DT_Q4_K) {
            bulk_g2s(st, reinterpret_cast<const uint8_t*>(a.xin.xi) + (size_t)sb * NT * kXiSbBytes, NT * kXiSbBytes,
                     bar);
            st += NT * kXiSbBytes;
            bulk_g2s(st, reinterpret_cast<const uint8_t*>(a.xin.x3) + (size_t)sb * NT * kX3SbBytes, NT * kX3SbBytes,
                     bar);
            st += NT * kX3SbBytes;
            bulk_g2s(st, reinterpret_cast<const uint8_t*>(a.xin.xc) + (size_t)sb * NT * kXcSbBytes, NT * kXcSbBytes,
                     bar);
            st += NT * kXcSbBytes;
          } else {
            bulk_g2s(st, reinterpret_cast<const uint8_t*>(a.xin.xf) + (size_t)sb * NT * kXfSbBytes, NT * kXfSbBytes,
                     bar);
            st += NT * kXfSbBytes;
          }
          bulk_g2s(st, reinterpret_cast<const uint8_t*>(a.xin.xs) + (size_t)sb * NT * kXsSbBytes, NT * kXsSbBytes, bar);
        };
        // the activations of this phase may be read once what they depend on is done
        auto resolve = [&]() {
          if (!pdl_done) {
            pdl_wait();
            pdl_done = true;
          }
          if (need > passed) {
            // target of barrier `need`, published by this CTA's consumers on arrival
            uint32_t k = 0;
            while (s_tgt[need - 1] == 0ull && ++k < kSpinLimit) {
            }
            const unsigned long long tgt = s_tgt[need - 1];
            if (tgt == 0ull) report_error(a.err, DEV_TIMEOUT_SMEM);
            else grid_wait(ca.gbar + need, tgt, a.err, (blockIdx.x << 8) | ((uint32_t)p << 1) | 1u, ca.grid_spin);
            passed = need;
          }
          dep = true;
          for (int j = 0; j < npend; ++j) issue_x(pend_s[j], pend_sb[j], pend_dt[j]);
          npend = 0;
          RB_TS(p, 6);
        };
        const int pf = (ca.prefetch >= 0 && ca.prefetch < S) ? ca.prefetch : S;
        for (int i = 0; i < pr.n_units; ++i) {
          if (!dep && npend >= pf) resolve();
          const int s = rp.s;
          if (issued >= (uint32_t)S) {
            ok = mbar_wait(&empty[s], (rp.round - 1) & 1, a.err, DEV_TIMEOUT_EMPTY);
            if (!ok) break;
          }
          const long long u = pr.u0 + i;
          const int dt = u < U1 ? a.dtype : a.dtype2;
          const int UB = unit_bytes(dt);
          mbar_arrive_expect_tx(&full[s], UB + x_stage_bytes(dt, NT));
          const uint8_t* wsrc = u < U1 ? a.w + u * (long long)UB : a.w2 + (u - U1) * (long long)UB;
          bulk_g2s_evict_first(ring + (size_t)s * SB, wsrc, UB, &full[s], pol);
          if (i == 0) RB_TS(p, 5);
          if (i + 1 == pr.n_units) RB_TS(p, 7);
          if (dep) {
            issue_x(s, x_sb, dt);
          } else {
            pend_s[npend] = s;
            pend_sb[npend] = x_sb;
            pend_dt[npend] = dt;
            ++npend;
          }
          if (++x_sb == a.nsb) x_sb = 0;
          rp.next(S);
          ++issued;
          if (!dep && (npend >= pf || i + 1 == pr.n_units)) resolve();
        }
      }
      // drain: every issued copy must land before this CTA may exit
      const uint32_t first = issued > (uint32_t)S ? issued - S : 0u;
      for (uint32_t j = first; j < issued; ++j)
        mbar_wait(&full[j % S], (j / S) & 1, a0.err, DEV_TIMEOUT_DRAIN);
    }
    return;
  }

  // ---- consumers ----
  pdl_wait();
  RingPos rp;
  bool alive = true;
  int passed = 0;  // highest grid barrier these consumers have waited for
  for (int p = 0; p < ca.n_phases; ++p) {
    const GemvArgs& a = ca.ph[p];
    const PhaseRange pr = phase_range(a);
    const int need = last_barrier(ca.bar_mask, p);
    const bool wg = need > passed && pr.n_units > 0;
    const unsigned long long my_target = wg ? s_tgt[need - 1] : 0ull;
    if (wg) passed = need;
    switch (a.dtype) {
      case DT_Q4_K:
        // 8-row steps: every Q4_K phase runs the mixed loop (a phase without a
        // second weight never reaches its Q6_K part), one inlined copy fewer
        if constexpr (NT == 1)
          consume_phase<DT_Q4_K, DT_Q6_K, NT>(a, p, ca.n_phases, pr, ring, S, SB, full, empty, inv_rms, red, T, rp,
                                              alive, ca.gbar + need, wg, my_target, ca.grid_spin);
        else
          consume_phase<DT_Q4_K, DT_Q4_K, NT>(a, p, ca.n_phases, pr, ring, S, SB, full, empty, inv_rms, red, T, rp,
                                              alive, ca.gbar + need, wg, my_target, ca.grid_spin);
        break;
      case DT_Q6_K: consume_phase<DT_Q6_K, DT_Q6_K, NT>(a, p, ca.n_phases, pr, ring, S, SB, full, empty, inv_rms, red, T, rp, alive,
                                         ca.gbar + need, wg, my_target, ca.grid_spin); break;
      default: consume_phase<DT_Q8_0, DT_Q8_0, NT>(a, p, ca.n_phases, pr, ring, S, SB, full, empty, inv_rms, red, T, rp, alive,
                                         ca.gbar + need, wg, my_target, ca.grid_spin); break;
    }
    if (p + 1 < ca.n_phases && ((ca.bar_mask >> (p + 1)) & 1u)) {
      // this CTA is done with phase p (epilogue writes included): arrive
      named_bar(1, 32 * kConsumerWarps);
      if (threadIdx.x == 0) {
        // one counter per barrier slot: every CTA arrives at each slot exactly
        // once per launch, so a ticket always lies in its own launch's window
        const unsigned long long t = atom_add_release_u64(ca.gbar + (p + 1), 1ull);
        RB_TS(p, 17);
        // (the failure-detection hook moves one barrier's target a grid beyond reach)
        s_tgt[p] = (t / gridDim.x + 1 + (ca.fail_bar == p + 1 ? 1 : 0)) * gridDim.x;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Plain rows -> activation fragments (+ RMSNorm sums of squares).
// Grid (K/256, ceil(M/8)): one CTA per (super-block, 8-token n-tile), 128 threads.
__global__ void xfrag_kernel(const float* x, int ldx, const float* w, int m, int k, int nt, XFrags out, float* ss,
                             int ld_ss) {
  __shared__ float T[256 * 8];
  __shared__ float scratch[32];
  const int sb = blockIdx.x, n0 = blockIdx.y * 8;
  const int ntok = (m - n0) < 8 ? (m - n0) : 8;
  for (int e = threadIdx.x; e < 256 * 8; e += blockDim.x) {
    const int kk = e >> 3, t = e & 7;
    T[e] = t < ntok ? x[(size_t)(n0 + t) * ldx + sb * 256 + kk] : 0.f;
  }
  __syncthreads();
  if (ss) {
    // sums of squares of the raw rows per 128 columns
    for (int e = threadIdx.x; e < 2 * ntok; e += blockDim.x) {
      const int hg = e / ntok, t = e % ntok;
      float q = 0.f;
      for (int i = 0; i < 128; ++i) {
        const float v = T[(hg * 128 + i) * 8 + t];
        q += v * v;
      }
      ss[(size_t)(sb * 2 + hg) * ld_ss + n0 + t] = q;
    }
  }
  frags_write(T, 8, 1, 256, 8, sb * 256, n0, w, out, nt, scratch, threadIdx.x, blockDim.x, [] { __syncthreads(); });
}

// ---------------------------------------------------------------------------
// Repack GGUF -> tiles (one CTA of 128 threads per tile).
// ---------------------------------------------------------------------------
struct RowSrc {
  const uint8_t* p;
  int row;
};

__device__ __forceinline__ RowSrc tiled_row_source(int R, const uint8_t* a, int rows_a, const uint8_t* b, int rows_b,
                                                   int mode) {
  if (mode == 0) return {R < rows_a ? a : nullptr, R};
  if (mode == 1) {
    if (R < rows_a) return {a, R};
    return {(R - rows_a) < rows_b ? b : nullptr, R - rows_a};
  }
  // interleave-8: tile rows 0-7 from a, 8-15 from b, output index t*8 + r%8
  const int t = R >> 4, r = R & 15, o = t * 8 + (r & 7);
  if (r < 8) return {o < rows_a ? a : nullptr, o};
  return {o < rows_b ? b : nullptr, o};
}

template <int DT>
__global__ void repack_kernel(const uint8_t* a, int rows_a, const uint8_t* b, int rows_b, int mode, int k,
                              uint8_t* out, int n_rg) {
  constexpr int BB = block_bytes(DT);
  constexpr int BPS = kSuperK / block_elems(DT);  // GGUF blocks per 256 columns
  constexpr int TB = tile_bytes(DT);
  __shared__ __align__(16) uint8_t src[16 * BB * BPS];
  const int nsb = k / kSuperK;
  const long long tile = blockIdx.x;  // ((rg * nsb + sb) * 8 + mt)
  const int mt = (int)(tile % kUnitTiles);
  const int sb = (int)((tile / kUnitTiles) % nsb);
  const int rg = (int)(tile / kUnitTiles / nsb);
  const size_t row_bytes = (size_t)(k / block_elems(DT)) * BB;
  for (int i = threadIdx.x; i < 16 * BB * BPS; i += blockDim.x) {
    const int r = i / (BB * BPS), off = i % (BB * BPS);
    const RowSrc rs = tiled_row_source(rg * kRowGroup + mt * kTileRows + r, a, rows_a, b, rows_b, mode);
    src[i] = rs.p ? rs.p[(size_t)rs.row * row_bytes + (size_t)sb * BB * BPS + off] : 0;
  }
  __syncthreads();
  uint8_t* o = out + tile * TB;
  const int t = threadIdx.x;
  if (DT == DT_Q4_K) {
    if (t < 16) {
      for (int i = 0; i < 16; ++i) o[t * 16 + i] = src[t * BB + i];
    }
    // int8-MMA A fragments (m16n8k32): 4 chunks (64 columns) x 32 lanes x 4 words;
    // word w: sub-block 2*chunk + w/2, columns +16*(w&1); byte i holds the quants of
    // rows g (low nibble) and g+8 (high nibble) at column 32j + 4c + i
    for (int idx = t; idx < 4 * 32 * 4; idx += blockDim.x) {
      const int ch = idx / 128, lane = (idx / 4) % 32, w = idx % 4;
      const int j = 2 * ch + (w >> 1), g = lane >> 2, c = lane & 3;
      uint32_t word = 0;
      for (int i = 0; i < 4; ++i) {
        const int e = 32 * j + 16 * (w & 1) + 4 * c + i;
        word |= (uint32_t)q4k_quant(src + g * BB + 16, e) << (8 * i);
        word |= (uint32_t)q4k_quant(src + (g + 8) * BB + 16, e) << (8 * i + 4);
      }
      *reinterpret_cast<uint32_t*>(o + 256 + (ch * 32 + lane) * 16 + w * 4) = word;
    }
  } else if (DT == DT_Q6_K) {
    if (t < 16) {
      o[t * 2] = src[t * BB + 208];
      o[t * 2 + 1] = src[t * BB + 209];
      for (int i = 0; i < 16; ++i) o[32 + t * 16 + i] = src[t * BB + 192 + i];
    }
    for (int idx = t; idx < 16 * 32; idx += blockDim.x) {  // (ks, lane)
      const int ks = idx / 32, lane = idx % 32;
      uint32_t word = 0, hbits = 0;
      for (int i = 0; i < 8; ++i) {
        int row, col;
        frag_pos(lane, i, row, col);
        const int e = ks * 16 + col;
        const uint32_t q = (uint32_t)(q6k_quant(src + row * BB, e) + 32);  // 0..63
        word |= (q & 0xF) << (4 * i);
        hbits |= (q >> 4) << (i < 4 ? 2 * i : 8 + 2 * (i - 4));
      }
      const int ch = ks / 4, w = ks % 4;
      *reinterpret_cast<uint32_t*>(o + 288 + (ch * 32 + lane) * 16 + w * 4) = word;
      const int hc = ks / 8, hw = (ks & 7) >> 1;
      uint16_t* hp = reinterpret_cast<uint16_t*>(o + 288 + 2048 + (hc * 32 + lane) * 16 + hw * 4);
      hp[ks & 1] = (uint16_t)hbits;
    }
  } else {  // Q8_0
    for (int idx = t; idx < 16 * 8; idx += blockDim.x) {
      const int r = idx / 8, bk = idx % 8;
      o[(r * 8 + bk) * 2] = src[(r * BPS + bk) * BB];
      o[(r * 8 + bk) * 2 + 1] = src[(r * BPS + bk) * BB + 1];
    }
    for (int idx = t; idx < 16 * 32; idx += blockDim.x) {  // (ks, lane)
      const int ks = idx / 32, lane = idx % 32;
      uint8_t bytes[8];
      for (int i = 0; i < 8; ++i) {
        int row, col;
        frag_pos(lane, i, row, col);
        const int e = ks * 16 + col;
        const int8_t q = (int8_t)src[(row * BPS + e / 32) * BB + 2 + (e % 32)];
        bytes[i] = (uint8_t)((int)q + 128);
      }
      // [v0 v4 v1 v5 | v2 v6 v3 v7]
      const uint8_t ord[8] = {bytes[0], bytes[4], bytes[1], bytes[5], bytes[2], bytes[6], bytes[3], bytes[7]};
      const int ch = ks / 2;
      uint8_t* dst = o + 256 + (ch * 32 + lane) * 16 + (ks & 1) * 8;
      for (int i = 0; i < 8; ++i) dst[i] = ord[i];
    }
  }
}

// Inverse of repack for plain mode (test hook: tiled -> GGUF bytes).
template <int DT>
__global__ void unpack_kernel(const uint8_t* tiled, int n, int k, uint8_t* out) {
  constexpr int BB = block_bytes(DT);
  constexpr int BPS = kSuperK / block_elems(DT);
  constexpr int TB = tile_bytes(DT);
  const int nsb = k / kSuperK;
  const long long tile = blockIdx.x;
  const int mt = (int)(tile % kUnitTiles);
  const int sb = (int)((tile / kUnitTiles) % nsb);
  const int rg = (int)(tile / kUnitTiles / nsb);
  const uint8_t* o = tiled + tile * TB;
  const size_t row_bytes = (size_t)(k / block_elems(DT)) * BB;
  __shared__ __align__(16) uint8_t dst[16 * BB * BPS];
  for (int i = threadIdx.x; i < 16 * BB * BPS; i += blockDim.x) dst[i] = 0;
  __syncthreads();
  const int t = threadIdx.x;
  if (DT == DT_Q4_K) {
    if (t < 16)
      for (int i = 0; i < 16; ++i) dst[t * BB + i] = o[t * 16 + i];
    __syncthreads();
    for (int idx = t; idx < 16 * 256; idx += blockDim.x) {
      const int row = idx / 256, e = idx % 256;
      const int j = e / 32, within = e % 32, hi16 = within / 16, c = (within % 16) / 4, i = within % 4;
      const int g = row & 7, lane = g * 4 + c, w = 2 * (j & 1) + hi16;
      const uint32_t word = *reinterpret_cast<const uint32_t*>(o + 256 + ((j >> 1) * 32 + lane) * 16 + w * 4);
      const uint32_t q = (word >> (8 * i + 4 * (row >> 3))) & 0xF;
      const int grp = e >> 6, wq = e & 63;
      uint8_t* qb = dst + row * BB + 16 + 32 * grp + (wq & 31);
      if (wq < 32) atomicOr(reinterpret_cast<unsigned int*>((size_t)qb & ~(size_t)3), q << (8 * ((size_t)qb & 3)));
      else atomicOr(reinterpret_cast<unsigned int*>((size_t)qb & ~(size_t)3), (q << 4) << (8 * ((size_t)qb & 3)));
    }
  }
  __syncthreads();
  for (int i = t; i < 16 * BB * BPS; i += blockDim.x) {
    const int r = i / (BB * BPS), off = i % (BB * BPS);
    const int row = rg * kRowGroup + mt * kTileRows + r;
    if (row < n) out[(size_t)row * row_bytes + (size_t)sb * BB * BPS + off] = dst[i];
  }
}

__global__ void dequant_kernel(int dtype, const uint8_t* blocks, size_t nblocks, float* out) {
  const size_t be = block_elems(dtype), bb = block_bytes(dtype);
  const size_t total = nblocks * be;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const uint8_t* blk = blocks + (i / be) * bb;
    const int e = (int)(i % be);
    out[i] = dtype == DT_Q4_K ? dequant_q4k_elem(blk, e) : dtype == DT_Q6_K ? dequant_q6k_elem(blk, e)
                                                                           : dequant_q80_elem(blk, e);
  }
}

// Quantisers (own design; the reference has none). Every step is an IEEE-rounded
// operation, so a CPU implementation of the same steps reproduces the bytes.
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
__device__ __forceinline__ uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

__global__ void quantize_kernel(int dtype, const float* x, size_t nblocks, uint8_t* out) {
  const size_t bi = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (bi >= nblocks) return;
  if (dtype == DT_Q4_K) {
    const float* v = x + bi * 256;
    uint8_t* o = out + bi * 144;
    float scale[8], minv[8], max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; ++j) {
      float mn = v[32 * j], mx = v[32 * j];
      for (int i = 1; i < 32; ++i) {
        const float t = v[32 * j + i];
        mn = (t < mn) ? t : mn;
        mx = (mx < t) ? t : mx;
      }
      if (mn > 0.f) mn = 0.f;
      scale[j] = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
      minv[j] = -mn;
      max_scale = (max_scale < scale[j]) ? scale[j] : max_scale;
      max_min = (max_min < minv[j]) ? minv[j] : max_min;
    }
    const uint16_t dh = f2h_bits(__fdiv_rn(max_scale, 63.0f)), mh = f2h_bits(__fdiv_rn(max_min, 63.0f));
    const float df = half_bits_to_float(dh), dmf = half_bits_to_float(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
      sc[j] = df > 0.f ? clampi(__float2int_rn(__fdiv_rn(scale[j], df)), 0, 63) : 0;
      m[j] = dmf > 0.f ? clampi(__float2int_rn(__fdiv_rn(minv[j], dmf)), 0, 63) : 0;
    }
    o[0] = dh & 0xff; o[1] = dh >> 8; o[2] = mh & 0xff; o[3] = mh >> 8;
    for (int j = 0; j < 4; ++j) {
      o[4 + j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
      o[4 + j + 4] = (uint8_t)(m[j] | ((m[j + 4] >> 4) << 6));
      o[4 + j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    for (int i = 0; i < 4; ++i)
      for (int l = 0; l < 32; ++l) {
        int qq[2];
        for (int hh = 0; hh < 2; ++hh) {
          const int j = 2 * i + hh, e = 64 * i + 32 * hh + l;
          const float dd = __fmul_rn(df, (float)sc[j]), mm = __fmul_rn(dmf, (float)m[j]);
          qq[hh] = dd > 0.f ? clampi(__float2int_rn(__fdiv_rn(__fadd_rn(v[e], mm), dd)), 0, 15) : 0;
        }
        o[16 + 32 * i + l] = (uint8_t)(qq[0] | (qq[1] << 4));
      }
  } else if (dtype == DT_Q6_K) {
    const float* v = x + bi * 256;
    uint8_t* o = out + bi * 210;
    float s[16], smax = 0.f;
    for (int g = 0; g < 16; ++g) {
      float amax = 0.f;
      for (int i = 0; i < 16; ++i) {
        const float t = fabsf(v[16 * g + i]);
        amax = (amax < t) ? t : amax;
      }
      s[g] = __fdiv_rn(amax, 31.0f);
      smax = (smax < s[g]) ? s[g] : smax;
    }
    const uint16_t dh = f2h_bits(__fdiv_rn(smax, 127.0f));
    const float df = half_bits_to_float(dh);
    int8_t sc[16];
    for (int g = 0; g < 16; ++g) sc[g] = (int8_t)(df > 0.f ? clampi(__float2int_rn(__fdiv_rn(s[g], df)), -128, 127) : 0);
    uint8_t q[256];
    for (int i = 0; i < 256; ++i) {
      const float dd = __fmul_rn(df, (float)sc[i / 16]);
      q[i] = (uint8_t)((dd != 0.f ? clampi(__float2int_rn(__fdiv_rn(v[i], dd)), -32, 31) : 0) + 32);
    }
    for (int h = 0; h < 2; ++h)
      for (int l = 0; l < 32; ++l) {
        const uint8_t* qq = q + 128 * h;
        const uint8_t q1 = qq[l], q2 = qq[l + 32], q3 = qq[l + 64], q4 = qq[l + 96];
        o[64 * h + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
        o[64 * h + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
        o[128 + 32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
      }
    for (int g = 0; g < 16; ++g) o[192 + g] = (uint8_t)sc[g];
    o[208] = dh & 0xff;
    o[209] = dh >> 8;
  } else {  // Q8_0
    const float* v = x + bi * 32;
    uint8_t* o = out + bi * 34;
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) {
      const float t = fabsf(v[i]);
      amax = (amax < t) ? t : amax;
    }
    const uint16_t dh = f2h_bits(__fdiv_rn(amax, 127.0f));
    const float df = half_bits_to_float(dh);
    uint8_t blk[34];
    blk[0] = (uint8_t)(dh & 0xffu);
    blk[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 32; ++i) {
      const int q = df > 0.f ? clampi(__float2int_rn(__fdiv_rn(v[i], df)), -128, 127) : 0;
      blk[2 + i] = (uint8_t)(q & 0xff);
    }
    for (int i = 0; i < 34; ++i) o[i] = blk[i];
  }
}

template <int NT>
cudaError_t launch_chain_t(ChainArgs ca, int num_sms, cudaStream_t s, int pdl) {
  int sb = 0;
  for (int p = 0; p < ca.n_phases; ++p) {
    sb = max(sb, stage_bytes(ca.ph[p].dtype, NT));
    if (ca.ph[p].n_rg2) sb = max(sb, stage_bytes(ca.ph[p].dtype2, NT));
  }
  sb = (sb + 127) & ~127;
  const int fit = (kSmemBudget - 4 * tile_floats(NT) - 4096) / sb;
  ca.stages = fit > kMaxStages ? kMaxStages : fit < 1 ? 1 : fit;
  ca.stage_bytes = sb;
  int smem = chain_smem(ca.stages, sb, NT).total;
  if (ca.n_phases > 1 && smem < kChainMinSmem) smem = kChainMinSmem;  // one CTA per SM
  auto kern = gemv_kernel<NT>;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cudaError_t e = ensure_smem_attr(kern, kSmemBudget + 8192, dev)) return e;
  if (ca.n_phases > 1) {
    // grid barriers need every CTA resident at once: one CTA per SM must fit
    // (checked once per device and footprint)
    static std::mutex mu;
    static std::set<std::pair<int, int>> ok;
    std::lock_guard<std::mutex> lock(mu);
    if (!ok.count({dev, smem})) {
      int per_sm = 0;
      if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem)) return e;
      if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
      ok.insert({dev, smem});
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ca.n_phases == 1 ? gemv_ctas(num_sms, ca.ph[0].n_rg + ca.ph[0].n_rg2, ca.ph[0].nsb) : num_sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, ca);
}


// ===========================================================================
// tcgen05 dequant-GEMM for 16..64 rows (prefill chunks, large scheduler
// steps), where the GEMV above is bound by its mma.sync issue rate.
//
// D[128 weight rows][N tokens] accumulates in tensor memory (TMEM) from
// tcgen05.mma kind::f16 (M = 128, N = 16..64, K = 16), A and B in shared
// memory in the canonical K-major no-swizzle layout: 8 x 16-byte core
// matrices, rows 16 bytes apart, 8-row groups 128 bytes apart (SBO), 8-column
// chunks LBO apart. Eight warps dequantise one 64-column slice of a 128-row
// weight tile per stage straight from the tiled layout: every weight becomes
// w * 2^e_row (w bit-exact as dequantize_* computes it; e_row a per-row power
// of two chosen at upload so |w| * 2^e < 2^14 fits fp16) split into fp16
// hi + lo. The activations come from the fp16 hi/lo fragments (xfrag.cuh).
// Three MMAs per k-step (hi.hi + hi.lo + lo.hi) give ~22-bit products with
// fp32 accumulation. One thread issues the MMAs and commits each stage to an
// mbarrier that frees the stage for the producers. Units (128-row tile x
// 64-column slice) are split evenly over a persistent grid (stream-K); every
// segment of one tile ends in a drain of TMEM into a fixed partial slot, and
// qgemm_epi_kernel sums a tile's slots in CTA order (deterministic), undoes
// 2^e_row and runs the GEMV's fused epilogue. Every mbarrier wait is bounded.
// ===========================================================================
constexpr int kQgRows = 128;
constexpr int kQgKc = 64;
constexpr int kQgMaxStages = 3;                          // A/B operand stages (2 or 3 by format)
constexpr int kQgCompute = 256;                          // dequantising threads (warps 0-7)
constexpr int kQgThreads = kQgCompute + 64;              // + the loader warp + the MMA warp
constexpr int kQgAPlane = kQgRows * kQgKc * 2;           // 16 KB
constexpr int kQgBPlane = kMaxTokens * kQgKc * 2;        // 8 KB
constexpr int kQgStage = 2 * kQgAPlane + 2 * kQgBPlane;  // 48 KB
constexpr int kQgALbo = kQgRows * 16;                    // bytes between 8-column chunks (A)
constexpr int kQgBLbo = kMaxTokens * 16;                 // (B)
constexpr int kQgTmemCols = 128;  // two accumulators of kMaxTokens columns
constexpr int kQgSmemUse = 220 * 1024;  // operand stages + quantised weight ring
constexpr int kQgMaxQStages = 8;
constexpr int kQgSmem = kQgSmemUse + 1024;

__device__ __forceinline__ uint32_t qg_aoff(int row, int col) {
  return (uint32_t)((col >> 3) * kQgALbo + (row >> 3) * 128 + (row & 7) * 16 + (col & 7) * 2);
}
__device__ __forceinline__ uint32_t qg_boff(int t, int col) {
  return (uint32_t)((col >> 3) * kQgBLbo + (t >> 3) * 128 + (t & 7) * 16 + (col & 7) * 2);
}
__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }  // e in [-126, 127]
// v (0 <= v < 2^23) as a float, exactly: 2^23 + v built in the mantissa, minus 2^23
__device__ __forceinline__ float u2f(uint32_t v) { return __fsub_rn(__uint_as_float(0x4B000000u | v), 8388608.0f); }

// fp16 hi + lo of two values (hi = RN(x), lo = RN(x - hi)), packed as half2 words
__device__ __forceinline__ void hilo2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 f = __half22float2(h);
  hi = h2_as_u32(h);
  lo = h2_as_u32(__floats2half2_rn(__fsub_rn(x0, f.x), __fsub_rn(x1, f.y)));
}

__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void sts64(uint32_t addr, uint32_t v0, uint32_t v1) {
  asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(v0), "r"(v1) : "memory");
}

// ---- tcgen05 wrappers (PTX ISA, sm_100a) ----
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  // start >> 4 [0,14), LBO >> 4 [16,30), SBO >> 4 [32,46), version 1 [46,48), no swizzle [61,64)
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// kind::f16 instruction descriptor: f32 accumulate, f16 A and B, both K-major
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Stream-K owner of unit u: the largest CTA c with floor(c * U / G) <= u.
__host__ __device__ __forceinline__ int qg_owner(long long u, long long U, int G) {
  return (int)(((u + 1) * G - 1) / U);
}

struct QgemmArgs {
  const uint8_t* w = nullptr;
  int32_t dtype = 0, n_rg = 0, nsb = 0, m = 0, nt_x = 0;
  const uint4* xf = nullptr;  // fp16 hi/lo fragments, n-tile stride nt_x
  const uint32_t* xs = nullptr;  // sub-block sums (Q4_K min term of the exact-weight GEMM)
  const uint8_t* bprep = nullptr;  // exact-weight GEMM: prepared activation planes (q2_bprep_kernel)
  const int8_t* rexp = nullptr;
  float* part = nullptr;      // [n_rt][slots][64 tokens][128 rows]
  int32_t slots = 0;
  int32_t dbg = 0;  // measurement hook: bit 0 skips the weight dequant, bit 1 the MMAs, bit 2 the activations
  uint32_t* err = nullptr;
};

// One 64-column slice (group kg & 3 of its super-block) of the 128-row weight
// tile whose eight 16-row tiles sit at `tiles` in shared memory, dequantised into
// the A planes at sA (hi) / sA + kQgAPlane (lo). grow: global row of tile row 0.
template <int DT>
__device__ __forceinline__ void qg_produce_a(const QgemmArgs& a, const uint8_t* tiles, int grow, int kg, uint32_t sA,
                                             int warp, int lane) {
  constexpr int TB = tile_bytes(DT);
  const int g = lane >> 2, c = lane & 3;
  const int grp = kg & 3;
  const uint8_t* tile = tiles + warp * TB;
  const int rowA = warp * 16 + g, rowB = rowA + 8;  // rows within the 128-row tile
  const float sAe = pow2f(a.rexp[grow + rowA]), sBe = pow2f(a.rexp[grow + rowB]);
  const uint32_t lo_plane = kQgAPlane;
  auto ld128 = [](const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); };
  if (DT == DT_Q4_K) {
    const uint4 hA = ld128(tile + g * 16), hB = ld128(tile + (g + 8) * 16);
    const float dA = guard_scale(half_bits_to_float(hA.x & 0xffffu), 0.00000006f);
    const float mA = guard_scale(half_bits_to_float(hA.x >> 16), 0.00000024f);
    const float dB = guard_scale(half_bits_to_float(hB.x & 0xffffu), 0.00000006f);
    const float mB = guard_scale(half_bits_to_float(hB.x >> 16), 0.00000024f);
    uint8_t scA[12], scB[12];
    const uint32_t wa[3] = {hA.y, hA.z, hA.w}, wb[3] = {hB.y, hB.z, hB.w};
#pragma unroll
    for (int i = 0; i < 12; ++i) {
      scA[i] = (uint8_t)(wa[i >> 2] >> (8 * (i & 3)));
      scB[i] = (uint8_t)(wb[i >> 2] >> (8 * (i & 3)));
    }
    const uint4 q = ld128(tile + 256 + grp * 512 + lane * 16);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = 2 * grp + h;
      int sca, ma, scb, mb;
      q4k_scale_min(j, scA, sca, ma);
      q4k_scale_min(j, scB, scb, mb);
      // w 2^e = (d1 2^e) q - m1 2^e (the power of two is exact); fused, so within half an ulp of w
      const float d1a = __fmul_rn(__fmul_rn(dA, (float)sca), sAe), m1a = __fmul_rn(__fmul_rn(mA, (float)ma), sAe);
      const float d1b = __fmul_rn(__fmul_rn(dB, (float)scb), sBe), m1b = __fmul_rn(__fmul_rn(mB, (float)mb), sBe);
#pragma unroll
      for (int half2i = 0; half2i < 2; ++half2i) {  // w0: columns 4c.., w1: 16 + 4c..
        const uint32_t wd = half2i ? (h ? q.w : q.y) : (h ? q.z : q.x);
        const int col = 32 * h + 16 * half2i + 4 * c;
        float va[4], vb[4];
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint32_t byte = (wd >> (8 * b)) & 0xffu;
          va[b] = fmaf(d1a, u2f(byte & 0xF), -m1a);
          vb[b] = fmaf(d1b, u2f(byte >> 4), -m1b);
        }
        uint32_t h0, l0, h1, l1;
        hilo2(va[0], va[1], h0, l0);
        hilo2(va[2], va[3], h1, l1);
        sts64(sA + qg_aoff(rowA, col), h0, h1);
        sts64(sA + lo_plane + qg_aoff(rowA, col), l0, l1);
        hilo2(vb[0], vb[1], h0, l0);
        hilo2(vb[2], vb[3], h1, l1);
        sts64(sA + qg_aoff(rowB, col), h0, h1);
        sts64(sA + lo_plane + qg_aoff(rowB, col), l0, l1);
      }
    }
  } else if (DT == DT_Q6_K) {
    const uint16_t* dd = reinterpret_cast<const uint16_t*>(tile);
    const float dA = guard_scale(half_bits_to_float(dd[g]), 0.00000006f);
    const float dB = guard_scale(half_bits_to_float(dd[g + 8]), 0.00000006f);
    const uint32_t scAw = *reinterpret_cast<const uint32_t*>(tile + 32 + g * 16 + grp * 4);
    const uint32_t scBw = *reinterpret_cast<const uint32_t*>(tile + 32 + (g + 8) * 16 + grp * 4);
    const uint4 ql = ld128(tile + 288 + grp * 512 + lane * 16);
    const uint4 qh = ld128(tile + 288 + 2048 + (grp >> 1) * 512 + lane * 16);
    const uint32_t qw[4] = {ql.x, ql.y, ql.z, ql.w};
    const uint32_t hws[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
      const int ks = grp * 4 + wi;
      const uint32_t H = (ks & 1) ? (hws[(ks & 7) >> 1] >> 16) : (hws[(ks & 7) >> 1] & 0xffffu);
      const float fa = __fmul_rn(__fmul_rn(dA, (float)(int8_t)(scAw >> (8 * wi))), sAe);
      const float fb = __fmul_rn(__fmul_rn(dB, (float)(int8_t)(scBw >> (8 * wi))), sBe);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        float v[2];
#pragma unroll
        for (int up = 0; up < 2; ++up) {
          const int nib = (int)((qw[wi] >> (4 * (r + 4 * up))) & 0xFu);
          const int hb = (int)((H >> (2 * r + 8 * up)) & 3u);
          v[up] = __fmul_rn((r & 1) ? fb : fa, u2f((uint32_t)(nib | (hb << 4))) - 32.0f);
        }
        uint32_t hh, ll;
        hilo2(v[0], v[1], hh, ll);
        const int row = (r & 1) ? rowB : rowA;
        const int col = 16 * wi + 2 * c + ((r & 2) ? 8 : 0);
        sts32(sA + qg_aoff(row, col), hh);
        sts32(sA + lo_plane + qg_aoff(row, col), ll);
      }
    }
  } else {  // Q8_0: chunks 2 grp and 2 grp + 1 (32 columns each)
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int ch = 2 * grp + cc;
      const float da = __fmul_rn(half_bits_to_float(reinterpret_cast<const uint16_t*>(tile + g * 16)[ch]), sAe);
      const float db = __fmul_rn(half_bits_to_float(reinterpret_cast<const uint16_t*>(tile + (g + 8) * 16)[ch]), sBe);
      const uint4 q = ld128(tile + 256 + ch * 512 + lane * 16);
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {
        const uint32_t w0 = s2 ? q.z : q.x, w1 = s2 ? q.w : q.y;
        const int col0 = 32 * cc + 16 * s2 + 2 * c;
#pragma unroll
        for (int r = 0; r < 4; ++r) {  // A-fragment register r: bytes (2(r&1), 2(r&1)+1) of w0 / w1
          const uint32_t wd = (r & 2) ? w1 : w0;
          const int sh = (r & 1) ? 16 : 0;
          const float qa = u2f((wd >> sh) & 0xffu) - 128.0f;
          const float qb = u2f((wd >> (sh + 8)) & 0xffu) - 128.0f;
          const float d = (r & 1) ? db : da;
          uint32_t hh, ll;
          hilo2(__fmul_rn(qa, d), __fmul_rn(qb, d), hh, ll);
          const int row = (r & 1) ? rowB : rowA;
          const int col = col0 + ((r & 2) ? 8 : 0);
          sts32(sA + qg_aoff(row, col), hh);
          sts32(sA + lo_plane + qg_aoff(row, col), ll);
        }
      }
    }
  }
}

// Activations of 64-column group kg (fp16 hi/lo fragments, tokens >= m as zeros):
// loaded one unit ahead into registers, stored into the B planes at
// sB (hi) / sB + kQgBPlane (lo).
constexpr int kQgBItems = 4;  // per compute thread: 4 k-steps x 8 n-tiles x 32 lanes / 256
__device__ __forceinline__ void qg_load_b(const QgemmArgs& a, int kg, int ntn, int tid, uint4 bv[kQgBItems]) {
  const int sb = kg >> 2, ks0 = (kg & 3) * 4;
  const int per_ks = ntn * 32, n_items = 4 * per_ks;
#pragma unroll
  for (int i = 0; i < kQgBItems; ++i) {
    const int e = tid + i * kQgCompute;
    bv[i] = make_uint4(0u, 0u, 0u, 0u);
    if (e < n_items) {
      const int ksl = e / per_ks, rem = e - ksl * per_ks, nt = rem >> 5, l = rem & 31;
      if (nt * 8 + (l >> 2) < a.m) bv[i] = __ldg(a.xf + (((size_t)sb * a.nt_x + nt) * 16 + ks0 + ksl) * 32 + l);
    }
  }
}
__device__ __forceinline__ void qg_store_b(int ntn, uint32_t sB, int tid, const uint4 bv[kQgBItems]) {
  const int per_ks = ntn * 32, n_items = 4 * per_ks;
#pragma unroll
  for (int i = 0; i < kQgBItems; ++i) {
    const int e = tid + i * kQgCompute;
    if (e < n_items) {
      const int ksl = e / per_ks, rem = e - ksl * per_ks, nt = rem >> 5, l = rem & 31;
      const int t = nt * 8 + (l >> 2), col = 16 * ksl + 2 * (l & 3);
      // the fragments hold x ~= 256 hi + lo; the GEMM's planes take x ~= hi + lo
      uint32_t w[4] = {bv[i].x, bv[i].y, bv[i].z, bv[i].w};
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float2 h = __half22float2(u32_as_h2(w[q])), lo = __half22float2(u32_as_h2(w[q + 2]));
        hilo2(fmaf(256.0f, h.x, lo.x), fmaf(256.0f, h.y, lo.y), w[q], w[q + 2]);
      }
      sts32(sB + qg_boff(t, col), w[0]);
      sts32(sB + qg_boff(t, col + 8), w[1]);
      sts32(sB + kQgBPlane + qg_boff(t, col), w[2]);
      sts32(sB + kQgBPlane + qg_boff(t, col + 8), w[3]);
    }
  }
}

// Walks a CTA's units as segments (maximal runs inside one 128-row tile).
struct QgWalk {
  long long u, u1, seg_end;
  int kG, rt;
  __device__ QgWalk(long long u0, long long u1_, int kG_) : u(u0), u1(u1_), seg_end(0), kG(kG_), rt(0) {}
  __device__ bool next_segment() {
    if (u >= u1) return false;
    rt = (int)(u / kG);
    seg_end = min(u1, (long long)(rt + 1) * kG);
    return true;
  }
};

// Q4_K (18 KB per half row-group) affords three operand stages next to a
// four-deep weight ring; the larger formats keep two.
template <int DT>
__host__ __device__ constexpr int qg_stages() {
  return DT == DT_Q4_K ? 3 : 2;
}
template <int DT>
__host__ __device__ constexpr int qg_qstages() {
  return ((kQgSmemUse - qg_stages<DT>() * kQgStage) / (8 * tile_bytes(DT))) > kQgMaxQStages
             ? kQgMaxQStages
             : (kQgSmemUse - qg_stages<DT>() * kQgStage) / (8 * tile_bytes(DT));
}

// Warp roles: 0-7 dequantise weights and stage activations; 8 streams each
// super-block's half row-group (8 tiles, contiguous in the tiled layout) into
// a ring with the bulk-copy engine (no multicast); 9 issues the MMAs into one
// of two TMEM accumulators (one per segment, alternating) and commits stages
// back to the producers. Every hand-off is an mbarrier with a bounded wait.
template <int DT>
__global__ void __launch_bounds__(kQgThreads, 1) qgemm_kernel(const __grid_constant__ QgemmArgs a) {
  constexpr int UB = unit_bytes(DT), TB = tile_bytes(DT), HU = 8 * TB, QS = qg_qstages<DT>();
  constexpr int kQgStages = qg_stages<DT>();
  constexpr int kCw = kQgCompute / 32;
  extern __shared__ __align__(1024) uint8_t qg_smem_raw[];
  __shared__ uint64_t sfull[kQgMaxStages], sfree[kQgMaxStages];
  __shared__ uint64_t qfull[kQgMaxQStages], qempty[kQgMaxQStages];
  __shared__ uint64_t accfull[2], accempty[2];
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(qg_smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  uint8_t* qring = smem + kQgStages * kQgStage;
  const int n_rt = 2 * a.n_rg, kG = 4 * a.nsb;
  const long long U = (long long)n_rt * kG;
  const int G = gridDim.x, cta = blockIdx.x;
  const long long u0 = U * cta / G, u1 = U * (cta + 1) / G;
  const int N = (a.m + 15) & ~15, ntn = N >> 3;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(kQgTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < kQgStages; ++i) {
      mbar_init(&sfull[i], kCw);
      mbar_init(&sfree[i], 1);
    }
    for (int i = 0; i < QS; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], kCw);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], kCw);
    }
    fence_barrier_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (warp == kCw) {
    // ---- loader: the weights do not depend on the previous kernel ----
    if (lane == 0) {
      long long iq = 0;
      bool ok = true;
      QgWalk w(u0, u1, kG);
      while (ok && w.next_segment()) {
        const int rg = w.rt >> 1, half = w.rt & 1;
        while (w.u < w.seg_end) {
          const int sb = (int)((w.u - (long long)w.rt * kG) >> 2);
          const int q = (int)(iq % QS);
          if (iq >= QS && !mbar_wait(&qempty[q], (uint32_t)((iq / QS - 1) & 1), a.err, DEV_TIMEOUT_SMEM)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&qfull[q], HU);
          bulk_g2s(qring + (size_t)q * HU, a.w + ((size_t)rg * a.nsb + sb) * UB + (size_t)half * 8 * TB, HU, &qfull[q]);
          ++iq;
          w.u = min(w.seg_end, (long long)w.rt * kG + (sb + 1) * 4);
        }
      }
      // copies still in flight land before the CTA's shared memory goes away
      for (long long j = iq > QS ? iq - QS : 0; j < iq; ++j)
        mbar_wait(&qfull[j % QS], (uint32_t)((j / QS) & 1), nullptr, 0);
    }
    __syncwarp();
  } else if (warp == kCw + 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(kQgRows, N);
      long long it = 0;
      int seg = 0;
      bool ok = true;
      QgWalk w(u0, u1, kG);
      while (ok && w.next_segment()) {
        const int b = seg & 1;
        if (seg >= 2 && !mbar_wait(&accempty[b], (uint32_t)((seg / 2 - 1) & 1), a.err, DEV_TIMEOUT_DRAIN)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * kMaxTokens);
        bool first = true;
        for (; w.u < w.seg_end; ++w.u, ++it) {
          const int s = (int)(it % kQgStages);
          if (!mbar_wait(&sfull[s], (uint32_t)((it / kQgStages) & 1), a.err, DEV_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + s * kQgStage;
#pragma unroll
          for (int ks = 0; ks < ((a.dbg & 2) ? 0 : kQgKc / 16); ++ks) {
            const uint64_t ah = umma_desc(st + ks * 2 * kQgALbo, kQgALbo, 128);
            const uint64_t al = umma_desc(st + kQgAPlane + ks * 2 * kQgALbo, kQgALbo, 128);
            const uint64_t bh = umma_desc(st + 2 * kQgAPlane + ks * 2 * kQgBLbo, kQgBLbo, 128);
            const uint64_t bl = umma_desc(st + 2 * kQgAPlane + kQgBPlane + ks * 2 * kQgBLbo, kQgBLbo, 128);
            umma_f16(acc, ah, bh, idesc, (first && ks == 0) ? 0u : 1u);
            umma_f16(acc, ah, bl, idesc, 1u);
            umma_f16(acc, al, bh, idesc, 1u);
          }
          umma_commit(&sfree[s]);
          first = false;
        }
        if (!ok) break;
        umma_commit(&accfull[b]);
        ++seg;
      }
      if (it > 0) {  // own MMAs complete before the accumulators are freed
        const long long last = it - 1;
        mbar_wait(&sfree[last % kQgStages], (uint32_t)((last / kQgStages) & 1), nullptr, 0);
      }
    }
    __syncwarp();
  } else {
    // ---- producers (warps 0-7) ----
    pdl_wait();
    bool alive = true;
    long long it = 0, iq = 0;
    int seg = 0;
    uint4 bv[kQgBItems];
    if (u0 < u1 && !(a.dbg & 4)) qg_load_b(a, (int)(u0 % kG), ntn, tid, bv);
    QgWalk w(u0, u1, kG);
    while (alive && w.next_segment()) {
      const int grow = w.rt * kQgRows;
      bool first = true;
      for (; w.u < w.seg_end; ++w.u, ++it) {
        const int kg = (int)(w.u - (long long)w.rt * kG);
        const bool sb_first = first || (kg & 3) == 0;
        const bool sb_last = (kg & 3) == 3 || w.u + 1 == w.seg_end;
        const int q = (int)(iq % QS);
        if (sb_first) alive = alive && mbar_wait(&qfull[q], (uint32_t)((iq / QS) & 1), a.err, DEV_TIMEOUT_FULL);
        const int s = (int)(it % kQgStages);
        if (it >= kQgStages)  // the MMAs that last read stage s are done
          alive = alive && mbar_wait(&sfree[s], (uint32_t)((it / kQgStages - 1) & 1), a.err, DEV_TIMEOUT_EMPTY);
        if (!alive) break;
        const uint32_t st = sbase + s * kQgStage;
        if (!(a.dbg & 1)) qg_produce_a<DT>(a, qring + (size_t)q * HU, grow, kg, st, warp, lane);
        if (!(a.dbg & 4)) {
          qg_store_b(ntn, st + 2 * kQgAPlane, tid, bv);
          if (w.u + 1 < u1) qg_load_b(a, (int)((w.u + 1) % kG), ntn, tid, bv);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sfull[s]);
          if (sb_last) mbar_arrive(&qempty[q]);
        }
        __syncwarp();
        if (sb_last) ++iq;
        first = false;
      }
      if (!alive) break;
      // segment end: drain accumulator seg & 1 into this CTA's slot of tile rt
      const int b = seg & 1;
      alive = mbar_wait(&accfull[b], (uint32_t)((seg / 2) & 1), a.err, DEV_TIMEOUT_DRAIN);
      __syncwarp();
      if (!alive) break;
      tc_fence_after();
      const int quarter = warp & 3, colh = warp >> 2;
      if (colh * 32 < N) {
        const int slot = cta - qg_owner((long long)w.rt * kG, U, G);
        float* dst = a.part + ((size_t)w.rt * a.slots + slot) * kMaxTokens * kQgRows + 32 * quarter + lane;
#pragma unroll
        for (int h16 = 0; h16 < 2; ++h16) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(b * kMaxTokens + colh * 32 + h16 * 16), v);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int t = colh * 32 + h16 * 16 + i;
            if (t < a.m) dst[(size_t)t * kQgRows] = v[i];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[b]);
      ++seg;
    }
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kQgTmemCols) : "memory");
  }
}

struct QgemmTail {
  const float* part = nullptr;
  const int8_t* rexp = nullptr;
  int32_t slots = 0, G = 0, kG = 0;
  long long U = 0;
};

// Sums each 256-row group's partial slots (CTA order), undoes 2^e_row and runs
// the GEMV epilogue (same fragment mapping: warp = 16-row tile of the group).
// One CTA per (256-row group, 8-token n-tile): the tokens of an epilogue are
// independent, so splitting them gives NT times the CTAs.
__global__ void __launch_bounds__(kConsumerWarps * 32) qgemm_epi_kernel(const __grid_constant__ GemvArgs ga,
                                                                        const __grid_constant__ QgemmTail q) {
  extern __shared__ __align__(16) float qe_smem[];
  float* red = qe_smem;                              // kConsumerWarps * kMaxTokens
  float* inv_rms = red + kConsumerWarps * kMaxTokens;  // kMaxTokens
  float* T = inv_rms + kMaxTokens;                   // tile_floats(1)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rg = blockIdx.x, t0 = 8 * blockIdx.y;
  pdl_wait();
  pdl_launch_dependents();
  if (t0 >= ga.m) return;
  // this CTA's tokens t0 .. t0 + 7 as tokens 0..7 of a narrower launch
  GemvArgs a = ga;
  a.m = min(8, ga.m - t0);
  a.xout_nt = ga.m <= 8 ? 1 : ga.m <= 16 ? 2 : ga.m <= 32 ? 4 : 8;  // gemv_nt_for
  a.xout_t0 = t0;
  if (a.y) a.y += (size_t)t0 * a.ldy;
  if (a.resid) a.resid += (size_t)t0 * a.ldr;
  if (a.q_out) a.q_out += (size_t)t0 * a.ldq;
  if (a.ss_out) a.ss_out += t0;
  if (a.ss_part) a.ss_part += t0;
  if (a.argmax) a.argmax += t0;
  if (a.row_pos) a.row_pos += t0;
  if (a.row_tenant) a.row_tenant += t0;
  if (a.ss_part) {  // as consume_phase: eight strided partial sums per token, added in a fixed order
    const int t = tid & 63, r = tid >> 6;
    if (t < a.m) {
      float ss = 0.f;
      for (int j = r; j < a.n_ss; j += 8) ss += __ldcg(a.ss_part + (size_t)j * a.ld_ss + t);
      red[r * 64 + t] = ss;
    }
    __syncthreads();
    if (tid < a.m) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) ss += red[k * 64 + tid];
      inv_rms[tid] = 1.0f / sqrtf(ss / (float)a.norm_dim + a.norm_eps);
    }
    __syncthreads();
  }
  const int rt = rg * 2 + (warp >> 3);
  const int rl = (warp & 7) * 16 + g;  // row within the 128-row tile (and rl + 8)
  const int c0 = qg_owner((long long)rt * q.kG, q.U, q.G), c1 = qg_owner((long long)rt * q.kG + q.kG - 1, q.U, q.G);
  float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
  for (int cc = c0; cc <= c1; ++cc) {
    const float* base = q.part + ((size_t)rt * q.slots + (cc - c0)) * kMaxTokens * kQgRows;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int t = 2 * c + (r & 1);
      if (t < a.m) acc[0][r] += __ldcg(base + (size_t)(t0 + t) * kQgRows + rl + ((r & 2) ? 8 : 0));
    }
  }
  const int row0 = rg * kRowGroup + warp * kTileRows + g;
  // the per-row 2^e of the hi/lo-weight GEMM (none for the exact-weight GEMM)
  const float sA = q.rexp ? pow2f(-(int)q.rexp[row0]) : 1.f, sB = q.rexp ? pow2f(-(int)q.rexp[row0 + 8]) : 1.f;
  acc[0][0] *= sA;
  acc[0][1] *= sA;
  acc[0][2] *= sB;
  acc[0][3] *= sB;
  epilogue<1>(a, 0, rg, warp, lane, acc, a.ss_part ? inv_rms : nullptr, red, T);
}

// Per-row exponent e with (bound of |w| over the row) * 2^e < 2^14, from the
// block scales alone: Q4_K |w| <= |d| 63 15 + |dmin| 63, Q6_K |d| 128 32,
// Q8_0 |d| 128 (NaN/Inf scales replaced as the fused kernels do).
__global__ void rowexp_kernel(const uint8_t* w, int dtype, int n_rg, int nsb, int8_t* out) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n_rg * kRowGroup) return;
  const int rg = row / kRowGroup, rr = row % kRowGroup, ti = rr / kTileRows, r16 = rr % kTileRows;
  const int UB = unit_bytes(dtype), TB = tile_bytes(dtype);
  float bound = 0.f;
  for (int sb = 0; sb < nsb; ++sb) {
    const uint8_t* tile = w + ((size_t)rg * nsb + sb) * UB + ti * TB;
    if (dtype == DT_Q4_K) {
      const uint32_t h = *reinterpret_cast<const uint32_t*>(tile + r16 * 16);
      const float d = guard_scale(half_bits_to_float(h & 0xffffu), 0.00000006f);
      const float dm = guard_scale(half_bits_to_float(h >> 16), 0.00000024f);
      bound = fmaxf(bound, fabsf(d) * 945.f + fabsf(dm) * 63.f);
    } else if (dtype == DT_Q6_K) {
      const float d = guard_scale(half_bits_to_float(reinterpret_cast<const uint16_t*>(tile)[r16]), 0.00000006f);
      bound = fmaxf(bound, fabsf(d) * 4096.f);
    } else {
      for (int i = 0; i < 8; ++i)
        bound = fmaxf(bound, fabsf(half_bits_to_float(reinterpret_cast<const uint16_t*>(tile + r16 * 16)[i])) * 128.f);
    }
  }
  int e = 0;
  if (bound > 0.f && isfinite(bound)) {
    int x;
    frexpf(bound, &x);  // bound < 2^x
    e = min(max(14 - x, -100), 100);
  }
  out[row] = (int8_t)e;
}

// ===========================================================================
// Exact-weight tcgen05 GEMM for Q4_K, 16..64 rows (prefill chunks, large
// scheduler steps).
//
// y = sum_sb d_sb * (sum_k sc_j q_k x_k) - dmin_sb * (sum_j m_j xsum_j) per row.
// The products sc_j * q_k are integers below 2^10, exact in fp16, so the A
// operand needs no hi/lo split: eight producer warps turn the 4-bit quants of
// a 128-row x 64-column slice into sc * q with two bit operations and one
// half2 fused multiply-add per pair. The activations come as fp16 hi/lo
// (x ~= 256 hi + lo, xfrag.cuh) stacked along N: N = 2 Np (hi rows, then lo
// rows), so one MMA per 16-column step accumulates both. The min term is a
// second MMA per slice with K = 16 (two live columns: the slice's two
// sub-blocks' mins times their activation sums). Each (128-row tile,
// super-block) run accumulates in its own TMEM pair (D, Dm; two pairs
// alternate) and four drain warps fold it into per-row registers with the
// super-block's d and dmin: y += d (256 D_hi + D_lo) - dmin (256 Dm_hi + Dm_lo).
// Work split, partial slots and the epilogue kernel are those of the hi/lo GEMM.
// Every mbarrier wait is bounded.
// ===========================================================================
constexpr int kQ2MaxStages = 6;
constexpr int kQ2SmemUse = 216 * 1024;
constexpr int kQ2Drain = 4;                     // warps 0-3: TMEM lanes 0-127
constexpr int kQ2Prod = 8;                      // warps 4-11: one 16-row tile each
constexpr int kQ2LoadWarp = kQ2Drain + kQ2Prod;  // 12: weight ring
constexpr int kQ2MmaWarp = kQ2LoadWarp + 1;      // 13
constexpr int kQ2BWarp = kQ2MmaWarp + 1;         // 14: activation planes
constexpr int kQ2Threads = 32 * (kQ2BWarp + 1);
constexpr int kQ2APlane = kQgRows * kQgKc * 2;   // 16 KB: 128 rows x 64 k fp16
constexpr int kQ2BPlane = 128 * kQgKc * 2;       // 16 KB: up to 128 N rows (hi, lo) x 64 k
constexpr int kQ2MPlane = 128 * 16 * 2;          // 4 KB: 128 rows x 16 k (min-term operands)
// stage: A plane | A min plane | B plane (N2 rows) | B min plane (N2 rows)
__host__ __device__ constexpr int q2_stage_bytes(int n2) { return kQ2APlane + kQ2MPlane + n2 * 64 * 2 + n2 * 16 * 2; }
constexpr int kQ2QStages = 3;  // weight ring: 18 KB per (128-row tile, super-block) run
__host__ __device__ constexpr int q2_stages(int n2) {
  return (kQ2SmemUse - kQ2QStages * 8 * 2304) / q2_stage_bytes(n2) > kQ2MaxStages
             ? kQ2MaxStages
             : (kQ2SmemUse - kQ2QStages * 8 * 2304) / q2_stage_bytes(n2);
}
constexpr int kQ2Lbo = 128 * 16;                 // bytes between 8-column chunks (all planes: 128 rows)
constexpr int kQ2Smem = kQ2SmemUse + 1024;

__device__ __forceinline__ uint32_t q2_off(int row, int col) {
  return (uint32_t)((col >> 3) * kQ2Lbo + (row >> 3) * 128 + (row & 7) * 16 + (col & 7) * 2);
}
// activation planes hold N2 = 2 Np rows: 8-column chunks N2 * 16 bytes apart
__host__ __device__ __forceinline__ uint32_t q2b_off(int n2, int row, int col) {
  return (uint32_t)((col >> 3) * n2 * 16 + (row >> 3) * 128 + (row & 7) * 16 + (col & 7) * 2);
}
// per 64-column slice, in global memory: the B plane (N2 x 64 fp16) then the
// min-term plane (N2 x 16 fp16), laid out as they sit in shared memory
__host__ __device__ constexpr int q2_bslice_bytes(int n2) { return n2 * 64 * 2 + n2 * 16 * 2; }
// half2 {v, v} of a small non-negative integer v (< 1024), exactly
__device__ __forceinline__ uint32_t h2_int(uint32_t v) {
  const uint32_t b = 0x6400u | v;  // fp16 1024 + v
  return hsub2_u(b | (b << 16), 0x64006400u);
}
// issues one 32-lane x 8-column load; tcgen05.wait::ld makes the registers valid
__device__ __forceinline__ void tmem_ld8_async(uint32_t taddr, uint32_t r[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float v[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// One 64-column slice (sub-blocks 2 grp, 2 grp + 1) of this warp's 16-row
// tile: A = sc * q at rows tw*16 + g, + 8; the mins of both sub-blocks into
// columns 0, 1 of the min plane; d, dmin into dd when `first` (run start).
__device__ __forceinline__ void q2_produce_a(const uint8_t* tile, int tw, int grp, int lane, uint32_t sA, uint32_t sAm,
                                             float2* dd, bool first) {
  const int g = lane >> 2, c = lane & 3;
  const uint4 hA = lds128(tile + g * 16);
  const uint4 hB = lds128(tile + (g + 8) * 16);
  const uint32_t scA_lo = hA.y & 0x3F3F3F3Fu, scA_hi = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
  const uint32_t mnA_lo = hA.z & 0x3F3F3F3Fu, mnA_hi = ((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u);
  const uint32_t scB_lo = hB.y & 0x3F3F3F3Fu, scB_hi = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
  const uint32_t mnB_lo = hB.z & 0x3F3F3F3Fu, mnB_hi = ((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u);
  const int rA = tw * 16 + g, rB = rA + 8;
  const uint4 q = lds128(tile + 256 + grp * 512 + lane * 16);
  const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int j = 2 * grp + h;
    const uint32_t sa = ((j < 4 ? scA_lo : scA_hi) >> (8 * (j & 3))) & 0xffu;
    const uint32_t sb = ((j < 4 ? scB_lo : scB_hi) >> (8 * (j & 3))) & 0xffu;
    const uint32_t ka = h2_int(sa), kb = h2_int(sb);
    const uint32_t na = h2_int(sa << 4) ^ 0x80008000u;     // -16 sc (x 64 below)
    const uint32_t nb = h2_int(sb << 4) ^ 0x80008000u;
    const uint32_t oa = h2_u32_mul(na, 0x54005400u);        // -16 sc * 64 = -1024 sc
    const uint32_t ob = h2_u32_mul(nb, 0x54005400u);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t w = wd[2 * h + half];
      const int col = 32 * h + 16 * half + 4 * c;
      const uint32_t w01 = prmt(w, 0u, 0x4140u), w23 = prmt(w, 0u, 0x4342u);
      const uint32_t s01 = w01 >> 4, s23 = w23 >> 4;
      // low nibbles: row g; high nibbles: row g + 8; (1024 + q) sc - 1024 sc = sc q
      const uint32_t a01 = hfma2_u(lop3_and_or(w01, 0x000F000Fu, 0x64006400u), ka, oa);
      const uint32_t a23 = hfma2_u(lop3_and_or(w23, 0x000F000Fu, 0x64006400u), ka, oa);
      const uint32_t b01 = hfma2_u(lop3_and_or(s01, 0x000F000Fu, 0x64006400u), kb, ob);
      const uint32_t b23 = hfma2_u(lop3_and_or(s23, 0x000F000Fu, 0x64006400u), kb, ob);
      sts64(sA + q2_off(rA, col), a01, a23);
      sts64(sA + q2_off(rB, col), b01, b23);
    }
  }
  if (c == 0) {
    // min plane: column 0 = m_{2 grp}, column 1 = m_{2 grp + 1} (the rest stays zero)
    const int j0 = 2 * grp, j1 = j0 + 1;
    const uint32_t ma0 = ((j0 < 4 ? mnA_lo : mnA_hi) >> (8 * (j0 & 3))) & 0xffu;
    const uint32_t ma1 = ((j1 < 4 ? mnA_lo : mnA_hi) >> (8 * (j1 & 3))) & 0xffu;
    const uint32_t mb0 = ((j0 < 4 ? mnB_lo : mnB_hi) >> (8 * (j0 & 3))) & 0xffu;
    const uint32_t mb1 = ((j1 < 4 ? mnB_lo : mnB_hi) >> (8 * (j1 & 3))) & 0xffu;
    sts32(sAm + q2_off(rA, 0), prmt(h2_int(ma0), h2_int(ma1), 0x5410u));
    sts32(sAm + q2_off(rB, 0), prmt(h2_int(mb0), h2_int(mb1), 0x5410u));
    if (first) {
      dd[rA] = make_float2(guard_scale(half_bits_to_float(hA.x), 0.00000006f),
                           guard_scale(half_bits_to_float(hA.x >> 16), 0.00000024f));
      dd[rB] = make_float2(guard_scale(half_bits_to_float(hB.x), 0.00000006f),
                           guard_scale(half_bits_to_float(hB.x >> 16), 0.00000024f));
    }
  }
}

// The activation planes of every 64-column slice, written once per GEMM from
// the fp16 hi/lo fragments: B rows [0, Np) the hi parts of tokens 0..Np-1,
// rows [Np, 2 Np) the lo parts (tokens >= m zero); the min-term plane holds the
// sums of the slice's two sub-blocks in columns 0, 1 (hi, lo rows likewise)
// and zeros in columns 2..15. One CTA per slice.
template <int NT>
__global__ void __launch_bounds__(256) q2_bprep_kernel(const uint4* xf, const uint32_t* xs, int m, int nt_x,
                                                       uint8_t* out) {
  constexpr int Np = 8 * NT, N2 = 2 * Np;
  const int kg = blockIdx.x, sb = kg >> 2, ks0 = (kg & 3) * 4;
  uint8_t* B = out + (size_t)kg * q2_bslice_bytes(N2);
  uint8_t* Bm = B + N2 * 64 * 2;
  pdl_wait();
  pdl_launch_dependents();
  for (int e = threadIdx.x; e < 4 * NT * 32; e += blockDim.x) {
    const int ksl = e / (NT * 32), rem = e % (NT * 32), nt = rem >> 5, l = rem & 31;
    const int t = nt * 8 + (l >> 2), col = 16 * ksl + 2 * (l & 3);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t < m) v = __ldg(xf + (((size_t)sb * nt_x + nt) * 16 + ks0 + ksl) * 32 + l);
    *reinterpret_cast<uint32_t*>(B + q2b_off(N2, t, col)) = v.x;
    *reinterpret_cast<uint32_t*>(B + q2b_off(N2, t, col + 8)) = v.y;
    *reinterpret_cast<uint32_t*>(B + q2b_off(N2, Np + t, col)) = v.z;
    *reinterpret_cast<uint32_t*>(B + q2b_off(N2, Np + t, col + 8)) = v.w;
  }
  for (int e = threadIdx.x; e < N2 * 8; e += blockDim.x) {  // (row, pair of columns)
    const int row = e >> 3, cp = (e & 7) * 2;
    uint32_t w = 0u;
    if (cp == 0) {
      const int t = row < Np ? row : row - Np;
      if (t < m) {
        const uint32_t* src = xs + (((size_t)sb * nt_x + (t >> 3)) * 8 + (t & 7)) * 8 + 2 * (kg & 3);
        const uint32_t s0 = __ldg(src), s1 = __ldg(src + 1);
        w = row < Np ? prmt(s0, s1, 0x5410u) : prmt(s0, s1, 0x7632u);
      }
    }
    *reinterpret_cast<uint32_t*>(Bm + q2b_off(N2, row, cp)) = w;
  }
}

template <int NT>
__global__ void __launch_bounds__(kQ2Threads, 1) qgemm2_kernel(const __grid_constant__ QgemmArgs a) {
  constexpr int Np = 8 * NT, N2 = 2 * Np;
  constexpr int TB = tile_bytes(DT_Q4_K), HU = 8 * TB;
  constexpr int QS = kQ2QStages;
  constexpr int kQ2Stages = q2_stages(N2), kQ2Stage = q2_stage_bytes(N2);
  constexpr int kOffAm = kQ2APlane, kOffB = kQ2APlane + kQ2MPlane, kOffBm = kOffB + N2 * 64 * 2;
  constexpr uint32_t kCols = 8 * Np <= 32 ? 32 : (8 * Np <= 64 ? 64 : (8 * Np <= 128 ? 128 : (8 * Np <= 256 ? 256 : 512)));
  static_assert(QS >= 2, "weight ring");
  extern __shared__ __align__(1024) uint8_t q2_smem_raw[];
  __shared__ uint64_t sfull[kQ2MaxStages], sfree[kQ2MaxStages];
  __shared__ uint64_t qfull[kQ2QStages], qempty[kQ2QStages];
  // d, dmin of each run's rows: four slots, so producers run up to four runs
  // ahead of the drain (the TMEM pairs alternate between two)
  constexpr int kDd = 4;
  __shared__ uint64_t accfull[2], accempty[2], ddfull[kDd], ddempty[kDd], bfull[kQ2MaxStages];
  __shared__ float2 dd[kDd][kQgRows];
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q2_smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  uint8_t* qring = smem + kQ2Stages * kQ2Stage;
  const int n_rt = 2 * a.n_rg, kG = 4 * a.nsb;
  const long long U = (long long)n_rt * kG;
  const int G = gridDim.x, cta = blockIdx.x;
  const long long u0 = U * cta / G, u1 = U * (cta + 1) / G;
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // the A min plane's unused columns 2..15 stay zero for the whole launch
  for (int i = tid; i < kQ2Stages * kQ2MPlane / 16; i += blockDim.x) {
    const int st = i / (kQ2MPlane / 16), r = i % (kQ2MPlane / 16);
    *reinterpret_cast<uint4*>(smem + st * kQ2Stage + kOffAm + r * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
  if (tid == 0) {
    for (int i = 0; i < kQ2Stages; ++i) {
      mbar_init(&sfull[i], kQ2Prod);
      mbar_init(&sfree[i], 1);
      mbar_init(&bfull[i], 1);
    }
    for (int i = 0; i < QS; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], kQ2Prod);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accfull[i], 1);
      mbar_init(&accempty[i], kQ2Drain);
    }
    for (int i = 0; i < kDd; ++i) {
      mbar_init(&ddfull[i], kQ2Prod);
      mbar_init(&ddempty[i], kQ2Drain);    }
    fence_barrier_init();
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // a run: a maximal stretch of slices inside one (128-row tile, super-block)
  auto run_end = [&](long long u) { return min(u1, (u / 4 + 1) * 4); };

  if (warp == kQ2LoadWarp) {
    // ---- loader: the eight 16-row tiles of each (tile, super-block) run ----
    if (lane == 0) {
      long long iq = 0;
      bool ok = true;
      for (long long u = u0; ok && u < u1; u = run_end(u)) {
        const int rt = (int)(u / kG), sb = (int)((u - (long long)rt * kG) >> 2);
        const int rg = rt >> 1, half = rt & 1;
        const int q = (int)(iq % QS);
        if (iq >= QS && !mbar_wait(&qempty[q], (uint32_t)((iq / QS - 1) & 1), a.err, DEV_TIMEOUT_SMEM)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&qfull[q], HU);
        bulk_g2s(qring + (size_t)q * HU, a.w + ((size_t)rg * a.nsb + sb) * unit_bytes(DT_Q4_K) + (size_t)half * 8 * TB,
                 HU, &qfull[q]);
        ++iq;
      }
      for (long long j = iq > QS ? iq - QS : 0; j < iq; ++j)
        mbar_wait(&qfull[j % QS], (uint32_t)((j / QS) & 1), nullptr, 0);
    }
    __syncwarp();
  } else if (warp == kQ2BWarp) {
    // ---- activation planes of every slice, copied from the prepared buffer ----
    if (lane == 0) {
      pdl_wait();
      constexpr uint32_t BB = N2 * 64 * 2, BM = N2 * 16 * 2;
      long long it = 0;
      for (long long u = u0; u < u1; ++u, ++it) {
        const int s = (int)(it % kQ2Stages);
        if (it >= kQ2Stages && !mbar_wait(&sfree[s], (uint32_t)((it / kQ2Stages - 1) & 1), a.err, DEV_TIMEOUT_EMPTY))
          break;
        // the planes sit back to back in the prepared buffer and in the stage
        const uint8_t* src = a.bprep + (size_t)(u % kG) * q2_bslice_bytes(N2);
        mbar_arrive_expect_tx(&bfull[s], BB + BM);
        bulk_g2s(smem + s * kQ2Stage + kOffB, src, BB + BM, &bfull[s]);
      }
      for (long long j = it > kQ2Stages ? it - kQ2Stages : 0; j < it; ++j)
        mbar_wait(&bfull[j % kQ2Stages], (uint32_t)((j / kQ2Stages) & 1), nullptr, 0);
    }
    __syncwarp();
  } else if (warp == kQ2MmaWarp) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_f16(kQgRows, N2);
      long long it = 0, gi = 0;
      bool ok = true;
      for (long long u = u0; ok && u < u1; ++gi) {
        const long long ue = run_end(u);
        const int b = (int)(gi & 1);
        if (gi >= 2 && !mbar_wait(&accempty[b], (uint32_t)((gi / 2 - 1) & 1), a.err, DEV_TIMEOUT_DRAIN)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dmain = tmem + (uint32_t)(b * 2 * N2), dmin = dmain + (uint32_t)N2;
        for (bool first = true; u < ue; ++u, ++it, first = false) {
          const int s = (int)(it % kQ2Stages);
          if (!mbar_wait(&sfull[s], (uint32_t)((it / kQ2Stages) & 1), a.err, DEV_TIMEOUT_FULL) ||
              !mbar_wait(&bfull[s], (uint32_t)((it / kQ2Stages) & 1), a.err, DEV_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + s * kQ2Stage;
          if (!(a.dbg & 2)) {
            constexpr uint32_t kBLbo = N2 * 16;
#pragma unroll
            for (int ks = 0; ks < kQgKc / 16; ++ks)
              umma_f16(dmain, umma_desc(st + ks * 2 * kQ2Lbo, kQ2Lbo, 128),
                       umma_desc(st + kOffB + ks * 2 * kBLbo, kBLbo, 128), idesc, (first && ks == 0) ? 0u : 1u);
            umma_f16(dmin, umma_desc(st + kOffAm, kQ2Lbo, 128), umma_desc(st + kOffBm, kBLbo, 128), idesc,
                     first ? 0u : 1u);
          }
          umma_commit(&sfree[s]);
        }
        if (!ok) break;
        umma_commit(&accfull[b]);
      }
      if (it > 0) {
        const long long last = it - 1;
        mbar_wait(&sfree[last % kQ2Stages], (uint32_t)((last / kQ2Stages) & 1), nullptr, 0);
      }
    }
    __syncwarp();
  } else if (warp >= kQ2Drain) {
    // ---- producers (warps 4-11): A = sc * q, min plane, d / dmin, activations ----
    const int pw = warp - kQ2Drain;
    bool alive = true;
    long long it = 0, iq = 0, gi = 0;
    for (long long u = u0; alive && u < u1; ++gi) {
      const long long ue = run_end(u);
      const int b = (int)(gi & 1);
      const int q = (int)(iq % QS);
      alive = mbar_wait(&qfull[q], (uint32_t)((iq / QS) & 1), a.err, DEV_TIMEOUT_FULL);
      // dd slot gi % kDd was last read by the drain of run gi - kDd
      const int ds = (int)(gi % kDd);
      if (alive && gi >= kDd)
        alive = mbar_wait(&ddempty[ds], (uint32_t)((gi / kDd - 1) & 1), a.err, DEV_TIMEOUT_DRAIN);
      for (bool first = true; alive && u < ue; ++u, ++it) {
        const int kg = (int)(u % kG);
        const int s = (int)(it % kQ2Stages);
        if (it >= kQ2Stages)
          alive = mbar_wait(&sfree[s], (uint32_t)((it / kQ2Stages - 1) & 1), a.err, DEV_TIMEOUT_EMPTY);
        if (!alive) break;
        const uint32_t st = sbase + s * kQ2Stage;
        if (!(a.dbg & 1))
          q2_produce_a(qring + (size_t)q * HU + pw * TB, pw, kg & 3, lane, st, st + kOffAm, dd[ds], first);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (first) mbar_arrive(&ddfull[ds]);
          mbar_arrive(&sfull[s]);
          if (u + 1 == ue) mbar_arrive(&qempty[q]);
        }
        __syncwarp();
        first = false;
      }
      ++iq;
    }
  } else {
    // ---- drain (warps 0-3): row 32 warp + lane of the 128-row tile ----
    const int row = 32 * warp + lane;
    float y[Np];
#pragma unroll
    for (int t = 0; t < Np; ++t) y[t] = 0.f;
    bool alive = true;
    long long gi = 0;
    for (long long u = u0; alive && u < u1; ++gi) {
      const long long ue = run_end(u);
      const int rt = (int)(u / kG);
      const int b = (int)(gi & 1);
      alive = mbar_wait(&accfull[b], (uint32_t)((gi / 2) & 1), a.err, DEV_TIMEOUT_DRAIN) &&
              mbar_wait(&ddfull[gi % kDd], (uint32_t)((gi / kDd) & 1), a.err, DEV_TIMEOUT_DRAIN);
      __syncwarp();
      if (!alive) break;
      tc_fence_after();
      const float d = dd[gi % kDd][row].x, dm = dd[gi % kDd][row].y;
      __syncwarp();
      if (lane == 0) mbar_arrive(&ddempty[gi % kDd]);
      const uint32_t tl = tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(b * 2 * N2);
#pragma unroll
      for (int t0 = 0; t0 < Np; t0 += 8) {
        uint32_t dh[8], dl[8], mh[8], ml[8];
        tmem_ld8_async(tl + t0, dh);
        tmem_ld8_async(tl + Np + t0, dl);
        tmem_ld8_async(tl + N2 + t0, mh);
        tmem_ld8_async(tl + N2 + Np + t0, ml);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 8; ++i)
          y[t0 + i] = fmaf(-dm, fmaf(256.0f, __uint_as_float(mh[i]), __uint_as_float(ml[i])),
                           fmaf(d, fmaf(256.0f, __uint_as_float(dh[i]), __uint_as_float(dl[i])), y[t0 + i]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[b]);
      u = ue;
      if (u == u1 || u % kG == 0) {
        // segment end: this CTA's share of tile rt into its partial slot
        const int slot = cta - qg_owner((long long)rt * kG, U, G);
        float* dst = a.part + ((size_t)rt * a.slots + slot) * kMaxTokens * kQgRows + row;
#pragma unroll
        for (int t = 0; t < Np; ++t) {
          if (t < a.m) dst[(size_t)t * kQgRows] = y[t];
          y[t] = 0.f;
        }
      }
    }
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

template <int NT>
cudaError_t launch_q2_bprep_t(const QgemmArgs& q, uint8_t* out, cudaStream_t s, int pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(4 * q.nsb);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, q2_bprep_kernel<NT>, q.xf, q.xs, q.m, q.nt_x, out);
}

template <int NT>
cudaError_t launch_qgemm2_t(const QgemmArgs& q, int G, cudaStream_t s, int pdl) {
  auto kern = qgemm2_kernel<NT>;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cudaError_t e = ensure_smem_attr(kern, kQ2Smem, dev)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kQ2Threads);
  cfg.dynamicSmemBytes = kQ2Smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, q);
}

cudaError_t launch_qgemm_epi(const GemvArgs& a, const QgemmTail& q, cudaStream_t s, int pdl) {
  const int smem = (kConsumerWarps * kMaxTokens + kMaxTokens + tile_floats(1)) * 4;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cudaError_t e = ensure_smem_attr(qgemm_epi_kernel, smem, dev)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_rg, gemv_nt_for(a.m));
  cfg.blockDim = dim3(kConsumerWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, qgemm_epi_kernel, a, q);
}

template <int DT>
cudaError_t launch_qgemm_t(const QgemmArgs& q, int G, cudaStream_t s, int pdl) {
  auto kern = qgemm_kernel<DT>;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cudaError_t e = ensure_smem_attr(kern, kQgSmem, dev)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kQgThreads);
  cfg.dynamicSmemBytes = kQgSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, q);
}

}  // namespace

int gemv_nt_for(int m) { return m <= 8 ? 1 : m <= 16 ? 2 : m <= 32 ? 4 : 8; }

int gemv_ctas(int num_sms, int n_rg, int nsb) {
  const long long U = (long long)n_rg * nsb;
  return (int)(U < num_sms ? U : num_sms);
}

size_t gemv_partials_floats(int num_ctas, int nt, int n_phases) {
  return (size_t)num_ctas * (n_phases > 1 ? 4 : 2) * kConsumerWarps * nt * 128;
}


cudaError_t gemv_chain_launch(const ChainArgs& c, int num_sms, cudaStream_t s, int pdl) {
  if (c.n_phases < 1 || c.n_phases > kMaxPhases) return cudaErrorInvalidValue;
  if (c.n_phases > 1 && !c.gbar) return cudaErrorInvalidValue;
  const int m = c.ph[0].m;
  for (int p = 0; p < c.n_phases; ++p) {
    const GemvArgs& a = c.ph[p];
    if (a.m != m || a.m < 1 || a.m > kMaxTokens) return cudaErrorInvalidValue;
    if (a.dtype != DT_Q4_K && a.dtype != DT_Q6_K && a.dtype != DT_Q8_0) return cudaErrorInvalidValue;
    // a second weight: same format, or Q6_K after Q4_K, in a QKV epilogue
    if (a.n_rg2 && (!a.w2 || a.epi != EPI_QKV ||
                    !(gemv_nt_for(a.m) == 1 ? (a.dtype == DT_Q4_K ? a.dtype2 == DT_Q6_K : a.dtype2 == a.dtype)
                                             : a.dtype2 == a.dtype)))
      return cudaErrorInvalidValue;
  }
  switch (gemv_nt_for(m)) {
    case 1: return launch_chain_t<1>(c, num_sms, s, pdl);
    case 2: return launch_chain_t<2>(c, num_sms, s, pdl);
    case 4: return launch_chain_t<4>(c, num_sms, s, pdl);
    default: return launch_chain_t<8>(c, num_sms, s, pdl);
  }
}

cudaError_t gemv_launch(const GemvArgs& a, int num_sms, cudaStream_t s, int pdl) {
  ChainArgs c;
  c.ph[0] = a;
  c.n_phases = 1;
  return gemv_chain_launch(c, num_sms, s, pdl);
}

cudaError_t repack_launch(const uint8_t* a, int rows_a, const uint8_t* b, int rows_b, int mode, int dtype, int k,
                          uint8_t* out, int n_rg, cudaStream_t s) {
  const long long tiles = (long long)n_rg * (k / kSuperK) * kUnitTiles;
  if (tiles == 0) return cudaSuccess;
  switch (dtype) {
    case DT_Q4_K: repack_kernel<DT_Q4_K><<<(unsigned)tiles, 128, 0, s>>>(a, rows_a, b, rows_b, mode, k, out, n_rg); break;
    case DT_Q6_K: repack_kernel<DT_Q6_K><<<(unsigned)tiles, 128, 0, s>>>(a, rows_a, b, rows_b, mode, k, out, n_rg); break;
    case DT_Q8_0: repack_kernel<DT_Q8_0><<<(unsigned)tiles, 128, 0, s>>>(a, rows_a, b, rows_b, mode, k, out, n_rg); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t unpack_launch(const uint8_t* tiled, int dtype, int n, int k, uint8_t* out, cudaStream_t s) {
  if (dtype != DT_Q4_K) return cudaErrorInvalidValue;
  const int n_rg = (n + kRowGroup - 1) / kRowGroup;
  const long long tiles = (long long)n_rg * (k / kSuperK) * kUnitTiles;
  unpack_kernel<DT_Q4_K><<<(unsigned)tiles, 128, 0, s>>>(tiled, n, k, out);
  return cudaGetLastError();
}

cudaError_t dequant_launch(int dtype, const uint8_t* blocks, size_t nblocks, float* out, cudaStream_t s) {
  if (nblocks == 0) return cudaSuccess;
  const size_t total = nblocks * block_elems(dtype);
  const unsigned grid = (unsigned)((total + 255) / 256 < 65535 * 16 ? (total + 255) / 256 : 65535 * 16);
  dequant_kernel<<<grid, 256, 0, s>>>(dtype, blocks, nblocks, out);
  return cudaGetLastError();
}

cudaError_t xfrag_launch(const float* x, int ldx, const float* w, int m, int k, int nt, const XFrags& out, float* ss,
                         int ld_ss, cudaStream_t s) {
  if (m < 1 || k % 256 || nt * 8 < m) return cudaErrorInvalidValue;
  xfrag_kernel<<<dim3(k / 256, (m + 7) / 8), 128, 0, s>>>(x, ldx, w, m, k, nt, out, ss, ld_ss);
  return cudaGetLastError();
}

cudaError_t quantize_launch(int dtype, const float* x, size_t n, uint8_t* out, cudaStream_t s) {
  const size_t be = block_elems(dtype);
  if (n % be) return cudaErrorInvalidValue;
  const size_t nb = n / be;
  if (nb == 0) return cudaSuccess;
  quantize_kernel<<<(unsigned)((nb + 127) / 128), 128, 0, s>>>(dtype, x, nb, out);
  return cudaGetLastError();
}


QgemmPlan qgemm_plan(int num_sms, int n_rg, int nsb) {
  QgemmPlan p;
  p.n_rt = 2 * n_rg;
  p.kG = 4 * nsb;
  p.U = (long long)p.n_rt * p.kG;
  p.G = (int)(p.U < num_sms ? p.U : num_sms);
  p.slots = 1;
  for (int rt = 0; rt < p.n_rt; ++rt) {
    const int c0 = qg_owner((long long)rt * p.kG, p.U, p.G), c1 = qg_owner((long long)rt * p.kG + p.kG - 1, p.U, p.G);
    p.slots = c1 - c0 + 1 > p.slots ? c1 - c0 + 1 : p.slots;
  }
  return p;
}

size_t qgemm_part_floats(const QgemmPlan& p) { return (size_t)p.n_rt * p.slots * kMaxTokens * kQgRows; }

cudaError_t rowexp_launch(const uint8_t* tiled, int dtype, int n_rg, int nsb, int8_t* out, cudaStream_t s) {
  const int rows = n_rg * kRowGroup;
  if (rows == 0) return cudaSuccess;
  rowexp_kernel<<<(rows + 255) / 256, 256, 0, s>>>(tiled, dtype, n_rg, nsb, out);
  return cudaGetLastError();
}

size_t qgemm_bprep_bytes(int nsb) { return (size_t)4 * nsb * q2_bslice_bytes(2 * kMaxTokens); }

cudaError_t qgemm_launch(const GemvArgs& a, float* part, uint8_t* bprep, const QgemmPlan& p, cudaStream_t s,
                         int pdl) {
  const int8_t* rexp = a.rexp;
  if (a.m < 16 || a.m > kMaxTokens || !a.xin.xf || !rexp || !part || p.G < 1 || a.n_rg2) return cudaErrorInvalidValue;
  QgemmArgs q;
  q.w = a.w;
  q.xs = a.xin.xs;
  q.dtype = a.dtype;
  q.n_rg = a.n_rg;
  q.nsb = a.nsb;
  q.m = a.m;
  q.nt_x = gemv_nt_for(a.m);
  q.xf = a.xin.xf;
  q.rexp = rexp;
  q.part = part;
  q.slots = p.slots;
  q.dbg = a.dbg >> 4;
  q.err = a.err;
  cudaError_t e;
  const bool exact = a.dtype == DT_Q4_K && a.xin.xs && bprep && !(a.dbg & 0x100);  // exact-weight GEMM for Q4_K
  q.bprep = bprep;
  switch (exact ? -1 : a.dtype) {
    case -1:
      switch (gemv_nt_for(a.m)) {
        case 2:
          e = launch_q2_bprep_t<2>(q, bprep, s, pdl);
          if (e == cudaSuccess) e = launch_qgemm2_t<2>(q, p.G, s, pdl);
          break;
        case 4:
          e = launch_q2_bprep_t<4>(q, bprep, s, pdl);
          if (e == cudaSuccess) e = launch_qgemm2_t<4>(q, p.G, s, pdl);
          break;
        default:
          e = launch_q2_bprep_t<8>(q, bprep, s, pdl);
          if (e == cudaSuccess) e = launch_qgemm2_t<8>(q, p.G, s, pdl);
          break;
      }
      break;
    case DT_Q4_K: e = launch_qgemm_t<DT_Q4_K>(q, p.G, s, pdl); break;
    case DT_Q6_K: e = launch_qgemm_t<DT_Q6_K>(q, p.G, s, pdl); break;
    case DT_Q8_0: e = launch_qgemm_t<DT_Q8_0>(q, p.G, s, pdl); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  QgemmTail t;
  t.part = part;
  t.rexp = exact ? nullptr : rexp;
  t.slots = p.slots;
  t.G = p.G;
  t.kG = p.kG;
  t.U = p.U;
  return launch_qgemm_epi(a, t, s, pdl);
}

}  // namespace rb
