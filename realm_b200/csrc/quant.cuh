// GGUF block formats, the tensor-core tile layout the GEMV streams, and the
// per-element device dequantisation (bit-exact with the reference's
// dequantize_q4_k / q6_k / q8_0, crates/realm-core/src/quant.rs:127-187,
// 393-451, 371-387).
#pragma once
#include "common.cuh"

namespace rb {

enum Dtype : int32_t { DT_F32 = 0, DT_F16 = 1, DT_Q8_0 = 8, DT_Q4_K = 12, DT_Q6_K = 14 };

// GGUF block geometry.
__host__ __device__ constexpr int block_bytes(int dt) {
  return dt == DT_Q4_K ? 144 : dt == DT_Q6_K ? 210 : dt == DT_Q8_0 ? 34 : dt == DT_F16 ? 2 : 4;
}
__host__ __device__ constexpr int block_elems(int dt) {
  return (dt == DT_Q4_K || dt == DT_Q6_K) ? 256 : dt == DT_Q8_0 ? 32 : 1;
}

// ---------------------------------------------------------------------------
// Tiled layout ("mma tiles"). A weight W[N][K] is cut into 16-row x 256-column
// tiles; 16 tiles stacked vertically (256 rows) at one 256-column position form
// a streaming unit. Units are stored row-group-major, then by K position, so a
// row group's whole K range is one contiguous run of bytes. Inside a tile the
// quantised values are pre-permuted into the m16n8k16 A-fragment order, so each
// lane fetches its operands with 16-byte shared-memory loads and never shuffles.
// The byte count equals the GGUF byte count (no expansion):
//   Q4_K tile 2304 B = 16 rows x 144 B:  [16 x {d, dmin, scales[12]}][qs 2048 B]
//   Q6_K tile 3360 B = 16 rows x 210 B:  [16 x d][16 x scales[16]][lo nibbles 2048 B][hi 2 bits 1024 B]
//   Q8_0 tile 4352 B = 16 rows x 8 x 34: [16 x 8 x d][q+128 as u8, 4096 B]
// Per k-step (16 columns) each lane owns 8 values v0..v7 of rows g=lane/4 and g+8
// at columns c2=2*(lane%4) (+1, +8, +9):
//   v0=(g,c2) v4=(g,c2+1) v1=(g+8,c2) v5=(g+8,c2+1) v2=(g,c2+8) v6=(g,c2+9) v3=(g+8,c2+8) v7=(g+8,c2+9)
// so that (word >> 4r) & 0x000F000F is A-fragment register r (low/high halves).
// ---------------------------------------------------------------------------
constexpr int kTileRows = 16;
constexpr int kUnitTiles = 16;  // tiles per unit => 256 rows per row group
constexpr int kRowGroup = kTileRows * kUnitTiles;
constexpr int kSuperK = 256;

__host__ __device__ constexpr int tile_bytes(int dt) {
  return dt == DT_Q4_K ? 2304 : dt == DT_Q6_K ? 3360 : dt == DT_Q8_0 ? 4352 : 0;
}
__host__ __device__ constexpr int unit_bytes(int dt) { return tile_bytes(dt) * kUnitTiles; }

// Position (row-in-tile, column-in-k-step) of value i (0..7) held by `lane`.
__host__ __device__ inline void frag_pos(int lane, int i, int& row, int& col) {
  const int g = lane >> 2, c2 = (lane & 3) * 2;
  const int r = i & 3, hi = i >> 2;  // r: register, hi: upper half
  row = g + ((r & 1) ? 8 : 0);
  col = c2 + ((r & 2) ? 8 : 0) + hi;
}

// ---- reference dequantisation of one GGUF element (bit-exact, no FMA) ----
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t* s, int& sc, int& m) {
  // crates/realm-core/src/quant.rs:108-122 get_scale_min_k4
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// element e (0..255) of a Q4_K block -> its 4-bit quant
__device__ __forceinline__ int q4k_quant(const uint8_t* qs, int e) {
  const int grp = e >> 6, w = e & 63;
  const uint8_t b = qs[32 * grp + (w & 31)];
  return (w < 32) ? (b & 0xF) : (b >> 4);
}

__device__ __forceinline__ float dequant_q4k_elem(const uint8_t* blk, int e) {
  const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
  const float mn = half_bits_to_float(blk[2] | (blk[3] << 8));
  int sc, m;
  q4k_scale_min(e >> 5, blk + 4, sc, m);
  const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(mn, (float)m);
  return __fsub_rn(__fmul_rn(d1, (float)q4k_quant(blk + 16, e)), m1);
}

// element e of a Q6_K block -> signed 6-bit quant (quant.rs:411-449 index map)
__device__ __forceinline__ int q6k_quant(const uint8_t* blk, int e) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  const int h = e >> 7, r = e & 127, t = r >> 5, l = r & 31;
  const uint8_t lo = ql[64 * h + l + ((t & 1) ? 32 : 0)];
  const int nib = (t & 2) ? (lo >> 4) : (lo & 0xF);
  const int hb = (qh[32 * h + l] >> (2 * t)) & 3;
  return (nib | (hb << 4)) - 32;
}
__device__ __forceinline__ int q6k_scale(const uint8_t* blk, int e) {
  return (int)(int8_t)blk[192 + (e >> 4)];
}
__device__ __forceinline__ float dequant_q6k_elem(const uint8_t* blk, int e) {
  const float d = half_bits_to_float(blk[208] | (blk[209] << 8));
  return __fmul_rn(__fmul_rn(d, (float)q6k_scale(blk, e)), (float)q6k_quant(blk, e));
}

__device__ __forceinline__ float dequant_q80_elem(const uint8_t* blk, int e) {
  const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
  return __fmul_rn((float)(int8_t)blk[2 + e], d);
}

}  // namespace rb
