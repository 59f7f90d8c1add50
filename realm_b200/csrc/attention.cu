// Paged KV cache + paged GQA decode attention (sm_100a).
//
// Replaces the reference's contiguous fp32 KVCache (crates/realm-models/src/kv_cache.rs:7-80),
// repeat_kv + StandardAttention (crates/realm-models/src/attention.rs:272-380,
// crates/realm-models/src/attention_stub/mod.rs:42-158). The reference has no paged
// cache; here K/V live in 16-token pages reached through a per-tenant page table.
//
// Decode attention, stream-K over pages: the 16-token pages of every
// (query row, kv head) pair form one sequence and each CTA takes an equal
// contiguous share, so every CTA streams the same number of bytes whatever the
// context lengths. Within a pair's segment each of the CTA's 4 warps streams
// every 4th page (K and V blocks of one kv head, contiguous) with the
// bulk-copy engine into a private ring, so every KV page is read from HBM once
// per GQA group. With fp16 K/V the scores and P.V run on the tensor cores
// (mma.sync m16n8k16; query and probabilities as fp16 hi + lo), with an online
// softmax per query head in fp32; fp32 K/V take a scalar path. Warps merge
// through shared memory; a pair split over CTAs is combined by the last CTA to
// finish it, in CTA order (deterministic, no spin waits).
#include "attention.cuh"
#include "common.cuh"
#include "xfrag.cuh"

namespace rb {

namespace {

constexpr int kAttnWarps = 4;
constexpr int kMaxRows = 64;

// Scratch of the decode kernel on num_ctas CTAs: two pair partials per CTA
// (query columns: attn_cols).
__host__ __device__ constexpr size_t decode_partials_floats(int num_ctas, int n_rep, int hd) {
  return (size_t)num_ctas * 2 * (n_rep < 4 ? 4 : n_rep) * (hd + 2);
}

// ring stages per warp: two CTAs of 4 warps per SM with three stages each keep
// ~190 KB of fp16 K/V in flight per SM at hd 128. (Three CTAs with two stages,
// the same bytes, measured 1.7 % slower per decode step once decode steps ran
// whole pairs: 3.601 vs 3.541 ms.)
__host__ __device__ constexpr int attn_ring(int hd, int f16, int nrep) {
  return hd == 128 ? (f16 ? 3 : 1) : 3;
}


template <int HD, int F16, int NREP = 1>
struct AttnCfg {
  static constexpr int ESZ = F16 ? 2 : 4;
  static constexpr int BLK = 16 * HD * ESZ;  // one page of one kv head (K or V), bytes
  static constexpr int NSW = attn_ring(HD, F16, NREP);
  // fp16 blocks arrive by TMA as HD / 64 boxes of 16 rows x 128 bytes with
  // 128-byte swizzle (each box 1024-byte aligned), fp32 blocks by a plain bulk copy
  static constexpr int SBLK = BLK;
  static constexpr int STAGE = 2 * SBLK;
};

// Query columns per (row group, kv head) pair: in the grouped variant (GR) the
// n_rep heads of up to NC / n_rep consecutive rows of one tenant (a prompt
// chunk) share every K/V page. fp16 pools only; 4 columns keep two CTAs per SM.
// Steps without such rows (decode) run the ungrouped variant and its smaller
// shared-memory footprint.
template <int NREP, int F16, int GR = 1>
__host__ __device__ constexpr int attn_cols() {
  return (GR && F16 && NREP < 4) ? 4 : NREP;
}

template <int HD, int NREP, int F16, int GR>
__host__ __device__ constexpr int attn_smem_bytes() {
  return 1024                                                           // ring alignment
         + kAttnWarps * AttnCfg<HD, F16, NREP>::NSW * AttnCfg<HD, F16, NREP>::STAGE  // rings
         + attn_cols<NREP, F16, GR>() * HD * 4                              // q
         + kAttnWarps * (NREP > 8 ? NREP : 8) * 16 * 4                 // probabilities
         + kAttnWarps * attn_cols<NREP, F16, GR>() * (HD + 2) * 4           // warp merge
         + kAttnWarps * AttnCfg<HD, F16, NREP>::NSW * 8                // mbarriers
         + kMaxRows * 8 + 64;                                          // row tables
}

__device__ __forceinline__ void to_f32(const uint4 raw, float* f, int f16) {
  if (f16) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __half22float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  } else {
    f[0] = __uint_as_float(raw.x);
    f[1] = __uint_as_float(raw.y);
    f[2] = __uint_as_float(raw.z);
    f[3] = __uint_as_float(raw.w);
  }
}

// Byte offset of (token row r, 16-byte chunk k of the head_dim row) in a block
// stored as 128-byte-swizzled boxes of 16 rows x 64 fp16 columns.
__device__ __forceinline__ int swz(int r, int k) {
  return (k >> 3) * 2048 + r * 128 + (((k & 7) ^ (r & 7)) << 4);
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
// two fp32 values -> packed fp16 hi and lo parts (x ~= hi + lo, ~22 bits)
// (paired conversions: hi = RN(x), lo = RN(x - hi), two values per instruction)
__device__ __forceinline__ void pack_hilo(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x0, x1);
  const float2 f = __half22float2(h);
  const __half2 l = __floats2half2_rn(x0 - f.x, x1 - f.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}
// 2^x by the hardware approximation (relative error below 2^-22; flushes
// subnormal results to zero, which the softmax weights absorb)
__device__ __forceinline__ float exp2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A segment: this CTA's share of one (row, kv head) pair, pages [p_begin, p_end)
// of the pair; x0, x1 its place in the global page sequence, ps, pe the pair's.
__device__ __forceinline__ void attn_stamp(const AttnArgs& a, int slot) {
  if (a.dbg_ts && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    a.dbg_ts[(size_t)blockIdx.x * 8 + slot] = t;
  }
}

// Row r belongs to a prompt chunk: a run of consecutive rows of one tenant at
// consecutive positions, at least two rows long.
__device__ __forceinline__ bool row_in_chunk(const int* rt, const int* rp, int n, int r) {
  return (r > 0 && rt[r - 1] == rt[r] && rp[r - 1] + 1 == rp[r]) ||
         (r + 1 < n && rt[r + 1] == rt[r] && rp[r] + 1 == rp[r + 1]);
}

struct UnitInfo {
  int row, nr, kvh, p_begin, p_end, len;  // row: first row of the group, nr rows
  long long x0, x1, ps, pe;
  bool valid;
};

template <int HD, int NREP, int F16, int GR>
__global__ void __launch_bounds__(kAttnWarps * 32, 3) attn_kernel(const __grid_constant__ AttnArgs a) {
  using C = AttnCfg<HD, F16, NREP>;
  constexpr int NSW = C::NSW;
  constexpr int NC = attn_cols<NREP, F16, GR>(), RG = NC / NREP;  // query columns, rows per group
  extern __shared__ __align__(128) uint8_t smem_raw[];
  // the swizzle pattern of TMA boxes follows shared-memory address bits: align to 1 KB
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* rings = smem;
  float* qs = reinterpret_cast<float*>(rings + kAttnWarps * NSW * C::STAGE);
  float* pb = qs + NC * HD;
  float* mrg = pb + kAttnWarps * (NREP > 8 ? NREP : 8) * 16;
  uint64_t* bars = reinterpret_cast<uint64_t*>(mrg + kAttnWarps * NC * (HD + 2));
  long long* row_pages = reinterpret_cast<long long*>(bars + kAttnWarps * NSW);  // prefix of pages per row group
  __shared__ int s_last, s_ng, s_whole;
  __shared__ int g_row0[kMaxRows], g_nr[kMaxRows];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kv = a.kv.n_kv;
  const int G = gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kAttnWarps * NSW; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  attn_stamp(a, 0);
  pdl_launch_dependents();
  // Positions, tenants and page tables are written before the previous kernel
  // (by the host or an earlier kernel), and so are all cached K/V except the
  // new tokens that the previous kernel appends: pages wholly below the
  // smallest position of this launch's rows are streamed before waiting for it.
  __shared__ int s_pos_min;
  // the rows' tenants and positions, read once (coalesced) into shared memory
  __shared__ int s_rt[kMaxRows], s_rp[kMaxRows];
  for (int i = threadIdx.x; i < a.n_rows; i += blockDim.x) {
    s_rt[i] = a.row_tenant[i];
    s_rp[i] = a.row_pos[i];
  }
  __syncthreads();
  // Rows group by tenant: up to RG consecutive rows of one tenant at
  // consecutive positions share a pair (the last has the largest position).
  // Stream-K over pages: the pages of all (row group, kv head) pairs form one
  // sequence (group-major, kv head, page); CTA b takes [P b / Gp, P (b+1) / Gp).
  if (threadIdx.x == 0) {
    long long acc = 0;
    int pmin = 0x7fffffff, ng = 0;
    for (int r = 0; r < a.n_rows;) {
      if (a.skip_chunked && row_in_chunk(s_rt, s_rp, a.n_rows, r)) {  // the prompt-chunk kernel's row
        ++r;
        continue;
      }
      int n = 1;
      while (n < RG && r + n < a.n_rows && s_rt[r + n] == s_rt[r] && s_rp[r + n] == s_rp[r + n - 1] + 1)
        ++n;
      g_row0[ng] = r;
      g_nr[ng] = n;
      row_pages[ng] = acc;
      acc += (long long)n_kv * ((s_rp[r + n - 1] >> 4) + 1);
      for (int i = 0; i < n; ++i) pmin = min(pmin, s_rp[r + i]);
      ++ng;
      r += n;
    }
    row_pages[ng] = acc;
    s_ng = ng;
    s_pos_min = pmin;
    // Whole pairs: CTA b takes pairs [b n / G, (b + 1) n / G) whole (no partials,
    // no merge) when even the worst CTA (ceil(n / G) pairs of the longest length)
    // stays within three times the even page share (whole_pairs > 1: that many
    // times); every CTA computes the same answer. At three CTAs per SM an 8-row
    // decode step (pairs of 9-32 pages) runs 1.3 % faster whole than split.
    int longest = 0;
    for (int gi = 0; gi < ng; ++gi)
      longest = max(longest, (s_rp[g_row0[gi] + g_nr[gi] - 1] >> 4) + 1);
    const long long n_pairs = (long long)ng * n_kv, share = (acc + G - 1) / G;
    s_whole = a.whole_pairs && (long long)longest * ((n_pairs + G - 1) / G) <= (a.whole_pairs == 1 ? 3 : a.whole_pairs) * share;
  }
  __syncthreads();
  const int pos_min = a.early_kv ? s_pos_min : -1;
  const int n_groups = s_ng;
  const long long P = row_pages[n_groups];
  // only the first Gp = min(G, P) CTAs take pages, so that none of them is empty
  const long long Gp = P < G ? P : G;
  long long P0 = (long long)blockIdx.x < Gp ? P * blockIdx.x / Gp : P;
  long long P1 = (long long)blockIdx.x < Gp ? P * (blockIdx.x + 1) / Gp : P;
  if (s_whole) {
    // pair q = (group q / n_kv, kv head q % n_kv) starts at page row_pages[group] + kv head * np
    const long long n_pairs = (long long)n_groups * n_kv;
    auto pair_start = [&](long long q) -> long long {
      if (q >= n_pairs) return P;
      const int gi = (int)(q / n_kv), kvh = (int)(q % n_kv);
      return row_pages[gi] + kvh * ((row_pages[gi + 1] - row_pages[gi]) / n_kv);
    };
    P0 = pair_start(n_pairs * blockIdx.x / G);
    P1 = pair_start(n_pairs * (blockIdx.x + 1) / G);
  }
  auto cta_start = [&](long long cc) { return P * cc / Gp; };

  auto seg_at = [&](long long x) -> UnitInfo {
    UnitInfo ui;
    ui.valid = x < P1;
    if (!ui.valid) return ui;
    int r = 0;
    while (r + 1 < n_groups && row_pages[r + 1] <= x) ++r;
    const int last_pos = s_rp[g_row0[r] + g_nr[r] - 1];
    const int np = (last_pos >> 4) + 1;
    const long long local = x - row_pages[r];
    ui.row = g_row0[r];
    ui.nr = g_nr[r];
    ui.kvh = (int)(local / np);
    ui.ps = row_pages[r] + (long long)ui.kvh * np;
    ui.pe = ui.ps + np;
    ui.x0 = x;
    ui.x1 = P1 < ui.pe ? P1 : ui.pe;
    ui.p_begin = (int)(x - ui.ps);
    ui.p_end = (int)(ui.x1 - ui.ps);
    ui.len = last_pos + 1;
    return ui;
  };

  uint8_t* myring = rings + warp * NSW * C::STAGE;
  uint64_t* mybars = bars + warp * NSW;
  const size_t kv_head_stride = (size_t)16 * HD;  // elements
  auto block_ptr = [&](int page, int which, int kvh) -> const uint8_t* {
    const size_t el = ((((size_t)page * a.kv.n_layers + a.layer) * 2 + which) * n_kv + kvh) * kv_head_stride;
    return reinterpret_cast<const uint8_t*>(a.kv.pool) + el * C::ESZ;
  };

  // producer iterator (uniform across the warp): CTA unit iteration + page
  int pp = -1;
  UnitInfo pu = seg_at(P0);
  if (pu.valid) pp = pu.p_begin + warp;
  auto prod_advance = [&]() {
    pp += kAttnWarps;
    while (pu.valid && pp >= pu.p_end) {
      pu = seg_at(pu.x1);
      pp = pu.valid ? pu.p_begin + warp : -1;
    }
  };
  // position the producer on its first item
  while (pu.valid && pp >= pu.p_end) {
    pu = seg_at(pu.x1);
    pp = pu.valid ? pu.p_begin + warp : -1;
  }
  int issued = 0, consumed = 0;
  // Page-table cache of this warp (uniform use): lane i holds the physical page
  // of page pc_base + 4 i of tenant pc_tenant, refilled with one coalesced load
  // per 32 of the warp's pages instead of one dependent load per page.
  int pc_tenant = -1, pc_base = 0, pc_val = 0;
  auto page_of = [&](int tenant, int p) -> int {
    if (tenant != pc_tenant || p < pc_base || ((p - pc_base) & (kAttnWarps - 1)) ||
        p >= pc_base + kAttnWarps * 32) {
      pc_tenant = tenant;
      pc_base = p;
      const int q = p + kAttnWarps * lane;
      pc_val = q < a.kv.ptab_stride ? a.kv.ptab[(size_t)tenant * a.kv.ptab_stride + q] : 0;
    }
    return __shfl_sync(0xffffffffu, pc_val, (p - pc_base) / kAttnWarps);
  };
  auto issue_upto = [&](int limit, bool old_only = false) {
    while (issued < limit && pu.valid && (!old_only || (pp + 1) * 16 <= pos_min)) {
      const int s = issued % NSW;
      const int page = page_of(s_rt[pu.row], pp);
      if (lane == 0) mbar_arrive_expect_tx(&mybars[s], 2 * C::BLK);
      if constexpr (F16) {
        // TMA boxes: K then V of (page, layer, kv head), HD / 64 boxes each
        if (lane == 0) {
          const int yk = ((((page * a.kv.n_layers + a.layer) * 2) * n_kv + pu.kvh) * 16);
#pragma unroll
          for (int which = 0; which < 2; ++which)
#pragma unroll
            for (int b = 0; b < HD / 64; ++b)
              tma_load_2d(myring + s * C::STAGE + which * C::SBLK + b * 2048, &a.kv_tmap, b * 64, yk + which * n_kv * 16,
                          &mybars[s]);
        }
      } else if (lane == 0) {
        bulk_g2s(myring + s * C::STAGE, block_ptr(page, 0, pu.kvh), C::BLK, &mybars[s]);
        bulk_g2s(myring + s * C::STAGE + C::SBLK, block_ptr(page, 1, pu.kvh), C::BLK, &mybars[s]);
      }
      ++issued;
      prod_advance();
    }
  };
  issue_upto(NSW, true);  // pages the previous kernel does not write
  pdl_wait();
  attn_stamp(a, 1);
  issue_upto(NSW);

  bool alive = true;
  const int j = lane & 15, hh = lane >> 4;
  constexpr int DPL = HD / 32;  // output dims per lane
  for (long long x = P0; x < P1;) {
    const UnitInfo ui = seg_at(x);
    x = ui.x1;
    // q of the n_rep heads that share this kv head, for each row of the group
    const int nc = ui.nr * NREP;  // query columns in use
    for (int i = threadIdx.x; i < nc * HD; i += blockDim.x) {
      const int col = i / HD;
      qs[i] = a.q[(size_t)(ui.row + col / NREP) * a.ldq + (size_t)(ui.kvh * NREP + col % NREP) * HD + i % HD];
    }
    __syncthreads();

    if constexpr (F16) {
      // Tensor-core path (fp16 K/V): per page of 16 tokens, S = K Q^T with
      // mma m16n8k16 (A = K tile by ldmatrix, B = the n_rep query heads as
      // fp16 hi + lo, ~22 bits, scale folded in), online softmax per head in
      // fp32, then O^T += V^T P^T (A = V tile by ldmatrix.trans, B = P as
      // fp16 hi + lo). Lane (g = lane/4, c = lane%4) owns heads 2c, 2c+1.
      constexpr int KS = HD / 16;
      // PK: at most 4 query columns, so the MMA's 8 columns carry the hi parts
      // (columns 0-3) and the lo parts (4-7) of the same heads: one MMA per
      // step instead of two. Lanes c and c ^ 2 then hold the two halves of the
      // same heads, summed by one shuffle; every lane works on heads
      // hb + 0, hb + 1 (hb = 2 (c & 1) packed, 2 c otherwise).
      constexpr bool PK = NC <= 4;
      const int g = lane >> 2, c = lane & 3;
      const int hb = PK ? 2 * (c & 1) : 2 * c;
      const float qscale = a.scale * 1.4426950408889634f;
      uint32_t qb[KS][2][2];  // [k-step][hi, lo][b0, b1] (packed: [k-step][0][b0, b1])
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          const int d = ks * 16 + 2 * c + 8 * b;
          const int hq = PK ? (g & 3) : g;
          // scores in base-2 units: scale * log2(e) folded into q
          const float x0 = hq < nc ? qs[hq * HD + d] * qscale : 0.f;
          const float x1 = hq < nc ? qs[hq * HD + d + 1] * qscale : 0.f;
          uint32_t hi, lo;
          pack_hilo(x0, x1, hi, lo);
          if (PK) {
            qb[ks][0][b] = g < 4 ? hi : lo;
          } else {
            qb[ks][0][b] = hi;
            qb[ks][1][b] = lo;
          }
        }
      float mh[2] = {-INFINITY, -INFINITY}, lh[2] = {0.f, 0.f};
      // causal limit of columns hb, hb + 1: their row's position + 1
      int lim[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) lim[h] = hb + h < nc ? s_rp[ui.row + (hb + h) / NREP] + 1 : 0;
      float ot[KS][4];
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) ot[mt][0] = ot[mt][1] = ot[mt][2] = ot[mt][3] = 0.f;
      float* pt = pb + warp * 16 * 8;  // [16 tokens][8 heads] transpose buffer
      const int mi = lane >> 3, rr = lane & 7;
      // this lane's ldmatrix addresses in a K block and a V block, per k-step
      int koff[KS], voff[KS];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        koff[ks] = swz(rr + (mi & 1) * 8, ks * 2 + (mi >> 1));
        voff[ks] = swz(rr + (mi >> 1) * 8, ks * 2 + (mi & 1));
      }
      for (int p = ui.p_begin + warp; p < ui.p_end; p += kAttnWarps) {
        issue_upto(consumed + NSW);
        const int s = consumed % NSW;
        if (alive) alive = mbar_wait(&mybars[s], (consumed / NSW) & 1, a.err, DEV_TIMEOUT_FULL);
        if (consumed == 0) attn_stamp(a, 2);
        const uint8_t* kb = myring + s * C::STAGE;
        const uint8_t* vb = kb + C::SBLK;
        // four independent accumulators (k-step parity x hi/lo) keep the MMA
        // dependency chains short; summed in a fixed order
        float sa[4][4];
#pragma unroll
        for (int q = 0; q < 4; ++q) sa[q][0] = sa[q][1] = sa[q][2] = sa[q][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          uint32_t af[4];
          ldsm_x4(af, kb + koff[ks]);
          if (PK) {
            mma_16816(sa[ks & 3], af, qb[ks][0][0], qb[ks][0][1]);
          } else {
            mma_16816(sa[(ks & 1) * 2], af, qb[ks][0][0], qb[ks][0][1]);
            mma_16816(sa[(ks & 1) * 2 + 1], af, qb[ks][1][0], qb[ks][1][1]);
          }
        }
        float sc[4];  // (tok g, head hb), (g, hb+1), (g+8, hb), (g+8, hb+1)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          sc[e] = (sa[0][e] + sa[2][e]) + (sa[1][e] + sa[3][e]);
          // packed: hi-part sums in lanes c < 2, lo-part sums in c >= 2
          if (PK) sc[e] += __shfl_xor_sync(0xffffffffu, sc[e], 2);
        }
        bool v0h[2], v1h[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          v0h[h] = p * 16 + g < lim[h];
          v1h[h] = p * 16 + g + 8 < lim[h];
        }
        // Online softmax with a lazily raised maximum: the running maximum of
        // heads 2c, 2c+1 changes only when some score of the page exceeds it
        // (a warp vote); then it is reduced over the lanes of each head and O
        // and the per-lane partial sums are rescaled. Sums stay per lane (every
        // lane of a head uses the same maximum) until the segment ends.
        float s0[2], s1[2], pr[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          s0[h] = v0h[h] ? sc[h] : -INFINITY;
          s1[h] = v1h[h] ? sc[2 + h] : -INFINITY;
        }
        const bool up = fmaxf(s0[0], s1[0]) > mh[0] || fmaxf(s0[1], s1[1]) > mh[1];
        if (__any_sync(0xffffffffu, up)) {
          float alpha[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float mx = fmaxf(s0[h], s1[h]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mn = fmaxf(mh[h], mx);
            alpha[h] = mh[h] == -INFINITY ? 0.f : exp2_fast(mh[h] - mn);
            lh[h] *= alpha[h];
            mh[h] = mn;
          }
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            ot[mt][0] *= alpha[0];
            ot[mt][1] *= alpha[1];
            ot[mt][2] *= alpha[0];
            ot[mt][3] *= alpha[1];
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          pr[h] = v0h[h] ? exp2_fast(s0[h] - mh[h]) : 0.f;
          pr[2 + h] = v1h[h] ? exp2_fast(s1[h] - mh[h]) : 0.f;
          lh[h] += pr[h] + pr[2 + h];
        }
        // P^T as the B operand: lane (g, c) needs heads g, tokens 2c, 2c+1, 2c+8, 2c+9
        if (!PK || c < 2) {
          pt[g * 8 + hb] = pr[0];
          pt[g * 8 + hb + 1] = pr[1];
          pt[(g + 8) * 8 + hb] = pr[2];
          pt[(g + 8) * 8 + hb + 1] = pr[3];
        }
        __syncwarp();
        const int hp = PK ? (g & 3) : g;
        uint32_t pbh0, pbl0, pbh1, pbl1;
        pack_hilo(pt[(2 * c) * 8 + hp], pt[(2 * c + 1) * 8 + hp], pbh0, pbl0);
        pack_hilo(pt[(2 * c + 8) * 8 + hp], pt[(2 * c + 9) * 8 + hp], pbh1, pbl1);
        __syncwarp();
        if (PK) {  // columns 0-3: the hi parts of P, 4-7: the lo parts
          if (g >= 4) {
            pbh0 = pbl0;
            pbh1 = pbl1;
          }
        }
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          uint32_t af[4];
          ldsm_x4_trans(af, vb + voff[mt]);
          mma_16816(ot[mt], af, pbh0, pbh1);
          if (!PK) mma_16816(ot[mt], af, pbl0, pbl1);
        }
        ++consumed;
      }
      // this warp's partial: O^T fragments -> mrg[head][dim], then m, l per head
      // (packed: the hi- and lo-weighted halves of a head sit in lanes c, c ^ 2)
#pragma unroll
      for (int mt = 0; mt < KS; ++mt)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float v = ot[mt][q];
          if (PK) v += __shfl_xor_sync(0xffffffffu, v, 2);
          const int head = hb + (q & 1), dim = mt * 16 + g + ((q & 2) ? 8 : 0);
          if (head < nc && (!PK || c < 2)) mrg[(warp * NC + head) * (HD + 2) + dim] = v;
        }
      // the per-lane partial sums of each head, then (m, l) in natural-log units
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        lh[h] += __shfl_xor_sync(0xffffffffu, lh[h], 4);
        lh[h] += __shfl_xor_sync(0xffffffffu, lh[h], 8);
        lh[h] += __shfl_xor_sync(0xffffffffu, lh[h], 16);
      }
      if (g == 0 && (!PK || c < 2))
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (hb + h < nc) {
            mrg[(warp * NC + hb + h) * (HD + 2) + HD] = mh[h] * 0.6931471805599453f;
            mrg[(warp * NC + hb + h) * (HD + 2) + HD + 1] = lh[h];
          }
    } else {
      float m[NREP], l[NREP], o[NREP][DPL];
  #pragma unroll
      for (int r = 0; r < NREP; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
  #pragma unroll
        for (int d = 0; d < DPL; ++d) o[r][d] = 0.f;
      }
      for (int p = ui.p_begin + warp; p < ui.p_end; p += kAttnWarps) {
        issue_upto(consumed + NSW);
        const int s = consumed % NSW;
        if (alive) alive = mbar_wait(&mybars[s], (consumed / NSW) & 1, a.err, DEV_TIMEOUT_FULL);
        const uint8_t* kb = myring + s * C::STAGE;
        const uint8_t* vb = kb + C::SBLK;
        // ---- scores: lane (j, hh) covers token j, dims [hh*HD/2, (hh+1)*HD/2)
        float dot[NREP];
  #pragma unroll
        for (int r = 0; r < NREP; ++r) dot[r] = 0.f;
        constexpr int EPV = 16 / C::ESZ;  // elements per 16-byte vector
  #pragma unroll 4
        for (int cidx = 0; cidx < (HD / 2) / EPV; ++cidx) {
          const int d0 = hh * (HD / 2) + cidx * EPV;
          const uint4 raw = *reinterpret_cast<const uint4*>(kb + ((size_t)j * HD + d0) * C::ESZ);
          float kf[8];
          to_f32(raw, kf, F16);
  #pragma unroll
          for (int r = 0; r < NREP; ++r) {
  #pragma unroll
            for (int e = 0; e < EPV; e += 4) {
              const float4 qv = *reinterpret_cast<const float4*>(qs + r * HD + d0 + e);
              dot[r] = fmaf(qv.x, kf[e], dot[r]);
              dot[r] = fmaf(qv.y, kf[e + 1], dot[r]);
              dot[r] = fmaf(qv.z, kf[e + 2], dot[r]);
              dot[r] = fmaf(qv.w, kf[e + 3], dot[r]);
            }
          }
        }
        const int tok = p * 16 + j;
        const bool valid = tok < ui.len;
        float alpha[NREP];
  #pragma unroll
        for (int r = 0; r < NREP; ++r) {
          const float sc = (dot[r] + __shfl_xor_sync(0xffffffffu, dot[r], 16)) * a.scale;
          float pm = valid ? sc : -INFINITY;
          pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 1));
          pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 2));
          pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 4));
          pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 8));
          const float mn = fmaxf(m[r], pm);
          alpha[r] = expf(m[r] - mn);
          const float pj = valid ? expf(sc - mn) : 0.f;
          float ps = pj;
          ps += __shfl_xor_sync(0xffffffffu, ps, 1);
          ps += __shfl_xor_sync(0xffffffffu, ps, 2);
          ps += __shfl_xor_sync(0xffffffffu, ps, 4);
          ps += __shfl_xor_sync(0xffffffffu, ps, 8);
          l[r] = l[r] * alpha[r] + ps;
          m[r] = mn;
          if (hh == 0) pb[(warp * NREP + r) * 16 + j] = pj;
        }
        __syncwarp();
        // ---- PV: lane owns dims [lane*DPL, lane*DPL + DPL)
  #pragma unroll
        for (int r = 0; r < NREP; ++r)
  #pragma unroll
          for (int d = 0; d < DPL; ++d) o[r][d] *= alpha[r];
        const int nvalid = min(16, ui.len - p * 16);
        for (int t = 0; t < nvalid; ++t) {
          float vf[DPL];
          if (F16) {
            const __half* vh = reinterpret_cast<const __half*>(vb) + (size_t)t * HD + lane * DPL;
  #pragma unroll
            for (int d = 0; d < DPL; d += 2) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vh + d));
              vf[d] = f.x;
              vf[d + 1] = f.y;
            }
          } else {
            const float* vp = reinterpret_cast<const float*>(vb) + (size_t)t * HD + lane * DPL;
  #pragma unroll
            for (int d = 0; d < DPL; ++d) vf[d] = vp[d];
          }
  #pragma unroll
          for (int r = 0; r < NREP; ++r) {
            const float pj = pb[(warp * NREP + r) * 16 + t];
  #pragma unroll
            for (int d = 0; d < DPL; ++d) o[r][d] = fmaf(pj, vf[d], o[r][d]);
          }
        }
        __syncwarp();
        ++consumed;
      }
      // ---- this warp's partial -> mrg
#pragma unroll
      for (int r = 0; r < NREP; ++r) {
        static_assert(F16 || NC == NREP, "fp32 pools keep one row per pair");
      float* w = mrg + (warp * NC + r) * (HD + 2);
#pragma unroll
        for (int d = 0; d < DPL; ++d) w[lane * DPL + d] = o[r][d];
        if (lane == 0) {
          w[HD] = m[r];
          w[HD + 1] = l[r];
        }
      }
    }
    // ---- merge the warps
    if (x >= P1) attn_stamp(a, 3);
    __syncthreads();
    // a pair split over CTAs: slot 0 for the CTA's first segment, 1 for its last
    const bool whole = ui.x0 == ui.ps && ui.x1 == ui.pe;
    const size_t slot = (size_t)blockIdx.x * 2 + (ui.x0 == P0 ? 0 : 1);
    // Final values go to shared memory (the q buffer is free now), then out to the
    // fp32 output and / or the activation fragments of the o-proj GEMV.
    float* ofin = qs;
    __shared__ float frag_scratch[16];
    auto finish = [&]() {
      __syncthreads();
      if (a.out)
        for (int i = threadIdx.x; i < nc * HD; i += blockDim.x) {
          const int col = i / HD;
          a.out[(size_t)(ui.row + col / NREP) * a.ldo + (size_t)(ui.kvh * NREP + col % NREP) * HD + i % HD] = ofin[i];
        }
      if (a.xout.xi || a.xout.xf)
        for (int rl = 0; rl < ui.nr; ++rl)
          frags_write(ofin + rl * NREP * HD, 1, 0, NREP * HD, 1, ui.kvh * NREP * HD, ui.row + rl, nullptr, a.xout,
                      a.xf_nt, frag_scratch, threadIdx.x, blockDim.x, [] { __syncthreads(); });
    };
    auto merge_warps = [&](int i, float& M, float& Lsum, float& O) {
      const int r = i / HD, d = i % HD;
      M = -INFINITY;
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, mrg[(w * NC + r) * (HD + 2) + HD]);
      Lsum = 0.f;
      O = 0.f;
      for (int w = 0; w < kAttnWarps; ++w) {
        const float* ww = mrg + (w * NC + r) * (HD + 2);
        const float f = (ww[HD] == -INFINITY) ? 0.f : expf(ww[HD] - M);
        Lsum += ww[HD + 1] * f;
        O += ww[d] * f;
      }
    };
    if (whole) {
      for (int i = threadIdx.x; i < nc * HD; i += blockDim.x) {
        float M, Lsum, O;
        merge_warps(i, M, Lsum, O);
        ofin[i] = Lsum > 0.f ? O / Lsum : 0.f;
      }
      finish();
    } else {
      for (int i = threadIdx.x; i < nc * HD; i += blockDim.x) {
        const int r = i / HD, d = i % HD;
        float M, Lsum, O;
        merge_warps(i, M, Lsum, O);
        float* dst = a.partials + (slot * NC + r) * (HD + 2);
        __stcg(dst + d, O);
        if (d == 0) {
          __stcg(dst + HD, M);
          __stcg(dst + HD + 1, Lsum);
        }
      }
      // contributors: the CTAs whose page ranges intersect the pair
      long long cf = ui.ps * Gp / P, cl = (ui.pe - 1) * Gp / P;
      while (cf + 1 < Gp && cta_start(cf + 1) <= ui.ps) ++cf;
      while (cf > 0 && cta_start(cf) > ui.ps) --cf;
      while (cl + 1 < Gp && cta_start(cl + 1) <= ui.pe - 1) ++cl;
      while (cl > 0 && cta_start(cl) > ui.pe - 1) --cl;
      const int ncon = (int)(cl - cf + 1);
      __syncthreads();  // partial stores of this CTA before thread 0's release
      if (threadIdx.x == 0) s_last = atom_add_acq_rel(a.counters + ui.row * n_kv + ui.kvh, 1) == ncon - 1;
      __syncthreads();
      if (s_last) {
        // contributor cc's partial is in its slot 0 iff the pair is its first segment
        auto part = [&](int j) {
          const long long cc = cf + j;
          const int sl = cta_start(cc) >= ui.ps ? 0 : 1;
          return a.partials + ((size_t)cc * 2 + sl) * NC * (HD + 2);
        };
        // (m, l) of every contributor and head into shared memory (mrg is free)
        float* tab = mrg;  // [ncon][NC][2]
        const bool fits = ncon * NC * 2 <= kAttnWarps * NC * (HD + 2);
        if (fits)
          for (int e = threadIdx.x; e < ncon * NC; e += blockDim.x) {
            const float* src = part(e / NC) + (e % NC) * (HD + 2);
            tab[2 * e] = __ldcg(src + HD);
            tab[2 * e + 1] = __ldcg(src + HD + 1);
          }
        __syncthreads();
        for (int i = threadIdx.x; i < nc * HD; i += blockDim.x) {
          const int r = i / HD, d = i % HD;
          auto mval = [&](int j) { return fits ? tab[2 * (j * NC + r)] : __ldcg(part(j) + r * (HD + 2) + HD); };
          auto lval = [&](int j) { return fits ? tab[2 * (j * NC + r) + 1] : __ldcg(part(j) + r * (HD + 2) + HD + 1); };
          float M = -INFINITY;
          for (int j = 0; j < ncon; ++j) M = fmaxf(M, mval(j));
          float Lsum = 0.f, O = 0.f;
          // output loads issued 8 at a time, summed in contributor order
          for (int j0 = 0; j0 < ncon; j0 += 8) {
            float ov[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (j0 + j < ncon) ov[j] = __ldcg(part(j0 + j) + r * (HD + 2) + d);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (j0 + j < ncon) {
                const float ms = mval(j0 + j);
                const float f = (ms == -INFINITY) ? 0.f : expf(ms - M);
                Lsum += lval(j0 + j) * f;
                O += ov[j] * f;
              }
          }
          ofin[i] = Lsum > 0.f ? O / Lsum : 0.f;
        }
        finish();
        if (threadIdx.x == 0) a.counters[ui.row * n_kv + ui.kvh] = 0;
      }
    }
    __syncthreads();
  }
  attn_stamp(a, 4);
  // every issued copy is consumed on the normal path; after a timed-out wait,
  // let the copies still in flight land before the CTA exits (bounded)
  if (!alive && lane == 0)
    for (int k = (issued > NSW ? issued - NSW : 0); k < issued; ++k)
      mbar_wait(&mybars[k % NSW], (k / NSW) & 1, a.err, DEV_TIMEOUT_DRAIN);
}

// ---------------------------------------------------------------------------
// Prompt-chunk attention (fp16 pools, n_rep 8). The rows of a chunk (a
// run of consecutive positions of one tenant, as a prefill step or a prompt
// chunk in a mixed step has) share their tenant's K/V pages, so the query
// vectors (row, head) of one kv head become the M dimension of the MMAs:
// 16 per warp, 64 per item (chunk, kv head, 64-vector tile). An item's pages
// (up to its last row's position) are cut into segments of SEG pages, SEG
// chosen per launch so that there are about two units (item, segment) per
// CTA; a unit streams its pages once through a shared ring (TMA boxes,
// 128-byte swizzle, a producer warp) for all 64 vectors:
//   S = Q K^T   mma m16n8k16, A = Q as fp16 hi + lo (~22 bits, scale and
//               log2 e folded in), B = K straight from the ldmatrix fragments;
//   online softmax per vector in fp32 (row maxima over the quad, raised
//               lazily by warp vote), causal limit = the vector's position;
//   O += P V    A = P from the S accumulators (hi + lo), B = V by
//               ldmatrix.trans.
// A single-segment item is written out directly; otherwise each unit leaves
// (O, m, l) in its slot and the last unit of the item to finish merges the
// slots in segment order (deterministic). Results go out as fp32 rows and / or
// the o-proj's activation fragments. At n_rep 8 a 64-row chunk reads each kv
// head's pages 8 times instead of 64.
// ---------------------------------------------------------------------------
constexpr int kChunkWarps = 4;                // consumers; warp kChunkWarps streams the pages
constexpr int kChunkVecs = 16 * kChunkWarps;  // query vectors per item
constexpr int kChunkStages = 6;
constexpr int kChunkCounterOff = 16384;       // item counters, past the decode kernel's pair counters

// Items of one launch for n_kv kv heads: per chunk n_kv x ceil(rows * n_rep / 64),
// at most n_kv x (64 * 8 / 64 + 32) over the <= 32 chunks of <= 64 rows.
__host__ __device__ constexpr int chunk_max_items(int n_kv) { return n_kv * (kMaxRows * 8 / kChunkVecs + kMaxRows / 2); }

template <int HD>
__host__ __device__ constexpr int chunk_smem_bytes() {
  return 1024                                // ring alignment (128-byte swizzle pattern)
         + kChunkStages * 2 * 16 * HD * 2    // ring: K and V of one page per stage
         + kChunkVecs * HD * 4               // results of one item
         + kChunkStages * 2 * 8;             // full / empty barriers
}

template <int HD, int NREP>
__global__ void __launch_bounds__((kChunkWarps + 1) * 32, 2) attn_chunk_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int BLK = 16 * HD * 2, STAGE = 2 * BLK, NS = kChunkStages, KS = HD / 16;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* ofin = reinterpret_cast<float*>(ring + NS * STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(ofin + kChunkVecs * HD);
  uint64_t* empty = full + NS;
  constexpr int kTiles = kMaxRows * NREP / kChunkVecs;  // tiles of a chunk of at most kMaxRows rows
  __shared__ int s_rt[kMaxRows], s_rp[kMaxRows], c_row0[kMaxRows / 2], c_nr[kMaxRows / 2];
  // units: chunk-major, then kv head, then tile, then segment. c_u0: units before
  // the chunk; c_hu: units of one kv head of it; t_u0: units before tile t within
  // one kv head; t_np: the tile's pages
  __shared__ int c_u0[kMaxRows / 2 + 1], c_hu[kMaxRows / 2], c_nt[kMaxRows / 2];
  __shared__ int t_u0[kMaxRows / 2][kTiles + 1], t_np[kMaxRows / 2][kTiles];
  __shared__ int s_nc, s_seg, s_last;
  __shared__ float frag_scratch[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kv = a.kv.n_kv;
  const int G = gridDim.x;
  float* partials = a.partials + decode_partials_floats(G, NREP, HD);  // past the decode kernel's
  int32_t* counters = a.counters + kChunkCounterOff;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kChunkWarps);
    }
    fence_barrier_init();
  }
  pdl_launch_dependents();
  // rows, queries and the chunk's own K/V come from the kernels before this one
  pdl_wait();
  for (int i = threadIdx.x; i < a.n_rows; i += blockDim.x) {
    s_rt[i] = a.row_tenant[i];
    s_rp[i] = a.row_pos[i];
  }
  __syncthreads();
  struct Item {
    int row0, tenant, kvh, v0, nv, npages;  // vectors v0 .. v0 + nv of the chunk (v = row * NREP + rep)
  };
  if (threadIdx.x == 0) {
    int nc = 0;
    long long total = 0;
    for (int r = 0; r < a.n_rows;) {
      if (!row_in_chunk(s_rt, s_rp, a.n_rows, r)) {
        ++r;
        continue;
      }
      int n = 1;
      while (r + n < a.n_rows && s_rt[r + n] == s_rt[r] && s_rp[r + n] == s_rp[r + n - 1] + 1) ++n;
      c_row0[nc] = r;
      c_nr[nc] = n;
      c_nt[nc] = (n * NREP + kChunkVecs - 1) / kChunkVecs;
      for (int t = 0; t < c_nt[nc]; ++t) {
        const int vl = min((t + 1) * kChunkVecs, n * NREP) - 1;  // the tile's last vector
        t_np[nc][t] = (s_rp[r + vl / NREP] >> 4) + 1;
        total += (long long)n_kv * t_np[nc][t];
      }
      ++nc;
      r += n;
    }
    // segment length: about two units per CTA, at least 4 pages
    const int seg = max(4, (int)((total + 2LL * G - 1) / (2LL * G)));
    int u = 0;
    for (int ci = 0; ci < nc; ++ci) {
      c_u0[ci] = u;
      int hu = 0;
      for (int t = 0; t < c_nt[ci]; ++t) {
        t_u0[ci][t] = hu;
        hu += (t_np[ci][t] + seg - 1) / seg;
      }
      t_u0[ci][c_nt[ci]] = hu;
      c_hu[ci] = hu;
      u += n_kv * hu;
    }
    c_u0[nc] = u;
    s_nc = nc;
    s_seg = seg;
  }
  __syncthreads();
  const int n_chunks = s_nc, seg = s_seg, n_units = c_u0[n_chunks];
  // unit -> item, its id (for the merge counter), segments, first and end page
  auto unit_at = [&](int u, Item& I, int& item_id, int& nseg, int& seg0, int& p0, int& p1) {
    int ci = 0;
    while (ci + 1 < n_chunks && c_u0[ci + 1] <= u) ++ci;
    const int local = u - c_u0[ci], hu = c_hu[ci];
    I.kvh = local / hu;
    const int r = local % hu;
    int t = 0;
    while (t + 1 < c_nt[ci] && t_u0[ci][t + 1] <= r) ++t;
    I.row0 = c_row0[ci];
    I.tenant = s_rt[I.row0];
    I.v0 = t * kChunkVecs;
    I.nv = min(kChunkVecs, c_nr[ci] * NREP - I.v0);
    I.npages = t_np[ci][t];
    seg0 = c_u0[ci] + I.kvh * hu + t_u0[ci][t];  // the item's first unit
    nseg = t_u0[ci][t + 1] - t_u0[ci][t];
    item_id = (ci * n_kv + I.kvh) * kTiles + t;  // < 32 * n_kv * 8 <= 16384 counters (n_kv <= 64)
    p0 = (u - seg0) * seg;
    p1 = min(I.npages, p0 + seg);
  };

  if (warp == kChunkWarps) {
    // ---- producer: the pages of this CTA's units, in order, through the ring
    if (lane == 0) {
      uint32_t issued = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < n_units && ok; u += G) {
        Item I;
        int item_id, nseg, seg0, p0, p1;
        unit_at(u, I, item_id, nseg, seg0, p0, p1);
        const int32_t* pt = a.kv.ptab + (size_t)I.tenant * a.kv.ptab_stride;
        for (int p = p0; p < p1; ++p) {
          const int s = issued % NS;
          if (issued >= (uint32_t)NS) {
            ok = mbar_wait(&empty[s], ((issued / NS) - 1) & 1, a.err, DEV_TIMEOUT_EMPTY);
            if (!ok) break;
          }
          const int page = pt[p];
          mbar_arrive_expect_tx(&full[s], 2 * BLK);
          const int yk = (((page * a.kv.n_layers + a.layer) * 2) * n_kv + I.kvh) * 16;
#pragma unroll
          for (int which = 0; which < 2; ++which)
#pragma unroll
            for (int b = 0; b < HD / 64; ++b)
              tma_load_2d(ring + s * STAGE + which * BLK + b * 2048, &a.kv_tmap, b * 64, yk + which * n_kv * 16,
                          &full[s]);
          ++issued;
        }
      }
      // every issued copy lands before the CTA may exit (the consumers may have stopped early)
      const uint32_t first = issued > (uint32_t)NS ? issued - NS : 0u;
      for (uint32_t j = first; j < issued; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, a.err, DEV_TIMEOUT_DRAIN);
    }
    return;
  }

  // ---- consumers
  constexpr int NTH = kChunkWarps * 32;
  const int g = lane >> 2, c = lane & 3;
  const int tid = threadIdx.x;
  const float qscale = a.scale * 1.4426950408889634f;  // scores in base-2 units
  // this lane's ldmatrix rows in a K block and a V block (addresses formed per use)
  const int mi = lane >> 3, rk = (lane & 7) + (mi & 1) * 8, rv = (lane & 7) + (mi >> 1) * 8;
  bool alive = true;
  uint32_t consumed = 0;
  for (int u = blockIdx.x; u < n_units; u += G) {
    Item I;
    int item_id, nseg, seg0, p0, p1;
    unit_at(u, I, item_id, nseg, seg0, p0, p1);
    // this thread's two query vectors: rows g and g + 8 of the warp's 16
    const int vA = warp * 16 + g, vB = vA + 8;
    const bool okA = vA < I.nv, okB = vB < I.nv;
    const int rowA = I.row0 + (I.v0 + vA) / NREP, rowB = I.row0 + (I.v0 + vB) / NREP;
    const int headA = I.kvh * NREP + (I.v0 + vA) % NREP, headB = I.kvh * NREP + (I.v0 + vB) % NREP;
    const float* qA = a.q + (size_t)rowA * a.ldq + (size_t)headA * HD;
    const float* qB = a.q + (size_t)rowB * a.ldq + (size_t)headB * HD;
    uint32_t qh[KS][4], ql[KS][4];  // A fragments of Q (hi, lo)
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int d = ks * 16 + 2 * c + ((e & 2) ? 8 : 0);
        const bool ok = (e & 1) ? okB : okA;
        const float* qp = (e & 1) ? qB : qA;
        const float2 v = ok ? *reinterpret_cast<const float2*>(qp + d) : make_float2(0.f, 0.f);
        pack_hilo(v.x * qscale, v.y * qscale, qh[ks][e], ql[ks][e]);
      }
    const int limA = okA ? s_rp[rowA] + 1 : 0, limB = okB ? s_rp[rowB] + 1 : 0;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
    float o[2 * KS][4];
#pragma unroll
    for (int j = 0; j < 2 * KS; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    for (int p = p0; p < p1; ++p, ++consumed) {
      const int s = consumed % NS;
      if (alive) alive = mbar_wait(&full[s], (consumed / NS) & 1, a.err, DEV_TIMEOUT_FULL);
      const uint8_t* kb = ring + s * STAGE;
      const uint8_t* vb = kb + BLK;
      // S: n-tile t = tokens 8t..8t+7 of the page; hi and lo parts apart
      float sh[2][4], sl[2][4];
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) sh[t][e] = sl[t][e] = 0.f;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t kf[4];  // K as an A fragment (tokens x dims) = B fragments of both n-tiles
        ldsm_x4(kf, kb + swz(rk, ks * 2 + (mi >> 1)));
        mma_16816(sh[0], qh[ks], kf[0], kf[2]);
        mma_16816(sl[0], ql[ks], kf[0], kf[2]);
        mma_16816(sh[1], qh[ks], kf[1], kf[3]);
        mma_16816(sl[1], ql[ks], kf[1], kf[3]);
      }
      // sc[t][e]: vector A (e < 2) or B, token 16p + 8t + 2c + (e & 1)
      float sc[2][4];
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = p * 16 + t * 8 + 2 * c + (e & 1);
          sc[t][e] = tok < ((e & 2) ? limB : limA) ? sh[t][e] + sl[t][e] : -INFINITY;
        }
      float xA = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
      float xB = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
      xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 1));
      xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 2));
      xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 1));
      xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 2));
      if (__any_sync(0xffffffffu, xA > mA || xB > mB)) {
        const float nA = fmaxf(mA, xA), nB = fmaxf(mB, xB);
        const float alA = mA == -INFINITY ? 0.f : exp2_fast(mA - nA);
        const float alB = mB == -INFINITY ? 0.f : exp2_fast(mB - nB);
        mA = nA;
        mB = nB;
        lA *= alA;
        lB *= alB;
#pragma unroll
        for (int j = 0; j < 2 * KS; ++j) {
          o[j][0] *= alA;
          o[j][1] *= alA;
          o[j][2] *= alB;
          o[j][3] *= alB;
        }
      }
      float pr[2][4];
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float m = (e & 2) ? mB : mA;
          pr[t][e] = sc[t][e] == -INFINITY ? 0.f : exp2_fast(sc[t][e] - m);
        }
      lA += (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
      lB += (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
      // P as the A fragment (vectors x tokens) of the P V step
      uint32_t ph[4], pl[4];
      pack_hilo(pr[0][0], pr[0][1], ph[0], pl[0]);
      pack_hilo(pr[0][2], pr[0][3], ph[1], pl[1]);
      pack_hilo(pr[1][0], pr[1][1], ph[2], pl[2]);
      pack_hilo(pr[1][2], pr[1][3], ph[3], pl[3]);
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        uint32_t vf[4];  // V^T as an A fragment (dims x tokens) = B fragments of two 8-dim n-tiles
        ldsm_x4_trans(vf, vb + swz(rv, mt * 2 + (mi & 1)));
        mma_16816(o[2 * mt], ph, vf[0], vf[2]);
        mma_16816(o[2 * mt], pl, vf[0], vf[2]);
        mma_16816(o[2 * mt + 1], ph, vf[1], vf[3]);
        mma_16816(o[2 * mt + 1], pl, vf[1], vf[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    lA += __shfl_xor_sync(0xffffffffu, lA, 1);
    lA += __shfl_xor_sync(0xffffffffu, lA, 2);
    lB += __shfl_xor_sync(0xffffffffu, lB, 1);
    lB += __shfl_xor_sync(0xffffffffu, lB, 2);
    named_bar_sync(1, NTH);  // the previous unit's results are written out
    if (nseg == 1) {
      const float iA = lA > 0.f ? 1.0f / lA : 0.f, iB = lB > 0.f ? 1.0f / lB : 0.f;
#pragma unroll
      for (int j = 0; j < 2 * KS; ++j) {
        const int d = j * 8 + 2 * c;
        *reinterpret_cast<float2*>(ofin + vA * HD + d) = make_float2(o[j][0] * iA, o[j][1] * iA);
        *reinterpret_cast<float2*>(ofin + vB * HD + d) = make_float2(o[j][2] * iB, o[j][3] * iB);
      }
    } else {
      // this unit's (O, m, l) per vector into its slot; the item's last unit merges
      float* slot = partials + (size_t)u * kChunkVecs * (HD + 2);
#pragma unroll
      for (int j = 0; j < 2 * KS; ++j) {
        const int d = j * 8 + 2 * c;
        __stcg(reinterpret_cast<float2*>(slot + vA * (HD + 2) + d), make_float2(o[j][0], o[j][1]));
        __stcg(reinterpret_cast<float2*>(slot + vB * (HD + 2) + d), make_float2(o[j][2], o[j][3]));
      }
      if (c == 0) {
        __stcg(reinterpret_cast<float2*>(slot + vA * (HD + 2) + HD), make_float2(mA, lA));
        __stcg(reinterpret_cast<float2*>(slot + vB * (HD + 2) + HD), make_float2(mB, lB));
      }
      named_bar_sync(1, NTH);  // the slot's stores before thread 0's release
      if (tid == 0) s_last = atom_add_acq_rel(counters + item_id, 1) == nseg - 1;
      named_bar_sync(1, NTH);
      if (!s_last) continue;
      // merge the item's slots in segment order, each thread on its own fragment
      // positions: per segment one batch of independent L2 loads, then
      // (M, L, O) <- (M, L, O) and (m, l, o) rescaled to the larger maximum
      const float* first = partials + (size_t)seg0 * kChunkVecs * (HD + 2);
      constexpr int JH = KS;  // 8-dim n-tiles per half of the head dimension
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float MA = -INFINITY, MB = -INFINITY, LA = 0.f, LB = 0.f;
        float acc[JH][4];
#pragma unroll
        for (int j = 0; j < JH; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        for (int q = 0; q < nseg; ++q) {
          const float* sq = first + (size_t)q * kChunkVecs * (HD + 2);
          const float2 mlA = __ldcg(reinterpret_cast<const float2*>(sq + vA * (HD + 2) + HD));
          const float2 mlB = __ldcg(reinterpret_cast<const float2*>(sq + vB * (HD + 2) + HD));
          float2 oa[JH], ob[JH];
#pragma unroll
          for (int j = 0; j < JH; ++j) {
            const int d = (h * JH + j) * 8 + 2 * c;
            oa[j] = __ldcg(reinterpret_cast<const float2*>(sq + vA * (HD + 2) + d));
            ob[j] = __ldcg(reinterpret_cast<const float2*>(sq + vB * (HD + 2) + d));
          }
          const float nA = fmaxf(MA, mlA.x), nB = fmaxf(MB, mlB.x);
          const float fA = MA == -INFINITY ? 0.f : exp2_fast(MA - nA), gA = mlA.x == -INFINITY ? 0.f : exp2_fast(mlA.x - nA);
          const float fB = MB == -INFINITY ? 0.f : exp2_fast(MB - nB), gB = mlB.x == -INFINITY ? 0.f : exp2_fast(mlB.x - nB);
          MA = nA;
          MB = nB;
          LA = LA * fA + mlA.y * gA;
          LB = LB * fB + mlB.y * gB;
#pragma unroll
          for (int j = 0; j < JH; ++j) {
            acc[j][0] = acc[j][0] * fA + oa[j].x * gA;
            acc[j][1] = acc[j][1] * fA + oa[j].y * gA;
            acc[j][2] = acc[j][2] * fB + ob[j].x * gB;
            acc[j][3] = acc[j][3] * fB + ob[j].y * gB;
          }
        }
        const float iA = LA > 0.f ? 1.0f / LA : 0.f, iB = LB > 0.f ? 1.0f / LB : 0.f;
#pragma unroll
        for (int j = 0; j < JH; ++j) {
          const int d = (h * JH + j) * 8 + 2 * c;
          *reinterpret_cast<float2*>(ofin + vA * HD + d) = make_float2(acc[j][0] * iA, acc[j][1] * iA);
          *reinterpret_cast<float2*>(ofin + vB * HD + d) = make_float2(acc[j][2] * iB, acc[j][3] * iB);
        }
      }
      if (tid == 0) counters[item_id] = 0;
    }
    named_bar_sync(1, NTH);
    // whole rows: the tile starts at a multiple of 64 vectors, a multiple of n_rep
    const int r0 = I.row0 + I.v0 / NREP, nrows = I.nv / NREP;
    if (a.out)
      for (int i = tid; i < I.nv * HD; i += NTH) {
        const int v = I.v0 + i / HD;
        a.out[(size_t)(I.row0 + v / NREP) * a.ldo + (size_t)(I.kvh * NREP + v % NREP) * HD + i % HD] = ofin[i];
      }
    if (a.xout.xi || a.xout.xf)
      for (int rl = 0; rl < nrows; ++rl)
        frags_write(ofin + rl * NREP * HD, 1, 0, NREP * HD, 1, I.kvh * NREP * HD, r0 + rl, nullptr, a.xout, a.xf_nt,
                    frag_scratch, tid, NTH, [] { named_bar_sync(1, kChunkWarps * 32); });
  }
}

template <int HD, int NREP>
cudaError_t launch_chunk_t(const AttnArgs& a, int num_sms, cudaStream_t s, int pdl) {
  constexpr int smem = chunk_smem_bytes<HD>();
  static_assert(2 * (smem + 1024) <= 228 * 1024, "two CTAs per SM");
  auto kern = attn_chunk_kernel<HD, NREP>;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cudaError_t e = ensure_smem_attr(kern, smem, dev)) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * num_sms);
  cfg.blockDim = dim3((kChunkWarps + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int HD, int NREP, int F16, int GR>
cudaError_t launch_attn_t(const AttnArgs& a, int num_sms, cudaStream_t s, int pdl) {
  constexpr int smem = attn_smem_bytes<HD, NREP, F16, GR>();
  auto kern = attn_kernel<HD, NREP, F16, GR>;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cudaError_t e = ensure_smem_attr(kern, smem, dev)) return e;
  static_assert(smem <= 227 * 1024, "shared memory of one CTA");
  // as many CTAs per SM as are resident at once (static shared memory and
  // registers included), at most attn_grid() / num_sms
  static int per_sm_cache[64] = {};
  int per_sm = dev < 64 ? per_sm_cache[dev] : 0;
  if (per_sm == 0) {
    if (cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kAttnWarps * 32, smem)) return e;
    per_sm = per_sm < 1 ? 1 : per_sm > 3 ? 3 : per_sm;
    if (dev < 64) per_sm_cache[dev] = per_sm;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms * per_sm);
  cfg.blockDim = dim3(kAttnWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int HD, int F16>
cudaError_t launch_attn_hd(const AttnArgs& a, int nrep, int num_sms, cudaStream_t s, int pdl) {
  const bool gr = F16 && a.group_rows;  // the grouped variant differs only for fp16 and n_rep < 4
  switch (nrep) {
    case 1: return gr ? launch_attn_t<HD, 1, F16, 1>(a, num_sms, s, pdl) : launch_attn_t<HD, 1, F16, 0>(a, num_sms, s, pdl);
    case 2: return gr ? launch_attn_t<HD, 2, F16, 1>(a, num_sms, s, pdl) : launch_attn_t<HD, 2, F16, 0>(a, num_sms, s, pdl);
    case 4: return launch_attn_t<HD, 4, F16, 0>(a, num_sms, s, pdl);
    case 8: return launch_attn_t<HD, 8, F16, 0>(a, num_sms, s, pdl);
  }
  return cudaErrorInvalidValue;
}

__global__ void kv_append_kernel(const KvView kv, int layer, int n_rows, const int32_t* row_tenant,
                                 const int32_t* row_pos, const float* k, const float* v) {
  const int row_elems = kv.n_kv * kv.hd;
  const long long total = (long long)n_rows * row_elems;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / row_elems), e = (int)(i % row_elems);
    const int head = e / kv.hd, d = e % kv.hd;
    const int pos = row_pos[r];
    const int page = kv.ptab[(size_t)row_tenant[r] * kv.ptab_stride + (pos >> 4)];
    for (int which = 0; which < 2; ++which) {
      const size_t off = ((((size_t)page * kv.n_layers + layer) * 2 + which) * kv.n_kv + head) * 16 * (size_t)kv.hd +
                         (size_t)(pos & 15) * kv.hd + d;
      const float val = which ? v[i] : k[i];
      if (kv.f16) reinterpret_cast<__half*>(kv.pool)[off] = __float2half_rn(val);
      else reinterpret_cast<float*>(kv.pool)[off] = val;
    }
  }
}

__global__ void kv_gather_kernel(const KvView kv, int layer, int tenant, int len, float* ko, float* vo) {
  const int row_elems = kv.n_kv * kv.hd;
  const long long total = (long long)len * row_elems;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int pos = (int)(i / row_elems), e = (int)(i % row_elems);
    const int head = e / kv.hd, d = e % kv.hd;
    const int page = kv.ptab[(size_t)tenant * kv.ptab_stride + (pos >> 4)];
    for (int which = 0; which < 2; ++which) {
      const size_t off = ((((size_t)page * kv.n_layers + layer) * 2 + which) * kv.n_kv + head) * 16 * (size_t)kv.hd +
                         (size_t)(pos & 15) * kv.hd + d;
      const float val = kv.f16 ? __half2float(reinterpret_cast<const __half*>(kv.pool)[off])
                               : reinterpret_cast<const float*>(kv.pool)[off];
      (which ? vo : ko)[i] = val;
    }
  }
}

}  // namespace

int attn_grid(int num_sms) { return 3 * num_sms; }  // upper bound on the attention grids

cudaError_t kv_tensor_map(const KvView& kv, size_t n_pages, CUtensorMap* out) {
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess) return e;
    if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  if (!kv.f16 || (kv.hd != 64 && kv.hd != 128)) return cudaErrorInvalidValue;
  const cuuint64_t rows = (cuuint64_t)n_pages * kv.n_layers * 2 * kv.n_kv * 16;
  const cuuint64_t dims[2] = {(cuuint64_t)kv.hd, rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kv.hd * 2};
  const cuuint32_t box[2] = {64, 16};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kv.pool, dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

size_t attn_partials_floats(int num_ctas, int n_rep, int hd, int n_kv) {
  // + the prompt-chunk kernel's unit slots: at most 2 per CTA plus one per item
  return decode_partials_floats(num_ctas, n_rep, hd) +
         (size_t)(2 * num_ctas + chunk_max_items(n_kv)) * kChunkVecs * (hd + 2);
}

cudaError_t attn_launch(const AttnArgs& a_in, int num_sms, cudaStream_t s, int pdl, int* launches) {
  if (a_in.n_rows < 1 || a_in.n_rows > kMaxRows) return cudaErrorInvalidValue;
  const int nrep = a_in.n_heads / a_in.kv.n_kv;
  AttnArgs a = a_in;
  // n_rep 8 only: at n_rep 4 the decode kernel packs a row's hi and lo query
  // parts into one MMA, so both need the same MMAs per page and the rows of a
  // chunk already share the pages through L2 (bench.py --case chunk)
  if (a.group_rows && a.kv.f16 && nrep == 8 && (a.kv.hd == 64 || a.kv.hd == 128) &&
      a.kv.n_kv <= 64) {
    // prompt chunks on their own kernel; the decode kernel takes the other rows
    cudaError_t e = a.kv.hd == 128 ? launch_chunk_t<128, 8>(a, num_sms, s, pdl) : launch_chunk_t<64, 8>(a, num_sms, s, pdl);
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
    a.skip_chunked = 1;
  }
  if (launches) ++*launches;
  if (a.kv.hd == 128) {
    return a.kv.f16 ? launch_attn_hd<128, 1>(a, nrep, num_sms, s, pdl) : launch_attn_hd<128, 0>(a, nrep, num_sms, s, pdl);
  } else if (a.kv.hd == 64) {
    return a.kv.f16 ? launch_attn_hd<64, 1>(a, nrep, num_sms, s, pdl) : launch_attn_hd<64, 0>(a, nrep, num_sms, s, pdl);
  }
  return cudaErrorInvalidValue;
}

cudaError_t kv_append_launch(const KvView& kv, int layer, int n_rows, const int32_t* row_tenant,
                             const int32_t* row_pos, const float* k, const float* v, cudaStream_t s) {
  const long long total = (long long)n_rows * kv.n_kv * kv.hd;
  if (total == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  kv_append_kernel<<<grid, 256, 0, s>>>(kv, layer, n_rows, row_tenant, row_pos, k, v);
  return cudaGetLastError();
}

cudaError_t kv_gather_launch(const KvView& kv, int layer, int tenant, int len, float* k_out, float* v_out,
                             cudaStream_t s) {
  const long long total = (long long)len * kv.n_kv * kv.hd;
  if (total == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  kv_gather_kernel<<<grid, 256, 0, s>>>(kv, layer, tenant, len, k_out, v_out);
  return cudaGetLastError();
}

}  // namespace rb
