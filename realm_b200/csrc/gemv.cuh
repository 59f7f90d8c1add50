// Host/device interface of the fused dequant GEMV/GEMM (y = x . W^T).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "xfrag.cuh"

namespace rb {

enum Epilogue : int32_t {
  EPI_STORE = 0,   // y[tok][row] = acc * inv_rms[tok]
  EPI_QKV = 1,     // RoPE + q store + paged K/V append
  EPI_RESID = 2,   // x[tok][row] += acc, row-group sums of squares, fragments of x*norm
  EPI_SWIGLU = 3,  // rows interleaved gate/up per 8: h = silu(g) * u (+ fragments of h)
  EPI_LOGITS = 4,  // optional logits store + greedy argmax (ties -> last index)
};

// Paged KV pool view (shared with the attention kernels).
// Element (page, layer, kv, head, slot, d) lives at
// ((((page * n_layers + layer) * 2 + kv) * n_kv + head) * 16 + slot) * hd + d.
struct KvView {
  void* pool = nullptr;
  int32_t f16 = 1;  // 1: fp16 elements, 0: fp32
  int32_t n_layers = 1, n_kv = 1, hd = 128;
  const int32_t* ptab = nullptr;  // [tenant][ptab_stride] physical page ids
  int32_t ptab_stride = 0;
};

struct GemvArgs {
  // weights (tiled layout) and geometry
  const uint8_t* w = nullptr;
  int32_t dtype = 0;
  int32_t n = 0;      // logical output rows
  int32_t n_rg = 0;   // 256-row groups (padded rows = n_rg * 256)
  int32_t nsb = 0;    // K / 256
  // optional second weight of the same K in the same phase (GEMV kernel only):
  // its row groups follow the first's in the unit space, so both share one
  // stream-K split and one tail (a QKV phase runs q|k and v together); its
  // rows start at qkv_row0_2 in the QKV epilogue. dtype2 is dtype, or Q6_K
  // after Q4_K in steps of at most 8 rows.
  const uint8_t* w2 = nullptr;
  int32_t dtype2 = 0, n2 = 0, n_rg2 = 0, qkv_row0_2 = 0;
  int32_t m = 0;      // tokens (x rows)
  // input: activation fragments (xfrag.cuh) of x[m][K] (times the fused norm weight)
  XFrags xin;
  const float* ss_part = nullptr;  // optional [n_ss][ld_ss] partial sums of squares -> 1/rms per token
  int32_t n_ss = 0, ld_ss = 64;
  float norm_eps = 1e-5f;
  int32_t norm_dim = 0;
  // epilogue
  int32_t epi = EPI_STORE;
  float* y = nullptr;   // STORE / SWIGLU output, LOGITS logits (optional)
  int32_t ldy = 0;
  float* resid = nullptr;  // RESID: x stream (read-modify-write), ld = ldr
  int32_t ldr = 0;
  float* ss_out = nullptr;  // RESID: [n_rg][ld_ss]
  XFrags xout;              // RESID / SWIGLU: fragments of the next GEMV's input
  int32_t xout_nt = 0;      //   their n-tile count (0: the kernel's own) and the
  int32_t xout_t0 = 0;      //   token of this launch's row 0 (token-split epilogues)
  const float* xf_norm = nullptr;  // RESID: norm weight the next GEMV fuses
  unsigned long long* argmax = nullptr;  // LOGITS: per token key
  // QKV
  int32_t qkv_row0 = 0, n_q_rows = 0, n_k_rows = 0;
  float* q_out = nullptr;
  int32_t ldq = 0;
  float rope_theta = 10000.f;
  int32_t head_dim = 128;
  int32_t layer = 0;
  const int32_t* row_tenant = nullptr;
  const int32_t* row_pos = nullptr;
  KvView kv;
  int32_t dbg = 0;  // measurement hook: bit 0 skips the consumer math, bit 1 records phase times
  unsigned long long* dbg_ts = nullptr;  // [cta][8] %globaltimer stamps when dbg & 2
  const int8_t* rexp = nullptr;  // per-row exponents of the tcgen05 GEMM (rowexp_launch)
  // scratch / status
  float* partials = nullptr;
  int32_t* counters = nullptr;
  uint32_t* err = nullptr;
};

// A chain of GEMVs run by one persistent launch (phase p + 1 may read what
// phase p wrote when bit p + 1 of bar_mask is set: a grid barrier separates
// them). A single GEMV is a chain of one phase.
constexpr int kMaxPhases = 6;
constexpr int kStampSlots = 24;  // %globaltimer stamps per CTA and phase (measurement hook)
struct ChainArgs {
  GemvArgs ph[kMaxPhases];
  int32_t n_phases = 0;
  uint32_t bar_mask = 0;
  unsigned long long* gbar = nullptr;  // [kMaxPhases] grid-barrier arrival counters (monotonic, start at 0)
  int32_t stages = 0, stage_bytes = 0;  // ring geometry, set by gemv_chain_launch
  // weight units a producer may issue for a phase before the grid barrier that
  // phase waits on has passed (< 0: the whole ring)
  int32_t prefetch = -1;
  // failure-detection test hook: barrier slot whose target is moved out of
  // reach (0: none), and the poll limit of every grid-barrier wait (0: default)
  int32_t fail_bar = 0;
  uint32_t grid_spin = 0;
};

// Scratch needed by one GEMV launch (partials in floats, counters in ints).
size_t gemv_partials_floats(int num_ctas, int nt, int n_phases = 1);
int gemv_ctas(int num_sms, int n_rg, int nsb);
int gemv_nt_for(int m);
// Launch with programmatic dependent launch enabled when pdl != 0. A chain of
// more than one phase runs on num_sms CTAs; all its phases use the same NT
// (same m). Split-K counters of different phases must not overlap.
cudaError_t gemv_launch(const GemvArgs& a, int num_sms, cudaStream_t s, int pdl);
cudaError_t gemv_chain_launch(const ChainArgs& c, int num_sms, cudaStream_t s, int pdl);

// tcgen05 dequant-GEMM for 16 <= m <= 64 (a.xin.xf fragments in, the same
// epilogues as the GEMV out): two launches (GEMM, then partial sums +
// epilogue). a.rexp: per-row exponents from rowexp_launch; part: scratch of
// qgemm_part_floats(plan) floats.
struct QgemmPlan {
  int G = 0, n_rt = 0, kG = 0, slots = 0;
  long long U = 0;
};
QgemmPlan qgemm_plan(int num_sms, int n_rg, int nsb);
size_t qgemm_part_floats(const QgemmPlan& p);
cudaError_t rowexp_launch(const uint8_t* tiled, int dtype, int n_rg, int nsb, int8_t* out, cudaStream_t s);
// Q4_K runs the exact-weight GEMM, which also needs bprep: qgemm_bprep_bytes(nsb)
// bytes of scratch for its activation planes (null: the hi/lo-weight GEMM).
size_t qgemm_bprep_bytes(int nsb);
cudaError_t qgemm_launch(const GemvArgs& a, float* part, uint8_t* bprep, const QgemmPlan& p, cudaStream_t s,
                         int pdl);

// Repack GGUF blocks into the tiled layout. Source rows come from up to two
// matrices: mode 0 plain (rows of a), 1 concat (a then b), 2 interleave-8
// (tile rows 0-7 from a, 8-15 from b, same output index).
cudaError_t repack_launch(const uint8_t* a, int rows_a, const uint8_t* b, int rows_b, int mode, int dtype,
                          int k, uint8_t* out, int n_rg, cudaStream_t s);
cudaError_t unpack_launch(const uint8_t* tiled, int dtype, int n, int k, uint8_t* out, cudaStream_t s);

// Element-wise dequant (GGUF layout) and quantisers.
cudaError_t dequant_launch(int dtype, const uint8_t* blocks, size_t nblocks, float* out, cudaStream_t s);
cudaError_t quantize_launch(int dtype, const float* x, size_t n, uint8_t* out, cudaStream_t s);

}  // namespace rb
