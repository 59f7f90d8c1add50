// Paged KV cache kernels and paged GQA decode attention.
#pragma once
#include <cuda.h>

#include "gemv.cuh"

namespace rb {

// fp16 pools are also described by a TMA tensor map: the pool as a 2-D
// tensor [page * layer * (K|V) * kv head * 16 token rows][head_dim] fp16,
// boxes of 16 rows x 64 columns (128 bytes) with 128-byte swizzle.
cudaError_t kv_tensor_map(const KvView& kv, size_t n_pages, CUtensorMap* out);

struct AttnArgs {
  CUtensorMap kv_tmap;             // fp16 pools (kv_tensor_map); unused for fp32
  int32_t n_rows = 0;              // query rows (tenant, position) pairs
  const int32_t* row_tenant = nullptr;
  const int32_t* row_pos = nullptr;  // row attends to positions [0, pos]
  const float* q = nullptr;        // [n_rows][ldq], head h at h*hd
  int32_t ldq = 0;
  float* out = nullptr;            // [n_rows][ldo] fp32 (optional)
  int32_t ldo = 0;
  XFrags xout;                     // optional: output as activation fragments (xfrag.cuh)
  int32_t xf_nt = 1;               //   for the next GEMV, with xf_nt n-tiles
  int32_t n_heads = 0;
  int32_t layer = 0;
  float scale = 0.f;
  KvView kv;
  float* partials = nullptr;       // attn_partials_floats(grid) floats (split pairs)
  int32_t* counters = nullptr;     // [n_rows * n_kv], zero between launches
  uint32_t* err = nullptr;
  // 1: positions, tenants, page tables and every cached token below the rows'
  // smallest position are final before the previous kernel starts, so those
  // pages may be read before it completes (the decode step); 0: wait first
  int32_t early_kv = 0;
  // 1: consecutive rows of one tenant at consecutive positions share K/V pages
  // (the grouped kernel variant: up to 4 query columns per pair on fp16 pools);
  // 0: one row per pair (decode steps, where no two rows share a tenant)
  int32_t group_rows = 1;
  // 1: when the pairs are few and even enough, each CTA takes one (row, kv head)
  // pair whole instead of an even share of all pages (no cross-CTA merge)
  int32_t whole_pairs = 1;
  // set by attn_launch when a prompt-chunk kernel takes the rows that belong to
  // runs of consecutive positions of one tenant: the decode kernel skips them
  int32_t skip_chunked = 0;
  unsigned long long* dbg_ts = nullptr;  // measurement hook: [cta][8] %globaltimer stamps (or null)
};

// Partial-result scratch for a launch on num_ctas CTAs (attn_grid) over a pool
// of n_kv kv heads.
size_t attn_partials_floats(int num_ctas, int n_rep, int hd, int n_kv);
int attn_grid(int num_sms);
// Enqueues the attention of a step: one kernel, or (fp16 pools, n_rep 4 or 8,
// group_rows) the prompt-chunk kernel for runs of consecutive rows of one
// tenant followed by the decode kernel for the other rows. *launches (if
// given) is increased by the number of kernels enqueued.
cudaError_t attn_launch(const AttnArgs& a, int num_sms, cudaStream_t s, int pdl, int* launches = nullptr);

// Standalone append of k/v rows ([n_rows][n_kv*hd] fp32) at (tenant, pos).
cudaError_t kv_append_launch(const KvView& kv, int layer, int n_rows, const int32_t* row_tenant,
                             const int32_t* row_pos, const float* k, const float* v, cudaStream_t s);
// Gather one tenant/layer's first `len` positions into [len][n_kv][hd] fp32.
cudaError_t kv_gather_launch(const KvView& kv, int layer, int tenant, int len, float* k_out, float* v_out,
                             cudaStream_t s);

}  // namespace rb
