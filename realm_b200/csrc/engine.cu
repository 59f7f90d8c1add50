// Host runtime behind the C ABI: contexts, resident weights, paged KV pools,
// models and the batched forward (decode step) with CUDA-graph replay.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <chrono>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <string>
#include <vector>

#include "../../include/realm_b200.h"
#include "attention.cuh"
#include "common.cuh"
#include "gemv.cuh"
#include "quant.cuh"
#include "sample.cuh"
#include "xfrag.cuh"

namespace rb {

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define RB_CUDA(call)                                                                         \
  do {                                                                                        \
    cudaError_t e_ = (call);                                                                  \
    if (e_ != cudaSuccess) return fail(RB_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

// ---------------------------------------------------------------------------
// small kernels owned by the runtime
// ---------------------------------------------------------------------------
struct StepDesc {  // device view of one forward step (filled by one H2D copy)
  int32_t n_rows;
  int32_t n_updates;
  int32_t* row_tenant;
  int32_t* row_pos;
  int32_t* tokens;
  int32_t* upd;  // [n_updates][3] (tenant, page index, physical page)
};

// Embedding rows (bit-exact dequant of token_embd, model.rs:579-596 /
// memory64_host.rs:2570-2583), page-table updates, argmax reset, the
// per-128-column sums of squares feeding the first fused RMSNorm, and the
// activation fragments of x * attn_norm for layer 0's q|k|v GEMV.
// Embedding rows (one CTA per row and 256-column block): dequantised token
// rows into x, sums of squares per 128 columns, and the activation fragments
// of x * norm_w for the first GEMV. CTA (0, 0) also applies the step's page
// table updates.
__global__ void embed_kernel(const uint8_t* embd, int dtype, int hidden, const int32_t* desc_i, int32_t* ptab,
                             int ptab_stride, float* x, int ldx, float* ss, int ld_ss, unsigned long long* argmax,
                             const float* norm_w, int nt, XFrags frags) {
  const int n_rows = desc_i[0], n_upd = desc_i[1];
  const int32_t* row_tokens = desc_i + 2 + 2 * 64;
  const int32_t* upd = desc_i + 2 + 3 * 64;
  const int r = blockIdx.x, c0 = blockIdx.y * 256;
  if (r == 0 && blockIdx.y == 0) {
    for (int i = threadIdx.x; i < n_upd; i += blockDim.x)
      ptab[(size_t)upd[3 * i] * ptab_stride + upd[3 * i + 1]] = upd[3 * i + 2];
  }
  if (r >= n_rows) return;
  if (threadIdx.x == 0 && blockIdx.y == 0 && argmax) argmax[r] = 0ull;
  const int tok = row_tokens[r];
  const int be = block_elems(dtype), bb = block_bytes(dtype);
  const size_t row_bytes = (size_t)(hidden / be) * bb;
  const uint8_t* src = embd + (size_t)tok * row_bytes;
  float* xr = x + (size_t)r * ldx;
  __shared__ float T[256];
  __shared__ float red[8];
  for (int j = threadIdx.x; j < 256; j += blockDim.x) {
    const int i = c0 + j;
    float v = 0.f;
    if (i < hidden) {
      const uint8_t* blk = src + (size_t)(i / be) * bb;
      const int e = i % be;
      v = dtype == DT_Q4_K ? dequant_q4k_elem(blk, e)
        : dtype == DT_Q6_K ? dequant_q6k_elem(blk, e)
        : dtype == DT_Q8_0 ? dequant_q80_elem(blk, e)
                           : reinterpret_cast<const float*>(embd)[(size_t)tok * hidden + i];
      xr[i] = v;
    }
    T[j] = v;
  }
  __syncthreads();
  if (ss) {
    // one sum of squares per 128 columns, in the order a single thread would add
    // warp-reduced parts: 4 warps x 32 lanes over each 128-column half
    for (int hlf = 0; hlf < 2; ++hlf) {
      float sq = 0.f;
      if (threadIdx.x < 128) {
        const float v = T[hlf * 128 + threadIdx.x];
        sq = v * v;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      if ((threadIdx.x & 31) == 0 && threadIdx.x < 128) red[hlf * 4 + (threadIdx.x >> 5)] = sq;
    }
    __syncthreads();
    if (threadIdx.x < 2 && c0 + threadIdx.x * 128 < hidden) {
      const float* q = red + threadIdx.x * 4;
      ss[(size_t)(c0 / 128 + threadIdx.x) * ld_ss + r] = (q[0] + q[1]) + (q[2] + q[3]);
    }
  }
  if (!frags.xi && !frags.xf) return;
  __shared__ float scratch[8];
  __syncthreads();
  frags_write(T, 1, 0, 256, 1, c0, r, norm_w, frags, nt, scratch, threadIdx.x, blockDim.x, [] { __syncthreads(); });
}

__global__ void zero_u64_kernel(unsigned long long* p, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = 0ull;
}

// Plain tiled fp32 GEMM for the candle_matmul host functions (not on the decode path).
__global__ void sgemm_kernel(const float* A, const float* B, float* Cm, int M, int K, int N, int b_trans) {
  __shared__ float As[16][17], Bs[16][17];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
  float acc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    As[ty][tx] = (row < M && k0 + tx < K) ? A[(size_t)row * K + k0 + tx] : 0.f;
    const int bk = k0 + ty;
    Bs[ty][tx] = (bk < K && col < N) ? (b_trans ? B[(size_t)col * K + bk] : B[(size_t)bk * N + col]) : 0.f;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) acc = fmaf(As[ty][kk], Bs[kk][tx], acc);
    __syncthreads();
  }
  if (row < M && col < N) Cm[(size_t)row * N + col] = acc;
}

// ---------------------------------------------------------------------------
// resources
// ---------------------------------------------------------------------------
struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p(o.p), n(o.n) { o.p = nullptr; o.n = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) { release(); p = o.p; n = o.n; o.p = nullptr; o.n = 0; }
    return *this;
  }
  ~DevBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  cudaError_t alloc(size_t bytes) {
    release();
    if (bytes == 0) return cudaSuccess;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) n = bytes;
    return e;
  }
  template <class T> T* as() const { return reinterpret_cast<T*>(p); }
};

struct Weight {
  int dtype = 0, n = 0, k = 0, n_rg = 0;
  int k_in = 0;  // caller's K; k is K rounded up to 256 (Q8_0 rows are zero-padded)
  DevBuf tiled;
  DevBuf rexp;   // per-row power-of-two exponent of the tcgen05 GEMM's fp16 operands (int8)
};

// Device storage for one GEMV input's activation fragments (xfrag.cuh).
struct FragBuf {
  DevBuf f, i, i3, c, s;
  cudaError_t alloc(int k, int nt) {
    cudaError_t e;
    if ((e = f.alloc(xf_bytes(k, nt))) != cudaSuccess) return e;
    if ((e = i.alloc(xi_bytes(k, nt))) != cudaSuccess) return e;
    if ((e = i3.alloc(x3_bytes(k, nt))) != cudaSuccess) return e;
    if ((e = c.alloc(xc_bytes(k, nt))) != cudaSuccess) return e;
    return s.alloc(xs_bytes(k, nt));
  }
  XFrags view() const {
    XFrags v;
    v.xf = f.as<uint4>();
    v.xi = i.as<uint4>();
    v.x3 = i3.as<uint2>();
    v.xc = c.as<float>();
    v.xs = s.as<uint32_t>();
    return v;
  }
  // the encodings a GEMV of this dtype reads (producers skip the others):
  // Q4_K int8 limbs, scales and sums; Q6_K / Q8_0 fp16 hi/lo and sums; -1
  // (the tcgen05 GEMM of any dtype) fp16 hi/lo and sums
  XFrags view_for(int consumer_dtype) const {
    XFrags v = view();
    if (consumer_dtype == DT_Q4_K) v.xf = nullptr;
    else v.xi = nullptr, v.x3 = nullptr, v.xc = nullptr;
    return v;
  }
};

struct KvTenant {
  bool live = false;
  std::vector<int> len;    // per layer
  std::vector<int> pages;  // physical ids
};

struct KvPool {
  int n_layers = 0, n_kv = 0, hd = 0, f16 = 1, max_tenants = 0, max_seq = 0, max_pages_per_tenant = 0;
  int n_pages = 0;
  DevBuf pool, ptab;
  CUtensorMap tmap;  // fp16 pools: the pool as a TMA tensor (kv_tensor_map)
  std::vector<int32_t> h_ptab;
  std::vector<int> free_list;  // stack; back() is handed out next
  std::vector<KvTenant> tenants;
  KvView view() const {
    KvView v;
    v.pool = pool.p;
    v.f16 = f16;
    v.n_layers = n_layers;
    v.n_kv = n_kv;
    v.hd = hd;
    v.ptab = ptab.as<int32_t>();
    v.ptab_stride = max_pages_per_tenant;
    return v;
  }
};

struct RawTensor {
  int dtype = -1;
  size_t bytes = 0;
  DevBuf d;
};

struct LayerW {
  RawTensor raw[9];  // attn_norm, q, k, v, o, ffn_norm, gate, up, down
  Weight qk, v, o, gu, down;
  bool v_fused = false;
};

struct Model {
  rb_model_config cfg{};
  int pool = -1;
  RawTensor embd, out_norm, out_raw;
  Weight out;
  std::vector<LayerW> layers;
  bool finalized = false;
  // step buffers
  DevBuf x, q, ss, logits, argmax, desc;
  // activation fragments: q|k|v and LM-head input (a), o-proj (o), gate/up (f), down (d)
  FragBuf fa, fo, ff, fd;
  int max_rows = 0;
  std::map<int, cudaGraphExec_t> graphs;  // by 2 * row count + grouped attention
  std::map<int, int> graph_launches;
};

struct Ctx {
  int device = 0, num_sms = 148, max_rows = 64;
  bool pdl = true, graphs = true;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  DevBuf gemv_partials, counters, attn_partials, err;
  size_t attn_partials_cap = 0;
  DevBuf stage_in, stage_out;  // generic device staging for host-pointer calls
  FragBuf xf_scratch;          // activation fragments for rb_weight_matmul inputs
  int xf_scratch_k = 0;
  void* pinned = nullptr;      // step descriptor staging
  size_t pinned_bytes = 0;
  cudaEvent_t pinned_ev = nullptr;  // last copy out of `pinned` (reuse waits on it)
  std::vector<std::unique_ptr<Weight>> weights;
  std::vector<std::unique_ptr<KvPool>> pools;
  std::vector<std::unique_ptr<Model>> models;
  float last_ms = 0.f;
  int last_launches = 0;
  int gemv_dbg = 0;  // measurement hook (RB_GEMV_DBG): bit 0 skips the GEMV math, bit 1 phase stamps
  DevBuf dbg_ts, attn_ts;
  // GEMVs queued to run as one multi-phase launch (chain_add / chain_flush)
  GemvArgs chain_ph[kMaxPhases];
  int chain_n = 0;
  uint32_t chain_mask = 0;
  bool chains = true;  // RB_NO_CHAIN=1 launches every GEMV on its own
  DevBuf gbar;         // grid-barrier arrival counters (one per barrier slot) of multi-phase launches
  int last_chain_phases = 1;
  // tcgen05 GEMM routing (RB_QGEMM): 0 never; 1 every format from 16 rows (test
  // and measurement mode); 2 (default) Q4_K from 33 rows, where the
  // exact-weight GEMM beats the mma.sync GEMV on B200 (16-32 rows stay on the GEMV)
  int qgemm = 2;
  bool gemm_step = false;  // the step being enqueued runs its projections on the tcgen05 GEMM
  int chain_prefetch = -1;  // RB_CHAIN_PREFETCH: next-phase weight units issued ahead of a grid barrier
  int attn_group = 1;       // RB_ATTN_GROUP=0: one attention pair per row (no K/V sharing in prefill chunks)
  bool step_grouped = false;  // the step has consecutive rows of one tenant (a prompt chunk)
  int attn_whole = 1;         // RB_ATTN_WHOLE: 0 always split attention pages evenly over the CTAs; k > 1 whole pairs within k x the even share (1: 3x)
  bool merge_v = true;        // RB_MERGE_V=0: v runs as a phase of its own after q|k
  DevBuf qg_part;      // tcgen05 GEMM partial sums
  DevBuf qg_bprep;     // tcgen05 exact-weight GEMM: activation planes
  // failure-detection test hook (rb_test_fail_next_grid_barrier): when nonzero,
  // the next multi-phase GEMV launch with a grid barrier gets its first
  // barrier's target out of reach and this poll limit for every barrier wait
  uint32_t test_fail_spin = 0;
  // measurement hook (rb_forward_profile): when set, an event is recorded
  // after every launch of the step, tagged with the launch's kind
  std::vector<std::pair<int, cudaEvent_t>>* prof = nullptr;
};

enum ProfKind { PROF_EMBED = 0, PROF_GEMV = 1, PROF_ATTN = 2, PROF_QGEMM = 3, PROF_KINDS = 4 };

void prof_mark(Ctx* c, int kind) {
  if (!c->prof) return;
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return;
  cudaEventRecord(e, c->stream);
  c->prof->push_back({kind, e});
}

// With RB_QGEMM=1, batches of at least this many rows take the tcgen05 dequant-GEMM.
constexpr int kQgemmMinRows = 16;
constexpr int kQgemmAutoMinRows = 33;
// whether a batch of m rows runs its matmuls on the tcgen05 GEMM (Q4_K in the default mode)
bool gemm_rows(const Ctx* c, int m) {
  return (c->qgemm == 1 && m >= kQgemmMinRows) || (c->qgemm == 2 && m >= kQgemmAutoMinRows);
}
bool gemm_for(const Ctx* c, int m, int dtype) { return gemm_rows(c, m) && (c->qgemm == 1 || dtype == DT_Q4_K); }

constexpr int kMaxRowsAbi = 64;
constexpr int kCounters = 1 << 16;
constexpr int kChainCounterStride = 2048;  // split-K counters per chain phase (>= row groups of any GEMV)

int check_err(Ctx* c) {
  uint32_t e[4] = {0, 0, 0, 0};
  RB_CUDA(cudaMemcpyAsync(e, c->err.p, 16, cudaMemcpyDeviceToHost, c->stream));
  RB_CUDA(cudaStreamSynchronize(c->stream));
  if (e[0]) {
    cudaMemsetAsync(c->err.p, 0, 16, c->stream);
    // a timed-out multi-phase launch may have left the barrier count off its grid multiple
    if (c->gbar.p) cudaMemsetAsync(c->gbar.p, 0, 8 * kMaxPhases, c->stream);
    cudaStreamSynchronize(c->stream);
    if (e[0] == DEV_TIMEOUT_GRID)
      return fail(RB_ERR_TIMEOUT, "device wait timed out (grid barrier: target %u, seen %u, cta %u phase %u %s)",
                  e[1], e[2], e[3] >> 8, (e[3] >> 1) & 127, (e[3] & 1) ? "producer" : "consumers");
    return fail(RB_ERR_TIMEOUT, "device wait timed out (code %u)", e[0]);
  }
  return RB_OK;
}

// Bounded host wait on the stream.
int sync_ctx(Ctx* c, double timeout_s = 60.0) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(c->stream);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return fail(RB_ERR_CUDA, "stream: %s", cudaGetErrorString(e));
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > timeout_s)
      return fail(RB_ERR_TIMEOUT, "stream did not finish within %.0f s", timeout_s);
  }
  return check_err(c);
}

// Stage a caller buffer on the device (copy if host). Returns device pointer.
struct Staged {
  DevBuf own;
  const void* dptr = nullptr;
};
int stage(Ctx* c, const void* src, size_t bytes, uint32_t flags, Staged& out) {
  if (flags & RB_PTR_DEVICE) {
    out.dptr = src;
    return RB_OK;
  }
  RB_CUDA(out.own.alloc(bytes ? bytes : 1));
  if (bytes) RB_CUDA(cudaMemcpyAsync(out.own.p, src, bytes, cudaMemcpyHostToDevice, c->stream));
  out.dptr = out.own.p;
  return RB_OK;
}

int ensure_attn_partials(Ctx* c, size_t floats) {
  if (floats <= c->attn_partials_cap) return RB_OK;
  RB_CUDA(c->attn_partials.alloc(floats * 4));
  c->attn_partials_cap = floats;
  return RB_OK;
}

int upload_tiled(Ctx* c, Weight& w, int dtype, int n, int k, const uint8_t* a, int rows_a, const uint8_t* b,
                 int rows_b, int mode) {
  if (dtype != DT_Q4_K && dtype != DT_Q6_K && dtype != DT_Q8_0)
    return fail(RB_ERR_UNSUPPORTED, "dtype %d has no tiled GEMV", dtype);
  // Q8_0 (32-element blocks) rows whose K is not a multiple of 256 are padded
  // with zero blocks up to the next 256-column super-block
  const bool pad = dtype == DT_Q8_0 && (k % kSuperK) != 0;
  if (dtype == DT_Q8_0 ? (k % 32) != 0 : (k % kSuperK) != 0)
    return fail(RB_ERR_UNSUPPORTED, "K=%d must be a multiple of %d", k, dtype == DT_Q8_0 ? 32 : 256);
  const int kp = (k + kSuperK - 1) / kSuperK * kSuperK;
  DevBuf pa, pb;
  if (pad) {
    const size_t row_in = (size_t)(k / 32) * 34, row_out = (size_t)(kp / 32) * 34;
    RB_CUDA(pa.alloc(row_out * rows_a));
    RB_CUDA(cudaMemsetAsync(pa.p, 0, row_out * rows_a, c->stream));
    RB_CUDA(cudaMemcpy2DAsync(pa.p, row_out, a, row_in, row_in, rows_a, cudaMemcpyDeviceToDevice, c->stream));
    a = pa.as<uint8_t>();
    if (b && rows_b) {
      RB_CUDA(pb.alloc(row_out * rows_b));
      RB_CUDA(cudaMemsetAsync(pb.p, 0, row_out * rows_b, c->stream));
      RB_CUDA(cudaMemcpy2DAsync(pb.p, row_out, b, row_in, row_in, rows_b, cudaMemcpyDeviceToDevice, c->stream));
      b = pb.as<uint8_t>();
    }
  }
  w.dtype = dtype;
  w.n = n;
  w.k = kp;
  w.k_in = k;
  w.n_rg = (n + kRowGroup - 1) / kRowGroup;
  RB_CUDA(w.tiled.alloc((size_t)w.n_rg * (kp / kSuperK) * unit_bytes(dtype)));
  RB_CUDA(repack_launch(a, rows_a, b, rows_b, mode, dtype, kp, w.tiled.as<uint8_t>(), w.n_rg, c->stream));
  RB_CUDA(w.rexp.alloc((size_t)w.n_rg * kRowGroup));
  RB_CUDA(rowexp_launch(w.tiled.as<uint8_t>(), dtype, w.n_rg, kp / kSuperK, w.rexp.as<int8_t>(), c->stream));
  if (pad) RB_CUDA(cudaStreamSynchronize(c->stream));  // the padded copies are freed on return
  return RB_OK;
}

GemvArgs base_args(Ctx* c, const Weight& w, int m) {
  GemvArgs a;
  a.w = w.tiled.as<uint8_t>();
  a.dtype = w.dtype;
  a.n = w.n;
  a.n_rg = w.n_rg;
  a.nsb = w.k / kSuperK;
  a.m = m;
  a.rexp = w.rexp.as<int8_t>();
  a.partials = c->gemv_partials.as<float>();
  a.counters = c->counters.as<int32_t>();
  a.err = c->err.as<uint32_t>();
  a.dbg = c->gemv_dbg;
  if (c->gemv_dbg & 2) {
    a.dbg_ts = c->dbg_ts.as<unsigned long long>();
  }
  return a;
}

int launch_gemv(Ctx* c, const GemvArgs& a, int* launches) {
  RB_CUDA(gemv_launch(a, c->num_sms, c->stream, c->pdl ? 1 : 0));
  prof_mark(c, PROF_GEMV);
  if (launches) ++*launches;
  return RB_OK;
}

// Grows the tcgen05 GEMM's partial-sum scratch to cover a weight of n_rg row
// groups and nsb super-blocks (never during a stream capture: call first).
int ensure_qg_part(Ctx* c, int n_rg, int nsb) {
  const size_t need = qgemm_part_floats(qgemm_plan(c->num_sms, n_rg, nsb)) * 4;
  if (c->qg_part.n < need) {
    if (c->qg_part.p) RB_CUDA(cudaStreamSynchronize(c->stream));  // earlier launches may still read it
    RB_CUDA(c->qg_part.alloc(need));
  }
  const size_t bneed = qgemm_bprep_bytes(nsb);
  if (c->qg_bprep.n < bneed) {
    if (c->qg_bprep.p) RB_CUDA(cudaStreamSynchronize(c->stream));
    RB_CUDA(c->qg_bprep.alloc(bneed));
  }
  return RB_OK;
}

// y = x . W^T through the tcgen05 GEMM (a.m >= kQgemmMinRows; a.xin.xf holds x):
// the GEMM, then the partial sums and the fused epilogue (two launches).
int launch_qgemm(Ctx* c, const GemvArgs& a, int* launches) {
  const QgemmPlan p = qgemm_plan(c->num_sms, a.n_rg, a.nsb);
  if (c->qg_part.n < qgemm_part_floats(p) * 4 || c->qg_bprep.n < qgemm_bprep_bytes(a.nsb))
    return fail(RB_ERR_INVALID, "GEMM scratch not sized for this weight");
  RB_CUDA(qgemm_launch(a, c->qg_part.as<float>(), c->qg_bprep.as<uint8_t>(), p, c->stream, c->pdl ? 1 : 0));
  prof_mark(c, PROF_QGEMM);
  if (launches) *launches += a.dtype == DT_Q4_K ? 3 : 2;
  return RB_OK;
}

// Measurement hook (RB_GEMV_DBG bit 1): per phase, over the CTAs that had
// units, min / mean / max of each stamp (microseconds after the first CTA's
// first stamp) of the most recent GEMV launch.
void dump_stamps(Ctx* c, int n_phases) {
  const int G = c->num_sms;
  std::vector<unsigned long long> ts((size_t)G * kMaxPhases * kStampSlots);
  if (cudaMemcpy(ts.data(), c->dbg_ts.p, ts.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return;
  unsigned long long t0 = ~0ull;
  for (unsigned long long v : ts)
    if (v) t0 = std::min(t0, v);
  const char* names[kStampSlots] = {"cons_start", "cons_dep_ok", "cons_first_full", "cons_last_unit",
                                    "cons_done", "prod_first_w", "prod_x_released", "prod_last_w",
                                    "seg_begin", "seg_deposited", "seg_ticket", "seg_summed",
                                    "seg_epi_done", "resid_elems", "resid_ss", "resid_frags",
                                    "seg_fenced", "grid_arrived", "s18", "s19", "s20", "s21", "s22", "s23"};
  for (int p = 0; p < n_phases; ++p)
    for (int k = 0; k < kStampSlots; ++k) {
      double mn = 1e30, mx = 0, sum = 0;
      int n = 0;
      for (int b = 0; b < G; ++b) {
        const unsigned long long v = ts[((size_t)b * kMaxPhases + p) * kStampSlots + k];
        if (!v) continue;
        const double d = (double)(v - t0) / 1000.0;
        mn = std::min(mn, d);
        mx = std::max(mx, d);
        sum += d;
        ++n;
      }
      if (n) fprintf(stderr, "[gemv phase %d] %-16s n %3d min %8.2f mean %8.2f max %8.2f us\n", p, names[k], n, mn,
                     sum / n, mx);
    }
  // the three CTAs with the longest tail (last unit -> done), slots relative to their last unit
  for (int p = 0; p < n_phases; ++p) {
    std::vector<std::pair<double, int>> tails;
    for (int b = 0; b < G; ++b) {
      const unsigned long long* t = &ts[((size_t)b * kMaxPhases + p) * kStampSlots];
      if (t[3] && t[4]) tails.push_back({(double)(t[4] - t[3]) / 1000.0, b});
    }
    std::sort(tails.rbegin(), tails.rend());
    for (size_t i = 0; i < tails.size() && i < 3; ++i) {
      const int b = tails[i].second;
      const unsigned long long* t = &ts[((size_t)b * kMaxPhases + p) * kStampSlots];
      fprintf(stderr, "[gemv phase %d] slow cta %3d tail %6.2f us:", p, b, tails[i].first);
      for (int k = 8; k < kStampSlots; ++k)
        if (t[k]) fprintf(stderr, " %s %+.2f", names[k], ((double)t[k] - (double)t[3]) / 1000.0);
      fprintf(stderr, "\n");
    }
  }
  cudaMemset(c->dbg_ts.p, 0, ts.size() * 8);
  if (c->attn_ts.p) {  // the most recent attention launch
    const int GA = attn_grid(c->num_sms);
    std::vector<unsigned long long> at((size_t)GA * 8);
    if (cudaMemcpy(at.data(), c->attn_ts.p, at.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return;
    unsigned long long a0 = ~0ull;
    for (int b = 0; b < GA; ++b)
      if (at[b * 8]) a0 = std::min(a0, at[b * 8]);
    const char* an[5] = {"start", "dep_ok", "first_page", "last_merge", "done"};
    for (int k = 0; k < 5; ++k) {
      double mn = 1e30, mx = 0, sum = 0;
      int n = 0;
      for (int b = 0; b < GA; ++b) {
        const unsigned long long v = at[b * 8 + k];
        if (!v) continue;
        const double d = (double)(v - a0) / 1000.0;
        mn = std::min(mn, d);
        mx = std::max(mx, d);
        sum += d;
        ++n;
      }
      if (n) fprintf(stderr, "[attn] %-11s n %3d min %8.2f mean %8.2f max %8.2f us\n", an[k], n, mn, sum / n, mx);
    }
    cudaMemset(c->attn_ts.p, 0, at.size() * 8);
  }
}

// Queued GEMVs run as one persistent multi-phase launch (gemv.cu). A phase
// that reads what the phase before it wrote is separated from it by a grid
// barrier; the first phase of a launch depends on the previous kernel.
int chain_flush(Ctx* c, int* launches) {
  if (c->chain_n == 0) return RB_OK;
  ChainArgs ca;
  for (int p = 0; p < c->chain_n; ++p) ca.ph[p] = c->chain_ph[p];
  ca.n_phases = c->chain_n;
  ca.bar_mask = c->chain_mask;
  ca.gbar = c->gbar.as<unsigned long long>();
  ca.prefetch = c->chain_prefetch;
  if (c->test_fail_spin && c->chain_mask) {
    int b = 1;
    while (!((c->chain_mask >> b) & 1u)) ++b;
    ca.fail_bar = b;
    ca.grid_spin = c->test_fail_spin;
    c->test_fail_spin = 0;
  }
  c->last_chain_phases = c->chain_n;
  c->chain_n = 0;
  c->chain_mask = 0;
  RB_CUDA(gemv_chain_launch(ca, c->num_sms, c->stream, c->pdl ? 1 : 0));
  prof_mark(c, PROF_GEMV);
  if (launches) ++*launches;
  return RB_OK;
}

int chain_add(Ctx* c, GemvArgs a, bool reads_previous, int* launches) {
  if (c->gemm_step && a.dtype == DT_Q4_K) {  // 16+ rows: Q4_K phases run the tcgen05 GEMM + epilogue
    if (int rc = chain_flush(c, launches)) return rc;
    return launch_qgemm(c, a, launches);
  }
  if (!c->chains) {
    a.counters = c->counters.as<int32_t>();
    return launch_gemv(c, a, launches);
  }
  if (c->chain_n == kMaxPhases)
    if (int rc = chain_flush(c, launches)) return rc;
  const int p = c->chain_n;
  // partial-sum slots alternate between phases: two barrier-free transitions
  // in a row would reuse a slot that may still be read, so add a barrier
  if (p >= 2 && !((c->chain_mask >> (p - 1)) & 1u)) reads_previous = true;
  if (p > 0 && reads_previous) c->chain_mask |= 1u << p;
  a.counters = c->counters.as<int32_t>() + p * kChainCounterStride;
  c->chain_ph[p] = a;
  ++c->chain_n;
  return RB_OK;
}

// ---------------------------------------------------------------------------
// model forward (enqueue only). Every GEMV reads activation fragments written by
// the kernel before it: embed -> (q|k, v) -> attention -> o (+residual) ->
// gate/up (SwiGLU) -> down (+residual) -> next layer / LM head.
// ---------------------------------------------------------------------------
int enqueue_layer(Ctx* c, Model& M, int l, int m, const int32_t* d_tenant, const int32_t* d_pos, int* launches) {
  const rb_model_config& cf = M.cfg;
  KvPool& P = *c->pools[M.pool];
  LayerW& L = M.layers[l];
  const int H = cf.hidden, hd = cf.head_dim, Hq = cf.n_heads, Hkv = cf.n_kv_heads;
  const int n_ss = (H + 127) / 128;
  const int NT = gemv_nt_for(m);
  float* x = M.x.as<float>();
  float* ss = M.ss.as<float>();
  // q|k (+v) with fused RMSNorm (weight in the fragments, 1/rms in the epilogue),
  // RoPE and the paged KV append
  GemvArgs a = base_args(c, L.qk, m);
  a.xin = M.fa.view();
  a.ss_part = ss;
  a.n_ss = n_ss;
  a.ld_ss = kMaxRowsAbi;
  a.norm_eps = cf.layer_eps;
  a.norm_dim = H;
  a.epi = EPI_QKV;
  a.qkv_row0 = 0;
  a.n_q_rows = Hq * hd;
  a.n_k_rows = Hkv * hd;
  a.q_out = M.q.as<float>();
  a.ldq = Hq * hd;
  a.rope_theta = cf.rope_theta;
  a.head_dim = hd;
  a.layer = l;
  a.row_tenant = d_tenant;
  a.row_pos = d_pos;
  a.kv = P.view();
  // v joins the q|k phase as its second weight (one stream-K split, one tail)
  // unless the step runs its Q4_K projections on the tcgen05 GEMM
  const bool merge_v = c->merge_v && !L.v_fused && !c->gemm_step && L.v.k == L.qk.k &&
                       (m <= 8 ? (L.qk.dtype == DT_Q4_K ? L.v.dtype == DT_Q6_K : L.v.dtype == L.qk.dtype)
                               : L.v.dtype == L.qk.dtype);
  if (merge_v) {
    a.w2 = L.v.tiled.as<uint8_t>();
    a.dtype2 = L.v.dtype;
    a.n2 = L.v.n;
    a.n_rg2 = L.v.n_rg;
    a.qkv_row0_2 = (Hq + Hkv) * hd;
  }
  if (int rc = chain_add(c, a, true, launches)) return rc;
  if (!L.v_fused && !merge_v) {
    GemvArgs av = a;
    av.w = L.v.tiled.as<uint8_t>();
    av.dtype = L.v.dtype;
    av.n = L.v.n;
    av.n_rg = L.v.n_rg;
    av.nsb = L.v.k / kSuperK;
    av.qkv_row0 = (Hq + Hkv) * hd;
    if (int rc = chain_add(c, av, false, launches)) return rc;
  }
  if (int rc = chain_flush(c, launches)) return rc;
  // paged GQA attention -> fragments of the o-proj input
  AttnArgs at;
  at.n_rows = m;
  at.row_tenant = d_tenant;
  at.row_pos = d_pos;
  at.q = M.q.as<float>();
  at.ldq = Hq * hd;
  at.out = nullptr;
  at.xout = M.fo.view_for(c->gemm_step ? -1 : L.o.dtype);
  at.xf_nt = NT;
  at.n_heads = Hq;
  at.layer = l;
  at.scale = 1.0f / sqrtf((float)hd);  // attention_stub/mod.rs:57
  at.kv = P.view();
  at.kv_tmap = P.tmap;
  at.partials = c->attn_partials.as<float>();
  at.counters = c->counters.as<int32_t>() + kCounters / 2;
  at.err = c->err.as<uint32_t>();
  at.early_kv = 1;  // the step's descriptor and page tables precede the step's first kernel
  at.group_rows = c->attn_group && c->step_grouped;
  at.whole_pairs = c->attn_whole;
  if (c->gemv_dbg & 2) at.dbg_ts = c->attn_ts.as<unsigned long long>();
  RB_CUDA(attn_launch(at, c->num_sms, c->stream, c->pdl ? 1 : 0, launches));
  prof_mark(c, PROF_ATTN);
  // o-proj + residual; writes fragments of x * ffn_norm
  GemvArgs ao = base_args(c, L.o, m);
  ao.xin = M.fo.view();
  ao.epi = EPI_RESID;
  ao.resid = x;
  ao.ldr = H;
  ao.ss_out = ss;
  ao.ld_ss = kMaxRowsAbi;
  ao.xout = M.ff.view_for(c->gemm_step ? -1 : L.gu.dtype);
  ao.xf_norm = L.raw[5].d.as<float>();
  if (int rc = chain_add(c, ao, true, launches)) return rc;
  // gate/up (interleaved) with fused RMSNorm and SwiGLU -> fragments of h
  GemvArgs ag = base_args(c, L.gu, m);
  ag.xin = M.ff.view();
  ag.ss_part = ss;
  ag.n_ss = n_ss;
  ag.ld_ss = kMaxRowsAbi;
  ag.norm_eps = cf.layer_eps;
  ag.norm_dim = H;
  ag.epi = EPI_SWIGLU;
  ag.xout = M.fd.view_for(c->gemm_step ? -1 : L.down.dtype);
  if (int rc = chain_add(c, ag, true, launches)) return rc;
  // down + residual; writes fragments of x * (next layer's attn_norm | output_norm)
  GemvArgs ad = base_args(c, L.down, m);
  ad.xin = M.fd.view();
  ad.epi = EPI_RESID;
  ad.resid = x;
  ad.ldr = H;
  ad.ss_out = ss;
  ad.ld_ss = kMaxRowsAbi;
  ad.xout = M.fa.view();
  ad.xf_norm = (l + 1 < (int)cf.n_layers) ? M.layers[l + 1].raw[0].d.as<float>() : M.out_norm.d.as<float>();
  // left queued: the next layer's q|k, v (or the LM head) join this launch
  return chain_add(c, ad, true, launches);
}

int enqueue_head(Ctx* c, Model& M, int m, bool want_logits, int* launches) {
  const rb_model_config& cf = M.cfg;
  GemvArgs a = base_args(c, M.out, m);
  a.xin = M.fa.view();
  a.ss_part = M.ss.as<float>();
  a.n_ss = (cf.hidden + 127) / 128;
  a.ld_ss = kMaxRowsAbi;
  a.norm_eps = cf.rms_eps;
  a.norm_dim = cf.hidden;
  a.epi = EPI_LOGITS;
  a.y = want_logits ? M.logits.as<float>() : nullptr;
  a.ldy = cf.vocab;
  a.argmax = M.argmax.as<unsigned long long>();
  if (int rc = chain_add(c, a, true, launches)) return rc;
  return chain_flush(c, launches);
}

// Descriptor layout in int32s: [n_rows, n_upd, tenant[64], pos[64], tokens[64], upd[...][3]]
constexpr int kDescTenant = 2, kDescPos = 2 + 64, kDescTok = 2 + 128, kDescUpd = 2 + 192;

int enqueue_step(Ctx* c, Model& M, int m, int* launches) {
  const rb_model_config& cf = M.cfg;
  c->gemm_step = gemm_rows(c, m);
  KvPool& P = *c->pools[M.pool];
  int32_t* desc = M.desc.as<int32_t>();
  embed_kernel<<<dim3(m, (cf.hidden + 255) / 256), 128, 0, c->stream>>>(
      M.embd.d.as<uint8_t>(), M.embd.dtype, cf.hidden, desc, P.ptab.as<int32_t>(),
                                         P.max_pages_per_tenant, M.x.as<float>(), cf.hidden, M.ss.as<float>(),
                                         kMaxRowsAbi, M.argmax.as<unsigned long long>(),
                                         M.layers[0].raw[0].d.as<float>(), gemv_nt_for(m), M.fa.view());
  RB_CUDA(cudaGetLastError());
  prof_mark(c, PROF_EMBED);
  if (launches) ++*launches;
  for (int l = 0; l < (int)cf.n_layers; ++l)
    if (int rc = enqueue_layer(c, M, l, m, desc + kDescTenant, desc + kDescPos, launches)) return rc;
  return enqueue_head(c, M, m, true, launches);
}

}  // namespace rb

// ===========================================================================
// C ABI
// ===========================================================================
using namespace rb;

struct rb_ctx : Ctx {};

namespace {

__global__ void ptab_update_kernel(const int32_t* desc, int32_t* ptab, int stride) {
  const int n_upd = desc[1];
  const int32_t* upd = desc + kDescUpd;
  for (int i = threadIdx.x; i < n_upd; i += blockDim.x) ptab[(size_t)upd[3 * i] * stride + upd[3 * i + 1]] = upd[3 * i + 2];
}

KvPool* get_pool(rb_ctx* c, int32_t pool) {
  if (!c || pool < 0 || pool >= (int)c->pools.size() || !c->pools[pool]) return nullptr;
  return c->pools[pool].get();
}
Model* get_model(rb_ctx* c, int32_t model) {
  if (!c || model < 0 || model >= (int)c->models.size() || !c->models[model]) return nullptr;
  return c->models[model].get();
}

// Rows for one step: validates positions, allocates pages, fills the pinned
// descriptor. rank_layer < 0 checks all layers' lengths (model forward).
struct RowPlan {
  std::vector<int> tenant, pos, tok;
  std::vector<int> upd;  // triples
};

int plan_rows(KvPool& P, int n, const uint32_t* tenants, const uint32_t* tokens, const uint32_t* positions,
              int layer, RowPlan& rp) {
  rp.tenant.assign(n, 0);
  rp.pos.assign(n, 0);
  rp.tok.assign(n, 0);
  rp.upd.clear();
  std::map<int, int> rank;
  for (int r = 0; r < n; ++r) {
    const uint32_t t = tenants[r];
    if (t >= (uint32_t)P.max_tenants || !P.tenants[t].live) return fail(RB_ERR_NOT_FOUND, "tenant %u not created", t);
    KvTenant& T = P.tenants[t];
    const int base = T.len[layer < 0 ? 0 : layer];
    if (layer < 0)
      for (int l = 1; l < P.n_layers; ++l)
        if (T.len[l] != base) return fail(RB_ERR_INVALID, "tenant %u layers out of step", t);
    const int expect = base + rank[t]++;
    const int pos = positions ? (int)positions[r] : expect;
    if (pos != expect) return fail(RB_ERR_INVALID, "row %d: position %d != cache length %d", r, pos, expect);
    if (pos >= P.max_seq)
      return fail(RB_ERR_KV_OVERFLOW, "KV cache overflow: %d + 1 > %d", pos, P.max_seq);
    rp.tenant[r] = (int)t;
    rp.pos[r] = pos;
    rp.tok[r] = tokens ? (int)tokens[r] : 0;
  }
  // page allocation (all-or-nothing)
  std::vector<std::pair<int, int>> taken;
  for (int r = 0; r < n; ++r) {
    KvTenant& T = P.tenants[rp.tenant[r]];
    const int idx = rp.pos[r] >> 4;
    while ((int)T.pages.size() <= idx) {
      if (P.free_list.empty()) {
        for (auto it = taken.rbegin(); it != taken.rend(); ++it) {
          P.tenants[it->first].pages.pop_back();
          P.free_list.push_back(it->second);
        }
        return fail(RB_ERR_KV_POOL_EXHAUSTED, "KV page pool exhausted");
      }
      const int pg = P.free_list.back();
      P.free_list.pop_back();
      T.pages.push_back(pg);
      taken.push_back({rp.tenant[r], pg});
      const int pi = (int)T.pages.size() - 1;
      P.h_ptab[(size_t)rp.tenant[r] * P.max_pages_per_tenant + pi] = pg;
      rp.upd.insert(rp.upd.end(), {rp.tenant[r], pi, pg});
    }
  }
  return RB_OK;
}

// Whether some row continues the previous row's tenant at the next position:
// such rows attend as a group (shared K/V pages).
bool rows_grouped(const RowPlan& rp) {
  for (size_t r = 1; r < rp.tenant.size(); ++r)
    if (rp.tenant[r] == rp.tenant[r - 1] && rp.pos[r] == rp.pos[r - 1] + 1) return true;
  return false;
}

int upload_desc(rb_ctx* c, const RowPlan& rp, int32_t* d_desc) {
  const int n = (int)rp.tenant.size(), nu = (int)rp.upd.size() / 3;
  const size_t ints = kDescUpd + 3 * (size_t)nu;
  if (ints * 4 > c->pinned_bytes) return fail(RB_ERR_INVALID, "descriptor too large");
  // an earlier asynchronous call may still be copying out of the staging buffer
  RB_CUDA(cudaEventSynchronize(c->pinned_ev));
  int32_t* h = reinterpret_cast<int32_t*>(c->pinned);
  h[0] = n;
  h[1] = nu;
  for (int r = 0; r < n; ++r) {
    h[kDescTenant + r] = rp.tenant[r];
    h[kDescPos + r] = rp.pos[r];
    h[kDescTok + r] = rp.tok[r];
  }
  std::copy(rp.upd.begin(), rp.upd.end(), h + kDescUpd);
  RB_CUDA(cudaMemcpyAsync(d_desc, h, ints * 4, cudaMemcpyHostToDevice, c->stream));
  RB_CUDA(cudaEventRecord(c->pinned_ev, c->stream));
  return RB_OK;
}

int copy_out(rb_ctx* c, void* dst, const void* src, size_t bytes, uint32_t flags) {
  RB_CUDA(cudaMemcpyAsync(dst, src, bytes,
                          (flags & RB_PTR_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, c->stream));
  return RB_OK;
}

int pool_create(rb_ctx* c, int n_layers, int n_kv, int hd, int kv_dtype, int n_pages, int max_tenants, int max_seq) {
  if (n_layers < 1 || n_kv < 1 || (hd != 64 && hd != 128) || n_pages < 1 || max_tenants < 1 || max_seq < 1)
    return fail(RB_ERR_UNSUPPORTED, "kv pool geometry (layers %d, kv %d, hd %d) unsupported", n_layers, n_kv, hd);
  if (kv_dtype != RB_F16 && kv_dtype != RB_F32) return fail(RB_ERR_UNSUPPORTED, "kv dtype %d", kv_dtype);
  auto P = std::make_unique<KvPool>();
  P->n_layers = n_layers;
  P->n_kv = n_kv;
  P->hd = hd;
  P->f16 = kv_dtype == RB_F16;
  P->n_pages = n_pages;
  P->max_tenants = max_tenants;
  P->max_seq = max_seq;
  P->max_pages_per_tenant = (max_seq + 15) / 16;
  const size_t page_bytes = (size_t)n_layers * 2 * n_kv * 16 * hd * (P->f16 ? 2 : 4);
  if (P->pool.alloc(page_bytes * n_pages) != cudaSuccess) return fail(RB_ERR_OOM, "kv pool of %zu bytes", page_bytes * n_pages);
  RB_CUDA(cudaMemsetAsync(P->pool.p, 0, page_bytes * n_pages, c->stream));
  if (P->f16) RB_CUDA(kv_tensor_map(P->view(), (size_t)n_pages, &P->tmap));
  P->h_ptab.assign((size_t)max_tenants * P->max_pages_per_tenant, 0);
  RB_CUDA(P->ptab.alloc(P->h_ptab.size() * 4));
  RB_CUDA(cudaMemsetAsync(P->ptab.p, 0, P->h_ptab.size() * 4, c->stream));
  for (int i = n_pages - 1; i >= 0; --i) P->free_list.push_back(i);
  P->tenants.resize(max_tenants);
  const int n_rep_max = 8;
  if (int rc = ensure_attn_partials(c, attn_partials_floats(attn_grid(c->num_sms), n_rep_max, hd, n_kv))) return rc;
  c->pools.push_back(std::move(P));
  return (int)c->pools.size() - 1;
}

void tenant_release(KvPool& P, int t) {
  KvTenant& T = P.tenants[t];
  for (auto it = T.pages.rbegin(); it != T.pages.rend(); ++it) P.free_list.push_back(*it);
  T.pages.clear();
  std::fill(T.len.begin(), T.len.end(), 0);
}

// Sizes the tcgen05 GEMM scratch for every projection of the model.
int ensure_qg_model(Ctx* c, Model& M) {
  for (LayerW& L : M.layers)
    for (const Weight* w : {&L.qk, &L.v, &L.o, &L.gu, &L.down})
      if (w->n_rg)
        if (int rc = ensure_qg_part(c, w->n_rg, w->k / kSuperK)) return rc;
  return ensure_qg_part(c, M.out.n_rg, M.out.k / kSuperK);
}

int run_forward(rb_ctx* c, Model& M, int m, bool use_graph) {
  int launches = 0;
  if (c->test_fail_spin) use_graph = false;  // the armed hook must not be baked into a cached graph
  if (gemm_rows(c, m))
    if (int rc = ensure_qg_model(c, M)) return rc;
  RB_CUDA(cudaEventRecord(c->ev0, c->stream));
  if (use_graph) {
    const int key = 2 * m + (c->step_grouped ? 1 : 0);  // the attention variant is part of the graph
    auto it = M.graphs.find(key);
    if (it == M.graphs.end()) {
      cudaGraph_t g = nullptr;
      RB_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
      int rc = enqueue_step(c, M, m, &launches);
      cudaError_t e = cudaStreamEndCapture(c->stream, &g);
      if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      if (e != cudaSuccess) return fail(RB_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
      cudaGraphExec_t ex = nullptr;
      e = cudaGraphInstantiate(&ex, g, 0);
      cudaGraphDestroy(g);
      if (e != cudaSuccess) return fail(RB_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
      it = M.graphs.emplace(key, ex).first;
      M.graph_launches[key] = launches;
    }
    RB_CUDA(cudaGraphLaunch(it->second, c->stream));
    launches = M.graph_launches[key];
  } else {
    if (int rc = enqueue_step(c, M, m, &launches)) return rc;
  }
  RB_CUDA(cudaEventRecord(c->ev1, c->stream));
  c->last_launches = launches;
  return RB_OK;
}

}  // namespace

extern "C" {

int32_t rb_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return (int32_t)g_last_error.size();
  const size_t n = std::min(len - 1, g_last_error.size());
  std::memcpy(buf, g_last_error.data(), n);
  buf[n] = 0;
  return (int32_t)n;
}

int32_t rb_ctx_create(const rb_config* cfg, rb_ctx** out) {
  if (!out) return fail(RB_ERR_INVALID, "out is NULL");
  rb_config def{0, 64, 1, 1};
  if (!cfg) cfg = &def;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(RB_ERR_DISABLED, "no CUDA device");
  if (cfg->device < 0 || cfg->device >= ndev) return fail(RB_ERR_NOT_FOUND, "device %d not present", cfg->device);
  RB_CUDA(cudaSetDevice(cfg->device));
  cudaDeviceProp prop;
  RB_CUDA(cudaGetDeviceProperties(&prop, cfg->device));
  if (prop.major != 10) return fail(RB_ERR_UNSUPPORTED, "device %s is sm_%d%d; this build targets sm_100a", prop.name, prop.major, prop.minor);
  auto c = std::make_unique<rb_ctx>();
  c->device = cfg->device;
  c->num_sms = prop.multiProcessorCount;
  c->max_rows = cfg->max_rows ? std::min<int>(cfg->max_rows, kMaxRowsAbi) : kMaxRowsAbi;
  c->pdl = cfg->use_pdl != 0;
  c->graphs = cfg->use_graphs != 0;
  if (const char* d = getenv("RB_GEMV_DBG")) c->gemv_dbg = atoi(d);
  if (c->gemv_dbg & 2) {
    RB_CUDA(c->dbg_ts.alloc((size_t)c->num_sms * kMaxPhases * kStampSlots * 8));
    RB_CUDA(cudaMemset(c->dbg_ts.p, 0, (size_t)c->num_sms * kMaxPhases * kStampSlots * 8));
    RB_CUDA(c->attn_ts.alloc((size_t)attn_grid(c->num_sms) * 8 * 8));
    RB_CUDA(cudaMemset(c->attn_ts.p, 0, (size_t)attn_grid(c->num_sms) * 8 * 8));
  }
  if (const char* d = getenv("RB_NO_CHAIN")) c->chains = atoi(d) == 0;
  if (const char* d = getenv("RB_QGEMM")) c->qgemm = atoi(d);
  if (const char* d = getenv("RB_CHAIN_PREFETCH")) c->chain_prefetch = atoi(d);
  if (const char* d = getenv("RB_ATTN_GROUP")) c->attn_group = atoi(d) != 0;
  if (const char* d = getenv("RB_ATTN_WHOLE")) c->attn_whole = atoi(d);
  if (const char* d = getenv("RB_MERGE_V")) c->merge_v = atoi(d) != 0;
  RB_CUDA(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
  RB_CUDA(cudaEventCreate(&c->ev0));
  RB_CUDA(cudaEventCreate(&c->ev1));
  RB_CUDA(cudaEventCreateWithFlags(&c->pinned_ev, cudaEventDisableTiming));
  RB_CUDA(cudaEventRecord(c->pinned_ev, c->stream));
  RB_CUDA(c->gemv_partials.alloc(gemv_partials_floats(c->num_sms, 8, kMaxPhases) * 4));
  RB_CUDA(c->counters.alloc(kCounters * 4));
  RB_CUDA(cudaMemsetAsync(c->counters.p, 0, kCounters * 4, c->stream));
  RB_CUDA(c->err.alloc(16));
  RB_CUDA(cudaMemsetAsync(c->err.p, 0, 16, c->stream));
  RB_CUDA(c->gbar.alloc(8 * kMaxPhases));
  RB_CUDA(cudaMemsetAsync(c->gbar.p, 0, 8 * kMaxPhases, c->stream));
  c->pinned_bytes = 64 << 10;
  RB_CUDA(cudaMallocHost(&c->pinned, c->pinned_bytes));
  RB_CUDA(c->stage_in.alloc(c->pinned_bytes));
  RB_CUDA(cudaStreamSynchronize(c->stream));
  *out = c.release();
  return RB_OK;
}

int32_t rb_ctx_destroy(rb_ctx* c) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (auto& m : c->models)
    if (m)
      for (auto& g : m->graphs) cudaGraphExecDestroy(g.second);
  c->models.clear();
  c->pools.clear();
  c->weights.clear();
  if (c->pinned) cudaFreeHost(c->pinned);
  cudaEventDestroy(c->ev0);
  cudaEventDestroy(c->ev1);
  cudaEventDestroy(c->pinned_ev);
  cudaStreamDestroy(c->stream);
  delete c;
  return RB_OK;
}

int32_t rb_sync(rb_ctx* c) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  return sync_ctx(c);
}
void* rb_stream(rb_ctx* c) { return c ? (void*)c->stream : nullptr; }
int32_t rb_num_sms(rb_ctx* c) { return c ? c->num_sms : fail(RB_ERR_BAD_HANDLE, "null context"); }

int32_t rb_test_fail_next_grid_barrier(rb_ctx* c, uint32_t spin_polls) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  c->test_fail_spin = spin_polls ? spin_polls : 1;
  return RB_OK;
}

int32_t rb_kernel_binary_version(rb_ctx* c, int32_t* version) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  if (!version) return fail(RB_ERR_INVALID, "null output");
  RB_CUDA(cudaSetDevice(c->device));
  cudaFuncAttributes fa{};
  RB_CUDA(cudaFuncGetAttributes(&fa, embed_kernel));
  *version = fa.binaryVersion;
  return RB_OK;
}

int32_t rb_dequantize(rb_ctx* c, int32_t dtype, const void* blocks, size_t nblocks, float* out, uint32_t flags) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  if (dtype != DT_Q4_K && dtype != DT_Q6_K && dtype != DT_Q8_0) return fail(RB_ERR_UNSUPPORTED, "dtype %d", dtype);
  const size_t n = nblocks * block_elems(dtype);
  Staged in;
  if (int rc = stage(c, blocks, nblocks * block_bytes(dtype), flags, in)) return rc;
  DevBuf tmp;
  float* dout = out;
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(tmp.alloc(n * 4 + 4));
    dout = tmp.as<float>();
  }
  RB_CUDA(dequant_launch(dtype, (const uint8_t*)in.dptr, nblocks, dout, c->stream));
  if (!(flags & RB_PTR_DEVICE)) RB_CUDA(cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)n;
}

int32_t rb_quantize(rb_ctx* c, int32_t dtype, const float* x, size_t n, void* out_blocks, uint32_t flags) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  if (dtype != DT_Q4_K && dtype != DT_Q6_K && dtype != DT_Q8_0) return fail(RB_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (n % block_elems(dtype)) return fail(RB_ERR_INVALID, "n %% %d != 0", block_elems(dtype));
  const size_t nb = n / block_elems(dtype), ob = nb * block_bytes(dtype);
  Staged in;
  if (int rc = stage(c, x, n * 4, flags, in)) return rc;
  DevBuf tmp;
  uint8_t* dout = (uint8_t*)out_blocks;
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(tmp.alloc(ob + 16));
    dout = tmp.as<uint8_t>();
  }
  RB_CUDA(quantize_launch(dtype, (const float*)in.dptr, n, dout, c->stream));
  if (!(flags & RB_PTR_DEVICE)) RB_CUDA(cudaMemcpyAsync(out_blocks, dout, ob, cudaMemcpyDeviceToHost, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)nb;
}

int32_t rb_weight_upload(rb_ctx* c, int32_t dtype, uint32_t n, uint32_t k, const void* blocks, size_t nbytes,
                         uint32_t flags, int32_t* handle) {
  if (!c || !handle) return fail(RB_ERR_BAD_HANDLE, "null context/handle");
  if (dtype != DT_Q4_K && dtype != DT_Q6_K && dtype != DT_Q8_0) return fail(RB_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (dtype == DT_Q8_0 ? (k % 32) != 0 : (k % kSuperK) != 0)
    return fail(RB_ERR_UNSUPPORTED, "K dimension %u must be multiple of %d", k, dtype == DT_Q8_0 ? 32 : 256);
  const size_t expect = (size_t)n * (k / block_elems(dtype)) * block_bytes(dtype);
  if (nbytes != expect) return fail(RB_ERR_INVALID, "expected %zu bytes, got %zu", expect, nbytes);
  Staged in;
  if (int rc = stage(c, blocks, nbytes, flags, in)) return rc;
  auto w = std::make_unique<Weight>();
  if (int rc = upload_tiled(c, *w, dtype, n, k, (const uint8_t*)in.dptr, n, nullptr, 0, 0)) return rc;
  if (int rc = sync_ctx(c)) return rc;
  c->weights.push_back(std::move(w));
  *handle = (int32_t)c->weights.size() - 1;
  return RB_OK;
}

int32_t rb_weight_free(rb_ctx* c, int32_t h) {
  if (!c || h < 0 || h >= (int)c->weights.size() || !c->weights[h]) return fail(RB_ERR_BAD_HANDLE, "weight %d", h);
  cudaStreamSynchronize(c->stream);
  c->weights[h].reset();
  return RB_OK;
}

static int ensure_xf_scratch(rb_ctx* c, int k) {
  if (c->xf_scratch_k < k) {
    RB_CUDA(c->xf_scratch.alloc(k, 8));
    c->xf_scratch_k = k;
  }
  return RB_OK;
}

static int weight_matmul_dev(rb_ctx* c, const Weight& w, const float* din, float* dout, uint32_t batch) {
  if (int rc = ensure_xf_scratch(c, w.k)) return rc;
  DevBuf xpad;
  if (w.k_in != w.k) {  // zero-padded K (Q8_0): pad the input rows to match
    RB_CUDA(xpad.alloc((size_t)batch * w.k * 4));
    RB_CUDA(cudaMemsetAsync(xpad.p, 0, (size_t)batch * w.k * 4, c->stream));
    RB_CUDA(cudaMemcpy2DAsync(xpad.p, (size_t)w.k * 4, din, (size_t)w.k_in * 4, (size_t)w.k_in * 4, batch,
                              cudaMemcpyDeviceToDevice, c->stream));
    din = xpad.as<float>();
  }
  for (uint32_t b0 = 0; b0 < batch; b0 += kMaxRowsAbi) {
    const int m = (int)std::min<uint32_t>(kMaxRowsAbi, batch - b0);
    const int nt = gemv_nt_for(m);
    RB_CUDA(xfrag_launch(din + (size_t)b0 * w.k, w.k, nullptr, m, w.k, nt, c->xf_scratch.view(), nullptr, 0,
                         c->stream));
    GemvArgs a = base_args(c, w, m);
    a.xin = c->xf_scratch.view();
    a.epi = EPI_STORE;
    a.y = dout + (size_t)b0 * w.n;
    a.ldy = w.n;
    if (gemm_for(c, m, w.dtype)) {
      if (int rc = ensure_qg_part(c, w.n_rg, w.k / kSuperK)) return rc;
      if (int rc = launch_qgemm(c, a, nullptr)) return rc;
    } else if (int rc = launch_gemv(c, a, nullptr)) {
      return rc;
    }
  }
  return RB_OK;
}

int32_t rb_weight_matmul(rb_ctx* c, int32_t h, const float* input, float* output, uint32_t batch, uint32_t flags) {
  if (!c || h < 0 || h >= (int)c->weights.size() || !c->weights[h]) return fail(RB_ERR_BAD_HANDLE, "weight %d", h);
  const Weight& w = *c->weights[h];
  if (batch == 0) return 0;
  Staged in;
  if (int rc = stage(c, input, (size_t)batch * w.k_in * 4, flags, in)) return rc;
  DevBuf tmp;
  float* dout = output;
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(tmp.alloc((size_t)batch * w.n * 4));
    dout = tmp.as<float>();
  }
  if (int rc = weight_matmul_dev(c, w, (const float*)in.dptr, dout, batch)) return rc;
  if (!(flags & RB_PTR_DEVICE)) RB_CUDA(cudaMemcpyAsync(output, dout, (size_t)batch * w.n * 4, cudaMemcpyDeviceToHost, c->stream));
  if ((flags & RB_PTR_DEVICE) && (flags & RB_ASYNC)) return (int32_t)(batch * w.n);
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)(batch * w.n);
}

int32_t rb_weight_matmul_timing(rb_ctx* c, const int32_t* handles, uint32_t n_handles, uint32_t batch, uint32_t iters,
                                uint32_t reps, float* avg_us) {
  if (!c || !handles || !avg_us || n_handles == 0 || iters == 0 || reps == 0) return fail(RB_ERR_INVALID, "bad arguments");
  if (batch == 0 || batch > (uint32_t)kMaxRowsAbi) return fail(RB_ERR_INVALID, "batch %u not in [1, 64]", batch);
  std::vector<const Weight*> ws;
  int k = -1, nmax = 0;
  for (uint32_t i = 0; i < n_handles; ++i) {
    const int32_t h = handles[i];
    if (h < 0 || h >= (int)c->weights.size() || !c->weights[h]) return fail(RB_ERR_BAD_HANDLE, "weight %d", h);
    if (k >= 0 && c->weights[h]->k != k) return fail(RB_ERR_INVALID, "weights differ in K");
    k = c->weights[h]->k;
    nmax = std::max(nmax, c->weights[h]->n);
    ws.push_back(c->weights[h].get());
  }
  const int m = (int)batch, nt = gemv_nt_for(m);
  DevBuf x, y;
  RB_CUDA(x.alloc((size_t)m * k * 4));
  RB_CUDA(y.alloc((size_t)m * nmax * 4));
  RB_CUDA(cudaMemsetAsync(x.p, 0, x.n, c->stream));
  if (int rc = ensure_xf_scratch(c, k)) return rc;
  RB_CUDA(xfrag_launch(x.as<float>(), k, nullptr, m, k, nt, c->xf_scratch.view(), nullptr, 0, c->stream));
  for (const Weight* w : ws)
    if (int rc = ensure_qg_part(c, w->n_rg, w->k / kSuperK)) return rc;
  cudaGraph_t g = nullptr;
  RB_CUDA(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  int rc = RB_OK;
  for (uint32_t i = 0; i < iters && rc == RB_OK; ++i) {
    const Weight& w = *ws[i % ws.size()];
    GemvArgs a = base_args(c, w, m);
    a.xin = c->xf_scratch.view();
    a.epi = EPI_STORE;
    a.y = y.as<float>();
    a.ldy = w.n;
    rc = gemm_for(c, m, w.dtype) ? launch_qgemm(c, a, nullptr) : launch_gemv(c, a, nullptr);
  }
  cudaError_t e = cudaStreamEndCapture(c->stream, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return fail(RB_ERR_CUDA, "capture: %s", cudaGetErrorString(e));
  cudaGraphExec_t ex = nullptr;
  e = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(RB_ERR_CUDA, "instantiate: %s", cudaGetErrorString(e));
  RB_CUDA(cudaGraphLaunch(ex, c->stream));  // warm-up
  RB_CUDA(cudaEventRecord(c->ev0, c->stream));
  for (uint32_t r = 0; r < reps; ++r) RB_CUDA(cudaGraphLaunch(ex, c->stream));
  RB_CUDA(cudaEventRecord(c->ev1, c->stream));
  rc = sync_ctx(c);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, c->ev0, c->ev1);
  cudaGraphExecDestroy(ex);
  if (rc) return rc;
  *avg_us = ms * 1000.f / (float)(reps * iters);
  if ((c->gemv_dbg & 2) && c->dbg_ts.p) dump_stamps(c, 1);
  return RB_OK;
}

int32_t rb_weight_matmul_path(rb_ctx* c, uint32_t batch) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  return gemm_for(c, (int)batch, DT_Q4_K) ? 1 : 0;
}

int32_t rb_weight_export(rb_ctx* c, int32_t h, void* out_blocks, size_t nbytes, uint32_t flags) {
  if (!c || h < 0 || h >= (int)c->weights.size() || !c->weights[h]) return fail(RB_ERR_BAD_HANDLE, "weight %d", h);
  const Weight& w = *c->weights[h];
  if (w.dtype != DT_Q4_K) return fail(RB_ERR_UNSUPPORTED, "export supports Q4_K");
  const size_t bytes = (size_t)w.n * (w.k / 256) * 144;
  if (nbytes < bytes) return fail(RB_ERR_INVALID, "buffer too small");
  DevBuf tmp;
  uint8_t* d = (uint8_t*)out_blocks;
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(tmp.alloc(bytes));
    d = tmp.as<uint8_t>();
  }
  RB_CUDA(unpack_launch(w.tiled.as<uint8_t>(), w.dtype, w.n, w.k, d, c->stream));
  if (!(flags & RB_PTR_DEVICE)) RB_CUDA(cudaMemcpyAsync(out_blocks, d, bytes, cudaMemcpyDeviceToHost, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)bytes;
}

int32_t rb_fused_dequant_matmul(rb_ctx* c, int32_t dtype, const void* blocks, size_t nblocks, const float* input,
                                float* output, uint32_t batch, uint32_t n, uint32_t k, uint32_t flags) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  if (dtype == DT_Q4_K || dtype == DT_Q6_K) {
    if (k % 256) return fail(RB_ERR_UNSUPPORTED, "K dimension %u must be multiple of 256", k);
    if (nblocks != (size_t)n * (k / 256)) return fail(RB_ERR_INVALID, "Expected %zu blocks, got %zu", (size_t)n * (k / 256), nblocks);
  } else if (dtype == DT_Q8_0) {
    if (nblocks != ((size_t)n * k + 31) / 32) return fail(RB_ERR_INVALID, "Wrong number of blocks: expected %zu, got %zu", ((size_t)n * k + 31) / 32, nblocks);
    if (k % 32) return fail(RB_ERR_UNSUPPORTED, "Q8_0 GEMV needs K %% 32 == 0 (K=%u)", k);
  } else {
    return fail(RB_ERR_UNSUPPORTED, "dtype %d", dtype);
  }
  if (batch == 0) return 0;
  Staged in;
  if (int rc = stage(c, blocks, nblocks * block_bytes(dtype), flags, in)) return rc;
  Weight w;
  if (int rc = upload_tiled(c, w, dtype, n, k, (const uint8_t*)in.dptr, n, nullptr, 0, 0)) return rc;
  Staged xin;
  if (int rc = stage(c, input, (size_t)batch * k * 4, flags, xin)) return rc;
  DevBuf tmp;
  float* dout = output;
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(tmp.alloc((size_t)batch * n * 4));
    dout = tmp.as<float>();
  }
  if (int rc = weight_matmul_dev(c, w, (const float*)xin.dptr, dout, batch)) return rc;
  if (!(flags & RB_PTR_DEVICE)) RB_CUDA(cudaMemcpyAsync(output, dout, (size_t)batch * n * 4, cudaMemcpyDeviceToHost, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)(batch * n);
}

static int32_t candle_mm(rb_ctx* c, const float* a, const float* b, float* cm, uint32_t m, uint32_t k, uint32_t n,
                         uint32_t flags, int bt) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  if (m == 0 || k == 0 || n == 0) return fail(RB_ERR_INVALID, "empty matmul");
  Staged sa, sb;
  if (int rc = stage(c, a, (size_t)m * k * 4, flags, sa)) return rc;
  if (int rc = stage(c, b, (size_t)k * n * 4, flags, sb)) return rc;
  DevBuf tmp;
  float* d = cm;
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(tmp.alloc((size_t)m * n * 4));
    d = tmp.as<float>();
  }
  dim3 grid((n + 15) / 16, (m + 15) / 16), block(16, 16);
  sgemm_kernel<<<grid, block, 0, c->stream>>>((const float*)sa.dptr, (const float*)sb.dptr, d, m, k, n, bt);
  RB_CUDA(cudaGetLastError());
  if (!(flags & RB_PTR_DEVICE)) RB_CUDA(cudaMemcpyAsync(cm, d, (size_t)m * n * 4, cudaMemcpyDeviceToHost, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)(m * n);
}

int32_t rb_candle_matmul(rb_ctx* c, const float* a, const float* b, float* cm, uint32_t m, uint32_t k, uint32_t n,
                         uint32_t flags) {
  return candle_mm(c, a, b, cm, m, k, n, flags, 0);
}
int32_t rb_candle_matmul_transposed(rb_ctx* c, const float* a, const float* b, float* cm, uint32_t m, uint32_t k,
                                    uint32_t n, uint32_t flags) {
  return candle_mm(c, a, b, cm, m, k, n, flags, 1);
}

// ---- KV ----
int32_t rb_kv_pool_create(rb_ctx* c, uint32_t n_layers, uint32_t n_kv, uint32_t hd, int32_t kv_dtype,
                          uint32_t n_pages, uint32_t max_tenants, uint32_t max_seq, int32_t* pool) {
  if (!c || !pool) return fail(RB_ERR_BAD_HANDLE, "null context/pool");
  int rc = pool_create(c, n_layers, n_kv, hd, kv_dtype, n_pages, max_tenants, max_seq);
  if (rc < 0) return rc;
  *pool = rc;
  if (int e = sync_ctx(c)) return e;
  return RB_OK;
}

int32_t rb_kv_pool_destroy(rb_ctx* c, int32_t pool) {
  if (!get_pool(c, pool)) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  cudaStreamSynchronize(c->stream);
  c->pools[pool].reset();
  return RB_OK;
}

int32_t rb_kv_pool_shuffle(rb_ctx* c, int32_t pool, uint64_t seed) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  std::mt19937_64 g(seed);
  std::shuffle(P->free_list.begin(), P->free_list.end(), g);
  return RB_OK;
}

int32_t rb_kv_pool_free_pages(rb_ctx* c, int32_t pool) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  return (int32_t)P->free_list.size();
}

int32_t rb_kv_create(rb_ctx* c, int32_t pool, uint32_t t) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  if (t >= (uint32_t)P->max_tenants) return fail(RB_ERR_OUT_OF_BOUNDS, "tenant %u >= %d", t, P->max_tenants);
  if (P->tenants[t].live) tenant_release(*P, t);
  P->tenants[t].live = true;
  P->tenants[t].len.assign(P->n_layers, 0);
  return RB_OK;
}

int32_t rb_kv_destroy(rb_ctx* c, int32_t pool, uint32_t t) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  if (t >= (uint32_t)P->max_tenants || !P->tenants[t].live) return fail(RB_ERR_NOT_FOUND, "tenant %u", t);
  tenant_release(*P, t);
  P->tenants[t].live = false;
  return RB_OK;
}

int32_t rb_kv_clear(rb_ctx* c, int32_t pool, uint32_t t) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  if (t >= (uint32_t)P->max_tenants || !P->tenants[t].live) return fail(RB_ERR_NOT_FOUND, "tenant %u", t);
  cudaStreamSynchronize(c->stream);
  tenant_release(*P, t);
  return RB_OK;
}

int32_t rb_kv_len(rb_ctx* c, int32_t pool, uint32_t t, uint32_t layer) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  if (t >= (uint32_t)P->max_tenants || !P->tenants[t].live) return fail(RB_ERR_NOT_FOUND, "tenant %u", t);
  if (layer >= (uint32_t)P->n_layers) return fail(RB_ERR_NOT_FOUND, "layer %u", layer);
  return P->tenants[t].len[layer];
}

static int kv_append_rows(rb_ctx* c, KvPool& P, int layer, int n, const uint32_t* tenants, const uint32_t* positions,
                          const float* k, const float* v, uint32_t flags, RowPlan& rp) {
  if (int rc = plan_rows(P, n, tenants, nullptr, positions, layer, rp)) return rc;
  int32_t* d_desc = c->stage_in.as<int32_t>();
  if (int rc = upload_desc(c, rp, d_desc)) return rc;
  ptab_update_kernel<<<1, 128, 0, c->stream>>>(d_desc, P.ptab.as<int32_t>(), P.max_pages_per_tenant);
  RB_CUDA(cudaGetLastError());
  const size_t bytes = (size_t)n * P.n_kv * P.hd * 4;
  Staged sk, sv;
  if (int rc = stage(c, k, bytes, flags, sk)) return rc;
  if (int rc = stage(c, v, bytes, flags, sv)) return rc;
  RB_CUDA(kv_append_launch(P.view(), layer, n, d_desc + kDescTenant, d_desc + kDescPos, (const float*)sk.dptr,
                           (const float*)sv.dptr, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  for (int r = 0; r < n; ++r) P.tenants[rp.tenant[r]].len[layer] = std::max(P.tenants[rp.tenant[r]].len[layer], rp.pos[r] + 1);
  return RB_OK;
}

int32_t rb_kv_append(rb_ctx* c, int32_t pool, uint32_t t, uint32_t layer, const float* k, const float* v,
                     uint32_t seq_len, uint32_t flags) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  if (t >= (uint32_t)P->max_tenants || !P->tenants[t].live) return fail(RB_ERR_NOT_FOUND, "tenant %u", t);
  if (layer >= (uint32_t)P->n_layers) return fail(RB_ERR_NOT_FOUND, "layer %u", layer);
  if (P->tenants[t].len[layer] + (int)seq_len > P->max_seq)
    return fail(RB_ERR_KV_OVERFLOW, "KV cache overflow: %d + %u > %d", P->tenants[t].len[layer], seq_len, P->max_seq);
  for (uint32_t s0 = 0; s0 < seq_len; s0 += kMaxRowsAbi) {
    const int n = (int)std::min<uint32_t>(kMaxRowsAbi, seq_len - s0);
    std::vector<uint32_t> tv(n, t);
    RowPlan rp;
    const size_t off = (size_t)s0 * P->n_kv * P->hd;
    if (int rc = kv_append_rows(c, *P, layer, n, tv.data(), nullptr, k + off, v + off, flags, rp)) return rc;
  }
  return P->tenants[t].len[layer];
}

int32_t rb_kv_gather(rb_ctx* c, int32_t pool, uint32_t t, uint32_t layer, float* k_out, float* v_out, uint32_t flags) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  if (t >= (uint32_t)P->max_tenants || !P->tenants[t].live) return fail(RB_ERR_NOT_FOUND, "tenant %u", t);
  if (layer >= (uint32_t)P->n_layers) return fail(RB_ERR_NOT_FOUND, "layer %u", layer);
  const int len = P->tenants[t].len[layer];
  const size_t bytes = (size_t)len * P->n_kv * P->hd * 4;
  if (len == 0) return 0;
  DevBuf tk, tv;
  float *dk = k_out, *dv = v_out;
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(tk.alloc(bytes));
    RB_CUDA(tv.alloc(bytes));
    dk = tk.as<float>();
    dv = tv.as<float>();
  }
  RB_CUDA(kv_gather_launch(P->view(), layer, t, len, dk, dv, c->stream));
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(cudaMemcpyAsync(k_out, dk, bytes, cudaMemcpyDeviceToHost, c->stream));
    RB_CUDA(cudaMemcpyAsync(v_out, dv, bytes, cudaMemcpyDeviceToHost, c->stream));
  }
  if (int rc = sync_ctx(c)) return rc;
  return len;
}

int32_t rb_attention_forward(rb_ctx* c, int32_t pool, uint32_t layer, uint32_t n_rows, const uint32_t* tenants,
                             const uint32_t* positions, const float* q, const float* k_new, const float* v_new,
                             float* out, uint32_t n_heads, float scale, uint32_t flags) {
  KvPool* P = get_pool(c, pool);
  if (!P) return fail(RB_ERR_BAD_HANDLE, "pool %d", pool);
  if (n_rows == 0 || n_rows > (uint32_t)kMaxRowsAbi) return fail(RB_ERR_INVALID, "n_rows %u not in [1, 64]", n_rows);
  if (layer >= (uint32_t)P->n_layers) return fail(RB_ERR_NOT_FOUND, "layer %u", layer);
  if (n_heads % P->n_kv) return fail(RB_ERR_UNSUPPORTED, "n_heads %u not a multiple of n_kv %d", n_heads, P->n_kv);
  const int nrep = n_heads / P->n_kv;
  if (nrep != 1 && nrep != 2 && nrep != 4 && nrep != 8) return fail(RB_ERR_UNSUPPORTED, "GQA group %d", nrep);
  RowPlan rp;
  int32_t* d_desc = c->stage_in.as<int32_t>();
  if (k_new || v_new) {
    if (!k_new || !v_new) return fail(RB_ERR_INVALID, "k_new and v_new go together");
    if (int rc = kv_append_rows(c, *P, layer, n_rows, tenants, positions, k_new, v_new, flags, rp)) return rc;
  } else {
    rp.tenant.resize(n_rows);
    rp.pos.resize(n_rows);
    rp.tok.assign(n_rows, 0);
    for (uint32_t r = 0; r < n_rows; ++r) {
      const uint32_t t = tenants[r];
      if (t >= (uint32_t)P->max_tenants || !P->tenants[t].live) return fail(RB_ERR_NOT_FOUND, "tenant %u", t);
      const int len = P->tenants[t].len[layer];
      const int pos = positions ? (int)positions[r] : len - 1;
      if (pos < 0 || pos >= len) return fail(RB_ERR_OUT_OF_BOUNDS, "row %u position %d outside cache [0,%d)", r, pos, len);
      rp.tenant[r] = (int)t;
      rp.pos[r] = pos;
    }
    if (int rc = upload_desc(c, rp, d_desc)) return rc;
  }
  const size_t qbytes = (size_t)n_rows * n_heads * P->hd * 4;
  Staged sq;
  if (int rc = stage(c, q, qbytes, flags, sq)) return rc;
  DevBuf tmp;
  float* dout = out;
  if (!(flags & RB_PTR_DEVICE)) {
    RB_CUDA(tmp.alloc(qbytes));
    dout = tmp.as<float>();
  }
  AttnArgs at;
  at.n_rows = n_rows;
  at.row_tenant = d_desc + kDescTenant;
  at.row_pos = d_desc + kDescPos;
  at.q = (const float*)sq.dptr;
  at.ldq = n_heads * P->hd;
  at.out = dout;
  at.ldo = n_heads * P->hd;
  at.n_heads = n_heads;
  at.layer = layer;
  at.scale = scale;
  at.kv = P->view();
  at.kv_tmap = P->tmap;
  at.partials = c->attn_partials.as<float>();
  at.counters = c->counters.as<int32_t>() + kCounters / 2;
  at.err = c->err.as<uint32_t>();
  at.group_rows = c->attn_group && rows_grouped(rp);
  at.whole_pairs = c->attn_whole;
  RB_CUDA(cudaEventRecord(c->ev0, c->stream));
  int n_launch = 0;
  RB_CUDA(attn_launch(at, c->num_sms, c->stream, 0, &n_launch));
  RB_CUDA(cudaEventRecord(c->ev1, c->stream));
  if (!(flags & RB_PTR_DEVICE)) RB_CUDA(cudaMemcpyAsync(out, dout, qbytes, cudaMemcpyDeviceToHost, c->stream));
  if ((flags & RB_PTR_DEVICE) && (flags & RB_ASYNC)) {
    c->last_launches = n_launch;
    return (int32_t)(n_rows * n_heads * P->hd);
  }
  if (int rc = sync_ctx(c)) return rc;
  cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1);
  c->last_launches = n_launch;
  return (int32_t)(n_rows * n_heads * P->hd);
}

// ---- model ----
int32_t rb_model_create(rb_ctx* c, const rb_model_config* cfg, int32_t* model) {
  if (!c || !cfg || !model) return fail(RB_ERR_BAD_HANDLE, "null argument");
  const rb_model_config& f = *cfg;
  if (f.hidden % 256 || f.ffn % 256 || (f.n_heads * f.head_dim) % 256 || f.n_heads % f.n_kv_heads)
    return fail(RB_ERR_UNSUPPORTED, "hidden/ffn/heads*head_dim must be multiples of 256");
  const int nrep = f.n_heads / f.n_kv_heads;
  if (nrep != 1 && nrep != 2 && nrep != 4 && nrep != 8) return fail(RB_ERR_UNSUPPORTED, "GQA group %d", nrep);
  if (f.ffn % 8) return fail(RB_ERR_UNSUPPORTED, "ffn %% 8");
  auto M = std::make_unique<Model>();
  M->cfg = f;
  if (M->cfg.max_tenants == 0) M->cfg.max_tenants = 64;
  const int pages = f.kv_pages ? (int)f.kv_pages : (int)(M->cfg.max_tenants * ((f.max_seq + 15) / 16));
  const int p = pool_create(c, f.n_layers, f.n_kv_heads, f.head_dim, f.kv_dtype, pages, M->cfg.max_tenants, f.max_seq);
  if (p < 0) return p;
  M->pool = p;
  M->layers.resize(f.n_layers);
  const int R = kMaxRowsAbi;
  RB_CUDA(M->x.alloc((size_t)R * f.hidden * 4));
  RB_CUDA(M->q.alloc((size_t)R * f.n_heads * f.head_dim * 4));
  const int NTmax = gemv_nt_for(R);
  RB_CUDA(M->fa.alloc(f.hidden, NTmax));
  RB_CUDA(M->fo.alloc(f.n_heads * f.head_dim, NTmax));
  RB_CUDA(M->ff.alloc(f.hidden, NTmax));
  RB_CUDA(M->fd.alloc(f.ffn, NTmax));
  RB_CUDA(M->ss.alloc((size_t)((f.hidden + 127) / 128) * R * 4));
  RB_CUDA(M->logits.alloc((size_t)R * f.vocab * 4));
  RB_CUDA(M->argmax.alloc((size_t)R * 8));
  RB_CUDA(M->desc.alloc((kDescUpd + 3 * R) * 4));
  RB_CUDA(cudaMemsetAsync(M->x.p, 0, M->x.n, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  c->models.push_back(std::move(M));
  *model = (int32_t)c->models.size() - 1;
  return RB_OK;
}

int32_t rb_model_destroy(rb_ctx* c, int32_t model) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  cudaStreamSynchronize(c->stream);
  for (auto& g : M->graphs) cudaGraphExecDestroy(g.second);
  const int p = M->pool;
  c->models[model].reset();
  if (p >= 0 && p < (int)c->pools.size()) c->pools[p].reset();
  return RB_OK;
}

static bool tensor_shape(const rb_model_config& f, int which, size_t& rows, size_t& cols) {
  const size_t H = f.hidden, Q = (size_t)f.n_heads * f.head_dim, KV = (size_t)f.n_kv_heads * f.head_dim;
  switch (which) {
    case RB_W_TOKEN_EMBD: rows = f.vocab; cols = H; return true;
    case RB_W_OUTPUT_NORM: case RB_W_ATTN_NORM: case RB_W_FFN_NORM: rows = 1; cols = H; return true;
    case RB_W_OUTPUT: rows = f.vocab; cols = H; return true;
    case RB_W_Q: rows = Q; cols = H; return true;
    case RB_W_K: case RB_W_V: rows = KV; cols = H; return true;
    case RB_W_O: rows = H; cols = Q; return true;
    case RB_W_GATE: case RB_W_UP: rows = f.ffn; cols = H; return true;
    case RB_W_DOWN: rows = H; cols = f.ffn; return true;
  }
  return false;
}

int32_t rb_model_set_weight(rb_ctx* c, int32_t model, int32_t which, int32_t layer, int32_t dtype, const void* data,
                            size_t nbytes, uint32_t flags) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  size_t rows, cols;
  if (!tensor_shape(M->cfg, which, rows, cols)) return fail(RB_ERR_NOT_FOUND, "weight id %d", which);
  const bool global = which < 10;
  if (!global && (layer < 0 || layer >= (int)M->cfg.n_layers)) return fail(RB_ERR_NOT_FOUND, "layer %d", layer);
  const bool is_norm = which == RB_W_OUTPUT_NORM || which == RB_W_ATTN_NORM || which == RB_W_FFN_NORM;
  if (is_norm && dtype != RB_F32) return fail(RB_ERR_UNSUPPORTED, "norm weights are f32");
  if (!is_norm && dtype != RB_Q4_K && dtype != RB_Q6_K && dtype != RB_Q8_0 && !(which == RB_W_TOKEN_EMBD && dtype == RB_F32))
    return fail(RB_ERR_UNSUPPORTED, "dtype %d for weight %d", dtype, which);
  const size_t expect = rows * (cols / block_elems(dtype)) * block_bytes(dtype);
  if (cols % block_elems(dtype) || nbytes != expect)
    return fail(RB_ERR_INVALID, "weight %d: expected %zu bytes, got %zu", which, expect, nbytes);
  RawTensor* t = nullptr;
  if (which == RB_W_TOKEN_EMBD) t = &M->embd;
  else if (which == RB_W_OUTPUT_NORM) t = &M->out_norm;
  else if (which == RB_W_OUTPUT) t = &M->out_raw;
  else t = &M->layers[layer].raw[which - RB_W_ATTN_NORM];
  t->dtype = dtype;
  t->bytes = nbytes;
  RB_CUDA(t->d.alloc(nbytes));
  RB_CUDA(cudaMemcpyAsync(t->d.p, data, nbytes, (flags & RB_PTR_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  M->finalized = false;
  return (int32_t)nbytes;
}

int32_t rb_model_finalize(rb_ctx* c, int32_t model) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  const rb_model_config& f = M->cfg;
  if (M->embd.dtype < 0 || M->out_norm.dtype < 0 || M->out_raw.dtype < 0) return fail(RB_ERR_NOT_FOUND, "global weights missing");
  const int H = f.hidden, Q = f.n_heads * f.head_dim, KV = f.n_kv_heads * f.head_dim;
  for (int l = 0; l < (int)f.n_layers; ++l) {
    LayerW& L = M->layers[l];
    for (int i = 0; i < 9; ++i)
      if (L.raw[i].dtype < 0) return fail(RB_ERR_NOT_FOUND, "layer %d weight %d missing", l, RB_W_ATTN_NORM + i);
    RawTensor &q = L.raw[1], &k = L.raw[2], &v = L.raw[3], &o = L.raw[4], &g = L.raw[6], &u = L.raw[7], &d = L.raw[8];
    if (q.dtype != k.dtype) return fail(RB_ERR_UNSUPPORTED, "layer %d: wq and wk dtypes differ", l);
    if (g.dtype != u.dtype) return fail(RB_ERR_UNSUPPORTED, "layer %d: gate and up dtypes differ", l);
    if (int rc = upload_tiled(c, L.qk, q.dtype, Q + KV, H, q.d.as<uint8_t>(), Q, k.d.as<uint8_t>(), KV, 1)) return rc;
    if (int rc = upload_tiled(c, L.v, v.dtype, KV, H, v.d.as<uint8_t>(), KV, nullptr, 0, 0)) return rc;
    L.v_fused = false;
    if (int rc = upload_tiled(c, L.o, o.dtype, H, Q, o.d.as<uint8_t>(), H, nullptr, 0, 0)) return rc;
    if (int rc = upload_tiled(c, L.gu, g.dtype, 2 * f.ffn, H, g.d.as<uint8_t>(), f.ffn, u.d.as<uint8_t>(), f.ffn, 2)) return rc;
    if (int rc = upload_tiled(c, L.down, d.dtype, H, f.ffn, d.d.as<uint8_t>(), H, nullptr, 0, 0)) return rc;
  }
  if (int rc = upload_tiled(c, M->out, M->out_raw.dtype, f.vocab, H, M->out_raw.d.as<uint8_t>(), f.vocab, nullptr, 0, 0)) return rc;
  if (int rc = sync_ctx(c)) return rc;
  for (auto& g : M->graphs) cudaGraphExecDestroy(g.second);
  M->graphs.clear();
  M->finalized = true;
  return RB_OK;
}

int32_t rb_model_get_config(rb_ctx* c, int32_t model, rb_model_config* out) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  if (!out) return fail(RB_ERR_INVALID, "null config");
  *out = M->cfg;
  if (out->kv_pages == 0) out->kv_pages = (uint32_t)c->pools[M->pool]->n_pages;
  return RB_OK;
}

int32_t rb_ctx_max_rows(rb_ctx* c) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  return c->max_rows;
}

int32_t rb_model_kv_pool(rb_ctx* c, int32_t model) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  return M->pool;
}

int32_t rb_tenant_create(rb_ctx* c, int32_t model, uint32_t t) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  return rb_kv_create(c, M->pool, t);
}

int32_t rb_tenant_reset(rb_ctx* c, int32_t model, uint32_t t) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  return rb_kv_clear(c, M->pool, t);
}

int32_t rb_forward(rb_ctx* c, int32_t model, uint32_t n_rows, const uint32_t* tenants, const uint32_t* tokens,
                   const uint32_t* positions, float* logits, uint32_t* argmax, uint32_t flags) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  if (!M->finalized) return fail(RB_ERR_INVALID, "model not finalized");
  if (n_rows == 0 || n_rows > (uint32_t)c->max_rows) return fail(RB_ERR_INVALID, "n_rows %u not in [1, %d]", n_rows, c->max_rows);
  if (!tenants || !tokens) return fail(RB_ERR_INVALID, "tenants/tokens NULL");
  for (uint32_t r = 0; r < n_rows; ++r)
    if (tokens[r] >= M->cfg.vocab) return fail(RB_ERR_INVALID, "token %u >= vocab", tokens[r]);
  KvPool& P = *c->pools[M->pool];
  RowPlan rp;
  if (int rc = plan_rows(P, n_rows, tenants, tokens, positions, -1, rp)) return rc;
  if (int rc = upload_desc(c, rp, M->desc.as<int32_t>())) return rc;
  c->step_grouped = rows_grouped(rp);
  if (int rc = run_forward(c, *M, n_rows, c->graphs)) return rc;
  // outputs
  std::vector<unsigned long long> keys(n_rows);
  RB_CUDA(cudaMemcpyAsync(keys.data(), M->argmax.p, n_rows * 8, cudaMemcpyDeviceToHost, c->stream));
  if (logits) {
    if (int rc = copy_out(c, logits, M->logits.p, (size_t)n_rows * M->cfg.vocab * 4, flags)) return rc;
  }
  if (int rc = sync_ctx(c)) return rc;
  cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1);
  if ((c->gemv_dbg & 2) && c->dbg_ts.p) dump_stamps(c, c->last_chain_phases);
  for (uint32_t r = 0; r < n_rows; ++r) {
    KvTenant& T = P.tenants[rp.tenant[r]];
    for (auto& l : T.len) l = std::max(l, rp.pos[r] + 1);
  }
  if (argmax) {
    if (flags & RB_PTR_DEVICE) {
      std::vector<uint32_t> ids(n_rows);
      for (uint32_t r = 0; r < n_rows; ++r) ids[r] = (uint32_t)(keys[r] & 0xffffffffu);
      RB_CUDA(cudaMemcpy(argmax, ids.data(), n_rows * 4, cudaMemcpyHostToDevice));
    } else {
      for (uint32_t r = 0; r < n_rows; ++r) argmax[r] = (uint32_t)(keys[r] & 0xffffffffu);
    }
  }
  return (int32_t)n_rows;
}

int32_t rb_forward_profile(rb_ctx* c, int32_t model, uint32_t n_rows, const uint32_t* tenants,
                           const uint32_t* tokens, float* kind_ms) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  if (!M->finalized) return fail(RB_ERR_INVALID, "model not finalized");
  if (!kind_ms) return fail(RB_ERR_INVALID, "null output");
  if (n_rows == 0 || n_rows > (uint32_t)c->max_rows) return fail(RB_ERR_INVALID, "n_rows %u not in [1, %d]", n_rows, c->max_rows);
  for (uint32_t r = 0; r < n_rows; ++r)
    if (tokens[r] >= M->cfg.vocab) return fail(RB_ERR_INVALID, "token %u >= vocab", tokens[r]);
  KvPool& P = *c->pools[M->pool];
  RowPlan rp;
  if (int rc = plan_rows(P, n_rows, tenants, tokens, nullptr, -1, rp)) return rc;
  if (int rc = upload_desc(c, rp, M->desc.as<int32_t>())) return rc;
  c->step_grouped = rows_grouped(rp);
  std::vector<std::pair<int, cudaEvent_t>> marks;
  cudaEvent_t start = nullptr;
  RB_CUDA(cudaEventCreate(&start));
  const bool pdl = c->pdl;
  c->pdl = false;  // serialised launches: each interval is one kernel
  RB_CUDA(cudaEventRecord(start, c->stream));
  c->prof = &marks;
  int rc = run_forward(c, *M, (int)n_rows, false);
  c->prof = nullptr;
  c->pdl = pdl;
  if (!rc) rc = sync_ctx(c);
  for (int k = 0; k < PROF_KINDS; ++k) kind_ms[k] = 0.f;
  cudaEvent_t prev = start;
  for (auto& mk : marks) {
    float ms = 0.f;
    if (!rc) cudaEventElapsedTime(&ms, prev, mk.second);
    kind_ms[mk.first] += ms;
    prev = mk.second;
  }
  for (auto& mk : marks) cudaEventDestroy(mk.second);
  cudaEventDestroy(start);
  if (rc) return rc;
  for (uint32_t r = 0; r < n_rows; ++r) {
    KvTenant& T = P.tenants[rp.tenant[r]];
    for (auto& l : T.len) l = std::max(l, rp.pos[r] + 1);
  }
  return (int32_t)marks.size();
}

static int sample_rows(rb_ctx* c, const float* d_logits, uint32_t ld, uint32_t n_rows, uint32_t vocab,
                       const rb_sampling* params, const uint32_t* prev, const uint32_t* prev_off,
                       const float* uniforms, uint32_t* out, uint32_t flags) {
  if (!params || !uniforms || !out) return fail(RB_ERR_INVALID, "params/uniforms/out NULL");
  if (n_rows == 0) return 0;
  if (vocab == 0 || vocab > (uint32_t)kSampleMaxVocab || ld < vocab)
    return fail(RB_ERR_UNSUPPORTED, "vocab %u not in [1, %d] or ld %u < vocab", vocab, kSampleMaxVocab, ld);
  if ((prev == nullptr) != (prev_off == nullptr)) return fail(RB_ERR_INVALID, "prev_tokens and prev_offsets go together");
  const bool dev = flags & RB_PTR_DEVICE;
  uint32_t n_prev = 0;
  if (prev_off && !dev) n_prev = prev_off[n_rows];
  Staged sp, sprev, soff, su;
  if (int rc = stage(c, params, (size_t)n_rows * sizeof(rb_sampling), flags, sp)) return rc;
  if (prev_off) {
    if (int rc = stage(c, prev_off, (size_t)(n_rows + 1) * 4, flags, soff)) return rc;
    if (int rc = stage(c, prev, dev ? 0 : (size_t)n_prev * 4, flags, sprev)) return rc;
  }
  if (int rc = stage(c, uniforms, (size_t)n_rows * 4, flags, su)) return rc;
  DevBuf dout;
  uint32_t* o = out;
  if (!dev) {
    RB_CUDA(dout.alloc((size_t)n_rows * 4));
    o = dout.as<uint32_t>();
  }
  RB_CUDA(sample_launch(d_logits, (int)ld, (int)n_rows, (int)vocab, (const rb_sampling*)sp.dptr,
                        prev_off ? (const uint32_t*)sprev.dptr : nullptr, prev_off ? (const uint32_t*)soff.dptr : nullptr,
                        (const float*)su.dptr, o, c->stream));
  std::vector<uint32_t> h(n_rows);
  RB_CUDA(cudaMemcpyAsync(h.data(), o, (size_t)n_rows * 4, cudaMemcpyDeviceToHost, c->stream));
  if (int rc = sync_ctx(c)) return rc;
  for (uint32_t r = 0; r < n_rows; ++r)
    if (h[r] == 0xffffffffu) return fail(RB_ERR_INVALID, "row %u: Failed to create weighted index", r);
  if (!dev) std::copy(h.begin(), h.end(), out);
  return (int32_t)n_rows;
}

int32_t rb_sample_logits(rb_ctx* c, const float* logits, uint32_t ld, uint32_t n_rows, uint32_t vocab,
                         const rb_sampling* params, const uint32_t* prev_tokens, const uint32_t* prev_offsets,
                         const float* uniforms, uint32_t* out_tokens, uint32_t flags) {
  if (!c) return fail(RB_ERR_BAD_HANDLE, "null context");
  if (!logits) return fail(RB_ERR_INVALID, "logits NULL");
  Staged sl;
  if (int rc = stage(c, logits, (size_t)n_rows * ld * 4, flags, sl)) return rc;
  return sample_rows(c, (const float*)sl.dptr, ld, n_rows, vocab, params, prev_tokens, prev_offsets, uniforms,
                     out_tokens, flags);
}

float rb_sampling_uniform(uint64_t seed, uint64_t counter) {
  // SplitMix64 (Steele, Lea, Flood 2014) of seed + counter * golden gamma; top 23 bits
  uint64_t z = seed + counter * 0x9E3779B97F4A7C15ull + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 41) * (1.0f / 8388608.0f);
}

int32_t rb_forward_sample(rb_ctx* c, int32_t model, uint32_t n_rows, const uint32_t* tenants, const uint32_t* tokens,
                          const uint32_t* positions, const rb_sampling* params, const uint32_t* prev_tokens,
                          const uint32_t* prev_offsets, const float* uniforms, uint32_t* out_tokens, float* logits) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  std::vector<uint32_t> am(n_rows ? n_rows : 1);
  const int32_t rc = rb_forward(c, model, n_rows, tenants, tokens, positions, logits, am.data(), RB_PTR_HOST);
  if (rc < 0) return rc;
  // the step's logits stay in the model's device buffer until its next forward
  return sample_rows(c, M->logits.as<float>(), M->cfg.vocab, n_rows, M->cfg.vocab, params, prev_tokens, prev_offsets,
                     uniforms, out_tokens, RB_PTR_HOST);
}

int32_t rb_embed_tokens(rb_ctx* c, int32_t model, const uint32_t* ids, uint32_t n, float* out, uint32_t flags) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  if (M->embd.dtype < 0) return fail(RB_ERR_NOT_FOUND, "token_embd missing");
  const int H = M->cfg.hidden;
  for (uint32_t s0 = 0; s0 < n; s0 += kMaxRowsAbi) {
    const int m = (int)std::min<uint32_t>(kMaxRowsAbi, n - s0);
    RowPlan rp;
    rp.tenant.assign(m, 0);
    rp.pos.assign(m, 0);
    rp.tok.resize(m);
    for (int r = 0; r < m; ++r) {
      if (ids[s0 + r] >= M->cfg.vocab) return fail(RB_ERR_INVALID, "token %u >= vocab", ids[s0 + r]);
      rp.tok[r] = (int)ids[s0 + r];
    }
    int32_t* d = c->stage_in.as<int32_t>();
    if (int rc = upload_desc(c, rp, d)) return rc;
    KvPool& P = *c->pools[M->pool];
    embed_kernel<<<dim3(m, (H + 255) / 256), 128, 0, c->stream>>>(M->embd.d.as<uint8_t>(), M->embd.dtype, H, d,
                                                                  P.ptab.as<int32_t>(),
                                           P.max_pages_per_tenant, M->x.as<float>(), H, nullptr, kMaxRowsAbi,
                                           nullptr, nullptr, 1, XFrags());
    RB_CUDA(cudaGetLastError());
    if (int rc = copy_out(c, (uint8_t*)out + (size_t)s0 * H * 4, M->x.p, (size_t)m * H * 4, flags)) return rc;
    if (int rc = sync_ctx(c)) return rc;
  }
  return (int32_t)((size_t)n * H * 4);
}

int32_t rb_forward_layer(rb_ctx* c, int32_t model, uint32_t t, uint32_t layer, const float* hidden,
                         uint32_t hidden_len, uint32_t position, float* out, uint32_t flags) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  if (!M->finalized) return fail(RB_ERR_INVALID, "model not finalized");
  const int H = M->cfg.hidden;
  if (layer >= M->cfg.n_layers) return fail(RB_ERR_NOT_FOUND, "layer %u", layer);
  if (hidden_len == 0 || hidden_len % H) return fail(RB_ERR_INVALID, "hidden_len %u not a multiple of %d", hidden_len, H);
  const uint32_t S = hidden_len / H;
  if (S > (uint32_t)kMaxRowsAbi) return fail(RB_ERR_INVALID, "%u rows > 64", S);
  KvPool& P = *c->pools[M->pool];
  std::vector<uint32_t> tv(S, t), pv(S);
  for (uint32_t i = 0; i < S; ++i) pv[i] = position + i;
  RowPlan rp;
  if (int rc = plan_rows(P, S, tv.data(), nullptr, pv.data(), (int)layer, rp)) return rc;
  if (int rc = upload_desc(c, rp, M->desc.as<int32_t>())) return rc;
  ptab_update_kernel<<<1, 128, 0, c->stream>>>(M->desc.as<int32_t>(), P.ptab.as<int32_t>(), P.max_pages_per_tenant);
  RB_CUDA(cudaMemcpyAsync(M->x.p, hidden, (size_t)S * H * 4,
                          (flags & RB_PTR_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, c->stream));
  RB_CUDA(xfrag_launch(M->x.as<float>(), H, M->layers[layer].raw[0].d.as<float>(), (int)S, H, gemv_nt_for((int)S),
                       M->fa.view(), M->ss.as<float>(), kMaxRowsAbi, c->stream));
  int launches = 2;
  c->gemm_step = gemm_rows(c, (int)S);
  c->step_grouped = S > 1;  // one tenant at consecutive positions
  if (c->gemm_step)
    if (int rc = ensure_qg_model(c, *M)) return rc;
  RB_CUDA(cudaEventRecord(c->ev0, c->stream));
  const int32_t* d = M->desc.as<int32_t>();
  if (int rc = enqueue_layer(c, *M, (int)layer, (int)S, d + kDescTenant, d + kDescPos, &launches)) return rc;
  if (int rc = chain_flush(c, &launches)) return rc;
  RB_CUDA(cudaEventRecord(c->ev1, c->stream));
  if (int rc = copy_out(c, out, M->x.p, (size_t)S * H * 4, flags)) return rc;
  if (int rc = sync_ctx(c)) return rc;
  cudaEventElapsedTime(&c->last_ms, c->ev0, c->ev1);
  c->last_launches = launches;
  P.tenants[t].len[layer] = position + S;
  return (int32_t)((size_t)S * H * 4);
}

int32_t rb_compute_logits(rb_ctx* c, int32_t model, const float* hidden, uint32_t hidden_len, float* out,
                          uint32_t flags) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  if (!M->finalized) return fail(RB_ERR_INVALID, "model not finalized");
  const int H = M->cfg.hidden;
  if (hidden_len != (uint32_t)H) return fail(RB_ERR_INVALID, "hidden_len %u != %d", hidden_len, H);
  RB_CUDA(cudaMemcpyAsync(M->x.p, hidden, (size_t)H * 4,
                          (flags & RB_PTR_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, c->stream));
  RB_CUDA(xfrag_launch(M->x.as<float>(), H, M->out_norm.d.as<float>(), 1, H, 1, M->fa.view(), M->ss.as<float>(),
                       kMaxRowsAbi, c->stream));
  zero_u64_kernel<<<1, 64, 0, c->stream>>>(M->argmax.as<unsigned long long>(), 1);
  RB_CUDA(cudaGetLastError());
  c->gemm_step = false;
  if (int rc = enqueue_head(c, *M, 1, true, nullptr)) return rc;
  if (int rc = copy_out(c, out, M->logits.p, (size_t)M->cfg.vocab * 4, flags)) return rc;
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)(M->cfg.vocab * 4);
}

int32_t rb_memory64_load_layer(rb_ctx* c, int32_t model, uint32_t layer_id, void* dst, uint32_t max_size) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  if (layer_id >= M->cfg.n_layers) return fail(RB_ERR_NOT_FOUND, "layer %u not found", layer_id);
  LayerW& L = M->layers[layer_id];
  const int order[7] = {1, 2, 3, 4, 6, 7, 8};
  size_t total = 0;
  for (int i : order) {
    if (L.raw[i].dtype < 0) return fail(RB_ERR_NOT_FOUND, "layer %u incomplete", layer_id);
    total += L.raw[i].bytes;
  }
  if (total > max_size) return fail(RB_ERR_INVALID, "buffer too small: %zu > %u", total, max_size);
  if (total > 0x7fffffffu) return fail(RB_ERR_PTR_OVERFLOW, "layer larger than 2 GiB");
  size_t off = 0;
  for (int i : order) {
    RB_CUDA(cudaMemcpyAsync((uint8_t*)dst + off, L.raw[i].d.p, L.raw[i].bytes, cudaMemcpyDeviceToHost, c->stream));
    off += L.raw[i].bytes;
  }
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)total;
}

// The Memory64 image: layer 0's wq, wk, wv, wo, w_gate, w_up, w_down bytes, then
// layer 1's, ... (the order rb_memory64_load_layer copies one layer in).
static const int kMem64Order[7] = {1, 2, 3, 4, 6, 7, 8};

int32_t rb_memory64_size(rb_ctx* c, int32_t model, uint64_t* size) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  if (!size) return fail(RB_ERR_INVALID, "null size");
  uint64_t total = 0;
  for (const LayerW& L : M->layers)
    for (int i : kMem64Order) total += L.raw[i].bytes;
  *size = total;
  return RB_OK;
}

int32_t rb_memory64_read(rb_ctx* c, int32_t model, uint64_t offset, void* mem, uint32_t mem_size,
                         uint32_t mem_offset, uint32_t size, uint32_t flags) {
  Model* M = get_model(c, model);
  if (!M) return fail(RB_ERR_BAD_HANDLE, "model %d", model);
  // memory64_host.rs:785-805: destination overflow (-4), then bounds (-5)
  const uint64_t end_ptr = (uint64_t)mem_offset + size;
  if (end_ptr > 0xffffffffull) return fail(RB_ERR_IO, "memory pointer overflow: %u + %u", mem_offset, size);
  if (end_ptr > mem_size)
    return fail(RB_ERR_NO_MEMORY, "memory pointer out of bounds: %u + %u > %u", mem_offset, size, mem_size);
  if (size > 0x7fffffffu) return fail(RB_ERR_PTR_OVERFLOW, "read larger than 2 GiB");
  // memory64_host.rs:808-813 / 298-330: the read must lie inside the image (-2)
  uint64_t total = 0;
  for (const LayerW& L : M->layers)
    for (int i : kMem64Order) total += L.raw[i].bytes;
  if (offset > total || size > total - offset)
    return fail(RB_ERR_NOT_FOUND, "memory64_read failed at offset %llu: %u bytes exceed the %llu-byte image",
                (unsigned long long)offset, size, (unsigned long long)total);
  if (size && !mem) return fail(RB_ERR_INVALID, "null destination");
  const cudaMemcpyKind kind = (flags & RB_PTR_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
  uint64_t base = 0, done = 0;
  for (const LayerW& L : M->layers)
    for (int i : kMem64Order) {
      const RawTensor& t = L.raw[i];
      const uint64_t lo = base, hi = base + t.bytes;
      base = hi;
      if (done == size || hi <= offset + done || t.bytes == 0) continue;
      if (!t.d.p) return fail(RB_ERR_NOT_FOUND, "weight bytes of the image are not resident");
      const uint64_t from = offset + done - lo;
      const uint64_t n = std::min<uint64_t>(t.bytes - from, size - done);
      RB_CUDA(cudaMemcpyAsync((uint8_t*)mem + mem_offset + done, (const uint8_t*)t.d.p + from, n, kind, c->stream));
      done += n;
    }
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)size;
}

float rb_last_forward_ms(rb_ctx* c) { return c ? c->last_ms : -1.f; }
int32_t rb_last_forward_launches(rb_ctx* c) { return c ? c->last_launches : fail(RB_ERR_BAD_HANDLE, "null context"); }

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free GEMV (rb_weight_matmul_noalloc).
//
// Some callers cannot allocate device memory at the point where they run a
// matmul: a host that hands the library a fixed memory budget up front, code
// running under an allocator that must not grow (or that another runtime owns),
// or a serving loop that forbids cudaMalloc/cudaFree on its hot path because
// they synchronise the device. For them this entry point takes device pointers
// for the input and output and keeps every other byte it needs (activation
// fragments, split-K partial sums, split-K counters) in one file-scope device
// array of fixed size, which each GPU that loads the library holds until the
// process exits.
//
// Limits (calls beyond them fail with RB_ERR_INVALID and a message naming the
// limit): batch <= 8 rows, K <= 16384, N <= 131072 (512 groups of 256 rows),
// and at most 160 GEMV CTAs (the device's SM count when the weight has that
// many 256-row x 256-column units). The array is 3,565,568 bytes. Q8_0 weights
// whose K is not a multiple of 256 (zero-padded at upload) are refused with
// RB_ERR_UNSUPPORTED.
//
// The array is shared by every call on a device, from every context, and keeps
// the contents of the last call; the counters are cleared on the stream at the
// start of each call. Calls whose GPU work overlaps (two streams, two
// contexts, or two host threads without ordering) race on it and give wrong
// results: order them on one stream.
//
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress (with that device current) and caches it; make that
// first call before any stream capture on the device. The cached address
// belongs to the device's primary context: after cudaDeviceReset in this
// process it is stale, so no call may follow a reset.
// ---------------------------------------------------------------------------
namespace {

constexpr int kNaMaxBatch = 8;
constexpr int kNaMaxK = 16384;
constexpr int kNaMaxRowGroups = 512;
constexpr int kNaMaxCtas = 160;
constexpr int kNaMaxDevices = 64;
constexpr size_t kNaXf = (size_t)(kNaMaxK / 256) * kXfSbBytes;   // NT = 1
constexpr size_t kNaXi = (size_t)(kNaMaxK / 256) * kXiSbBytes;
constexpr size_t kNaX3 = (size_t)(kNaMaxK / 256) * kX3SbBytes;
constexpr size_t kNaXc = (size_t)(kNaMaxK / 256) * kXcSbBytes;
constexpr size_t kNaXs = (size_t)(kNaMaxK / 256) * kXsSbBytes;
constexpr size_t kNaPartials = (size_t)kNaMaxCtas * 2 * 16 * 128 * 4;  // gemv_partials_floats(160, 1) floats
constexpr size_t kNaCounters = (size_t)kNaMaxRowGroups * 4;
constexpr size_t kNaOffXi = kNaXf, kNaOffX3 = kNaOffXi + kNaXi, kNaOffXc = kNaOffX3 + kNaX3,
                 kNaOffXs = kNaOffXc + kNaXc, kNaOffPart = kNaOffXs + kNaXs, kNaOffCnt = kNaOffPart + kNaPartials,
                 kNaBytes = kNaOffCnt + kNaCounters;
static_assert(kNaOffXi % 256 == 0 && kNaOffX3 % 256 == 0 && kNaOffXc % 256 == 0 && kNaOffXs % 256 == 0 &&
                  kNaOffPart % 256 == 0 && kNaOffCnt % 256 == 0,
              "scratch sections must stay 256-byte aligned");
static_assert(kNaBytes == 3565568, "the documented size of the no-alloc scratch array");

// Host code sees only a stand-in for this symbol; its device address comes from
// cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNaBytes];

int noalloc_scratch(Ctx* c, uint8_t** out) {
  static std::mutex mu;
  static uint8_t* addr[kNaMaxDevices] = {};
  if (c->device < 0 || c->device >= kNaMaxDevices) return fail(RB_ERR_INVALID, "device %d out of range", c->device);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[c->device]) {
    int prev = 0;
    RB_CUDA(cudaGetDevice(&prev));
    RB_CUDA(cudaSetDevice(c->device));
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    cudaSetDevice(prev);
    if (e != cudaSuccess || !p)
      return fail(RB_ERR_CUDA, "cudaGetSymbolAddress of the no-alloc scratch: %s", cudaGetErrorString(e));
    addr[c->device] = static_cast<uint8_t*>(p);
  }
  *out = addr[c->device];
  return RB_OK;
}

}  // namespace

extern "C" int32_t rb_weight_matmul_noalloc(rb_ctx* c, int32_t h, const float* input, float* output, uint32_t batch,
                                            uint32_t flags) {
  if (!c || h < 0 || h >= (int)c->weights.size() || !c->weights[h]) return fail(RB_ERR_BAD_HANDLE, "weight %d", h);
  const Weight& w = *c->weights[h];
  if (!(flags & RB_PTR_DEVICE))
    return fail(RB_ERR_INVALID, "rb_weight_matmul_noalloc takes device pointers only (RB_PTR_DEVICE)");
  if (batch == 0) return 0;
  if (!input || !output) return fail(RB_ERR_INVALID, "null input or output");
  if (batch > (uint32_t)kNaMaxBatch)
    return fail(RB_ERR_INVALID, "batch %u exceeds the no-alloc maximum of %d rows", batch, kNaMaxBatch);
  if (w.k > kNaMaxK) return fail(RB_ERR_INVALID, "K=%d exceeds the no-alloc maximum of %d", w.k, kNaMaxK);
  if (w.k_in != w.k) return fail(RB_ERR_UNSUPPORTED, "K=%d is not a multiple of 256", w.k_in);
  if (w.n_rg > kNaMaxRowGroups)
    return fail(RB_ERR_INVALID, "N=%d exceeds the no-alloc maximum of %d", w.n, kNaMaxRowGroups * kRowGroup);
  if (gemv_ctas(c->num_sms, w.n_rg, w.k / kSuperK) > kNaMaxCtas)
    return fail(RB_ERR_INVALID, "%d SMs exceed the no-alloc maximum of %d GEMV CTAs", c->num_sms, kNaMaxCtas);
  if (gemv_partials_floats(gemv_ctas(c->num_sms, w.n_rg, w.k / kSuperK), 1) * 4 > kNaPartials)
    return fail(RB_ERR_INVALID, "split-K partials exceed the no-alloc scratch");
  uint8_t* base = nullptr;
  if (int rc = noalloc_scratch(c, &base)) return rc;
  RB_CUDA(cudaSetDevice(c->device));
  XFrags xf;
  xf.xf = reinterpret_cast<uint4*>(base);
  xf.xi = reinterpret_cast<uint4*>(base + kNaOffXi);
  xf.x3 = reinterpret_cast<uint2*>(base + kNaOffX3);
  xf.xc = reinterpret_cast<float*>(base + kNaOffXc);
  xf.xs = reinterpret_cast<uint32_t*>(base + kNaOffXs);
  int32_t* counters = reinterpret_cast<int32_t*>(base + kNaOffCnt);
  const int m = (int)batch;
  RB_CUDA(cudaMemsetAsync(counters, 0, (size_t)w.n_rg * 4, c->stream));
  RB_CUDA(xfrag_launch(input, w.k, nullptr, m, w.k, 1, xf, nullptr, 0, c->stream));
  GemvArgs a = base_args(c, w, m);
  a.dbg = 0;
  a.dbg_ts = nullptr;
  a.partials = reinterpret_cast<float*>(base + kNaOffPart);
  a.counters = counters;
  a.xin = xf;
  a.epi = EPI_STORE;
  a.y = output;
  a.ldy = w.n;
  RB_CUDA(gemv_launch(a, c->num_sms, c->stream, c->pdl ? 1 : 0));
  if (flags & RB_ASYNC) return (int32_t)(batch * w.n);
  if (int rc = sync_ctx(c)) return rc;
  return (int32_t)(batch * w.n);
}
