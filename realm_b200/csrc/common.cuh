// Shared device helpers for the realm-b200 decode path (sm_100a only).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef __CUDACC__
#error "compile with nvcc"
#endif

#include <mutex>
#include <set>
#include <utility>

namespace rb {

// Raises a kernel's dynamic shared-memory limit once per (kernel, device).
// Thread-safe: contexts on different host threads may launch concurrently.
inline cudaError_t ensure_smem_attr_impl(const void* kern, int bytes, int dev) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kern, dev})) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.insert({kern, dev});
  return e;
}
template <class K>
inline cudaError_t ensure_smem_attr(K kern, int bytes, int dev) {
  return ensure_smem_attr_impl(reinterpret_cast<const void*>(kern), bytes, dev);
}

// ---- device error word (bounded waits report here instead of hanging) ----
enum DevErr : uint32_t {
  DEV_OK = 0,
  DEV_TIMEOUT_FULL = 1,
  DEV_TIMEOUT_EMPTY = 2,
  DEV_TIMEOUT_DRAIN = 3,
  DEV_TIMEOUT_GRID = 4,  // grid barrier between the phases of a multi-phase GEMV
  DEV_TIMEOUT_SMEM = 5,  // producer waiting for its consumers' barrier ticket
};

// Spin limit for every mbarrier wait: ~2^26 polls is far beyond any legal
// wait (a few microseconds) yet ends in well under a second.
constexpr uint32_t kSpinLimit = 1u << 26;

__device__ __forceinline__ void report_error(uint32_t* err, uint32_t code) {
  if (err) atomicCAS(err, 0u, code);
}

// ---- mbarrier / bulk copy (TMA engine, no multicast) ----
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code`) if the phase never flips.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err, uint32_t code) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  report_error(err, code);
  return false;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same with an L2 eviction hint: streamed weights are read once per step.
__device__ __forceinline__ void bulk_g2s_evict_first(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                                     uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- programmatic dependent launch ----
// ---- grid barrier (co-resident CTAs of one cooperative launch) ----
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Atomic add with acquire-release (or release) semantics at GPU scope: the
// prior writes of the CTA (ordered by a barrier) are visible before it, and
// reads after it (acq_rel) see what the writers released.
__device__ __forceinline__ int atom_add_acq_rel(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int atom_add_relaxed(int32_t* p, int v) {
  int old;
  asm volatile("atom.relaxed.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ unsigned long long atom_add_release_u64(unsigned long long* p, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.release.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}

// Waits until *ctr >= target (bounded, then reports and returns false).
// On a timeout the first reporter also leaves err[1..3] = target, the counter
// it last saw (low 32 bits each) and `who` (caller-defined) for the host.
// `limit` polls at most (0: the default 2^22, about half a second).
__device__ __forceinline__ bool grid_wait(const unsigned long long* ctr, unsigned long long target, uint32_t* err,
                                          uint32_t who, uint32_t limit = 0) {
  unsigned long long v = 0;
  const uint32_t n = limit ? limit : (1u << 22);
  for (uint32_t i = 0; i < n; ++i) {
    v = ld_acquire_u64(ctr);
    if (v >= target) return true;
    if (i > 64) __nanosleep(100);
  }
  if (err && atomicCAS(err, 0u, (uint32_t)DEV_TIMEOUT_GRID) == 0u) {
    err[1] = (uint32_t)target;
    err[2] = (uint32_t)v;
    err[3] = who;
  }
  return false;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- tensor-core MMA (register accumulators: per-32-K scales need them) ----
__device__ __forceinline__ void mma_16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_1688(float c[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t d;
  // (a & mask) | orv  ->  immLut = (0xF0 & 0xCC) | 0xAA = 0xEA
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(orv));
  return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
  return h2_as_u32(__hfma2(u32_as_h2(a), u32_as_h2(b), u32_as_h2(c)));
}
__device__ __forceinline__ uint32_t h2_u32_mul(uint32_t a, uint32_t b) {
  return h2_as_u32(__hmul2(u32_as_h2(a), u32_as_h2(b)));
}
__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
  return h2_as_u32(__hsub2(u32_as_h2(a), u32_as_h2(b)));
}

// fp32 -> (hi, lo) fp16 pair with x ~= hi + lo to ~22 bits; lo is the rounded residual.
__device__ __forceinline__ void split_hilo(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

// Order-preserving float -> uint32 map (larger float -> larger key); used for
// argmax via 64-bit atomicMax with the index in the low word (ties -> larger index).
__device__ __forceinline__ uint32_t float_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

}  // namespace rb
