// Fused sampling of a batch of logits rows on the device: LogitsProcessor::sample
// (crates/realm-models/src/sampling.rs:107-300) with the strategy picked as
// LogitsProcessor::with_params does (:63-100), one CTA of 1024 threads per row,
// the row held in shared memory (in padded per-thread chunks).
//
//  1. repetition penalty once per occurrence of each previous token (:107-122);
//     the occurrences of one token are applied in list order by one thread;
//  2. temperature < 1e-7: argmax, ties to the last index (:141-148);
//  3. x / (temperature as f32), softmax (:125-137);
//  4. top-k: 4-pass radix select of the k-th largest probability on its bits;
//     ties at the threshold keep the lowest indices (the reference's unstable
//     selection leaves them unspecified); renormalise;
//  5. top-p: keep a token while the probability mass ranked before it (value
//     descending, index ascending, as the reference's stable sort) is below p;
//     the boundary value is found by the same radix walk over per-bin counts and
//     sums; renormalise;
//  6. WeightedIndex (rand 0.8.5): total, Uniform(0, total) scale, chosen =
//     u * scale, index = number of cumulative weights (all but the last) <= chosen.
//
// Sums are deterministic: fixed-order tree reductions for floats; the top-p bin
// sums are 2^-40 fixed point with integer atomics (order independent). They
// differ from the reference's sequential f32 sums by rounding only, which can
// move a top-p or sampling boundary when a draw or a cumulative sum lands within
// rounding of it.
#include "common.cuh"
#include "sample.cuh"

namespace rb {

namespace {

constexpr int kST = 1024;  // threads per row
constexpr int kSW = kST / 32;
constexpr double kFix = 1099511627776.0;  // 2^40

struct Red {
  float f[kSW];
  unsigned long long u[kSW];
  uint32_t c[kSW];
};

__device__ float block_sum(float v, Red& r) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) r.f[w] = v;
  __syncthreads();
  float t = lane < kSW ? r.f[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

__device__ float block_max(float v, Red& r) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) r.f[w] = v;
  __syncthreads();
  float t = lane < kSW ? r.f[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

__device__ unsigned long long block_max_u64(unsigned long long v, Red& r) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, v, o);
    v = x > v ? x : v;
  }
  __syncthreads();
  if (lane == 0) r.u[w] = v;
  __syncthreads();
  unsigned long long t = lane < kSW ? r.u[lane] : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, t, o);
    t = x > t ? x : t;
  }
  return t;
}

// exclusive prefix (in thread order) of per-thread counts
__device__ uint32_t block_excl_scan(uint32_t v, Red& r) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) r.c[w] = x;
  __syncthreads();
  uint32_t base = 0;
  for (int i = 0; i < w; ++i) base += r.c[i];
  return base + x - v;
}

// exclusive prefix (in thread order) of per-thread float sums, fixed order
__device__ float block_excl_scan_f(float v, Red& r) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) r.f[w] = x;
  __syncthreads();
  float base = 0.f;
  for (int i = 0; i < w; ++i) base += r.f[i];
  return base + (x - v);
}

__device__ __forceinline__ uint32_t fkey(float f) { return __float_as_uint(f); }  // f >= 0: order preserved

// The row is held as 1024 contiguous chunks of C elements (chunk t belongs to
// thread t, so scans run in index order), each chunk padded to an odd stride:
// a warp walking its 32 chunks in step then touches 32 different banks.
__host__ __device__ __forceinline__ int chunk_len(int V) { return (V + 1023) / 1024; }
__host__ __device__ __forceinline__ int chunk_stride(int C) { return (C & 1) ? C : C + 1; }

// One radix-select pass over the row (contiguous chunks of C per thread, every
// lane taking the same number of steps): histogram of digit `pass` of the keys
// whose higher digits equal `pre`, with the 2^-40 fixed-point sum of their
// values when `sums`. Lanes of a warp that hit the same bin combine first
// (match + popc / redux), so a bin takes one shared-memory atomic per group:
// softmax outputs share few exponent bytes, and per-element atomics on them
// serialise.
__device__ __forceinline__ void radix_hist(const float* sc, int i0, int i1, int C, uint32_t pre, uint32_t hmask,
                                           int pass, bool sums, uint32_t* hc, unsigned long long* hs) {
  const int lane = threadIdx.x & 31;
  for (int k = 0; k < C; ++k) {
    const int i = i0 + k;
    const bool in = i < i1;
    const uint32_t key = in ? fkey(sc[k]) : 0u;
    const bool act = in && (key & hmask) == pre;
    const unsigned am = __ballot_sync(0xffffffffu, act);
    if (act) {
      const uint32_t bin = (key >> (8 * pass)) & 255u;
      const unsigned grp = __match_any_sync(am, bin);
      const bool leader = lane == __ffs(grp) - 1;
      if (leader) atomicAdd(&hc[bin], (uint32_t)__popc(grp));
      if (sums) {
        const unsigned long long v = (unsigned long long)((double)sc[k] * kFix);  // <= 2^40
        const uint32_t lo = __reduce_add_sync(grp, (uint32_t)(v & 0xfffffu));      // 20-bit halves: no overflow
        const uint32_t hi = __reduce_add_sync(grp, (uint32_t)(v >> 20));
        if (leader) atomicAdd(&hs[bin], ((unsigned long long)hi << 20) + lo);
      }
    }
  }
}

// Warp 0 picks the bin of a radix pass (lane l owns bins 255 - 8l down to 248 - 8l).
// Top-k: the highest bin b where the count from the top through b reaches rem;
// rem becomes rem minus the count above b.
__device__ __forceinline__ void pick_topk_bin(const uint32_t* hc, uint32_t& rem, int& bin) {
  const int lane = threadIdx.x & 31;
  uint32_t own = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) own += hc[255 - 8 * lane - i];
  uint32_t incl = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const unsigned hit = __ballot_sync(0xffffffffu, incl >= rem);
  const int L = hit ? __ffs(hit) - 1 : 31;
  const uint32_t excl = __shfl_sync(0xffffffffu, incl - own, L);
  if (lane == 0) {
    uint32_t r = rem - excl;
    int b = 255 - 8 * L;
    for (int i = 0; i < 8 && b > 0; ++i, --b) {
      if (hc[b] >= r) break;
      r -= hc[b];
    }
    rem = r;
    bin = b;
  }
}
// Top-p: the lowest non-empty bin whose mass above it (acc + higher bins) is below P.
__device__ __forceinline__ void pick_topp_bin(const uint32_t* hc, const unsigned long long* hs,
                                              unsigned long long P, unsigned long long& acc, int& bin) {
  const int lane = threadIdx.x & 31;
  unsigned long long own = 0ull;
#pragma unroll
  for (int i = 0; i < 8; ++i) own += hs[255 - 8 * lane - i];
  unsigned long long incl = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  unsigned long long a = acc + (incl - own), best_a = 0ull;
  int best = -1;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int b = 255 - 8 * lane - i;
    if (hc[b] && a < P) {
      best = b;
      best_a = a;
    }
    a += hs[b];
  }
  const unsigned has = __ballot_sync(0xffffffffu, best >= 0);
  const int L = has ? 31 - __clz(has) : 0;  // the highest lane holds the lowest bins
  const int b_out = __shfl_sync(0xffffffffu, best, L);
  const unsigned long long a_out = __shfl_sync(0xffffffffu, best_a, L);
  if (lane == 0) {
    if (has) {
      bin = b_out;
      acc = a_out;
    } else {
      bin = 255;  // unreachable: the top element always qualifies
    }
  }
}

__global__ void __launch_bounds__(kST) sample_kernel(const float* logits, int ld, int V, const rb_sampling* prm,
                                                     const uint32_t* prev, const uint32_t* prev_off, const float* uni,
                                                     uint32_t* out) {
  extern __shared__ float sv[];  // 1024 chunks of C, stride CS
  __shared__ Red red;
  __shared__ uint32_t hc[256];
  __shared__ unsigned long long hs[256];
  __shared__ uint32_t sel_prefix, sel_rem;
  __shared__ unsigned long long sel_acc;
  const int row = blockIdx.x, tid = threadIdx.x;
  const rb_sampling p = prm[row];
  const float* lg = logits + (size_t)row * ld;
  const int C = chunk_len(V), CS = chunk_stride(C);
  auto at = [&](int i) -> float& { return sv[(i / C) * CS + i % C]; };
  for (int i = tid; i < V; i += kST) at(i) = lg[i];
  __syncthreads();
  // 1. repetition penalty: thread (token % 1024) applies every occurrence, in order
  if (p.repetition_penalty != 1.0f && prev_off) {
    const uint32_t j0 = prev_off[row], j1 = prev_off[row + 1];
    for (uint32_t j = j0; j < j1; ++j) {
      const uint32_t t = prev[j];
      if (t < (uint32_t)V && (int)(t % kST) == tid) {
        const float x = at((int)t);
        at((int)t) = x > 0.f ? __fdiv_rn(x, p.repetition_penalty) : __fmul_rn(x, p.repetition_penalty);
      }
    }
  }
  __syncthreads();
  const int i0 = min(tid * C, V), i1 = min(i0 + C, V);  // this thread's chunk
  float* sc = sv + tid * CS;                             // sc[i - i0] is element i
  // 2. greedy
  if (p.temperature < 1e-7) {
    unsigned long long best = 0ull;
    for (int i = i0; i < i1; ++i) {
      const unsigned long long k = ((unsigned long long)float_order_key(sc[i - i0]) << 32) | (unsigned)i;
      best = k > best ? k : best;
    }
    best = block_max_u64(best, red);
    if (tid == 0) out[row] = (uint32_t)(best & 0xffffffffu);
    return;
  }
  // 3. temperature + softmax
  const float tf = (float)p.temperature;
  float mx = -INFINITY;
  for (int i = i0; i < i1; ++i) {
    sc[i - i0] = __fdiv_rn(sc[i - i0], tf);
    mx = fmaxf(mx, sc[i - i0]);
  }
  mx = block_max(mx, red);
  float s = 0.f;
  for (int i = i0; i < i1; ++i) {
    sc[i - i0] = expf(sc[i - i0] - mx);
    s += sc[i - i0];
  }
  s = block_sum(s, red);
  for (int i = i0; i < i1; ++i) sc[i - i0] = __fdiv_rn(sc[i - i0], s);
  __syncthreads();
  // 4. top-k
  if (p.top_k > 0 && p.top_k < (uint32_t)V) {
    if (tid == 0) {
      sel_prefix = 0;
      sel_rem = p.top_k;
    }
    for (int pass = 3; pass >= 0; --pass) {
      if (tid < 256) hc[tid] = 0;
      __syncthreads();
      const uint32_t pre = sel_prefix, hmask = pass == 3 ? 0u : (0xffffffffu << (8 * (pass + 1)));
      radix_hist(sc, i0, i1, C, pre, hmask, pass, false, hc, hs);
      __syncthreads();
      if (tid < 32) {
        uint32_t rem = sel_rem;
        int b = 0;
        pick_topk_bin(hc, rem, b);
        if (tid == 0) {
          sel_prefix = pre | ((uint32_t)b << (8 * pass));
          sel_rem = rem;
        }
      }
      __syncthreads();
    }
    const uint32_t T = sel_prefix, keep_eq = sel_rem;
    uint32_t n_eq = 0;
    for (int i = i0; i < i1; ++i) n_eq += fkey(sc[i - i0]) == T;
    uint32_t rank = block_excl_scan(n_eq, red);
    float ks = 0.f;
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = fkey(sc[i - i0]);
      bool keep = k > T;
      if (k == T) keep = rank++ < keep_eq;
      if (!keep) sc[i - i0] = 0.f;
      ks += sc[i - i0];
    }
    ks = block_sum(ks, red);
    if (ks > 0.f)
      for (int i = i0; i < i1; ++i) sc[i - i0] = __fdiv_rn(sc[i - i0], ks);
    __syncthreads();
  }
  // 5. top-p
  const float top_p = (float)p.top_p;
  if (p.top_p > 0.0 && p.top_p < 1.0) {
    const unsigned long long P = (unsigned long long)((double)top_p * kFix);
    if (tid == 0) {
      sel_prefix = 0;
      sel_acc = 0ull;
    }
    for (int pass = 3; pass >= 0; --pass) {
      if (tid < 256) {
        hc[tid] = 0;
        hs[tid] = 0ull;
      }
      __syncthreads();
      const uint32_t pre = sel_prefix, hmask = pass == 3 ? 0u : (0xffffffffu << (8 * (pass + 1)));
      radix_hist(sc, i0, i1, C, pre, hmask, pass, true, hc, hs);
      __syncthreads();
      if (tid < 32) {
        unsigned long long acc = sel_acc;
        int b = 255;
        pick_topp_bin(hc, hs, P, acc, b);
        if (tid == 0) {
          sel_prefix = pre | ((uint32_t)b << (8 * pass));
          sel_acc = acc;
        }
      }
      __syncthreads();
    }
    const uint32_t T = sel_prefix;
    const unsigned long long above = sel_acc, tq = (unsigned long long)((double)__uint_as_float(T) * kFix);
    uint32_t n_eq = 0;
    for (int i = i0; i < i1; ++i) n_eq += fkey(sc[i - i0]) == T;
    uint32_t rank = block_excl_scan(n_eq, red);
    float ps = 0.f;
    for (int i = i0; i < i1; ++i) {
      const uint32_t k = fkey(sc[i - i0]);
      bool keep = k > T;
      if (k == T) keep = above + (unsigned long long)(rank++) * tq < P;
      if (!keep) sc[i - i0] = 0.f;
      ps += sc[i - i0];
    }
    ps = block_sum(ps, red);
    if (ps > 0.f)
      for (int i = i0; i < i1; ++i) sc[i - i0] = __fdiv_rn(sc[i - i0], ps);
    __syncthreads();
  }
  // 6. WeightedIndex
  float cs = 0.f;
  for (int i = i0; i < i1; ++i) cs += sc[i - i0];
  const float total = block_sum(cs, red);
  if (!(total > 0.f) || !isfinite(total)) {
    if (tid == 0) out[row] = 0xffffffffu;
    return;
  }
  const float max_rand = 1.0f - 1.1920928955078125e-07f;
  float scale = total;
  while (__fmul_rn(scale, max_rand) >= total) scale = nextafterf(scale, 0.0f);
  const float chosen = __fmul_rn(uni[row], scale);
  float run = block_excl_scan_f(cs, red);
  unsigned long long first = 0ull;  // max over (~index): the smallest index with cum > chosen
  for (int i = i0; i < i1 && i < V - 1; ++i) {
    run += sc[i - i0];
    if (run > chosen) {
      first = 0xffffffffull - (unsigned)i + 1ull;
      break;
    }
  }
  first = block_max_u64(first, red);
  if (tid == 0) out[row] = first ? (uint32_t)(0xffffffffull - first + 1ull) : (uint32_t)(V - 1);
}

}  // namespace

size_t sample_smem_bytes(int vocab) { return (size_t)1024 * chunk_stride(chunk_len(vocab)) * 4; }

cudaError_t sample_launch(const float* logits, int ld, int n_rows, int vocab, const rb_sampling* params,
                          const uint32_t* prev, const uint32_t* prev_off, const float* uniforms, uint32_t* out,
                          cudaStream_t s) {
  if (n_rows < 1 || vocab < 1 || vocab > kSampleMaxVocab || ld < vocab) return cudaErrorInvalidValue;
  int dev = 0;
  cudaGetDevice(&dev);
  if (cudaError_t e = ensure_smem_attr(sample_kernel, (int)sample_smem_bytes(kSampleMaxVocab), dev)) return e;
  sample_kernel<<<n_rows, kST, sample_smem_bytes(vocab), s>>>(logits, ld, vocab, params, prev, prev_off, uniforms, out);
  return cudaGetLastError();
}

}  // namespace rb
