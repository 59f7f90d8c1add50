// Paged KV cache + paged GQA decode attention (sm_100a).
//
// Replaces the reference's contiguous fp32 KVCache (crates/realm-models/src/kv_cache.rs:7-80),
// repeat_kv + StandardAttention (crates/realm-models/src/attention.rs:272-380,
// crates/realm-models/src/attention_stub/mod.rs:42-158). The reference has no paged
// cache; here K/V live in 16-token pages reached through a per-tenant page table.
//
// Decode attention: a work unit is (query row, kv head, split of 16 pages). Each of
// the CTA's 4 warps streams its share of the split's pages (K and V blocks of one
// kv head, contiguous) with the bulk-copy engine into a private ring, so every KV
// page is read from HBM once per GQA group, and keeps an online-softmax state
// (max, sum, output) for all n_rep query heads of the group. Warps merge through
// shared memory; splits of one (row, kv head) are merged by the last CTA to finish
// in a fixed order (deterministic, no spin waits).
#include "attention.cuh"
#include "common.cuh"
#include "xfrag.cuh"

namespace rb {

namespace {

constexpr int kAttnWarps = 4;
constexpr int kMaxRows = 64;

__host__ __device__ constexpr int attn_ring(int hd, int f16) { return (hd == 128 && !f16) ? 2 : 3; }

template <int HD, int F16>
struct AttnCfg {
  static constexpr int ESZ = F16 ? 2 : 4;
  static constexpr int BLK = 16 * HD * ESZ;  // one page of one kv head (K or V)
  static constexpr int NSW = attn_ring(HD, F16);
  static constexpr int STAGE = 2 * BLK;
};

template <int HD, int NREP, int F16>
__host__ __device__ constexpr int attn_smem_bytes() {
  return kAttnWarps * AttnCfg<HD, F16>::NSW * AttnCfg<HD, F16>::STAGE  // rings
         + NREP * HD * 4                                               // q
         + kAttnWarps * NREP * 16 * 4                                  // probabilities
         + kAttnWarps * NREP * (HD + 2) * 4                            // warp merge
         + kAttnWarps * AttnCfg<HD, F16>::NSW * 8                      // mbarriers
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

struct UnitInfo {
  int row, kvh, split, p_begin, p_end, len;
  bool valid;
};

template <int HD, int NREP, int F16>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(const AttnArgs a) {
  using C = AttnCfg<HD, F16>;
  constexpr int NSW = C::NSW;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* rings = smem;
  float* qs = reinterpret_cast<float*>(rings + kAttnWarps * NSW * C::STAGE);
  float* pb = qs + NREP * HD;
  float* mrg = pb + kAttnWarps * NREP * 16;
  uint64_t* bars = reinterpret_cast<uint64_t*>(mrg + kAttnWarps * NREP * (HD + 2));
  int* row_units = reinterpret_cast<int*>(bars + kAttnWarps * NSW);  // prefix of units per row
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kv = a.kv.n_kv;
  const int G = gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kAttnWarps * NSW; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  pdl_launch_dependents();
  pdl_wait();
  // per-row unit prefix (units = n_kv * splits)
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int r = 0; r < a.n_rows; ++r) {
      row_units[r] = acc;
      const int np = (a.row_pos[r] >> 4) + 1;
      acc += n_kv * ((np + kAttnPagesPerSplit - 1) / kAttnPagesPerSplit);
    }
    row_units[a.n_rows] = acc;
  }
  __syncthreads();
  const int total = row_units[a.n_rows];

  auto decode = [&](int it) -> UnitInfo {
    UnitInfo ui;
    const int u = blockIdx.x + it * G;
    ui.valid = u < total;
    if (!ui.valid) return ui;
    int r = 0;
    while (r + 1 < a.n_rows && row_units[r + 1] <= u) ++r;
    const int np = (a.row_pos[r] >> 4) + 1;
    const int ns = (np + kAttnPagesPerSplit - 1) / kAttnPagesPerSplit;
    const int local = u - row_units[r];
    ui.row = r;
    ui.kvh = local / ns;
    ui.split = local % ns;
    ui.p_begin = ui.split * kAttnPagesPerSplit;
    ui.p_end = min(np, ui.p_begin + kAttnPagesPerSplit);
    ui.len = a.row_pos[r] + 1;
    return ui;
  };

  uint8_t* myring = rings + warp * NSW * C::STAGE;
  uint64_t* mybars = bars + warp * NSW;
  const size_t kv_head_stride = (size_t)16 * HD;  // elements
  auto block_ptr = [&](int tenant, int p, int which, int kvh) -> const uint8_t* {
    const int page = a.kv.ptab[(size_t)tenant * a.kv.ptab_stride + p];
    const size_t el = ((((size_t)page * a.kv.n_layers + a.layer) * 2 + which) * n_kv + kvh) * kv_head_stride;
    return reinterpret_cast<const uint8_t*>(a.kv.pool) + el * C::ESZ;
  };

  // producer iterator (uniform across the warp): CTA unit iteration + page
  int pit = 0, pp = -1;
  UnitInfo pu = decode(0);
  if (pu.valid) pp = pu.p_begin + warp;
  auto prod_advance = [&]() {
    pp += kAttnWarps;
    while (pu.valid && pp >= pu.p_end) {
      ++pit;
      pu = decode(pit);
      pp = pu.valid ? pu.p_begin + warp : -1;
    }
  };
  // position the producer on its first item
  while (pu.valid && pp >= pu.p_end) {
    ++pit;
    pu = decode(pit);
    pp = pu.valid ? pu.p_begin + warp : -1;
  }
  int issued = 0, consumed = 0;
  auto issue_upto = [&](int limit) {
    while (issued < limit && pu.valid) {
      if (lane == 0) {
        const int s = issued % NSW;
        mbar_arrive_expect_tx(&mybars[s], C::STAGE);
        const int tenant = a.row_tenant[pu.row];
        bulk_g2s(myring + s * C::STAGE, block_ptr(tenant, pp, 0, pu.kvh), C::BLK, &mybars[s]);
        bulk_g2s(myring + s * C::STAGE + C::BLK, block_ptr(tenant, pp, 1, pu.kvh), C::BLK, &mybars[s]);
      }
      ++issued;
      prod_advance();
    }
  };
  issue_upto(NSW);

  bool alive = true;
  const int j = lane & 15, hh = lane >> 4;
  constexpr int DPL = HD / 32;  // output dims per lane
  for (int it = 0;; ++it) {
    const UnitInfo ui = decode(it);
    if (!ui.valid) break;
    // q of the n_rep heads that share this kv head
    for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x)
      qs[i] = a.q[(size_t)ui.row * a.ldq + (size_t)ui.kvh * NREP * HD + i];
    __syncthreads();

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
      const uint8_t* vb = kb + C::BLK;
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
    // ---- merge the warps
#pragma unroll
    for (int r = 0; r < NREP; ++r) {
      float* w = mrg + (warp * NREP + r) * (HD + 2);
#pragma unroll
      for (int d = 0; d < DPL; ++d) w[lane * DPL + d] = o[r][d];
      if (lane == 0) {
        w[HD] = m[r];
        w[HD + 1] = l[r];
      }
    }
    __syncthreads();
    const int np_row = (a.row_pos[ui.row] >> 4) + 1;
    const int nsplit = (np_row + kAttnPagesPerSplit - 1) / kAttnPagesPerSplit;
    const size_t slot = ((size_t)ui.row * n_kv + ui.kvh) * a.max_splits + ui.split;
    // Final values go to shared memory (the q buffer is free now), then out to the
    // fp32 output and / or the activation fragments of the o-proj GEMV.
    float* ofin = qs;
    __shared__ float frag_scratch[16];
    auto finish = [&]() {
      __syncthreads();
      if (a.out)
        for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x)
          a.out[(size_t)ui.row * a.ldo + (size_t)ui.kvh * NREP * HD + i] = ofin[i];
      if (a.xout.xi || a.xout.xf)
        frags_write(ofin, 1, 0, NREP * HD, 1, ui.kvh * NREP * HD, ui.row, nullptr, a.xout, a.xf_nt, frag_scratch,
                    threadIdx.x, blockDim.x, [] { __syncthreads(); });
    };
    auto merge_warps = [&](int i, float& M, float& Lsum, float& O) {
      const int r = i / HD, d = i % HD;
      M = -INFINITY;
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, mrg[(w * NREP + r) * (HD + 2) + HD]);
      Lsum = 0.f;
      O = 0.f;
      for (int w = 0; w < kAttnWarps; ++w) {
        const float* ww = mrg + (w * NREP + r) * (HD + 2);
        const float f = (ww[HD] == -INFINITY) ? 0.f : expf(ww[HD] - M);
        Lsum += ww[HD + 1] * f;
        O += ww[d] * f;
      }
    };
    if (nsplit == 1) {
      for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x) {
        float M, Lsum, O;
        merge_warps(i, M, Lsum, O);
        ofin[i] = Lsum > 0.f ? O / Lsum : 0.f;
      }
      finish();
    } else {
      for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x) {
        const int r = i / HD, d = i % HD;
        float M, Lsum, O;
        merge_warps(i, M, Lsum, O);
        float* dst = a.partials + (slot * NREP + r) * (HD + 2);
        __stcg(dst + d, O);
        if (d == 0) {
          __stcg(dst + HD, M);
          __stcg(dst + HD + 1, Lsum);
        }
      }
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0)
        s_last = atomicAdd(a.counters + ui.row * n_kv + ui.kvh, 1) == nsplit - 1;
      __syncthreads();
      if (s_last) {
        __threadfence();
        const size_t base = ((size_t)ui.row * n_kv + ui.kvh) * a.max_splits;
        for (int i = threadIdx.x; i < NREP * HD; i += blockDim.x) {
          const int r = i / HD, d = i % HD;
          float M = -INFINITY;
          for (int s = 0; s < nsplit; ++s) M = fmaxf(M, __ldcg(a.partials + ((base + s) * NREP + r) * (HD + 2) + HD));
          float Lsum = 0.f, O = 0.f;
          for (int s = 0; s < nsplit; ++s) {
            const float* src = a.partials + ((base + s) * NREP + r) * (HD + 2);
            const float ms = __ldcg(src + HD);
            const float f = (ms == -INFINITY) ? 0.f : expf(ms - M);
            Lsum += __ldcg(src + HD + 1) * f;
            O += __ldcg(src + d) * f;
          }
          ofin[i] = Lsum > 0.f ? O / Lsum : 0.f;
        }
        finish();
        if (threadIdx.x == 0) a.counters[ui.row * n_kv + ui.kvh] = 0;
      }
    }
    __syncthreads();
  }
  // every issued copy is consumed on the normal path; after a timed-out wait,
  // let the copies still in flight land before the CTA exits (bounded)
  if (!alive && lane == 0)
    for (int k = (issued > NSW ? issued - NSW : 0); k < issued; ++k)
      mbar_wait(&mybars[k % NSW], (k / NSW) & 1, a.err, DEV_TIMEOUT_DRAIN);
}

template <int HD, int NREP, int F16>
cudaError_t launch_attn_t(const AttnArgs& a, int num_sms, cudaStream_t s, int pdl) {
  constexpr int smem = attn_smem_bytes<HD, NREP, F16>();
  auto kern = attn_kernel<HD, NREP, F16>;
  static unsigned long long attr_set = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_set & (1ull << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_set |= 1ull << dev;
  }
  const int per_sm = smem <= 110 * 1024 ? 2 : 1;
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
  switch (nrep) {
    case 1: return launch_attn_t<HD, 1, F16>(a, num_sms, s, pdl);
    case 2: return launch_attn_t<HD, 2, F16>(a, num_sms, s, pdl);
    case 4: return launch_attn_t<HD, 4, F16>(a, num_sms, s, pdl);
    case 8: return launch_attn_t<HD, 8, F16>(a, num_sms, s, pdl);
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

size_t attn_partials_floats(int max_rows, int n_kv, int n_rep, int hd, int max_splits) {
  return (size_t)max_rows * n_kv * max_splits * n_rep * (hd + 2);
}

cudaError_t attn_launch(const AttnArgs& a, int num_sms, cudaStream_t s, int pdl) {
  if (a.n_rows < 1 || a.n_rows > kMaxRows) return cudaErrorInvalidValue;
  const int nrep = a.n_heads / a.kv.n_kv;
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
