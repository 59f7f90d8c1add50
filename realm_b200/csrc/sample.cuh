// Fused sampling (sample.cu): one CTA per logits row.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/realm_b200.h"

namespace rb {

constexpr int kSampleMaxVocab = 53248;  // the row lives in shared memory (217 KB with chunk padding)

size_t sample_smem_bytes(int vocab);
// logits [n_rows][ld] (device), params [n_rows], previous tokens prev[prev_off[r] ..
// prev_off[r + 1]) per row (prev_off may be NULL: none), uniforms [n_rows] in [0, 1);
// out [n_rows]: the sampled id, or 0xffffffff where WeightedIndex::new would fail.
cudaError_t sample_launch(const float* logits, int ld, int n_rows, int vocab, const rb_sampling* params,
                          const uint32_t* prev, const uint32_t* prev_off, const float* uniforms, uint32_t* out,
                          cudaStream_t s);

}  // namespace rb
