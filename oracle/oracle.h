// CPU oracle for the realm-b200 decode path.
//
// TEST INFRASTRUCTURE ONLY. This is a plain C++ restatement of the reference
// (Querent-ai/realm, Rust) CPU path used as the parity checker and as the timed
// CPU baseline. Nothing in the product library links, loads or calls it; only
// tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
// arms may use it.
//
// Every function names the reference file:line it follows (paths relative to
// the reference project root). Build: oracle/Makefile (g++ -O2
// -ffp-contract=off so that a*b-c stays two rounded operations, as in Rust).
#pragma once
#include <cstddef>
#include <cstdint>

extern "C" {

// ---- block formats (crates/realm-core/src/quant.rs:52-59, 97-107, 189-198) ----
#pragma pack(push, 1)
struct OrBlockQ4K { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[128]; };
struct OrBlockQ6K { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; };
struct OrBlockQ80 { uint16_t d; int8_t qs[32]; };
#pragma pack(pop)

enum OrDtype { OR_F32 = 0, OR_Q4K = 12, OR_Q6K = 14, OR_Q80 = 8, OR_F16 = 1 };

float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);
void or_get_scale_min_k4(int j, const uint8_t* scales, uint8_t* sc, uint8_t* m);

// Whole-tensor dequantisation; bit-exact restatement of dequantize_q4_k / q6_k / q8_0.
int or_dequant(int dtype, const void* blocks, size_t nblocks, float* out);

// Quantisers (the reference has none; these follow the GGUF block definitions).
int or_quantize(int dtype, const float* x, size_t n, void* out);
size_t or_block_bytes(int dtype);
size_t or_block_elems(int dtype);

// Fused dequant GEMV/GEMM, crates/realm-compute-cpu/src/fused.rs:229-374 (Q4_K),
// :1128-1259 (Q6_K), :2451-2554 (Q8_0): y[m,n] = sum_k x[m,k] * W[n,k].
// threads == 1 is the reference's single-threaded kernel with its AVX2 lane and
// horizontal-sum order; threads > 1 splits output rows across OpenMP threads
// (each output element is still computed in exactly the same order).
int or_fused_matmul(int dtype, const void* blocks, size_t nblocks, const float* x,
                    float* y, size_t m, size_t n, size_t k, int threads);

// CandleCpuBackend semantics (crates/realm-compute-cpu/src/candle_cpu_backend.rs:92-114):
// dequantise then an fp32 GEMM; here with a sequential fp32 sum per output.
int or_dequant_matmul(int dtype, const void* blocks, size_t nblocks, const float* x,
                      float* y, size_t m, size_t n, size_t k, int threads);
// The same sums computed one output element at a time (bit-identical check).
int or_dequant_matmul_scalar(int dtype, const void* blocks, size_t nblocks, const float* x,
                             float* y, size_t m, size_t n, size_t k, int threads);
// Same, accumulated in double (error-bound shadow for tolerance checks).
int or_dequant_matmul_f64(int dtype, const void* blocks, size_t nblocks, const float* x,
                          double* y, size_t m, size_t n, size_t k, int threads);

// ---- model pieces (crates/realm-models/src) ----
void or_rms_norm(const float* x, const float* w, float eps, size_t rows, size_t h, float* y);
void or_rope(float* t, size_t start_pos, size_t seq_len, size_t n_heads, size_t hd, float theta);
// compute_attention + StandardAttention::forward (attention.rs:310-380, attention_stub/mod.rs:42-158)
void or_attention(const float* q, const float* k, const float* v, size_t seq_len, size_t kv_len,
                  size_t position, size_t n_heads, size_t n_kv, size_t hd, float* out);

// KV cache (crates/realm-models/src/kv_cache.rs:7-80); kv_fp16 rounds to fp16 RNE on append.
void* or_kv_new(size_t max_seq, size_t n_kv, size_t hd, int kv_fp16);
void or_kv_free(void* kv);
int or_kv_append(void* kv, const float* k, const float* v, size_t n_floats);
size_t or_kv_len(void* kv);
void or_kv_data(void* kv, float* k_out, float* v_out);
void or_kv_clear(void* kv);

struct OrModelConfig {
  int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, max_seq;
  float rms_eps;     // final norm eps (model.rs:604-610, config.rms_norm_eps)
  float layer_eps;   // per-layer norm eps: config eps (memory64_host.rs:2069) or 1e-6 (layer.rs:57)
  float rope_theta;
  int32_t kv_fp16;
  int32_t threads;
};

// weight ids
enum OrWeight {
  OR_W_TOKEN_EMBD = 0, OR_W_OUTPUT_NORM = 1, OR_W_OUTPUT = 2,
  OR_W_ATTN_NORM = 10, OR_W_Q, OR_W_K, OR_W_V, OR_W_O, OR_W_FFN_NORM, OR_W_GATE, OR_W_UP, OR_W_DOWN
};

void* or_model_new(const OrModelConfig* cfg);
void or_model_free(void* model);
// layer = -1 for global tensors; bytes copied.
int or_model_set_weight(void* model, int which, int layer, int dtype, const void* data, size_t nbytes);
// Model::forward (model.rs:572-625): logits of the last token -> logits[vocab]
int or_model_forward(void* model, const uint32_t* tokens, size_t n, size_t position, float* logits);
// final hidden state (after final norm) of the last token, for debugging
int or_model_last_hidden(void* model, float* out);
void or_model_clear_kv(void* model);
int or_model_kv_fill(void* model, size_t n, uint64_t seed);
size_t or_model_kv_len(void* model, int layer);
void or_model_kv_data(void* model, int layer, float* k_out, float* v_out);
// Model::generate with greedy sampling (model.rs:749-847, sampling.rs:141-148) on token ids:
// writes n_gen generated ids to out_tokens and, if step_logits != NULL, the logits that
// produced each of them ([n_gen][vocab]).
int or_model_generate(void* model, const uint32_t* prompt, size_t n_prompt, size_t n_gen,
                      uint32_t* out_tokens, float* step_logits);
// argmax with ties to the LAST index (Rust Iterator::max_by, sampling.rs:141-148)
uint32_t or_argmax(const float* x, size_t n);

// LogitsProcessor::with_params(seed, temperature, top_p, top_k, repetition_penalty)
// then sample(logits) (crates/realm-models/src/sampling.rs:63-100, 107-300), with
// the random draw supplied: u in [0, 1) is the value rand 0.8.5's Uniform<f32>
// sampler would produce (a multiple of 2^-23). previous tokens: prev[n_prev]
// (the tokens this processor sampled before). logits is modified in place as the
// reference does. Writes the token to *out; returns 0, or -1 where the
// reference returns Err (WeightedIndex::new failed).
int or_sample(float* logits, size_t n, double temperature, double top_p, size_t top_k, float penalty,
              const uint32_t* prev, size_t n_prev, float u, uint32_t* out);
}
