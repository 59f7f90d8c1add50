/*
 * realm_b200.h — C ABI of the B200-native decode engine for Realm.
 *
 * One shared library (librealm_b200.so) replaces, for the decode hot path, the
 * reference's (Querent-ai/realm) host functions that WASM tenants call and the
 * GPU backend trait behind them. Every entry point names the reference
 * interface it stands in for (paths relative to the reference project root).
 *
 * Conventions
 *  - Every function returns int32_t: >= 0 is a count (elements or bytes, the
 *    same meaning as the host function it mirrors), < 0 is an error code.
 *  - Codes -1..-8 keep the meanings of crates/realm-runtime/src/host_functions.rs:145-155;
 *    codes from -20 on are specific to this library. rb_last_error() returns a
 *    thread-local message for the last failure on the calling thread.
 *  - Buffers passed with flags & RB_PTR_DEVICE are CUDA device pointers on the
 *    context's device; otherwise they are host pointers and the call copies
 *    in/out (pinned memory is fastest but not required).
 *  - One rb_ctx per GPU. Calls on one context are serialised on its stream and
 *    must come from one host thread at a time; contexts on different GPUs are
 *    independent (no global locks).
 *  - Weight bytes are GGUF block bytes exactly as stored in the reference's
 *    QuantizedTensor (crates/realm-runtime/src/model_storage.rs:44-77).
 */
#ifndef REALM_B200_H
#define REALM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---- */
#define RB_OK 0
#define RB_ERR_DISABLED (-1)        /* feature not available */
#define RB_ERR_NOT_FOUND (-2)       /* layer / resource not found */
#define RB_ERR_INVALID (-3)         /* buffer too small / validation failed */
#define RB_ERR_IO (-4)              /* read / write failed */
#define RB_ERR_NO_MEMORY (-5)       /* memory not available */
#define RB_ERR_PTR_OVERFLOW (-6)
#define RB_ERR_OUT_OF_BOUNDS (-7)
#define RB_ERR_WRITE (-8)
#define RB_ERR_BAD_HANDLE (-20)
#define RB_ERR_KV_POOL_EXHAUSTED (-21)
#define RB_ERR_KV_OVERFLOW (-22)    /* crates/realm-models/src/kv_cache.rs:48-53 */
#define RB_ERR_UNSUPPORTED (-23)    /* dtype / shape, e.g. K % 256 != 0 (fused.rs:238-243) */
#define RB_ERR_CUDA (-24)
#define RB_ERR_TIMEOUT (-25)        /* a bounded device wait gave up */
#define RB_ERR_OOM (-26)

/* ---- pointer-space flags ---- */
#define RB_PTR_HOST 0u
#define RB_PTR_DEVICE 1u
/* With RB_PTR_DEVICE: enqueue on the context stream and return without waiting
 * (rb_weight_matmul, rb_attention_forward); device-side failures surface at the
 * next rb_sync. Without RB_PTR_DEVICE the flag is ignored. */
#define RB_ASYNC 2u

/* ---- dtypes: GGML type ids (crates/realm-core/src/tensor.rs:7-40) ---- */
#define RB_F32 0
#define RB_F16 1
#define RB_Q8_0 8
#define RB_Q4_K 12
#define RB_Q6_K 14

typedef struct rb_ctx rb_ctx;

typedef struct rb_config {
  int32_t device;       /* CUDA device ordinal */
  uint32_t max_rows;    /* largest batch of query rows per call (<= 64) */
  uint32_t use_pdl;     /* programmatic dependent launch between kernels */
  uint32_t use_graphs;  /* capture decode steps as CUDA graphs */
} rb_config;

/* ---- context ---- */
int32_t rb_ctx_create(const rb_config* cfg, rb_ctx** out);
int32_t rb_ctx_destroy(rb_ctx* ctx);
int32_t rb_last_error(char* buf, size_t len);
/* Waits for all work on the context's stream (bounded: RB_ERR_TIMEOUT after ~60 s). */
int32_t rb_sync(rb_ctx* ctx);
/* The context's cudaStream_t, for callers that enqueue their own copies. */
void* rb_stream(rb_ctx* ctx);
int32_t rb_num_sms(rb_ctx* ctx);
/* Test hook: the architecture the library's kernels were compiled for, as the
 * CUDA runtime reports it for the loaded module (cudaFuncAttributes::binaryVersion,
 * 100 for sm_100a), written to *version. */
int32_t rb_kernel_binary_version(rb_ctx* ctx, int32_t* version);
/* Failure-detection test hook: the next multi-phase GEMV launch on this context
 * (the next rb_forward runs it outside any cached CUDA graph) gets its first
 * grid barrier's target out of reach, and every grid-barrier wait in it gives
 * up after spin_polls polls. The waits report through the device error word,
 * the kernel finishes, and the call returns RB_ERR_TIMEOUT (the reference's
 * host functions map such failures to a negative status as well,
 * crates/realm-runtime/src/host_functions.rs:145-155); the context stays usable.
 * Cache lengths are not advanced by the failed step. */
int32_t rb_test_fail_next_grid_barrier(rb_ctx* ctx, uint32_t spin_polls);

/* ---- quantised blocks ----
 * rb_dequantize: bit-exact dequantize_q4_k / q6_k / q8_0
 * (crates/realm-core/src/quant.rs:127-187, 393-451, 371-387; dispatch :663-939).
 * Returns elements written. */
int32_t rb_dequantize(rb_ctx* ctx, int32_t dtype, const void* blocks, size_t nblocks, float* out, uint32_t flags);
/* Quantiser (the reference has none; used to build the synthetic Q4_K_M weights).
 * Returns blocks written. */
int32_t rb_quantize(rb_ctx* ctx, int32_t dtype, const float* x, size_t n, void* out_blocks, uint32_t flags);

/* ---- fused dequant matmul ----
 * Mirrors fused_dequant_matmul_{q4k,q6k,q80}(blocks, input, output, batch_size, n, k)
 * (crates/realm-compute-cpu/src/fused.rs:229, 1128, 2451) and
 * GpuBackendTrait::fused_dequant_matmul_* (crates/realm-compute-gpu/src/gpu_backend_trait.rs:17-143):
 * output[b, j] = sum_i input[b, i] * W[j, i]; W is [n][k] GGUF blocks.
 * Validation as the reference: K % 256 for K-quants, block count, batch <= max_rows.
 * Returns batch_size * n. The blocks are staged and re-tiled on every call; use
 * rb_weight_upload + rb_weight_matmul to keep a weight resident. */
int32_t rb_fused_dequant_matmul(rb_ctx* ctx, int32_t dtype, const void* blocks, size_t nblocks, const float* input,
                                float* output, uint32_t batch_size, uint32_t n, uint32_t k, uint32_t flags);
/* Uploads a [n][k] GGUF weight once (tiled for the tensor-core GEMV). */
int32_t rb_weight_upload(rb_ctx* ctx, int32_t dtype, uint32_t n, uint32_t k, const void* blocks, size_t nbytes,
                         uint32_t flags, int32_t* handle);
int32_t rb_weight_free(rb_ctx* ctx, int32_t handle);
int32_t rb_weight_matmul(rb_ctx* ctx, int32_t handle, const float* input, float* output, uint32_t batch_size,
                         uint32_t flags);
/* Allocation-free variant of rb_weight_matmul; it has no counterpart in the
 * reference. For callers that cannot allocate device memory when they run a
 * matmul (a fixed memory budget handed over at start-up, an allocator owned by
 * another runtime, or a hot path where cudaMalloc/cudaFree and their device
 * synchronisation are not allowed): input [batch][k] and output [batch][n] are
 * caller-owned device buffers (flags must contain RB_PTR_DEVICE; RB_ASYNC
 * returns without waiting), and all other working memory is one fixed
 * 3,565,568-byte device array in the library, held on every GPU that loads it
 * until the process exits. Limits: batch <= 8, K <= 16384, N <= 131072, at most
 * 160 GEMV CTAs; larger calls fail with RB_ERR_INVALID. A Q8_0 weight whose K
 * is not a multiple of 256 (rows zero-padded at upload) is refused with
 * RB_ERR_UNSUPPORTED; rb_weight_matmul takes it. Every call on a device
 * shares the array (it keeps the last call's contents), so calls whose GPU
 * work overlaps race: order them on one stream. The first call on a device
 * looks up the array's address and caches it for the device's primary
 * context: make that call before any stream capture there, and do not call
 * again after the context was torn down (cudaDeviceReset) in this process.
 * Returns batch * n. */
int32_t rb_weight_matmul_noalloc(rb_ctx* ctx, int32_t handle, const float* input, float* output, uint32_t batch,
                                 uint32_t flags);
/* Timing hook: device time (microseconds) per launch of the GEMV kernel alone,
 * from a CUDA graph of `iters` back-to-back launches cycling over `n_handles`
 * resident weights (same K) with a fixed device-resident batch of `batch` rows
 * (activation fragments prepared once). The graph is replayed `reps` times and
 * the mean is returned in *avg_us. */
int32_t rb_weight_matmul_timing(rb_ctx* ctx, const int32_t* handles, uint32_t n_handles, uint32_t batch, uint32_t iters,
                                uint32_t reps, float* avg_us);
/* 1 when rb_weight_matmul of `batch` rows runs on the tcgen05 dequant-GEMM,
 * 0 when it runs on the mma.sync GEMV. */
int32_t rb_weight_matmul_path(rb_ctx* ctx, uint32_t batch);
/* Test hook: the resident tiled bytes converted back to GGUF layout (Q4_K). */
int32_t rb_weight_export(rb_ctx* ctx, int32_t handle, void* out_blocks, size_t nbytes, uint32_t flags);

/* candle_matmul (crates/realm-runtime/src/memory64_host.rs:861-969): C[m,n] = A[m,k] . B[k,n], f32.
 * candle_matmul_transposed (:975-1086): B given as [n,k]. Returns m*n. */
int32_t rb_candle_matmul(rb_ctx* ctx, const float* a, const float* b, float* c, uint32_t m, uint32_t k, uint32_t n,
                         uint32_t flags);
int32_t rb_candle_matmul_transposed(rb_ctx* ctx, const float* a, const float* b, float* c, uint32_t m, uint32_t k,
                                    uint32_t n, uint32_t flags);

/* ---- paged KV cache ----
 * The reference keeps one contiguous fp32 KVCache per layer
 * (crates/realm-models/src/kv_cache.rs:7-80) in a global map keyed by (model, layer)
 * (crates/realm-runtime/src/kv_cache_storage.rs:12-88). Here a pool holds
 * 16-token pages for all layers of a model geometry; each tenant owns a page
 * table and one length per layer. kv_dtype is RB_F32 (reference layout) or
 * RB_F16 (K/V rounded to fp16, nearest-even, on append). */
int32_t rb_kv_pool_create(rb_ctx* ctx, uint32_t n_layers, uint32_t n_kv_heads, uint32_t head_dim, int32_t kv_dtype,
                          uint32_t n_pages, uint32_t max_tenants, uint32_t max_seq, int32_t* pool);
int32_t rb_kv_pool_destroy(rb_ctx* ctx, int32_t pool);
/* Permutes the order in which free pages are handed out (deterministic in seed). */
int32_t rb_kv_pool_shuffle(rb_ctx* ctx, int32_t pool, uint64_t seed);
int32_t rb_kv_pool_free_pages(rb_ctx* ctx, int32_t pool);
/* KVCache::new (kv_cache.rs:24-34) for one tenant. */
int32_t rb_kv_create(rb_ctx* ctx, int32_t pool, uint32_t tenant);
int32_t rb_kv_destroy(rb_ctx* ctx, int32_t pool, uint32_t tenant);
/* KVCache::clear (kv_cache.rs:36-40): length 0, pages returned to the pool. */
int32_t rb_kv_clear(rb_ctx* ctx, int32_t pool, uint32_t tenant);
/* KVCache::current_seq_len */
int32_t rb_kv_len(rb_ctx* ctx, int32_t pool, uint32_t tenant, uint32_t layer);
/* KVCache::append (kv_cache.rs:44-70): k, v are [seq_len][n_kv][hd] f32.
 * Returns the new length, or RB_ERR_KV_OVERFLOW past max_seq. */
int32_t rb_kv_append(rb_ctx* ctx, int32_t pool, uint32_t tenant, uint32_t layer, const float* k, const float* v,
                     uint32_t seq_len, uint32_t flags);
/* KVCache::current_data (kv_cache.rs:73-79): writes [len][n_kv][hd] f32 each; returns len. */
int32_t rb_kv_gather(rb_ctx* ctx, int32_t pool, uint32_t tenant, uint32_t layer, float* k_out, float* v_out,
                     uint32_t flags);

/* ---- attention ----
 * The north star's attention_forward; defined after the reference's
 * Attention::forward trait (crates/realm-runtime/src/attention/mod.rs:34-45) and
 * compute_attention (crates/realm-models/src/attention.rs:310-380), over the paged cache.
 * Row r is a query of tenant tenants[r] at position positions[r]; it attends to
 * cached positions [0, positions[r]] of `layer` (causal mask, GQA grouping
 * n_heads / n_kv_heads). If k_new/v_new are given ([n_rows][n_kv][hd]) they are
 * appended at positions[r] first (positions[r] must equal that tenant's length).
 * q, out: [n_rows][n_heads][hd]. Returns n_rows * n_heads * hd. */
int32_t rb_attention_forward(rb_ctx* ctx, int32_t pool, uint32_t layer, uint32_t n_rows, const uint32_t* tenants,
                             const uint32_t* positions, const float* q, const float* k_new, const float* v_new,
                             float* out, uint32_t n_heads, float scale, uint32_t flags);

/* ---- model ---- */
typedef struct rb_model_config {
  uint32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, max_seq;
  float rms_eps;    /* final norm eps (crates/realm-models/src/model.rs:604-610) */
  float layer_eps;  /* per-layer norm eps (memory64_host.rs:2069, 2337 use the config eps) */
  float rope_theta;
  int32_t kv_dtype; /* RB_F32 or RB_F16 */
  uint32_t max_tenants;
  uint32_t kv_pages; /* 0: max_tenants * ceil(max_seq / 16) */
} rb_model_config;

/* weight ids (layer = -1 for the global ones) */
#define RB_W_TOKEN_EMBD 0
#define RB_W_OUTPUT_NORM 1
#define RB_W_OUTPUT 2
#define RB_W_ATTN_NORM 10
#define RB_W_Q 11
#define RB_W_K 12
#define RB_W_V 13
#define RB_W_O 14
#define RB_W_FFN_NORM 15
#define RB_W_GATE 16
#define RB_W_UP 17
#define RB_W_DOWN 18

int32_t rb_model_create(rb_ctx* ctx, const rb_model_config* cfg, int32_t* model);
int32_t rb_model_destroy(rb_ctx* ctx, int32_t model);
/* Stores one tensor (GGUF bytes, or f32 for norms). Returns bytes stored. */
int32_t rb_model_set_weight(rb_ctx* ctx, int32_t model, int32_t which, int32_t layer, int32_t dtype, const void* data,
                            size_t nbytes, uint32_t flags);
/* Tiles and fuses the stored tensors (q|k, gate/up interleave); call once after set_weight. */
int32_t rb_model_finalize(rb_ctx* ctx, int32_t model);
/* The KV pool holding this model's tenants (usable with the rb_kv_* calls). */
int32_t rb_model_kv_pool(rb_ctx* ctx, int32_t model);
/* The model's configuration as created (kv_pages resolved to the pool's page count). */
int32_t rb_model_get_config(rb_ctx* ctx, int32_t model, rb_model_config* out);
/* The context's largest batch of query rows per rb_forward (rb_config.max_rows, <= 64). */
int32_t rb_ctx_max_rows(rb_ctx* ctx);
int32_t rb_tenant_create(rb_ctx* ctx, int32_t model, uint32_t tenant);
int32_t rb_tenant_reset(rb_ctx* ctx, int32_t model, uint32_t tenant);

/* Batched forward over query rows (decode: one row per tenant; prefill chunk:
 * consecutive rows of one tenant). Row r feeds tokens[r] at positions[r]
 * (NULL: the tenant's cache length, then +1 per further row of that tenant),
 * which must equal the tenant's cache length plus the row's rank within the
 * tenant. Follows Model::forward (crates/realm-models/src/model.rs:572-625) per
 * row: embed, layers, final norm, LM head. logits: [n_rows][vocab] or NULL;
 * argmax: [n_rows] greedy ids (sampling.rs:141-148, ties -> last) or NULL.
 * Returns n_rows. */
int32_t rb_forward(rb_ctx* ctx, int32_t model, uint32_t n_rows, const uint32_t* tenants, const uint32_t* tokens,
                   const uint32_t* positions, float* logits, uint32_t* argmax, uint32_t flags);

/* Measurement hook: one decode step as rb_forward (positions = cache lengths,
 * no outputs), run without graph replay or programmatic dependent launch and
 * with an event after every kernel, so each interval is one kernel's device
 * time. kind_ms[4] receives the summed milliseconds of the embedding, GEMV
 * (multi-phase chain), attention and tcgen05 GEMM launches. Returns the
 * number of launches. */
int32_t rb_forward_profile(rb_ctx* ctx, int32_t model, uint32_t n_rows, const uint32_t* tenants,
                           const uint32_t* tokens, float* kind_ms);

/* realm_embed_tokens (crates/realm-runtime/src/memory64_host.rs:2483-2613): out [n][hidden]. Returns bytes. */
int32_t rb_embed_tokens(rb_ctx* ctx, int32_t model, const uint32_t* token_ids, uint32_t n, float* out,
                        uint32_t flags);
/* realm_forward_layer (memory64_host.rs:1918-2471): one transformer layer over
 * hidden [hidden_len / hidden][hidden] for `tenant`, appending to its cache at
 * `position` (must equal the layer's cache length). Returns bytes written. */
int32_t rb_forward_layer(rb_ctx* ctx, int32_t model, uint32_t tenant, uint32_t layer, const float* hidden,
                         uint32_t hidden_len, uint32_t position, float* out, uint32_t flags);
/* realm_compute_logits (memory64_host.rs:2742-2896): final norm + LM head of one
 * hidden row (hidden_len == hidden). Returns vocab * 4 bytes. */
int32_t rb_compute_logits(rb_ctx* ctx, int32_t model, const float* hidden, uint32_t hidden_len, float* out,
                          uint32_t flags);
/* memory64_load_layer (memory64_host.rs:688-763): copies layer `layer_id`'s GGUF
 * weight bytes (wq, wk, wv, wo, w_gate, w_up, w_down in that order) to dst.
 * Returns bytes, RB_ERR_NOT_FOUND (no such layer) or RB_ERR_INVALID (max_size too small). */
int32_t rb_memory64_load_layer(rb_ctx* ctx, int32_t model, uint32_t layer_id, void* dst, uint32_t max_size);
/* memory64_read (memory64_host.rs:767-825): copies `size` bytes at `offset` of the
 * model's Memory64 image into the caller's linear memory `mem` (mem_size bytes,
 * the WASM memory's extent) at `mem_offset`. The image is the layers' weight
 * bytes back to back, each layer laid out as rb_memory64_load_layer returns it.
 * Returns size, or the reference's codes: -4 (mem_offset + size overflows),
 * -5 (beyond mem_size), -2 (offset + size beyond the image). `mem` is host
 * memory unless flags has RB_PTR_DEVICE. */
int32_t rb_memory64_read(rb_ctx* ctx, int32_t model, uint64_t offset, void* mem, uint32_t mem_size,
                         uint32_t mem_offset, uint32_t size, uint32_t flags);
/* Total bytes of the model's Memory64 image (sum of every layer's weight bytes). */
int32_t rb_memory64_size(rb_ctx* ctx, int32_t model, uint64_t* size);

/* ---- GGUF files ----
 * rb_gguf is GGUFParser (crates/realm-core/src/formats/gguf.rs:100-479) over a
 * read-only memory mapping of the file (or caller-owned bytes), with the same
 * header rules and messages:
 *  - magic "GGUF" ("Invalid GGUF magic: 0x%08X");
 *  - version 2 or 3 ("Unsupported GGUF version: %u");
 *  - metadata of value types 0..12; an array of arrays is rejected ("Unknown
 *    typed value: 9");
 *  - tensor infos (name, dims, ggml type, offset relative to the data section).
 * Unknown ggml types parse, with nbytes 0 (gguf.rs:474-477 keeps parsing).
 * Errors: RB_ERR_INVALID for format errors, RB_ERR_IO for a truncated or
 * unreadable file.
 * Two deviations, both fixes of the reference:
 *  - tensor bytes are located at data section + offset. The data section
 *    starts at the end of the tensor infos, rounded up to general.alignment
 *    (default 32). model_storage.rs:444-464 drops the data-section offset.
 *  - nbytes uses the real ggml block sizes (Q8_0 34 bytes, Q4_0 18, Q8_K 292).
 *    tensor.rs:139-178 has 33, 16 and 322.
 * Every tensor's bytes are checked to lie inside the file. */
typedef struct rb_gguf rb_gguf;
typedef struct rb_gguf_tensor {
  const char* name;
  int32_t dtype;         /* ggml type id (RB_F32, RB_Q4_K, ...) */
  uint32_t n_dims;
  uint64_t dims[4];      /* ggml order: dims[0] is the contiguous (column) extent */
  uint64_t offset;       /* as stored: relative to the data section */
  uint64_t file_offset;  /* absolute position in the file */
  uint64_t nbytes;       /* 0 for ggml types this library does not know */
  const void* data;      /* host pointer into the mapping */
} rb_gguf_tensor;
/* metadata value types (gguf.rs:11-29) */
#define RB_GGUF_U8 0
#define RB_GGUF_I8 1
#define RB_GGUF_U16 2
#define RB_GGUF_I16 3
#define RB_GGUF_U32 4
#define RB_GGUF_I32 5
#define RB_GGUF_F32 6
#define RB_GGUF_BOOL 7
#define RB_GGUF_STRING 8
#define RB_GGUF_ARRAY 9
#define RB_GGUF_U64 10
#define RB_GGUF_I64 11
#define RB_GGUF_F64 12

int32_t rb_gguf_open(const char* path, rb_gguf** out);
/* Parses caller-owned bytes (GGUFParser over a Cursor); they must outlive the handle. */
int32_t rb_gguf_open_memory(const void* bytes, size_t nbytes, rb_gguf** out);
int32_t rb_gguf_close(rb_gguf* g);
int32_t rb_gguf_version(rb_gguf* g);
/* Start of the tensor data section in the file. */
int32_t rb_gguf_data_offset(rb_gguf* g, uint64_t* out);
int32_t rb_gguf_tensor_count(rb_gguf* g);
int32_t rb_gguf_tensor_info(rb_gguf* g, uint32_t index, rb_gguf_tensor* out);
/* Index of a tensor by name, or RB_ERR_NOT_FOUND ("Tensor not found: <name>"). */
int32_t rb_gguf_find_tensor(rb_gguf* g, const char* name);
int32_t rb_gguf_meta_count(rb_gguf* g);
/* Key and value type of metadata entry i (file order); for arrays also the element type and length. */
int32_t rb_gguf_meta_entry(rb_gguf* g, uint32_t index, const char** key, int32_t* type, int32_t* elem_type,
                           uint64_t* length);
/* Index of a metadata key, or RB_ERR_NOT_FOUND. */
int32_t rb_gguf_meta_find(rb_gguf* g, const char* key);
/* MetadataValue::as_u32 / as_f32 (gguf.rs:50-75): integer types cast to u32;
 * f32/f64 to f32; otherwise RB_ERR_INVALID. */
int32_t rb_gguf_meta_u32(rb_gguf* g, uint32_t index, uint32_t* out);
int32_t rb_gguf_meta_f32(rb_gguf* g, uint32_t index, float* out);
/* The raw little-endian bytes of a scalar value (cap >= its size); returns the size. */
int32_t rb_gguf_meta_scalar(rb_gguf* g, uint32_t index, void* out, size_t cap);
/* A string value (elem < 0) or element `elem` of a string array; not NUL-terminated. */
int32_t rb_gguf_meta_string(rb_gguf* g, uint32_t index, int64_t elem, const char** str, uint64_t* len);
/* Host pointer to the packed little-endian elements of a numeric or bool array. */
int32_t rb_gguf_meta_array_data(rb_gguf* g, uint32_t index, const void** data);
/* extract_config (gguf.rs:214-287): the transformer geometry from
 * "<arch>.*" keys, with the reference's fallbacks and defaults. head_dim =
 * hidden / n_heads; layer_eps = rms_eps; kv_dtype, max_tenants and kv_pages are
 * left 0 for the caller. */
int32_t rb_gguf_model_config(rb_gguf* g, rb_model_config* out);
/* Model::load_from_gguf (crates/realm-models/src/model.rs:291-540) onto the
 * device. It looks tensors up by name:
 *  - token_embd.weight, output_norm.weight, output.weight (else lm_head.weight,
 *    else the token embedding: tied weights);
 *  - blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm, ffn_gate,
 *    ffn_up, ffn_down}.weight.
 * cfg gives the geometry, as rb_gguf_model_config returns it and the caller
 * adjusts it (kv_dtype, max_tenants, kv_pages, max_seq). Shapes are checked
 * against it. Norm weights may be F32 or F16 (widened to f32). Creates and
 * finalizes a model; *model gets its handle. Returns RB_OK. */
int32_t rb_model_load_gguf(rb_ctx* ctx, rb_gguf* g, const rb_model_config* cfg, int32_t* model);

/* ---- sampling ----
 * LogitsProcessor (crates/realm-models/src/sampling.rs) on the device. The
 * strategy follows LogitsProcessor::with_params (:63-100):
 *  - temperature < 1e-7: argmax (ties to the last index);
 *  - else softmax(x / temperature), then top-k when 0 < top_k < vocab, then
 *    top-p when 0 < top_p < 1, then a multinomial draw.
 * The repetition penalty is applied before either, once per occurrence of each
 * previous token: a positive logit is divided by it, any other multiplied (:107-122).
 * The draw is rand 0.8.5's WeightedIndex over the probabilities with the uniform
 * value supplied by the caller. The reference's StdRng stream is not reproduced:
 * rb_sampling_uniform gives a counter-based uniform with the same 2^-23 grid. */
typedef struct rb_sampling {
  double temperature;       /* < 1e-7: greedy */
  double top_p;             /* used when 0 < top_p < 1 */
  uint32_t top_k;           /* used when 0 < top_k < vocab */
  float repetition_penalty; /* 1.0: off */
} rb_sampling;

/* Samples one token per row of logits [n_rows][ld] (vocab <= 53248). prev_tokens /
 * prev_offsets: row r's previous tokens are prev_tokens[prev_offsets[r] ..
 * prev_offsets[r + 1]) (both NULL: none). uniforms: [n_rows] values in [0, 1).
 * With RB_PTR_DEVICE every pointer is device memory; otherwise all are host
 * memory. Returns n_rows, or RB_ERR_INVALID ("Failed to create weighted index")
 * if a row has no positive probability left, as the reference's Err. */
int32_t rb_sample_logits(rb_ctx* ctx, const float* logits, uint32_t ld, uint32_t n_rows, uint32_t vocab,
                         const rb_sampling* params, const uint32_t* prev_tokens, const uint32_t* prev_offsets,
                         const float* uniforms, uint32_t* out_tokens, uint32_t flags);
/* The counter-based uniform draw in [0, 1) (a multiple of 2^-23) of (seed, counter):
 * SplitMix64 of seed + counter * 0x9E3779B97F4A7C15, top 23 bits. */
float rb_sampling_uniform(uint64_t seed, uint64_t counter);
/* rb_forward, then rb_sample_logits over the step's logits on the device (host
 * pointers; params, prev_* and uniforms per row as rb_sample_logits; logits: NULL,
 * or [n_rows][vocab] for the raw logits). Returns n_rows. */
int32_t rb_forward_sample(rb_ctx* ctx, int32_t model, uint32_t n_rows, const uint32_t* tenants, const uint32_t* tokens,
                          const uint32_t* positions, const rb_sampling* params, const uint32_t* prev_tokens,
                          const uint32_t* prev_offsets, const float* uniforms, uint32_t* out_tokens, float* logits);

/* ---- continuous batching ----
 * rb_batcher is ContinuousBatcher / BatchedRequest
 * (crates/realm-runtime/src/batching.rs:10-210) as host code, with the same rules:
 *  - rb_batcher_add_request appends to a FIFO queue; it fails with RB_ERR_INVALID
 *    ("Batch queue is full") when the queue already holds max_batch_size requests
 *    (batching.rs:95-104).
 *  - rb_batcher_get_batch REMOVES from the queue and returns, in FIFO order, up to
 *    max_batch_size requests that are not complete. Requests reached on the way
 *    that are complete, whose prompt + generated length is >= max_seq_len, or
 *    whose generated count is >= max_tokens, are dropped (batching.rs:109-139).
 *  - rb_batcher_update_request appends one generated token and marks the request
 *    complete once it has max_tokens (batching.rs:142-158).
 *  - update / remove of an id not in the queue fail with RB_ERR_NOT_FOUND
 *    ("Request <id> not found").
 *  - rb_batcher_stats: queued requests, those not complete, and the integer mean
 *    of their prompt + generated lengths (batching.rs:186-210).
 * One mutex guards each batcher, so its calls are safe from any thread. */
typedef struct rb_batcher rb_batcher;
typedef struct rb_request_list rb_request_list; /* the Vec<BatchedRequest> get_batch returns */
typedef struct rb_batched_request {
  uint64_t request_id;
  const uint32_t* prompt_tokens;
  uint32_t n_prompt;
  uint32_t n_generated;
  const uint32_t* generated_tokens;
  const char* prompt_text; /* NULL when the request has none */
  uint32_t max_tokens;
  uint32_t is_complete;
} rb_batched_request;
typedef struct rb_batch_stats {
  uint64_t total_requests, active_requests, average_sequence_length;
} rb_batch_stats;

int32_t rb_batcher_create(uint32_t max_batch_size, uint32_t max_seq_len, rb_batcher** out);
int32_t rb_batcher_destroy(rb_batcher* b);
/* BatchedRequest::new (prompt_text NULL) / ::with_prompt_text + add_request. */
int32_t rb_batcher_add_request(rb_batcher* b, uint64_t request_id, const uint32_t* prompt_tokens, uint32_t n_prompt,
                               const char* prompt_text, uint32_t max_tokens);
/* Returns the batch length; *out owns the requests (free with rb_request_list_free). */
int32_t rb_batcher_get_batch(rb_batcher* b, rb_request_list** out);
/* A view of request i of a list; its pointers stay valid until the list is freed. */
int32_t rb_request_list_get(const rb_request_list* list, uint32_t i, rb_batched_request* out);
int32_t rb_request_list_free(rb_request_list* list);
int32_t rb_batcher_update_request(rb_batcher* b, uint64_t request_id, uint32_t new_token);
int32_t rb_batcher_remove_request(rb_batcher* b, uint64_t request_id);
int32_t rb_batcher_active_count(rb_batcher* b);
int32_t rb_batcher_stats(rb_batcher* b, rb_batch_stats* out);

/* ---- decode scheduler ----
 * Continuous batching on one model, the step loop behind the reference's
 * batched dispatch (crates/realm-server/src/dispatcher.rs:560-700 with
 * batching.rs's admission rules). It has no single reference counterpart.
 * Requests wait in a FIFO queue and are admitted between steps while fewer than
 * max_batch_size are live and the KV pool can hold their worst case
 * (prompt + max_tokens - 1 tokens, capped at max_seq_len - 1). Admission is
 * strictly FIFO. Each admitted request gets a tenant id of its own in
 * [tenant_base, tenant_base + max_batch_size) and a fresh KV cache.
 * One step is one rb_forward over:
 *  - one row for every live request past its prompt (its last token), then
 *  - consecutive prompt rows of requests still prefilling, in admission order,
 *    at most prefill_chunk per request (0: no limit), while rows remain
 *    (rb_ctx_max_rows per step).
 * The greedy argmax of a request's last prompt row is its first generated
 * token, and of every decode row the next one. A request finishes, and its KV
 * pages go back to the pool before the next step, when:
 *  - it holds max_tokens generated tokens (RB_FINISH_MAX_TOKENS);
 *  - it generated eos_token (RB_FINISH_EOS);
 *  - prompt + generated reaches max_seq_len (RB_FINISH_LENGTH).
 * A prompt of max_seq_len tokens or more finishes at submission with none
 * generated (RB_FINISH_LENGTH), as get_batch drops it; max_tokens 0 finishes
 * with RB_FINISH_MAX_TOKENS.
 * rb_scheduler_submit, _cancel, _result, _release and _stats may be called from
 * any thread; rb_scheduler_step from one thread at a time (it uses the context). */
#define RB_NO_EOS 0xffffffffu
#define RB_FINISH_NONE 0
#define RB_FINISH_MAX_TOKENS 1
#define RB_FINISH_EOS 2
#define RB_FINISH_LENGTH 3
#define RB_FINISH_CANCELLED 4

typedef struct rb_scheduler rb_scheduler;
typedef struct rb_scheduler_config {
  uint32_t max_batch_size; /* live requests (<= rb_ctx_max_rows and <= the model's max_tenants) */
  uint32_t max_seq_len;    /* prompt + generated tokens per request (0: the model's max_seq) */
  uint32_t prefill_chunk;  /* prompt rows a request feeds per step (0: as many as fit) */
  uint32_t eos_token;      /* RB_NO_EOS: none */
  uint32_t tenant_base;    /* first tenant id the scheduler uses */
} rb_scheduler_config;
typedef struct rb_step_event {
  uint64_t request_id;
  uint32_t token;  /* generated token */
  uint32_t index;  /* its index among the request's generated tokens */
  int32_t finish;  /* RB_FINISH_NONE while the request continues */
} rb_step_event;
typedef struct rb_sched_stats {
  uint64_t steps, rows, prefill_rows, decode_rows, tokens_generated;
  uint32_t queued, live, finished;
  float device_ms; /* sum of rb_last_forward_ms over the steps */
} rb_sched_stats;

int32_t rb_scheduler_create(rb_ctx* ctx, int32_t model, const rb_scheduler_config* cfg, rb_scheduler** out);
/* Destroys the scheduler and the KV caches of its live requests. */
int32_t rb_scheduler_destroy(rb_scheduler* s);
/* Queues a request. RB_ERR_INVALID: duplicate id, empty prompt, token >= vocab;
 * RB_ERR_KV_POOL_EXHAUSTED: its worst case exceeds the whole pool. */
int32_t rb_scheduler_submit(rb_scheduler* s, uint64_t request_id, const uint32_t* prompt, uint32_t n_prompt,
                            uint32_t max_tokens);
/* Admits, runs one step and retires. events gets one entry per token generated
 * (cap >= max_batch_size); logits (NULL, or [cap][vocab] host floats) the
 * logits row each event's token came from. Returns the event count; 0 when
 * nothing was live or queued. On an error nothing of the step is kept. */
int32_t rb_scheduler_step(rb_scheduler* s, rb_step_event* events, uint32_t cap, float* logits);
/* The generated tokens of a live or finished request: writes min(n, cap) to
 * tokens (may be NULL) and its RB_FINISH_* state to *finish (may be NULL);
 * returns n. Queued requests return 0 with RB_FINISH_NONE. */
int32_t rb_scheduler_result(rb_scheduler* s, uint64_t request_id, uint32_t* tokens, uint32_t cap, int32_t* finish);
/* rb_scheduler_submit with a sampling strategy (LogitsProcessor::with_params,
 * crates/realm-models/src/sampling.rs:63-100) for this request: its tokens come from
 * rb_forward_sample with uniform draws rb_sampling_uniform(seed, i) for its i-th
 * generated token and its own generated tokens as the repetition-penalty history.
 * params NULL: greedy, as rb_scheduler_submit. */
int32_t rb_scheduler_submit_sampled(rb_scheduler* s, uint64_t request_id, const uint32_t* prompt, uint32_t n_prompt,
                                    uint32_t max_tokens, const rb_sampling* params, uint64_t seed);
/* Ends a queued or live request (RB_FINISH_CANCELLED; its KV pages are freed). */
int32_t rb_scheduler_cancel(rb_scheduler* s, uint64_t request_id);
/* Forgets a finished request. */
int32_t rb_scheduler_release(rb_scheduler* s, uint64_t request_id);
int32_t rb_scheduler_stats(rb_scheduler* s, rb_sched_stats* out);

/* Timing hook for benchmarks: device time (ms) of the last rb_forward. */
float rb_last_forward_ms(rb_ctx* ctx);
/* Kernel launches issued by the last rb_forward (graph replays count their kernels). */
int32_t rb_last_forward_launches(rb_ctx* ctx);

#ifdef __cplusplus
}
#endif
#endif /* REALM_B200_H */
