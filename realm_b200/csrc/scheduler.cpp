// Host runtime for request batching: the reference's ContinuousBatcher
// (crates/realm-runtime/src/batching.rs) and a continuous-batching decode
// scheduler that feeds rb_forward with the live requests of one model.
//
// Host code only, written against the public C ABI, so it runs without a GPU
// wherever it does not call into a model (the batcher never does).
#include <algorithm>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/realm_b200.h"

namespace rb {
int fail(int code, const char* fmt, ...);
}
using rb::fail;

namespace {

// BatchedRequest (batching.rs:10-73).
struct Request {
  uint64_t id = 0;
  std::vector<uint32_t> prompt;
  bool has_text = false;
  std::string text;
  std::vector<uint32_t> generated;
  uint32_t max_tokens = 0;
  bool complete = false;

  size_t seq_len() const { return prompt.size() + generated.size(); }
};

void fill_view(const Request& r, rb_batched_request* v) {
  v->request_id = r.id;
  v->prompt_tokens = r.prompt.data();
  v->n_prompt = (uint32_t)r.prompt.size();
  v->n_generated = (uint32_t)r.generated.size();
  v->generated_tokens = r.generated.data();
  v->prompt_text = r.has_text ? r.text.c_str() : nullptr;
  v->max_tokens = r.max_tokens;
  v->is_complete = r.complete ? 1u : 0u;
}

}  // namespace

struct rb_batcher {
  std::mutex mu;
  std::deque<Request> q;
  size_t max_batch = 0, max_seq = 0;
};

struct rb_request_list {
  std::vector<Request> items;
};

extern "C" {

int32_t rb_batcher_create(uint32_t max_batch_size, uint32_t max_seq_len, rb_batcher** out) {
  if (!out) return fail(RB_ERR_INVALID, "null output");
  auto* b = new rb_batcher;
  b->max_batch = max_batch_size;
  b->max_seq = max_seq_len;
  *out = b;
  return RB_OK;
}

int32_t rb_batcher_destroy(rb_batcher* b) {
  if (!b) return fail(RB_ERR_BAD_HANDLE, "null batcher");
  delete b;
  return RB_OK;
}

int32_t rb_batcher_add_request(rb_batcher* b, uint64_t request_id, const uint32_t* prompt_tokens, uint32_t n_prompt,
                               const char* prompt_text, uint32_t max_tokens) {
  if (!b) return fail(RB_ERR_BAD_HANDLE, "null batcher");
  if (n_prompt && !prompt_tokens) return fail(RB_ERR_INVALID, "null prompt");
  Request r;
  r.id = request_id;
  r.prompt.assign(prompt_tokens, prompt_tokens + n_prompt);
  if (prompt_text) {
    r.has_text = true;
    r.text = prompt_text;
  }
  r.max_tokens = max_tokens;
  std::lock_guard<std::mutex> g(b->mu);
  if (b->q.size() >= b->max_batch) return fail(RB_ERR_INVALID, "Batch queue is full");
  b->q.push_back(std::move(r));
  return RB_OK;
}

int32_t rb_batcher_get_batch(rb_batcher* b, rb_request_list** out) {
  if (!b) return fail(RB_ERR_BAD_HANDLE, "null batcher");
  if (!out) return fail(RB_ERR_INVALID, "null output");
  auto list = std::make_unique<rb_request_list>();
  {
    std::lock_guard<std::mutex> g(b->mu);
    // Front to back: drop what cannot run, take the rest until the batch is
    // full; whatever was not reached stays queued in order.
    while (!b->q.empty() && list->items.size() < b->max_batch) {
      Request r = std::move(b->q.front());
      b->q.pop_front();
      if (r.complete || r.seq_len() >= b->max_seq || r.generated.size() >= r.max_tokens) continue;
      list->items.push_back(std::move(r));
    }
  }
  const int32_t n = (int32_t)list->items.size();
  *out = list.release();
  return n;
}

int32_t rb_request_list_get(const rb_request_list* l, uint32_t i, rb_batched_request* out) {
  if (!l) return fail(RB_ERR_BAD_HANDLE, "null request list");
  if (!out) return fail(RB_ERR_INVALID, "null output");
  if (i >= l->items.size()) return fail(RB_ERR_OUT_OF_BOUNDS, "request %u of %zu", i, l->items.size());
  fill_view(l->items[i], out);
  return RB_OK;
}

int32_t rb_request_list_free(rb_request_list* l) {
  delete l;
  return RB_OK;
}

int32_t rb_batcher_update_request(rb_batcher* b, uint64_t request_id, uint32_t new_token) {
  if (!b) return fail(RB_ERR_BAD_HANDLE, "null batcher");
  std::lock_guard<std::mutex> g(b->mu);
  for (Request& r : b->q) {
    if (r.id != request_id) continue;
    r.generated.push_back(new_token);
    if (r.generated.size() >= r.max_tokens) r.complete = true;
    return RB_OK;
  }
  return fail(RB_ERR_NOT_FOUND, "Request %llu not found", (unsigned long long)request_id);
}

int32_t rb_batcher_remove_request(rb_batcher* b, uint64_t request_id) {
  if (!b) return fail(RB_ERR_BAD_HANDLE, "null batcher");
  std::lock_guard<std::mutex> g(b->mu);
  const size_t before = b->q.size();
  b->q.erase(std::remove_if(b->q.begin(), b->q.end(), [&](const Request& r) { return r.id == request_id; }),
             b->q.end());
  if (b->q.size() == before) return fail(RB_ERR_NOT_FOUND, "Request %llu not found", (unsigned long long)request_id);
  return RB_OK;
}

int32_t rb_batcher_active_count(rb_batcher* b) {
  if (!b) return fail(RB_ERR_BAD_HANDLE, "null batcher");
  std::lock_guard<std::mutex> g(b->mu);
  return (int32_t)std::count_if(b->q.begin(), b->q.end(), [](const Request& r) { return !r.complete; });
}

int32_t rb_batcher_stats(rb_batcher* b, rb_batch_stats* out) {
  if (!b) return fail(RB_ERR_BAD_HANDLE, "null batcher");
  if (!out) return fail(RB_ERR_INVALID, "null output");
  std::lock_guard<std::mutex> g(b->mu);
  out->total_requests = b->q.size();
  out->active_requests = 0;
  uint64_t sum = 0;
  for (const Request& r : b->q) {
    out->active_requests += r.complete ? 0 : 1;
    sum += r.seq_len();
  }
  out->average_sequence_length = b->q.empty() ? 0 : sum / b->q.size();
  return RB_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// decode scheduler
// ---------------------------------------------------------------------------
namespace {

constexpr uint32_t kPageTokens = 16;  // KV page size of the pool

struct Seq {
  uint64_t id = 0;
  std::vector<uint32_t> prompt, generated;
  uint32_t max_tokens = 0;
  int32_t finish = RB_FINISH_NONE;
  uint32_t tenant = 0;
  uint32_t cached = 0;    // tokens in the KV cache
  uint32_t reserve = 0;   // KV pages held back for the worst case
  bool cancel = false;    // cancelled while live: retired by the next step
  bool sampled = false;   // false: greedy argmax
  rb_sampling params{};
  uint64_t seed = 0;
};

uint32_t pages_for(uint32_t tokens) { return (tokens + kPageTokens - 1) / kPageTokens; }

}  // namespace

struct rb_scheduler {
  rb_ctx* ctx = nullptr;
  int32_t model = -1, pool = -1;
  rb_scheduler_config cfg{};
  uint32_t vocab = 0, max_rows = 0, total_pages = 0;

  std::mutex mu;  // guards everything below
  std::deque<std::unique_ptr<Seq>> queued;
  std::vector<std::unique_ptr<Seq>> live;  // admission order
  std::map<uint64_t, std::unique_ptr<Seq>> finished;
  std::vector<uint32_t> free_tenants;      // popped from the back
  rb_sched_stats stats{};

  std::vector<float> logits;               // [max_rows][vocab], on first use

  bool known(uint64_t id) const {
    if (finished.count(id)) return true;
    for (auto& s : queued)
      if (s->id == id) return true;
    for (auto& s : live)
      if (s->id == id) return true;
    return false;
  }
  // Worst-case cache length of a request: its last generated token is never fed.
  uint32_t worst_tokens(const Seq& s) const {
    const uint64_t w = (uint64_t)s.prompt.size() + (s.max_tokens ? s.max_tokens - 1 : 0);
    return (uint32_t)std::min<uint64_t>(w, cfg.max_seq_len - 1);
  }
};

namespace {

// Moves a live sequence to the finished map and gives its tenant back.
// Called with the mutex held, from the stepping thread.
int retire(rb_scheduler* s, size_t i, int32_t finish) {
  std::unique_ptr<Seq> q = std::move(s->live[i]);
  s->live.erase(s->live.begin() + (long)i);
  const int rc = rb_kv_destroy(s->ctx, s->pool, q->tenant);
  s->free_tenants.push_back(q->tenant);
  if (q->finish == RB_FINISH_NONE) q->finish = finish;
  s->finished[q->id] = std::move(q);
  return rc < 0 ? rc : RB_OK;
}

}  // namespace

extern "C" {

int32_t rb_scheduler_create(rb_ctx* ctx, int32_t model, const rb_scheduler_config* cfg, rb_scheduler** out) {
  if (!ctx || !cfg || !out) return fail(RB_ERR_BAD_HANDLE, "null argument");
  rb_model_config mc;
  if (int rc = rb_model_get_config(ctx, model, &mc)) return rc;
  const int32_t max_rows = rb_ctx_max_rows(ctx);
  if (max_rows < 0) return max_rows;
  const int32_t pool = rb_model_kv_pool(ctx, model);
  if (pool < 0) return pool;
  rb_scheduler_config c = *cfg;
  if (c.max_seq_len == 0) c.max_seq_len = mc.max_seq;
  if (c.max_batch_size == 0 || c.max_batch_size > (uint32_t)max_rows)
    return fail(RB_ERR_INVALID, "max_batch_size %u not in [1, %d]", c.max_batch_size, max_rows);
  if ((uint64_t)c.tenant_base + c.max_batch_size > mc.max_tenants)
    return fail(RB_ERR_INVALID, "tenants [%u, %u) beyond the model's %u", c.tenant_base,
                c.tenant_base + c.max_batch_size, mc.max_tenants);
  if (c.max_seq_len < 2 || c.max_seq_len > mc.max_seq)
    return fail(RB_ERR_INVALID, "max_seq_len %u not in [2, %u]", c.max_seq_len, mc.max_seq);
  auto s = std::make_unique<rb_scheduler>();
  s->ctx = ctx;
  s->model = model;
  s->pool = pool;
  s->cfg = c;
  s->vocab = mc.vocab;
  s->max_rows = (uint32_t)max_rows;
  s->total_pages = mc.kv_pages;
  for (uint32_t t = c.max_batch_size; t-- > 0;) s->free_tenants.push_back(c.tenant_base + t);
  *out = s.release();
  return RB_OK;
}

int32_t rb_scheduler_destroy(rb_scheduler* s) {
  if (!s) return fail(RB_ERR_BAD_HANDLE, "null scheduler");
  int rc = RB_OK;
  for (auto& q : s->live) {
    const int e = rb_kv_destroy(s->ctx, s->pool, q->tenant);
    if (e < 0 && rc == RB_OK) rc = e;
  }
  delete s;
  return rc;
}

int32_t rb_scheduler_submit(rb_scheduler* s, uint64_t request_id, const uint32_t* prompt, uint32_t n_prompt,
                            uint32_t max_tokens) {
  return rb_scheduler_submit_sampled(s, request_id, prompt, n_prompt, max_tokens, nullptr, 0);
}

int32_t rb_scheduler_submit_sampled(rb_scheduler* s, uint64_t request_id, const uint32_t* prompt, uint32_t n_prompt,
                                    uint32_t max_tokens, const rb_sampling* params, uint64_t seed) {
  if (!s) return fail(RB_ERR_BAD_HANDLE, "null scheduler");
  if (n_prompt == 0 || !prompt) return fail(RB_ERR_INVALID, "request %llu: empty prompt", (unsigned long long)request_id);
  for (uint32_t i = 0; i < n_prompt; ++i)
    if (prompt[i] >= s->vocab) return fail(RB_ERR_INVALID, "token %u >= vocab %u", prompt[i], s->vocab);
  auto q = std::make_unique<Seq>();
  q->id = request_id;
  q->prompt.assign(prompt, prompt + n_prompt);
  q->max_tokens = max_tokens;
  if (params && params->temperature >= 1e-7) {  // with_params: below 1e-7 is argmax
    q->sampled = true;
    q->params = *params;
    q->seed = seed;
  } else if (params && params->repetition_penalty != 1.0f) {
    q->sampled = true;  // greedy, but over penalised logits
    q->params = *params;
    q->seed = seed;
  }
  std::lock_guard<std::mutex> g(s->mu);
  if (s->known(request_id)) return fail(RB_ERR_INVALID, "request %llu already submitted", (unsigned long long)request_id);
  if (n_prompt >= s->cfg.max_seq_len || max_tokens == 0) {
    q->finish = max_tokens == 0 ? RB_FINISH_MAX_TOKENS : RB_FINISH_LENGTH;
    s->finished[request_id] = std::move(q);
    return RB_OK;
  }
  q->reserve = pages_for(s->worst_tokens(*q));
  if (q->reserve > s->total_pages)
    return fail(RB_ERR_KV_POOL_EXHAUSTED, "request %llu needs %u KV pages, the pool has %u",
                (unsigned long long)request_id, q->reserve, s->total_pages);
  s->queued.push_back(std::move(q));
  return RB_OK;
}

int32_t rb_scheduler_step(rb_scheduler* s, rb_step_event* events, uint32_t cap, float* logits_out) {
  if (!s) return fail(RB_ERR_BAD_HANDLE, "null scheduler");
  if (!events || cap < s->cfg.max_batch_size)
    return fail(RB_ERR_INVALID, "events capacity %u < max_batch_size %u", cap, s->cfg.max_batch_size);
  std::vector<uint32_t> tenants, tokens;
  struct Out { Seq* seq; uint32_t row; };
  std::vector<Out> outs;     // rows whose argmax is a generated token
  std::vector<std::pair<Seq*, uint32_t>> fed;  // rows each sequence feeds
  uint32_t n_prefill = 0, n_decode = 0;
  {
    std::lock_guard<std::mutex> g(s->mu);
    // Requests cancelled while live leave first.
    for (size_t i = s->live.size(); i-- > 0;)
      if (s->live[i]->cancel)
        if (int rc = retire(s, i, RB_FINISH_CANCELLED)) return rc;
    // Admission: FIFO while a tenant is free and the pool holds the worst case.
    int64_t free_pages = rb_kv_pool_free_pages(s->ctx, s->pool);
    if (free_pages < 0) return (int32_t)free_pages;
    for (auto& q : s->live) free_pages -= (int64_t)q->reserve - pages_for(q->cached);
    while (!s->queued.empty() && !s->free_tenants.empty() && (int64_t)s->queued.front()->reserve <= free_pages) {
      std::unique_ptr<Seq> q = std::move(s->queued.front());
      s->queued.pop_front();
      q->tenant = s->free_tenants.back();
      if (int rc = rb_kv_create(s->ctx, s->pool, q->tenant)) {
        s->queued.push_front(std::move(q));
        return rc;
      }
      s->free_tenants.pop_back();
      free_pages -= q->reserve;
      s->live.push_back(std::move(q));
    }
    // Rows: decode rows first (one per request past its prompt), then prompt chunks.
    for (auto& q : s->live) {
      if (q->cached < q->prompt.size()) continue;
      tenants.push_back(q->tenant);
      tokens.push_back(q->generated.back());
      outs.push_back({q.get(), (uint32_t)tokens.size() - 1});
      fed.push_back({q.get(), 1});
      ++n_decode;
    }
    for (auto& q : s->live) {
      const uint32_t left = (uint32_t)q->prompt.size() - std::min<uint32_t>(q->cached, (uint32_t)q->prompt.size());
      const uint32_t room = s->max_rows - (uint32_t)tokens.size();
      if (left == 0 || room == 0) continue;
      uint32_t n = std::min(left, room);
      if (s->cfg.prefill_chunk) n = std::min(n, s->cfg.prefill_chunk);
      for (uint32_t i = 0; i < n; ++i) {
        tenants.push_back(q->tenant);
        tokens.push_back(q->prompt[q->cached + i]);
      }
      if (n == left) outs.push_back({q.get(), (uint32_t)tokens.size() - 1});
      fed.push_back({q.get(), n});
      n_prefill += n;
    }
  }
  if (tokens.empty()) return 0;
  // The forward runs without the lock: submit/result/cancel stay responsive.
  const uint32_t n_rows = (uint32_t)tokens.size();
  std::vector<uint32_t> argmax(n_rows);
  float* lg = nullptr;
  if (logits_out) {
    s->logits.resize((size_t)s->max_rows * s->vocab);
    lg = s->logits.data();
  }
  bool any_sampled = false;
  for (const Out& o : outs) any_sampled = any_sampled || o.seq->sampled;
  int32_t rc;
  if (!any_sampled) {
    rc = rb_forward(s->ctx, s->model, n_rows, tenants.data(), tokens.data(), nullptr, lg, argmax.data(), RB_PTR_HOST);
  } else {
    // per-row strategies: rows without a token of their own stay greedy; the
    // sampled requests bring their history and their next uniform draw
    std::vector<rb_sampling> prm(n_rows);
    std::vector<float> uni(n_rows, 0.f);
    std::vector<uint32_t> off(n_rows + 1, 0), prev;
    std::vector<const Seq*> row_seq(n_rows, nullptr);
    for (const Out& o : outs) row_seq[o.row] = o.seq;
    for (uint32_t r = 0; r < n_rows; ++r) {
      prm[r] = rb_sampling{0.0, 1.0, 0u, 1.0f};
      off[r] = (uint32_t)prev.size();
      const Seq* q = row_seq[r];
      if (q && q->sampled) {
        prm[r] = q->params;
        uni[r] = rb_sampling_uniform(q->seed, q->generated.size());
        prev.insert(prev.end(), q->generated.begin(), q->generated.end());
      }
    }
    off[n_rows] = (uint32_t)prev.size();
    if (prev.empty()) prev.push_back(0);
    rc = rb_forward_sample(s->ctx, s->model, n_rows, tenants.data(), tokens.data(), nullptr, prm.data(), prev.data(),
                           off.data(), uni.data(), argmax.data(), lg);
  }
  if (rc < 0) return rc;
  std::lock_guard<std::mutex> g(s->mu);
  for (auto& [q, n] : fed) q->cached += n;
  uint32_t n_ev = 0;
  for (const Out& o : outs) {
    Seq* q = o.seq;
    if (q->cancel) continue;
    const uint32_t tok = argmax[o.row];
    q->generated.push_back(tok);
    if (q->generated.size() >= q->max_tokens) q->finish = RB_FINISH_MAX_TOKENS;
    else if (tok == s->cfg.eos_token) q->finish = RB_FINISH_EOS;
    else if (q->prompt.size() + q->generated.size() >= s->cfg.max_seq_len) q->finish = RB_FINISH_LENGTH;
    events[n_ev] = {q->id, tok, (uint32_t)q->generated.size() - 1, q->finish};
    if (logits_out)
      std::memcpy(logits_out + (size_t)n_ev * s->vocab, lg + (size_t)o.row * s->vocab, (size_t)s->vocab * 4);
    ++n_ev;
  }
  s->stats.steps += 1;
  s->stats.rows += n_rows;
  s->stats.prefill_rows += n_prefill;
  s->stats.decode_rows += n_decode;
  s->stats.tokens_generated += n_ev;
  s->stats.device_ms += rb_last_forward_ms(s->ctx);
  for (size_t i = s->live.size(); i-- > 0;) {
    Seq& q = *s->live[i];
    if (q.finish != RB_FINISH_NONE || q.cancel)
      if (int e = retire(s, i, q.cancel ? RB_FINISH_CANCELLED : q.finish)) return e;
  }
  return (int32_t)n_ev;
}

int32_t rb_scheduler_result(rb_scheduler* s, uint64_t request_id, uint32_t* tokens, uint32_t cap, int32_t* finish) {
  if (!s) return fail(RB_ERR_BAD_HANDLE, "null scheduler");
  std::lock_guard<std::mutex> g(s->mu);
  const Seq* q = nullptr;
  if (auto it = s->finished.find(request_id); it != s->finished.end()) q = it->second.get();
  for (auto& l : s->live)
    if (l->id == request_id) q = l.get();
  if (!q) {
    for (auto& w : s->queued)
      if (w->id == request_id) {
        if (finish) *finish = RB_FINISH_NONE;
        return 0;
      }
    return fail(RB_ERR_NOT_FOUND, "request %llu not found", (unsigned long long)request_id);
  }
  if (tokens) std::copy_n(q->generated.begin(), std::min<size_t>(cap, q->generated.size()), tokens);
  if (finish) *finish = q->finish;
  return (int32_t)q->generated.size();
}

int32_t rb_scheduler_cancel(rb_scheduler* s, uint64_t request_id) {
  if (!s) return fail(RB_ERR_BAD_HANDLE, "null scheduler");
  std::lock_guard<std::mutex> g(s->mu);
  for (auto it = s->queued.begin(); it != s->queued.end(); ++it)
    if ((*it)->id == request_id) {
      (*it)->finish = RB_FINISH_CANCELLED;
      s->finished[request_id] = std::move(*it);
      s->queued.erase(it);
      return RB_OK;
    }
  for (auto& l : s->live)
    if (l->id == request_id) {
      l->cancel = true;  // its KV pages are freed by the next step, on the stepping thread
      return RB_OK;
    }
  if (s->finished.count(request_id)) return RB_OK;
  return fail(RB_ERR_NOT_FOUND, "request %llu not found", (unsigned long long)request_id);
}

int32_t rb_scheduler_release(rb_scheduler* s, uint64_t request_id) {
  if (!s) return fail(RB_ERR_BAD_HANDLE, "null scheduler");
  std::lock_guard<std::mutex> g(s->mu);
  if (!s->finished.erase(request_id))
    return fail(RB_ERR_NOT_FOUND, "request %llu not finished", (unsigned long long)request_id);
  return RB_OK;
}

int32_t rb_scheduler_stats(rb_scheduler* s, rb_sched_stats* out) {
  if (!s) return fail(RB_ERR_BAD_HANDLE, "null scheduler");
  if (!out) return fail(RB_ERR_INVALID, "null output");
  std::lock_guard<std::mutex> g(s->mu);
  *out = s->stats;
  out->queued = (uint32_t)s->queued.size();
  out->live = (uint32_t)s->live.size();
  out->finished = (uint32_t)s->finished.size();
  return RB_OK;
}

}  // extern "C"
