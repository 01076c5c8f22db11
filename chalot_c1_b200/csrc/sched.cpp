// sched.cpp — continuous batching over chalot_forward_batch (the C ABI in
// include/chalot_b200.h, chalot_sched_*).
//
// The reference generates one prompt at a time (Engine::generate,
// src/model/engine.rs:497-548: prefill the prompt token by token, then feed
// back each greedy token). Here any number of such generations share the
// engine's batch slots: every step gives each decoding sequence one row (its
// last token at its next position) and the prefilling sequences chunks of
// their prompt (consecutive positions of one slot in one forward, which
// chalot_forward_batch runs as consecutive forwards would), so a sequence's
// tokens are exactly those of chalot_generate on its prompt alone. A sequence
// leaves after max_new tokens or a stop token (not returned), and its slot
// and K/V pages go back to the pool for the next waiting sequence.
//
// Admission with a paged K/V reserve counts pages: a sequence is admitted
// only if the pool's pages, less the most every running sequence may still
// take, cover its prompt + max_new - 1 positions, so a forward never runs out
// of pages.
#include <algorithm>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "capi_internal.h"

namespace {

struct Seq {
  uint64_t id = 0;
  std::vector<uint32_t> prompt;
  uint32_t max_new = 0;
  std::vector<uint32_t> stop;
  std::vector<uint32_t> out;
  int slot = -1;
  uint32_t fed = 0;       // prompt tokens already run
  uint32_t next = 0;      // the token to feed while decoding
  uint32_t pages = 0;     // pages its whole generation may take (paged reserve)
  bool done = false;
};

}  // namespace

struct chalot_sched {
  chalot_engine* e = nullptr;
  uint32_t max_rows = 0, n_slots = 0, max_seq = 0;
  uint32_t page_tokens = 0, total_pages = 0, committed = 0;  // pages the running sequences may take
  uint64_t next_id = 1;
  std::deque<Seq*> waiting;
  std::vector<Seq*> slot_seq;            // running sequence of each slot
  std::map<uint64_t, Seq*> all;          // every sequence not yet forgotten
  std::vector<uint32_t> r_slot, r_tok, r_pos, r_out;

  ~chalot_sched() {
    for (auto& kv : all) delete kv.second;
  }
};

using namespace chalot;

extern "C" {

__attribute__((visibility("default"))) int chalot_sched_create(chalot_engine* e, uint32_t max_rows,
                                                              chalot_sched** out) {
  if (!e || !out) return set_error(CHALOT_ERR_ARG, "sched_create: null argument");
  chalot_model_config c{};
  if (int rc = chalot_get_config(e, &c)) return rc;
  uint32_t nfree = 0, ntotal = 0, pt = 0;
  if (int rc = chalot_batch_kv_pages(e, &nfree, &ntotal, &pt)) return rc;
  uint32_t slots = 0;
  if (int rc = chalot_batch_capacity(e, &slots)) return rc;
  if (!slots) return set_error(CHALOT_ERR_STATE, "sched_create: reserve the batch first (chalot_batch_reserve)");
  if (max_rows < 1 || max_rows > slots) return set_error(CHALOT_ERR_ARG, "sched_create: max_rows must be in [1, max_seqs]");
  if (pt && nfree != ntotal) return set_error(CHALOT_ERR_STATE, "sched_create: the page pool is already in use");
  chalot_sched* s = new (std::nothrow) chalot_sched;
  if (!s) return set_error(CHALOT_ERR_OOM, "sched_create: out of host memory");
  s->e = e;
  s->max_rows = max_rows;
  s->n_slots = slots;
  s->max_seq = c.max_seq_len;
  s->page_tokens = pt;
  s->total_pages = ntotal;
  try {
    s->slot_seq.assign(slots, nullptr);
  } catch (const std::bad_alloc&) {
    delete s;
    return set_error(CHALOT_ERR_OOM, "sched_create: out of host memory");
  }
  *out = s;
  return CHALOT_OK;
}

__attribute__((visibility("default"))) void chalot_sched_free(chalot_sched* s) {
  if (!s) return;
  for (uint32_t i = 0; i < s->n_slots; ++i)
    if (s->slot_seq[i]) chalot_batch_release(s->e, i);
  delete s;
}

__attribute__((visibility("default"))) int chalot_sched_submit(chalot_sched* s, const uint32_t* prompt, size_t n,
                                                              uint32_t max_new, const uint32_t* stop,
                                                              size_t n_stop, uint64_t* id) {
  if (!s || !prompt || !id || (n_stop && !stop)) return set_error(CHALOT_ERR_ARG, "sched_submit: null argument");
  if (n < 1 || max_new < 1) return set_error(CHALOT_ERR_ARG, "sched_submit: need a prompt and max_new >= 1");
  if (n + max_new - 1 > s->max_seq)
    return set_error(CHALOT_ERR_ARG, "sched_submit: prompt + max_new - 1 exceeds max_seq_len");
  uint32_t pages = 0;
  if (s->page_tokens) {
    pages = (uint32_t)((n + max_new - 1 + s->page_tokens - 1) / s->page_tokens);
    if (pages > s->total_pages)
      return set_error(CHALOT_ERR_ARG, "sched_submit: the generation needs more K/V pages than the pool holds");
  }
  try {
    auto q = std::make_unique<Seq>();
    q->id = s->next_id;
    q->prompt.assign(prompt, prompt + n);
    q->max_new = max_new;
    q->stop.assign(stop, stop + n_stop);
    q->pages = pages;
    s->all[q->id] = q.get();
    s->waiting.push_back(q.get());
    *id = q->id;
    ++s->next_id;
    q.release();
  } catch (const std::bad_alloc&) {
    s->all.erase(s->next_id);
    return set_error(CHALOT_ERR_OOM, "sched_submit: out of host memory");
  }
  return CHALOT_OK;
}

// A generated token: kept unless it is a stop token; the sequence ends at a
// stop token or its max_new-th token.
static void take_token(Seq* q, uint32_t tok) {
  if (std::find(q->stop.begin(), q->stop.end(), tok) != q->stop.end()) {
    q->done = true;
    return;
  }
  q->out.push_back(tok);
  q->next = tok;
  if (q->out.size() >= q->max_new) q->done = true;
}

static int sched_step(chalot_sched* s, uint32_t* n_running, uint32_t* n_waiting, uint32_t* n_rows);

__attribute__((visibility("default"))) int chalot_sched_step(chalot_sched* s, uint32_t* n_running,
                                                            uint32_t* n_waiting, uint32_t* n_rows) {
  if (!s) return set_error(CHALOT_ERR_ARG, "sched_step: null scheduler");
  try {
    return sched_step(s, n_running, n_waiting, n_rows);
  } catch (const std::bad_alloc&) {
    return set_error(CHALOT_ERR_OOM, "sched_step: out of host memory");
  }
}

static int sched_step(chalot_sched* s, uint32_t* n_running, uint32_t* n_waiting, uint32_t* n_rows) {
  // admission: free slots, and pages for the whole generation
  for (uint32_t i = 0; i < s->n_slots && !s->waiting.empty(); ++i) {
    if (s->slot_seq[i]) continue;
    Seq* q = s->waiting.front();
    if (s->page_tokens && s->committed + q->pages > s->total_pages) break;  // first come, first served
    s->waiting.pop_front();
    q->slot = (int)i;
    s->slot_seq[i] = q;
    s->committed += q->pages;
  }
  // rows: one per decoding sequence, then prompt chunks in slot order
  s->r_slot.clear();
  s->r_tok.clear();
  s->r_pos.clear();
  struct Span {
    Seq* q;
    size_t first, count;
  };
  std::vector<Span> spans;
  for (uint32_t i = 0; i < s->n_slots && s->r_slot.size() < s->max_rows; ++i) {
    Seq* q = s->slot_seq[i];
    if (!q || q->fed < q->prompt.size()) continue;
    spans.push_back({q, s->r_slot.size(), 1});
    s->r_slot.push_back(i);
    s->r_tok.push_back(q->next);
    s->r_pos.push_back((uint32_t)(q->prompt.size() + q->out.size() - 1));
  }
  for (uint32_t i = 0; i < s->n_slots && s->r_slot.size() < s->max_rows; ++i) {
    Seq* q = s->slot_seq[i];
    if (!q || q->fed >= q->prompt.size()) continue;
    const size_t take = std::min<size_t>(q->prompt.size() - q->fed, s->max_rows - s->r_slot.size());
    spans.push_back({q, s->r_slot.size(), take});
    for (size_t k = 0; k < take; ++k) {
      s->r_slot.push_back(i);
      s->r_tok.push_back(q->prompt[q->fed + k]);
      s->r_pos.push_back(q->fed + (uint32_t)k);
    }
  }
  const uint32_t rows = (uint32_t)s->r_slot.size();
  if (rows) {
    s->r_out.assign(rows, 0);
    if (int rc = chalot_forward_batch(s->e, s->r_slot.data(), s->r_tok.data(), s->r_pos.data(), rows,
                                      s->r_out.data()))
      return rc;
    for (const Span& sp : spans) {
      Seq* q = sp.q;
      if (q->fed < q->prompt.size()) {  // a prompt chunk: the token after the prompt comes from its last row
        q->fed += (uint32_t)sp.count;
        if (q->fed == q->prompt.size()) take_token(q, s->r_out[sp.first + sp.count - 1]);
      } else {
        take_token(q, s->r_out[sp.first]);
      }
      if (q->done) {
        chalot_batch_release(s->e, (uint32_t)q->slot);
        s->slot_seq[q->slot] = nullptr;
        s->committed -= q->pages;
        q->slot = -1;
      }
    }
  }
  uint32_t running = 0;
  for (Seq* q : s->slot_seq) running += q != nullptr;
  if (n_running) *n_running = running;
  if (n_waiting) *n_waiting = (uint32_t)s->waiting.size();
  if (n_rows) *n_rows = rows;
  return CHALOT_OK;
}

__attribute__((visibility("default"))) int chalot_sched_poll(chalot_sched* s, uint64_t id, uint32_t* out,
                                                            size_t cap, size_t* n_out, int* done) {
  if (!s) return set_error(CHALOT_ERR_ARG, "sched_poll: null scheduler");
  auto it = s->all.find(id);
  if (it == s->all.end()) return set_error(CHALOT_ERR_ARG, "sched_poll: unknown sequence id");
  Seq* q = it->second;
  const size_t n = q->out.size();
  if (out && cap) std::memcpy(out, q->out.data(), std::min(cap, n) * sizeof(uint32_t));
  if (n_out) *n_out = n;
  if (done) *done = q->done ? 1 : 0;
  if (q->done && cap >= n) {  // everything handed over: forget it
    s->all.erase(it);
    delete q;
  }
  return CHALOT_OK;
}

}  // extern "C"
