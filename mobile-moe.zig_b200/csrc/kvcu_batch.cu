// kvcu_batch.cu — continuous batching over one shared pool (host code).
//
// Restates BatchScheduler (src/batch_queue.zig:75-232) with one change of
// structure: every request is a sequence of one kvcache (one shared block
// pool on the device) instead of owning a KVCache of its own
// (src/batch_queue.zig:33-52). The scheduler keeps, per request, its id (from
// 1, :83-90), status (waiting / running / paused / completed, :19-24),
// priority (low < normal < high < critical, :26-31, :185-192), its generated
// tokens and max_tokens (isFinished, :66-72) and its pool sequence. A reaped
// request's pool sequence is reset (its blocks go back to the pool's free
// list) and handed to the next request.
//
// Batch order (collectBatchIndices, :134-183): running or waiting requests
// that are not finished, by priority, then by arrival. The reference orders
// equal priorities by a millisecond timestamp; an arrival counter gives the
// same FIFO order without ties.
#include <algorithm>
#include <new>
#include <vector>

#include "kvcu_internal.h"

namespace {

struct Request {
  uint64_t id;
  int status;
  int priority;
  uint32_t max_tokens;
  uint32_t seq;        // the request's sequence in the pool
  uint64_t arrival;    // FIFO order within a priority
  std::vector<uint32_t> tokens;
  bool finished(uint32_t eos) const {
    if (status == KVCU_SEQ_COMPLETED) return true;
    if (tokens.size() >= max_tokens) return true;
    return !tokens.empty() && tokens.back() == eos;
  }
};

}  // namespace

struct kvcu_batch {
  kvcache* cache;
  uint32_t max_batch;
  uint64_t next_id = 1;
  uint64_t arrivals = 0;
  std::vector<Request> reqs;
  std::vector<uint32_t> free_seqs;  // pool sequences of reaped requests
  Request* find(uint64_t id) {
    for (auto& r : reqs)
      if (r.id == id) return &r;
    return nullptr;
  }
};

extern "C" {

kvcu_batch* kvcu_batch_create(kvcache* c, uint32_t max_batch_size) {
  if (!c || max_batch_size == 0) return nullptr;
  kvcu_batch* b = new (std::nothrow) kvcu_batch();
  if (!b) return nullptr;
  b->cache = c;
  b->max_batch = max_batch_size;
  return b;
}

int kvcu_batch_destroy(kvcu_batch* b) {
  delete b;
  return KVCU_OK;
}

int64_t kvcu_batch_add_request(kvcu_batch* b, uint32_t max_tokens, int priority) {
  if (!b || priority < KVCU_PRIORITY_LOW || priority > KVCU_PRIORITY_CRITICAL) return KVCU_ERR_INVALID_ARG;
  // a reaped request's (empty) pool sequence, else a new one; sequence 0 stays
  // the cache's single-sequence default and is never handed out
  uint32_t seq;
  if (!b->free_seqs.empty()) {
    seq = b->free_seqs.back();
    b->free_seqs.pop_back();
  } else {
    const int64_t s = kvcache_seq_create(b->cache);
    if (s < 0) return s;
    seq = (uint32_t)s;
  }
  Request r;
  r.id = b->next_id++;
  r.status = KVCU_SEQ_WAITING;
  r.priority = priority;
  r.max_tokens = max_tokens;
  r.seq = seq;
  r.arrival = b->arrivals++;
  b->reqs.push_back(std::move(r));
  return (int64_t)b->reqs.back().id;
}

uint32_t kvcu_batch_collect(kvcu_batch* b, uint32_t eos_token, uint64_t* ids_out, uint32_t* seqs_out,
                            uint32_t cap) {
  if (!b) return 0;
  std::vector<const Request*> cand;
  for (const auto& r : b->reqs)
    if ((r.status == KVCU_SEQ_RUNNING || r.status == KVCU_SEQ_WAITING) && !r.finished(eos_token))
      cand.push_back(&r);
  std::stable_sort(cand.begin(), cand.end(), [](const Request* x, const Request* y) {
    if (x->priority != y->priority) return x->priority > y->priority;
    return x->arrival < y->arrival;
  });
  const uint32_t n = (uint32_t)std::min<size_t>({cand.size(), (size_t)b->max_batch, (size_t)cap});
  for (uint32_t i = 0; i < n; ++i) {
    if (ids_out) ids_out[i] = cand[i]->id;
    if (seqs_out) seqs_out[i] = cand[i]->seq;
  }
  return n;
}

int kvcu_batch_mark_running(kvcu_batch* b, const uint64_t* ids, uint32_t n) {
  if (!b || (n && !ids)) return KVCU_ERR_INVALID_ARG;
  for (uint32_t i = 0; i < n; ++i)
    if (Request* r = b->find(ids[i]))
      if (r->status == KVCU_SEQ_WAITING) r->status = KVCU_SEQ_RUNNING;
  return KVCU_OK;
}

int kvcu_batch_set_status(kvcu_batch* b, uint64_t id, int status) {
  if (!b || status < KVCU_SEQ_WAITING || status > KVCU_SEQ_COMPLETED) return KVCU_ERR_INVALID_ARG;
  Request* r = b->find(id);
  if (!r) return KVCU_ERR_INVALID_ARG;
  r->status = status;
  return KVCU_OK;
}

int kvcu_batch_mark_completed(kvcu_batch* b, uint64_t id) {
  return kvcu_batch_set_status(b, id, KVCU_SEQ_COMPLETED);
}

int kvcu_batch_push_token(kvcu_batch* b, uint64_t id, uint32_t token) {
  Request* r = b ? b->find(id) : nullptr;
  if (!r) return KVCU_ERR_INVALID_ARG;
  r->tokens.push_back(token);
  return KVCU_OK;
}

int kvcu_batch_is_finished(kvcu_batch* b, uint64_t id, uint32_t eos_token) {
  Request* r = b ? b->find(id) : nullptr;
  if (!r) return KVCU_ERR_INVALID_ARG;
  return r->finished(eos_token) ? 1 : 0;
}

uint32_t kvcu_batch_reap_completed(kvcu_batch* b) {
  if (!b) return 0;
  uint32_t reaped = 0;
  for (size_t i = 0; i < b->reqs.size();) {
    if (b->reqs[i].status == KVCU_SEQ_COMPLETED) {
      kvcache_seq_reset(b->cache, b->reqs[i].seq);
      b->free_seqs.push_back(b->reqs[i].seq);
      b->reqs.erase(b->reqs.begin() + (ptrdiff_t)i);  // keeps the order of the rest (orderedRemove)
      ++reaped;
    } else {
      ++i;
    }
  }
  return reaped;
}

uint32_t kvcu_batch_reclaim_blocks(kvcu_batch* b) {
  if (!b) return 0;
  uint32_t reclaimed = 0;
  for (const auto& r : b->reqs) {
    if (r.status != KVCU_SEQ_PAUSED && r.status != KVCU_SEQ_COMPLETED) continue;
    const uint32_t before = kvcache_num_free_blocks(b->cache);
    kvcache_seq_reset(b->cache, r.seq);
    reclaimed += kvcache_num_free_blocks(b->cache) - before;
  }
  return reclaimed;
}

uint32_t kvcu_batch_running_count(const kvcu_batch* b) {
  if (!b) return 0;
  uint32_t n = 0;
  for (const auto& r : b->reqs) n += r.status == KVCU_SEQ_RUNNING;
  return n;
}

uint32_t kvcu_batch_size(const kvcu_batch* b) { return b ? (uint32_t)b->reqs.size() : 0; }

int64_t kvcu_batch_seq(const kvcu_batch* b, uint64_t id) {
  if (!b) return KVCU_ERR_INVALID_ARG;
  for (const auto& r : b->reqs)
    if (r.id == id) return r.seq;
  return KVCU_ERR_INVALID_ARG;
}

int kvcu_batch_status(const kvcu_batch* b, uint64_t id) {
  if (!b) return KVCU_ERR_INVALID_ARG;
  for (const auto& r : b->reqs)
    if (r.id == id) return r.status;
  return KVCU_ERR_INVALID_ARG;
}

}  // extern "C"
