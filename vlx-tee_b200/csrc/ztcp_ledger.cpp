// ztcp_ledger.cpp -- the keyring's per-page nonce and freshness tables in C++ (C ABI: ztcp_ledger.h).
//
// Per session: the burned 96-bit ChaCha20 nonces (sequence nonce, layer_id << 16 | head_group_id),
// the freshness watermark of every KV slot (model_id_hash, layer_id, head_group_id, page_token_hash)
// and the largest sequence nonce seen.  Batch operations validate every page against the tables and a
// batch-local overlay first and apply nothing unless all pages pass, which is the reference keyring's
// all-or-nothing behaviour (research/baseline_codec/fused_quant_crypto.py:263-342, :543-603).
#include "../../include/ztcp_ledger.h"

#include <cstring>
#include <mutex>
#include <new>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace {

inline uint64_t mix64(uint64_t x) {  // splitmix64 finalizer
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

struct Nonce {
  uint64_t seq;
  uint32_t loc;
  bool operator==(const Nonce& o) const { return seq == o.seq && loc == o.loc; }
};
struct NonceHash {
  size_t operator()(const Nonce& n) const { return (size_t)mix64(n.seq ^ mix64((uint64_t)n.loc + 0x9e37u)); }
};

struct Slot {
  uint64_t token;
  uint32_t model;
  uint32_t loc;  // layer_id << 16 | head_group_id
  bool operator==(const Slot& o) const { return token == o.token && model == o.model && loc == o.loc; }
};
struct SlotHash {
  size_t operator()(const Slot& s) const { return (size_t)mix64(s.token ^ mix64(((uint64_t)s.model << 32) | s.loc)); }
};

typedef unsigned __int128 u128;

struct Session {
  std::unordered_set<Nonce, NonceHash> used;
  std::unordered_map<Slot, uint64_t, SlotHash> watermark;
  u128 max_nonce = 0;  // may pass 2^64 - 1 through next_nonce, as the reference's Python integer does

  uint64_t mark(const Slot& s) const {
    auto it = watermark.find(s);
    return it == watermark.end() ? 0 : it->second;
  }
};

inline uint32_t loc_word(uint16_t layer, uint16_t hg) { return ((uint32_t)layer << 16) | hg; }

void set_err(ztcp_ledger_error* e, int32_t code, int32_t kind, int64_t index, uint64_t seq, uint64_t ref,
             uint32_t loc) {
  if (!e) return;
  e->code = code;
  e->kind = kind;
  e->index = index;
  e->seq = seq;
  e->ref = ref;
  e->loc = loc;
  e->reserved = 0;
}

inline uint64_t rd64(const uint8_t* p) {
  uint64_t v;
  std::memcpy(&v, p, 8);
  return v;
}
inline uint32_t rd32(const uint8_t* p) {
  uint32_t v;
  std::memcpy(&v, p, 4);
  return v;
}
inline uint16_t rd16(const uint8_t* p) {
  uint16_t v;
  std::memcpy(&v, p, 2);
  return v;
}

}  // namespace

struct ztcp_ledger {
  mutable std::mutex mu;
  std::unordered_map<uint64_t, Session> sessions;

  Session* find(uint64_t id) {
    auto it = sessions.find(id);
    return it == sessions.end() ? nullptr : &it->second;
  }
  const Session* find(uint64_t id) const {
    auto it = sessions.find(id);
    return it == sessions.end() ? nullptr : &it->second;
  }
};

struct ztcp_reservation {
  std::vector<std::pair<Slot, uint64_t>> slots;  // staged watermark per distinct slot
  uint64_t last_seq = 0;
  int64_t pages = 0;
};

extern "C" {

ztcp_ledger* ztcp_ledger_create(void) { return new (std::nothrow) ztcp_ledger(); }

void ztcp_ledger_destroy(ztcp_ledger* ledger) { delete ledger; }

int32_t ztcp_ledger_open(ztcp_ledger* ledger, uint64_t session) {
  if (!ledger) return ZTCP_LEDGER_EINVAL;
  std::lock_guard<std::mutex> g(ledger->mu);
  try {
    ledger->sessions[session] = Session();
  } catch (...) {
    return ZTCP_LEDGER_EINVAL;
  }
  return ZTCP_LEDGER_OK;
}

int32_t ztcp_ledger_close(ztcp_ledger* ledger, uint64_t session) {
  if (!ledger) return ZTCP_LEDGER_EINVAL;
  std::lock_guard<std::mutex> g(ledger->mu);
  return ledger->sessions.erase(session) ? 1 : 0;
}

int32_t ztcp_ledger_is_open(const ztcp_ledger* ledger, uint64_t session) {
  if (!ledger) return 0;
  std::lock_guard<std::mutex> g(ledger->mu);
  return ledger->find(session) != nullptr;
}

int32_t ztcp_ledger_next_nonce(ztcp_ledger* ledger, uint64_t session, uint64_t count, uint64_t* base_lo,
                               uint64_t* base_hi) {
  if (!ledger || !base_lo || !base_hi || count < 1) return ZTCP_LEDGER_EINVAL;
  std::lock_guard<std::mutex> g(ledger->mu);
  Session* s = ledger->find(session);
  if (!s) return ZTCP_LEDGER_ENOSESSION;
  const u128 base = s->max_nonce + 1;
  s->max_nonce = base + count - 1;
  *base_lo = (uint64_t)base;
  *base_hi = (uint64_t)(base >> 64);
  return ZTCP_LEDGER_OK;
}

int32_t ztcp_ledger_max_nonce(const ztcp_ledger* ledger, uint64_t session, uint64_t* max_lo, uint64_t* max_hi) {
  if (!ledger || !max_lo || !max_hi) return ZTCP_LEDGER_EINVAL;
  std::lock_guard<std::mutex> g(ledger->mu);
  const Session* s = ledger->find(session);
  if (!s) return ZTCP_LEDGER_ENOSESSION;
  *max_lo = (uint64_t)s->max_nonce;
  *max_hi = (uint64_t)(s->max_nonce >> 64);
  return ZTCP_LEDGER_OK;
}

int32_t ztcp_ledger_preflight(ztcp_ledger* ledger, uint64_t session, uint32_t model_id_hash, uint16_t layer_id,
                              uint16_t head_group_id, uint64_t base_sequence_nonce, const uint64_t* token_hashes,
                              int64_t n, ztcp_reservation** out, ztcp_ledger_error* err) {
  if (!ledger || !out || n < 1 || !token_hashes) return ZTCP_LEDGER_EINVAL;
  *out = nullptr;
  std::lock_guard<std::mutex> g(ledger->mu);
  Session* s = ledger->find(session);
  if (!s) return ZTCP_LEDGER_ENOSESSION;
  const uint32_t loc = loc_word(layer_id, head_group_id);
  try {
    std::unordered_map<Slot, uint64_t, SlotHash> staged;  // slot -> nonce of its latest page in the batch
    std::unordered_set<Nonce, NonceHash> batch;
    staged.reserve((size_t)n);
    batch.reserve((size_t)n);
    for (int64_t i = 0; i < n; ++i) {
      const uint64_t seq = base_sequence_nonce + (uint64_t)i;
      const Slot slot{token_hashes[i], model_id_hash, loc};
      auto st = staged.find(slot);
      const uint64_t prev = st != staged.end() ? st->second : s->mark(slot);
      if (seq < prev) {
        set_err(err, ZTCP_LEDGER_ESTALE, 0, i, seq, prev, loc);
        return ZTCP_LEDGER_ESTALE;
      }
      const Nonce nonce{seq, loc};
      if (s->used.count(nonce) || !batch.insert(nonce).second) {
        set_err(err, ZTCP_LEDGER_EREUSE, 0, i, seq, 0, loc);
        return ZTCP_LEDGER_EREUSE;
      }
      if (st != staged.end()) st->second = seq;
      else staged.emplace(slot, seq);
    }
    ztcp_reservation* r = new ztcp_reservation();
    r->slots.assign(staged.begin(), staged.end());
    r->last_seq = base_sequence_nonce + (uint64_t)(n - 1);
    r->pages = n;
    s->used.reserve(s->used.size() + batch.size());
    s->used.insert(batch.begin(), batch.end());
    if (r->last_seq > s->max_nonce) s->max_nonce = r->last_seq;
    *out = r;
  } catch (...) {
    return ZTCP_LEDGER_EINVAL;
  }
  return ZTCP_LEDGER_OK;
}

uint64_t ztcp_reservation_last_seq(const ztcp_reservation* r) { return r ? r->last_seq : 0; }
int64_t ztcp_reservation_pages(const ztcp_reservation* r) { return r ? r->pages : 0; }

int32_t ztcp_ledger_commit(ztcp_ledger* ledger, uint64_t session, const ztcp_reservation* r) {
  if (!ledger || !r) return ZTCP_LEDGER_EINVAL;
  std::lock_guard<std::mutex> g(ledger->mu);
  Session* s = ledger->find(session);
  if (!s) return ZTCP_LEDGER_ENOSESSION;
  try {
    for (const auto& kv : r->slots) {
      auto it = s->watermark.find(kv.first);
      if (it == s->watermark.end()) {
        if (kv.second > 0) s->watermark.emplace(kv.first, kv.second);
      } else if (kv.second > it->second) {
        it->second = kv.second;
      }
    }
  } catch (...) {
    return ZTCP_LEDGER_EINVAL;
  }
  if (r->last_seq > s->max_nonce) s->max_nonce = r->last_seq;
  return ZTCP_LEDGER_OK;
}

void ztcp_reservation_free(ztcp_reservation* r) { delete r; }

int32_t ztcp_ledger_freshness_batch(ztcp_ledger* ledger, uint64_t session, const ztcp_fresh_record* records,
                                    int64_t n, int32_t has_min, uint64_t min_sequence_nonce, ztcp_ledger_error* err) {
  if (!ledger || (n > 0 && !records) || n < 0) return ZTCP_LEDGER_EINVAL;
  std::lock_guard<std::mutex> g(ledger->mu);
  Session* s = ledger->find(session);
  if (!s) return ZTCP_LEDGER_ENOSESSION;
  try {
    std::unordered_map<Slot, uint64_t, SlotHash> staged;
    staged.reserve((size_t)n);
    u128 max_s = s->max_nonce;
    for (int64_t i = 0; i < n; ++i) {
      const ztcp_fresh_record& rec = records[i];
      const uint64_t seq = rec.sequence_nonce;
      const uint32_t loc = loc_word(rec.layer_id, rec.head_group_id);
      if (has_min && seq < min_sequence_nonce) {
        set_err(err, ZTCP_LEDGER_ESTALE, 1, i, seq, min_sequence_nonce, loc);
        return ZTCP_LEDGER_ESTALE;
      }
      const Slot slot{rec.page_token_hash, rec.model_id_hash, loc};
      auto st = staged.find(slot);
      const uint64_t latest = st != staged.end() ? st->second : s->mark(slot);
      if (seq < latest) {
        set_err(err, ZTCP_LEDGER_ESTALE, 0, i, seq, latest, loc);
        return ZTCP_LEDGER_ESTALE;
      }
      if (seq > latest) {
        if (st != staged.end()) st->second = seq;
        else staged.emplace(slot, seq);
      }
      if (seq > max_s) max_s = seq;
    }
    for (const auto& kv : staged) s->watermark[kv.first] = kv.second;
    s->max_nonce = max_s;
  } catch (...) {
    return ZTCP_LEDGER_EINVAL;
  }
  return ZTCP_LEDGER_OK;
}

int32_t ztcp_ledger_freshness_one(ztcp_ledger* ledger, uint64_t session, const ztcp_fresh_record* record,
                                  int32_t has_min, uint64_t min_sequence_nonce, int32_t has_expected,
                                  uint64_t expected_sequence_nonce, ztcp_ledger_error* err) {
  if (!ledger || !record) return ZTCP_LEDGER_EINVAL;
  std::lock_guard<std::mutex> g(ledger->mu);
  Session* s = ledger->find(session);
  if (!s) return ZTCP_LEDGER_ENOSESSION;
  const uint64_t seq = record->sequence_nonce;
  const uint32_t loc = loc_word(record->layer_id, record->head_group_id);
  if (has_expected && seq != expected_sequence_nonce) {
    set_err(err, ZTCP_LEDGER_EMISMATCH, 0, 0, seq, expected_sequence_nonce, loc);
    return ZTCP_LEDGER_EMISMATCH;
  }
  if (has_min && seq < min_sequence_nonce) {
    set_err(err, ZTCP_LEDGER_ESTALE, 1, 0, seq, min_sequence_nonce, loc);
    return ZTCP_LEDGER_ESTALE;
  }
  const Slot slot{record->page_token_hash, record->model_id_hash, loc};
  try {
    auto it = s->watermark.find(slot);
    const uint64_t latest = it == s->watermark.end() ? 0 : it->second;
    if (seq < latest) {
      set_err(err, ZTCP_LEDGER_ESTALE, 0, 0, seq, latest, loc);
      return ZTCP_LEDGER_ESTALE;
    }
    if (seq > latest) {
      if (it == s->watermark.end()) s->watermark.emplace(slot, seq);
      else it->second = seq;
    }
  } catch (...) {
    return ZTCP_LEDGER_EINVAL;
  }
  if (seq > s->max_nonce) s->max_nonce = seq;
  return ZTCP_LEDGER_OK;
}

int32_t ztcp_ledger_parse_headers(const uint8_t* blobs, int64_t stride, int64_t n, ztcp_fresh_record* out) {
  if (n < 0 || (n > 0 && (!blobs || !out)) || stride < 32) return ZTCP_LEDGER_EINVAL;
  for (int64_t i = 0; i < n; ++i) {
    const uint8_t* h = blobs + i * stride;  // <HBBIIHHQQ: magic, version, flags, tenant, model, layer, hg, token, seq
    out[i].model_id_hash = rd32(h + 8);
    out[i].layer_id = rd16(h + 12);
    out[i].head_group_id = rd16(h + 14);
    out[i].page_token_hash = rd64(h + 16);
    out[i].sequence_nonce = rd64(h + 24);
  }
  return ZTCP_LEDGER_OK;
}

}  // extern "C"
