// The generation loop: the reference's Worker (src/worker.rs) over the engine's C ABI.
//
// Host code only. One request at a time; between requests the worker keeps the prefix
// keys of what the engine's caches hold (the live cache) and of four snapshot slots,
// and resumes a new prompt from the longest cached strict prefix (worker.rs:118-180).
// Decoding follows worker.rs:195-255: with an MTP head, each step drafts one token,
// verifies [token, draft] in one 2-row forward with a checkpoint after the first row,
// and rolls the second row back when the draft is rejected; drafting pauses for 20
// requests when, after 16 drafts, the drafts cost more time than they saved.
//
// Sampling runs on the device (snl_engine_sample). The uniform draws come from a
// ChaCha12 stream on the host, taken one at a time in the reference Sampler's order:
// the device call receives the next two pending draws and reports how many it used, and
// only those leave the queue.
#include <algorithm>
#include <array>
#include <chrono>
#include <cstring>
#include <deque>
#include <random>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace snl {

size_t engine_hidden(const snl_engine* e);

namespace {

constexpr size_t kSpecTrial = 16;  // worker.rs:111
constexpr size_t kSpecPause = 20;  // worker.rs:113

// ---- ChaCha12 -------------------------------------------------------------------------

inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

void chacha_block(const uint32_t in[16], int rounds, uint32_t out[16]) {
  uint32_t x[16];
  memcpy(x, in, sizeof(x));
  auto qr = [&](int a, int b, int c, int d) {
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 16);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 12);
    x[a] += x[b]; x[d] = rotl32(x[d] ^ x[a], 8);
    x[c] += x[d]; x[b] = rotl32(x[b] ^ x[c], 7);
  };
  for (int r = 0; r < rounds; r += 2) {
    qr(0, 4, 8, 12); qr(1, 5, 9, 13); qr(2, 6, 10, 14); qr(3, 7, 11, 15);  // columns
    qr(0, 5, 10, 15); qr(1, 6, 11, 12); qr(2, 7, 8, 13); qr(3, 4, 9, 14);  // diagonals
  }
  for (int i = 0; i < 16; i++) out[i] = x[i] + in[i];
}

// A ChaCha12 word stream: 256-bit key, 64-bit block counter in words 12-13 from 0,
// stream id 0 in words 14-15; each block's 16 words are taken in order. A u64 seed is
// expanded into the key with PCG32 (XSH-RR output, O'Neill 2014), stepped before each
// 32-bit word, as rand documents for StdRng::seed_from_u64. A draw in [0, 1) is the
// top 24 bits of a word times 2^-24.
class ChaCha12 {
 public:
  explicit ChaCha12(uint64_t seed) {
    uint64_t st = seed;
    for (int i = 0; i < 8; i++) {
      st = st * 6364136223846793005ull + 11634580027462260723ull;
      const uint32_t xs = (uint32_t)(((st >> 18) ^ st) >> 27);
      const int rot = (int)(st >> 59);
      key_[i] = (xs >> rot) | (xs << ((32 - rot) & 31));
    }
  }
  uint32_t next_u32() {
    if (idx_ == 16) refill();
    return buf_[idx_++];
  }
  float next_f32() { return (float)(next_u32() >> 8) * (1.0f / 16777216.0f); }

 private:
  void refill() {
    const uint32_t in[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,  // "expand 32-byte k"
                             key_[0], key_[1], key_[2], key_[3], key_[4], key_[5], key_[6], key_[7],
                             (uint32_t)ctr_, (uint32_t)(ctr_ >> 32), 0u, 0u};
    chacha_block(in, 12, buf_);
    ctr_++;
    idx_ = 0;
  }
  uint32_t key_[8];
  uint32_t buf_[16];
  uint64_t ctr_ = 0;
  int idx_ = 16;
};

uint64_t entropy_seed() {
  std::random_device rd;
  return ((uint64_t)rd() << 32) ^ rd();
}

// ---- the engine behind snl_worker_create ---------------------------------------------

snl_engine* as_engine(void* s) { return static_cast<snl_engine*>(s); }
int e_forward(void* s, const uint32_t* t, size_t n, const uint32_t* pos, const uint32_t* ei, const float* em, size_t ne,
              size_t rows, int ckpt) {
  return snl_engine_forward_mm(as_engine(s), t, n, pos, ei, em, ne, rows, ckpt, nullptr);
}
int e_forward_greedy(void* s, const uint32_t* t, size_t n, const uint32_t* pos, size_t rows, int ckpt, uint32_t* out) {
  return snl_engine_forward_greedy(as_engine(s), t, n, pos, rows, ckpt, out);
}
int e_sample(void* s, size_t row, const snl_sample_p* p, const uint32_t* ht, const uint32_t* hc, size_t nh,
             const float* u, int64_t draft, uint32_t* out3) {
  return snl_engine_sample(as_engine(s), row, p, ht, hc, nh, u, draft, out3);
}
int e_mtp(void* s, size_t r0, const uint32_t* t, size_t n, const uint32_t* pos, size_t slot0, int draft, uint32_t* d) {
  return snl_engine_mtp(as_engine(s), r0, t, n, pos, slot0, draft, d);
}
int e_reset(void* s) { return snl_engine_reset(as_engine(s)); }
int e_snapshot(void* s, size_t slot) { return snl_engine_snapshot(as_engine(s), slot); }
int e_restore(void* s, size_t slot, size_t pos) { return snl_engine_restore(as_engine(s), slot, pos); }
int e_rollback(void* s) { return snl_engine_rollback(as_engine(s)); }
size_t e_hid_rows(void* s) { return snl_engine_hid_rows(as_engine(s)); }
size_t e_pos(void* s) { return snl_engine_pos(as_engine(s)); }

// A cached state is reusable only if its keys are a strict prefix of the prompt: the
// recurrent state cannot be rewound, and one token must still be fed for logits
// (worker.rs:115-120).
size_t shared_prefix(const std::vector<uint64_t>& cached, const std::vector<uint64_t>& prompt) {
  if (cached.size() < prompt.size() && std::equal(cached.begin(), cached.end(), prompt.begin())) return cached.size();
  return 0;
}

}  // namespace
}  // namespace snl

struct snl_worker {
  snl_worker_ops ops;
  std::vector<uint64_t> live;  // keys of the tokens in the caches
  struct Snap {
    bool used = false;
    std::vector<uint64_t> keys;
    uint64_t last = 0;
  };
  std::vector<Snap> snaps = std::vector<Snap>(SNL_WORKER_SNAPSHOTS);
  bool spec = false;
  size_t spec_pause = 0;
  uint64_t clock = 0;
};

namespace snl {
namespace {

double now_s(const snl_worker_ops& o) {
  if (o.now) return o.now(o.self);
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

// The request's sampler (sampler.rs Sampler): parameters, generator, pending draws and
// the counts of accepted tokens for the penalties.
struct Sampler {
  const snl_worker_ops& o;
  snl_sample_p p;
  ChaCha12 rng;
  std::deque<float> draws;
  std::unordered_map<uint32_t, uint32_t> counts;
  std::vector<uint32_t> ht, hc;
  bool greedy_fast;     // argmax of unpenalised logits: the engine's forward_greedy
  uint32_t greedy[2] = {0, 0};  // its per-row answers for the last forward

  Sampler(const snl_worker_ops& ops, const snl_sample_p& params, uint64_t seed)
      : o(ops), p(params), rng(seed) {
    greedy_fast = ops.forward_greedy && p.temperature <= 1e-5f && p.repetition_penalty == 1.0f &&
                  p.presence_penalty == 0.0f && p.frequency_penalty == 0.0f;
  }
  void accept(uint32_t t) { counts[t]++; }

  // sample (draft < 0) or verify on kept logit row `row`; returns token and acceptance.
  int pick(size_t row, int64_t draft, uint32_t* tok, bool* ok) {
    while (draws.size() < 2) draws.push_back(rng.next_f32());
    ht.clear();
    hc.clear();
    for (auto& kv : counts) {
      ht.push_back(kv.first);
      hc.push_back(kv.second);
    }
    const float u[2] = {draws[0], draws[1]};
    uint32_t out3[3] = {0, 0, 0};
    SNL_TRY(o.sample(o.self, row, &p, ht.data(), hc.data(), ht.size(), u, draft, out3));
    if (out3[2] > 2) return fail(SNL_E_STATE, "worker: sampler reported more than two draws");
    for (uint32_t i = 0; i < out3[2]; i++) draws.pop_front();
    *tok = out3[0];
    if (ok) *ok = out3[1] != 0;
    return SNL_OK;
  }
};

// The request in the worker's terms.
struct Req {
  std::vector<uint32_t> tokens;
  std::vector<uint64_t> keys;
  std::vector<uint32_t> pos;  // [n][3]
  std::vector<uint32_t> eidx;
  const float* embeds = nullptr;
  size_t n = 0;
};

// Emit (worker.rs:340-391) on token ids: EOS, the token limit and client disconnects.
struct Emit {
  const snl_gen_request* r;
  uint32_t* out;
  size_t cap;
  size_t generated = 0, max = 0;
  int reason = SNL_FINISH_LENGTH;
  bool cancelled = false;
  bool push(uint32_t t) {
    if (out && generated < cap) out[generated] = t;
    generated++;
    for (size_t i = 0; i < r->n_eos; i++)
      if (r->eos[i] == t) {
        reason = SNL_FINISH_STOP;
        return false;
      }
    if (r->on_token && !r->on_token(r->user, t)) {
      cancelled = true;
      return false;
    }
    return generated < max;
  }
};

// Worker::feed (worker.rs:298-338): prompt tokens from..to one engine chunk at a time,
// splicing the encoded media rows, and with drafting on, the MTP head fed with every
// (hidden row, next token) pair of the chunk.
int feed(snl_worker* w, const Req& q, size_t from, size_t to, bool want_logits) {
  const snl_worker_ops& o = w->ops;
  const size_t chunk = o.prefill_chunk;
  std::vector<uint32_t> ei;
  std::vector<float> er;
  for (size_t c0 = from; c0 < to;) {
    const size_t c1 = std::min(c0 + chunk, to);
    ei.clear();
    er.clear();
    for (size_t i = 0; i < q.eidx.size(); i++) {
      if (q.eidx[i] >= c0 && q.eidx[i] < c1) {
        ei.push_back(q.eidx[i] - (uint32_t)c0);
        er.insert(er.end(), q.embeds + i * o.hidden, q.embeds + (i + 1) * o.hidden);
      }
    }
    SNL_TRY(o.forward(o.self, q.tokens.data() + c0, c1 - c0, q.pos.data() + 3 * c0, ei.empty() ? nullptr : ei.data(),
                      er.empty() ? nullptr : er.data(), ei.size(), (want_logits && c1 == to) ? 1 : 0, 0));
    // Hidden row k of this step belongs to token c0 - 1 + k and pairs with token c0 + k;
    // row 0 needs an earlier token, and the last row's partner comes with the next step.
    const size_t r0 = c0 == 0 ? 1 : 0;
    if (w->spec && r0 < c1 - c0)
      SNL_TRY(o.mtp(o.self, r0, q.tokens.data() + c0 + r0, c1 - c0 - r0, q.pos.data() + 3 * (c0 + r0 - 1),
                    c0 + r0 - 1, 0, nullptr));
    c0 = c1;
  }
  return SNL_OK;
}

int run(snl_worker* w, const snl_gen_request* r, uint32_t* out_tokens, size_t out_cap, snl_finish* fin) {
  const snl_worker_ops& o = w->ops;
  const size_t ctx = o.ctx;
  const size_t n = r->n;
  if (n == 0) return fail(SNL_E_INVALID, "empty prompt");
  if (n >= ctx)
    return fail(SNL_E_RANGE, "prompt is " + std::to_string(n) + " tokens but the context size is " +
                                 std::to_string(ctx) + "; restart with a larger --ctx");
  Req q;
  q.n = n;
  q.tokens.assign(r->tokens, r->tokens + n);
  q.keys.resize(n);
  q.pos.resize(3 * n);
  for (size_t i = 0; i < n; i++) {
    q.keys[i] = r->keys ? r->keys[i] : (uint64_t)r->tokens[i];
    for (int k = 0; k < 3; k++) q.pos[3 * i + k] = r->pos ? r->pos[3 * i + k] : (uint32_t)i;
  }
  if (r->n_embeds) {
    if (!r->embed_idx || !r->embeds) return fail(SNL_E_INVALID, "worker: media rows without indices");
    for (size_t i = 0; i < r->n_embeds; i++)
      if (r->embed_idx[i] >= n) return fail(SNL_E_RANGE, "worker: media row beyond the prompt");
    q.eidx.assign(r->embed_idx, r->embed_idx + r->n_embeds);
    q.embeds = r->embeds;
  }
  const size_t max_tokens = std::min(r->max_tokens, ctx - n);
  const double t0 = now_s(o);
  w->spec = o.has_mtp && w->spec_pause == 0;
  w->spec_pause = w->spec_pause ? w->spec_pause - 1 : 0;

  // The longest cached strict prefix: the live cache, or a snapshot if it holds more
  // (ties between snapshots go to the higher slot, as Iterator::max_by_key).
  w->clock++;
  const size_t live_hit = shared_prefix(w->live, q.keys);
  int best = -1;
  size_t best_n = 0;
  for (int i = 0; i < (int)w->snaps.size(); i++) {
    if (!w->snaps[i].used) continue;
    const size_t k = shared_prefix(w->snaps[i].keys, q.keys);
    if (best < 0 || k >= best_n) {
      best = i;
      best_n = k;
    }
  }
  if (best >= 0 && best_n > live_hit) {
    SNL_TRY(o.restore(o.self, (size_t)best, best_n));
    w->snaps[best].last = w->clock;
    w->live = w->snaps[best].keys;
  } else if (live_hit == 0) {
    SNL_TRY(o.reset(o.self));
    w->live.clear();
  }
  const size_t cached = w->live.size();

  if (r->snapshot_at >= 0 && (size_t)r->snapshot_at > w->live.size() && (size_t)r->snapshot_at < n) {
    const size_t s = (size_t)r->snapshot_at;
    SNL_TRY(feed(w, q, w->live.size(), s, false));
    int slot = 0;  // least recently used; an empty slot counts as 0 (first minimum wins)
    for (int i = 1; i < (int)w->snaps.size(); i++) {
      const uint64_t ui = w->snaps[i].used ? w->snaps[i].last : 0;
      const uint64_t us = w->snaps[slot].used ? w->snaps[slot].last : 0;
      if (ui < us) slot = i;
    }
    SNL_TRY(o.snapshot(o.self, (size_t)slot));
    w->live.assign(q.keys.begin(), q.keys.begin() + s);
    w->snaps[slot].used = true;
    w->snaps[slot].keys = w->live;
    w->snaps[slot].last = w->clock;
  }
  SNL_TRY(feed(w, q, w->live.size(), n, true));
  w->live = q.keys;
  uint32_t rope = 0;  // Prompt::next_pos: one past the largest position component
  for (size_t i = 0; i < 3 * n; i++) rope = std::max(rope, q.pos[i] + 1);
  const double prefill_secs = now_s(o) - t0;

  const double t1 = now_s(o);
  Sampler sm(o, r->params, r->has_seed ? r->seed : entropy_seed());
  Emit out{r, out_tokens, out_cap};
  out.max = max_tokens;
  size_t drafted = 0, accepted = 0;
  double draft_secs = 0, verify_secs = 0;
  uint32_t tok = 0;
  SNL_TRY(sm.pick(0, -1, &tok, nullptr));
  // MTP input of the next draft: hidden rows from r0 of the last step, the tokens that
  // follow them, their positions and the first MTP cache slot.
  struct MtpIn {
    size_t r0;
    std::vector<uint32_t> toks;
    std::vector<uint32_t> pos;
    size_t slot0;
  } mi{o.hid_rows(o.self), {tok}, {q.pos[3 * (n - 1)], q.pos[3 * (n - 1) + 1], q.pos[3 * (n - 1) + 2]}, n - 1};

  while (out.push(tok)) {
    sm.accept(tok);
    const double t = now_s(o);
    bool have_draft = false;
    uint32_t d = 0;
    if (w->spec) {
      SNL_TRY(o.mtp(o.self, mi.r0, mi.toks.data(), mi.toks.size(), mi.pos.data(), mi.slot0, 1, &d));
      have_draft = true;
    }
    draft_secs += now_s(o) - t;
    if (!have_draft) {
      const uint32_t p1[3] = {rope, rope, rope};
      if (sm.greedy_fast) {
        SNL_TRY(o.forward_greedy(o.self, &tok, 1, p1, 1, 0, sm.greedy));
        w->live.push_back(tok);
        rope++;
        tok = sm.greedy[0];
      } else {
        SNL_TRY(o.forward(o.self, &tok, 1, p1, nullptr, nullptr, 0, 1, 0));
        w->live.push_back(tok);
        rope++;
        SNL_TRY(sm.pick(0, -1, &tok, nullptr));
      }
      continue;
    }
    // Verify the draft: one pass over [tok, draft] gives the distribution after tok (to
    // accept or replace the draft) and after the draft.
    const size_t slot = o.pos(o.self);
    const uint32_t two[2] = {tok, d};
    const uint32_t p2[6] = {rope, rope, rope, rope + 1, rope + 1, rope + 1};
    const double tv = now_s(o);
    if (sm.greedy_fast)
      SNL_TRY(o.forward_greedy(o.self, two, 2, p2, 2, 1, sm.greedy));
    else
      SNL_TRY(o.forward(o.self, two, 2, p2, nullptr, nullptr, 0, 2, 1));
    verify_secs += now_s(o) - tv;
    drafted++;
    // A step yields 1 + acceptance tokens for (draft + verify) time, where plain decoding
    // yields one token for about the verify time: stop drafting when drafts cost more
    // than the accepted tokens save.
    if (drafted == kSpecTrial && draft_secs > verify_secs * (double)accepted / (double)drafted) {
      w->spec = false;
      w->spec_pause = kSpecPause;
    }
    bool ok = false;
    uint32_t next = 0;
    if (sm.greedy_fast) {
      next = sm.greedy[0];
      ok = next == d;
    } else {
      SNL_TRY(sm.pick(0, (int64_t)d, &next, &ok));
    }
    w->live.push_back(tok);
    if (ok) {
      accepted++;
      w->live.push_back(d);
      if (!out.push(d)) break;
      sm.accept(d);
      if (sm.greedy_fast)
        tok = sm.greedy[1];
      else
        SNL_TRY(sm.pick(1, -1, &tok, nullptr));
      mi = MtpIn{1, {d, tok}, {rope, rope, rope, rope + 1, rope + 1, rope + 1}, slot};
      rope += 2;
    } else {
      SNL_TRY(o.rollback(o.self));
      tok = next;
      mi = MtpIn{1, {tok}, {rope, rope, rope}, slot};
      rope++;
    }
  }
  if (fin) {
    fin->reason = out.reason;
    fin->cancelled = out.cancelled ? 1 : 0;
    fin->prompt_tokens = n;
    fin->completion_tokens = out.generated;
    fin->cached_tokens = cached;
    fin->prefill_secs = prefill_secs;
    fin->decode_secs = now_s(o) - t1;
    fin->drafted = drafted;
    fin->accepted = accepted;
  }
  return SNL_OK;
}

int check_ops(const snl_worker_ops& o) {
  if (!o.forward || !o.sample || !o.reset || !o.snapshot || !o.restore || !o.rollback || !o.hid_rows || !o.pos)
    return fail(SNL_E_INVALID, "worker: engine operations missing");
  if (o.has_mtp && !o.mtp) return fail(SNL_E_INVALID, "worker: MTP engine without an mtp operation");
  if (o.prefill_chunk == 0 || o.ctx == 0) return fail(SNL_E_INVALID, "worker: zero context or chunk");
  return SNL_OK;
}

}  // namespace
}  // namespace snl

using namespace snl;

extern "C" int snl_worker_create_ops(const snl_worker_ops* ops, snl_worker** out) {
  if (!ops || !out) return fail(SNL_E_INVALID, "snl_worker_create_ops: null argument");
  *out = nullptr;
  SNL_TRY(check_ops(*ops));
  snl_worker* w = new snl_worker();
  w->ops = *ops;
  *out = w;
  return SNL_OK;
}

extern "C" int snl_worker_create(snl_engine* e, snl_worker** out) {
  if (!e || !out) return fail(SNL_E_INVALID, "snl_worker_create: null argument");
  snl_worker_ops o;
  memset(&o, 0, sizeof(o));
  o.self = e;
  o.ctx = snl_engine_ctx(e);
  o.prefill_chunk = snl_engine_prefill_chunk(e);
  o.hidden = engine_hidden(e);
  o.has_mtp = snl_engine_has_mtp(e);
  o.forward = e_forward;
  o.forward_greedy = e_forward_greedy;
  o.sample = e_sample;
  o.mtp = e_mtp;
  o.reset = e_reset;
  o.snapshot = e_snapshot;
  o.restore = e_restore;
  o.rollback = e_rollback;
  o.hid_rows = e_hid_rows;
  o.pos = e_pos;
  return snl_worker_create_ops(&o, out);
}

extern "C" void snl_worker_destroy(snl_worker* w) { delete w; }

extern "C" int snl_worker_run(snl_worker* w, const snl_gen_request* r, uint32_t* out_tokens, size_t out_cap,
                              snl_finish* fin) {
  if (!w || !r || (r->n && !r->tokens) || (r->n_eos && !r->eos))
    return fail(SNL_E_INVALID, "snl_worker_run: null argument");
  const int rc = run(w, r, out_tokens, out_cap, fin);
  if (rc != SNL_OK) {
    // Leave the caches in a known state after a failure (worker.rs:93-100).
    const std::string msg = snl_last_error();
    w->ops.reset(w->ops.self);
    w->live.clear();
    for (auto& s : w->snaps) s = snl_worker::Snap();
    set_error(msg);
  }
  return rc;
}

extern "C" int snl_worker_prefix(const snl_worker* w, int slot, uint64_t* keys, size_t cap, size_t* n,
                                 uint64_t* used) {
  if (!w || !n) return fail(SNL_E_INVALID, "snl_worker_prefix: null argument");
  if (slot >= (int)w->snaps.size()) return fail(SNL_E_RANGE, "snapshot slot out of range");
  const std::vector<uint64_t>* k = &w->live;
  uint64_t last = 0;
  if (slot >= 0) {
    const auto& s = w->snaps[slot];
    static const std::vector<uint64_t> none;
    k = s.used ? &s.keys : &none;
    last = s.used ? s.last : 0;
  }
  *n = k->size();
  if (keys) memcpy(keys, k->data(), std::min(cap, k->size()) * sizeof(uint64_t));
  if (used) *used = last;
  return SNL_OK;
}

extern "C" int snl_worker_spec(const snl_worker* w, int* spec, size_t* pause) {
  if (!w) return fail(SNL_E_INVALID, "snl_worker_spec: null worker");
  if (spec) *spec = w->spec ? 1 : 0;
  if (pause) *pause = w->spec_pause;
  return SNL_OK;
}

extern "C" int snl_rng_uniforms(uint64_t seed, size_t n, float* out) {
  if (n && !out) return fail(SNL_E_INVALID, "snl_rng_uniforms: null output");
  ChaCha12 g(seed);
  for (size_t i = 0; i < n; i++) out[i] = g.next_f32();
  return SNL_OK;
}

extern "C" int snl_chacha_block(const uint32_t in[16], int rounds, uint32_t out[16]) {
  if (!in || !out || rounds <= 0 || rounds % 2) return fail(SNL_E_INVALID, "snl_chacha_block: bad argument");
  chacha_block(in, rounds, out);
  return SNL_OK;
}
