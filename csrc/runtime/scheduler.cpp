// Continuous-batching scheduler and paged-KV block pool (see scheduler.h).
//
// Policy (the behaviour vLLM's V1 scheduler gives the reference):
//  1. Running requests first, in admission order: one token for a decode, the next prompt
//     chunk for a partial prefill, within the per-step token budget.  When the pool has no
//     block for a running request, the most recently admitted running request is preempted
//     (recompute: its blocks are released and it returns to the head of the waiting queue).
//  2. If nothing was preempted, waiting requests are admitted FCFS while the budget, the
//     sequence cap and the pool allow; prefix-cache hits skip their cached full blocks.
// The step's inputs are laid out decodes first (one query token each), then prefills, which
// is the order the attention kernels consume them in.
#include "scheduler.h"

#include <algorithm>
#include <stdexcept>

namespace b200 {
namespace rt {

// ------------------------------------------------------------------------------ BlockPool
BlockPool::BlockPool(int num_blocks)
    : num_blocks_(num_blocks),
      ref_(num_blocks, 0),
      hash_(num_blocks, 0),
      pos_(num_blocks),
      in_free_(num_blocks, true) {
  for (int b = 0; b < num_blocks; ++b) pos_[b] = free_.insert(free_.end(), b);
  free_count_ = num_blocks;
}

int BlockPool::allocate() {
  if (free_.empty()) return -1;
  const int b = free_.front();
  free_.pop_front();
  in_free_[b] = false;
  --free_count_;
  if (hash_[b] != 0) {
    auto it = cached_.find(hash_[b]);
    if (it != cached_.end() && it->second == b) cached_.erase(it);
    hash_[b] = 0;
  }
  ref_[b] = 1;
  return b;
}

void BlockPool::release(int b) {
  if (ref_[b] <= 0) throw std::runtime_error("BlockPool: double free");
  if (--ref_[b] == 0) {
    pos_[b] = free_.insert(free_.end(), b);
    in_free_[b] = true;
    ++free_count_;
  }
}

void BlockPool::touch(int b) {
  if (ref_[b] == 0 && in_free_[b]) {
    free_.erase(pos_[b]);
    in_free_[b] = false;
    --free_count_;
  }
  ++ref_[b];
}

int BlockPool::lookup(uint64_t h) const {
  auto it = cached_.find(h);
  return it == cached_.end() ? -1 : it->second;
}

void BlockPool::set_hash(int b, uint64_t h) {
  if (h == 0 || hash_[b] != 0) return;
  if (cached_.count(h)) return;  // an identical block is already cached
  hash_[b] = h;
  cached_[h] = b;
}

// ------------------------------------------------------------------------------ Scheduler
static inline uint64_t mix64(uint64_t x) {
  // splitmix64 finaliser
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

uint64_t Scheduler::block_hash(uint64_t parent, const int32_t* toks, int n) const {
  uint64_t h = mix64(parent ^ 0x5bd1e9955bd1e995ull);
  for (int i = 0; i < n; ++i) h = mix64(h ^ (uint64_t)(uint32_t)toks[i]);
  return h == 0 ? 1 : h;
}

Scheduler::Scheduler(const SchedulerConfig& cfg, int num_blocks, const StepBuffers& buf)
    : cfg_(cfg), pool_(num_blocks), buf_(buf) {
  for (int s = cfg_.max_num_seqs - 1; s >= 0; --s) free_slots_.push_back(s);
  if (cfg_.block_size <= 0) throw std::runtime_error("scheduler: block_size must be > 0");
  if ((int64_t)cfg_.max_blocks_per_seq * cfg_.block_size < cfg_.max_model_len)
    throw std::runtime_error("scheduler: block-table width cannot hold max_model_len");
  if (buf_.max_tokens < cfg_.max_num_batched_tokens || buf_.max_reqs < cfg_.max_num_seqs)
    throw std::runtime_error("scheduler: step buffers smaller than the batch limits");
}

void Scheduler::add_request(int64_t id, const std::vector<int32_t>& prompt,
                            const SamplingCfg& sp) {
  if (reqs_.count(id)) throw std::runtime_error("scheduler: duplicate request id");
  if (prompt.empty()) throw std::runtime_error("scheduler: empty prompt");
  if ((int)prompt.size() >= cfg_.max_model_len)
    throw std::runtime_error("scheduler: prompt length " + std::to_string(prompt.size()) +
                             " leaves no room below max_model_len " +
                             std::to_string(cfg_.max_model_len));
  Request r;
  r.id = id;
  r.tokens = prompt;
  r.num_prompt = (int)prompt.size();
  r.sp = sp;
  r.arrival_seq = arrival_seq_++;
  reqs_.emplace(id, std::move(r));
  enqueue_waiting(id, false);
}

// FCFS: new requests at the back, preempted ones back at the front.  Priority: both by
// (priority, arrival), so a preempted request returns to the place its priority gives it.
void Scheduler::enqueue_waiting(int64_t id, bool front) {
  if (!cfg_.priority_policy) {
    if (front)
      waiting_.push_front(id);
    else
      waiting_.push_back(id);
    return;
  }
  const Request& r = reqs_.at(id);
  auto later = [&](int64_t other) {
    const Request& o = reqs_.at(other);
    return o.sp.priority > r.sp.priority ||
           (o.sp.priority == r.sp.priority && o.arrival_seq > r.arrival_seq);
  };
  auto it = std::find_if(waiting_.begin(), waiting_.end(), later);
  waiting_.insert(it, id);
}

// The running request to preempt when blocks run out: the most recently admitted (FCFS), or
// the one that sorts last by (priority, arrival) among those not yet scheduled this step.
int64_t Scheduler::pick_victim(size_t from) const {
  // only requests not yet placed in this step's batch (index >= from) can give up blocks
  if (!cfg_.priority_policy) return running_.back();
  int64_t best = running_.back();
  for (size_t k = from; k < running_.size(); ++k) {
    const int64_t id = running_[k];
    const Request& a = reqs_.at(id);
    const Request& b = reqs_.at(best);
    if (a.sp.priority > b.sp.priority ||
        (a.sp.priority == b.sp.priority && a.arrival_seq > b.arrival_seq))
      best = id;
  }
  return best;
}

void Scheduler::release_slot(Request& r) {
  if (r.state_slot >= 0) {
    free_slots_.push_back(r.state_slot);
    r.state_slot = -1;
  }
}

void Scheduler::free_request_blocks(Request& r) {
  // reverse order: the tail blocks (least likely shared) are handed out first
  for (auto it = r.blocks.rbegin(); it != r.blocks.rend(); ++it) pool_.release(*it);
  r.blocks.clear();
  r.block_hashes.clear();
}

bool Scheduler::abort_request(int64_t id) {
  auto it = reqs_.find(id);
  if (it == reqs_.end() || it->second.status == kFinished) return false;
  Request& r = it->second;
  if (r.status == kWaiting) {
    waiting_.erase(std::remove(waiting_.begin(), waiting_.end(), id), waiting_.end());
  } else {
    running_.erase(std::remove(running_.begin(), running_.end(), id), running_.end());
  }
  free_request_blocks(r);
  release_slot(r);
  r.status = kFinished;
  r.reason = kAbort;
  r.finish_step = step_;
  return true;
}

void Scheduler::preempt(Request& r) {
  free_request_blocks(r);
  release_slot(r);
  r.num_computed = 0;
  r.num_cached_prefix = 0;
  r.status = kWaiting;
  r.num_preemptions++;
  enqueue_waiting(r.id, true);
}

bool Scheduler::ensure_blocks(Request& r, int num_tokens) {
  const int need = (num_tokens + cfg_.block_size - 1) / cfg_.block_size - (int)r.blocks.size();
  if (need <= 0) return true;
  if ((int)r.blocks.size() + need > cfg_.max_blocks_per_seq) return false;
  if (pool_.num_free() < need) return false;
  for (int i = 0; i < need; ++i) r.blocks.push_back(pool_.allocate());
  return true;
}

void Scheduler::admit_prefix(Request& r) {
  if (!cfg_.prefix_caching || r.sp.no_prefix_cache) return;
  const int bs = cfg_.block_size;
  const int n_full = ((int)r.tokens.size() - 1) / bs;  // keep >= 1 token to compute
  uint64_t parent = 0;
  for (int j = 0; j < n_full; ++j) {
    const uint64_t h = block_hash(parent, r.tokens.data() + j * bs, bs);
    pool_.cache_queries++;
    const int b = pool_.lookup(h);
    if (b < 0) break;
    pool_.cache_hits++;
    pool_.touch(b);
    r.blocks.push_back(b);
    r.block_hashes.push_back(h);
    parent = h;
  }
  r.num_computed = (int)r.blocks.size() * bs;
  r.num_cached_prefix = r.num_computed;
}

void Scheduler::register_full_blocks(Request& r) {
  if (!cfg_.prefix_caching) return;
  const int bs = cfg_.block_size;
  const int known = std::min(r.num_computed, (int)r.tokens.size());
  while ((int)r.block_hashes.size() < (int)r.blocks.size() &&
         ((int)r.block_hashes.size() + 1) * bs <= known) {
    const int j = (int)r.block_hashes.size();
    const uint64_t parent = j == 0 ? 0 : r.block_hashes[j - 1];
    const uint64_t h = block_hash(parent, r.tokens.data() + j * bs, bs);
    pool_.set_hash(r.blocks[j], h);
    r.block_hashes.push_back(h);
  }
}

// Keep the first ``cap`` drafts of a tree and, of those, the ones shallower than ``max_depth``
// (depth 0 = child of the pending token) whose parent is kept; parents are re-indexed.
// Returns the depth of every kept draft.
static std::vector<int> prune_tree(std::vector<int32_t>& tok, std::vector<int32_t>& par,
                                   int cap, int max_depth) {
  const int n = std::max(0, std::min((int)tok.size(), cap));
  std::vector<int> depth(n), remap(n, -1), kept;
  int m = 0;
  for (int j = 0; j < n; ++j) {
    const int p = par[j];
    depth[j] = p < 0 ? 0 : depth[p] + 1;
    if (depth[j] >= max_depth || (p >= 0 && remap[p] < 0)) continue;
    remap[j] = m;
    tok[m] = tok[j];
    par[m] = p < 0 ? -1 : remap[p];
    kept.push_back(depth[j]);
    ++m;
  }
  tok.resize(m);
  par.resize(m);
  return kept;
}

StepPlan Scheduler::schedule() {
  StepPlan plan;
  if (waiting_.empty() && running_.empty()) return plan;
  ++step_;
  struct Item {
    Request* r;
    int start, q;
    bool samples;
    int spec;  // draft tokens appended to a decode
    bool tree;
    std::vector<int> depth;  // tree drafts: depth of every node
  };
  std::vector<Item> items;
  items.reserve(running_.size() + 16);
  int budget = cfg_.max_num_batched_tokens;
  bool preempted = false;

  for (size_t i = 0; i < running_.size() && budget > 0; ++i) {
    Request& r = reqs_.at(running_[i]);
    const int remaining = (int)r.tokens.size() - r.num_computed;
    if (remaining <= 0) continue;
    int q = std::min(remaining, budget);
    if (cfg_.long_prefill_threshold > 0 && q > 1) q = std::min(q, cfg_.long_prefill_threshold);
    if (!cfg_.chunked_prefill && q < remaining) continue;
    int spec = 0;
    bool tree = false;
    std::vector<int> depth;
    if (remaining == 1 && !r.draft.empty()) {
      // verify drafts: never past the model length or the request's token budget
      const int len_room = cfg_.max_model_len - (int)r.tokens.size();
      const int tok_room = r.sp.max_tokens - r.num_output() - 1;
      if (r.draft_parent.empty()) {
        spec = std::max(0, std::min({(int)r.draft.size(), budget - 1, len_room, tok_room}));
      } else {
        // every node takes a KV slot; only paths up to tok_room tokens can be accepted
        depth = prune_tree(r.draft, r.draft_parent,
                           std::min({budget - 1, len_room, kMaxTreeDrafts}), tok_room);
        spec = (int)r.draft.size();
        tree = spec > 0;
      }
      q += spec;
    }
    bool self_preempted = false;
    while (!ensure_blocks(r, r.num_computed + q)) {
      const int64_t victim = pick_victim(i);
      running_.erase(std::find(running_.begin(), running_.end(), victim));
      preempted = true;
      plan.num_preempted++;
      preempt(reqs_.at(victim));
      if (victim == r.id) {
        self_preempted = true;
        break;
      }
    }
    if (self_preempted) break;
    items.push_back({&r, r.num_computed, q, r.num_computed + q - spec == (int)r.tokens.size(),
                     spec, tree, std::move(depth)});
    budget -= q;
  }

  while (!preempted && !waiting_.empty() && budget > 0 &&
         (int)running_.size() < cfg_.max_num_seqs) {
    Request& r = reqs_.at(waiting_.front());
    if (r.num_computed == 0 && r.blocks.empty()) admit_prefix(r);
    const int remaining = (int)r.tokens.size() - r.num_computed;
    int q = std::min(remaining, budget);
    if (cfg_.long_prefill_threshold > 0 && q > 1) q = std::min(q, cfg_.long_prefill_threshold);
    if ((!cfg_.chunked_prefill && q < remaining) || !ensure_blocks(r, r.num_computed + q)) {
      // not admitted this step: give back the prefix-cache blocks admit_prefix pinned, or
      // waiting requests could hold the whole pool while nothing runs
      free_request_blocks(r);
      r.num_computed = 0;
      r.num_cached_prefix = 0;
      break;
    }
    waiting_.pop_front();
    r.status = kRunning;
    if (r.state_slot < 0 && !free_slots_.empty()) {
      r.state_slot = free_slots_.back();
      free_slots_.pop_back();
    }
    running_.push_back(r.id);
    items.push_back({&r, r.num_computed, q, r.num_computed + q == (int)r.tokens.size(), 0,
                     false, {}});
    budget -= q;
  }

  // decodes (one query token) first, then prefills; stable within each class
  std::stable_partition(items.begin(), items.end(), [](const Item& it) { return it.q == 1; });

  const int bs = cfg_.block_size;
  int t = 0, s = 0;
  buf_.cu_q[0] = 0;
  last_sample_ids_.clear();
  last_sample_counts_.clear();
  for (const Item& it : items) plan.tree = plan.tree || it.tree;
  if (plan.tree && buf_.tree_mask == nullptr)
    throw std::runtime_error("scheduler: draft trees need the tree_mask step buffer");
  for (size_t i = 0; i < items.size(); ++i) {
    Item& it = items[i];
    Request& r = *it.r;
    r.last_path.clear();
    const int base = it.q - it.spec;  // step tokens before the drafts
    uint64_t anc[kMaxTreeDrafts];     // tree drafts: the node and its ancestors (bit = node)
    for (int j = 0; j < it.q; ++j) {
      const int pos = it.start + j;  // sequence index = KV slot
      const int d = j - base;
      buf_.input_ids[t] = d < 0 ? r.tokens[pos] : r.draft[d];
      buf_.positions[t] = d >= 0 && it.tree ? it.start + base + it.depth[d] : pos;
      buf_.slot_mapping[t] = r.blocks[pos / bs] * bs + pos % bs;
      if (plan.tree) {
        uint64_t m = 0;  // non-tree rows: causal
        if (it.tree) {
          if (d >= 0) {
            const int p = r.draft_parent[d];
            anc[d] = (1ull << d) | (p >= 0 ? anc[p] : 0ull);
            m = (anc[d] << 1) | 1ull;  // step token 0 is the pending token
          } else {
            m = 1ull;
          }
        }
        buf_.tree_mask[t] = (int64_t)m;
      }
      ++t;
    }
    buf_.cu_q[i + 1] = t;
    const int seq_len = it.start + it.q;
    buf_.seq_lens[i] = seq_len;
    if (buf_.state_slots) buf_.state_slots[i] = r.state_slot;
    plan.max_seq_len = std::max(plan.max_seq_len, seq_len);
    std::copy(r.blocks.begin(), r.blocks.end(),
              buf_.block_tables + (int64_t)i * cfg_.max_blocks_per_seq);
    if (it.q == 1)
      plan.num_decodes++;
    else {
      plan.num_prefills++;
      plan.num_prefill_tokens += it.q;
    }
    if (it.samples) {
      // one row per position that predicts a new token: the pending token's position and,
      // under verification, every draft position
      for (int j = 0; j <= it.spec; ++j) {
        buf_.logits_idx[s] = t - 1 - it.spec + j;
        buf_.temperature[s] = r.sp.temperature;
        buf_.top_k[s] = r.sp.top_k;
        buf_.top_p[s] = r.sp.top_p;
        buf_.min_p[s] = r.sp.min_p;
        buf_.seeds[s] = r.sp.seed;
        // same noise as without speculation: the output index the row's token would take
        buf_.steps[s] = r.num_output() + (j > 0 && it.tree ? it.depth[j - 1] + 1 : j);
        ++s;
      }
      if (r.sp.temperature > 0.f) plan.all_greedy = false;
      if (r.sp.temperature > 0.f && (r.sp.top_k > 0 || r.sp.top_p < 1.f || r.sp.min_p > 0.f))
        plan.any_filter = true;
      last_sample_ids_.push_back(r.id);
      last_sample_counts_.push_back(1 + it.spec);
      plan.sample_counts.push_back(1 + it.spec);
    }
    plan.num_spec_tokens += it.spec;
    plan.req_ids.push_back(r.id);
    if (it.spec > 0) {
      r.spec_start = it.start;
      r.draft.resize(it.spec);  // the drafts under verification
      spec_proposed_ += it.spec;
    } else {
      r.draft.clear();
      r.draft_parent.clear();
    }
    r.num_computed = seq_len;
    register_full_blocks(r);
  }
  plan.num_tokens = t;
  plan.num_reqs = (int)items.size();
  plan.num_samples = s;
  plan.sample_req_ids = last_sample_ids_;
  return plan;
}

std::vector<std::pair<int64_t, int>> Scheduler::update(const int64_t* sampled, int n) {
  int rows = 0;
  for (int c : last_sample_counts_) rows += c;
  if (n != rows)
    throw std::runtime_error("scheduler.update: expected " + std::to_string(rows) +
                             " sampled rows, got " + std::to_string(n));
  std::vector<std::pair<int64_t, int>> finished;
  kv_moves_.clear();
  int row = 0;
  for (size_t k = 0; k < last_sample_ids_.size(); ++k) {
    const int cnt = last_sample_counts_[k];
    const int64_t* y = sampled + row;
    row += cnt;
    auto itr = reqs_.find(last_sample_ids_[k]);
    if (itr == reqs_.end()) continue;
    Request& r = itr->second;
    if (r.status != kRunning) continue;  // aborted or preempted while in flight
    // tokens this step contributes: accepted drafts, then the token drawn at the first
    // position whose draft was rejected (or after the last draft).  rows[j] = sampling row of
    // the j-th contributed token.
    int accept = 0;
    const int d = cnt - 1;
    const bool tree = d > 0 && !r.draft_parent.empty();
    std::vector<int> rows(1, 0);
    r.last_path.clear();
    if (tree) {
      // walk down the tree: the child whose token equals the token drawn at its parent
      int cur = -1;
      for (;;) {
        const int32_t want = (int32_t)y[cur + 1];
        int next = -1;
        for (int c = cur + 1; c < d; ++c)
          if (r.draft_parent[c] == cur && r.draft[c] == want) {
            next = c;
            break;
          }
        if (next < 0) break;
        r.last_path.push_back(next);
        rows.push_back(next + 1);
        cur = next;
      }
      accept = (int)r.last_path.size();
    } else {
      while (accept < d && (int32_t)y[accept] == r.draft[accept]) ++accept;
      for (int j = 1; j <= accept; ++j) rows.push_back(j);
    }
    const int spec_start = r.spec_start;
    if (d > 0) {
      spec_accepted_ += accept;
      // KV is valid for the pending token and the accepted drafts only
      r.num_computed = r.spec_start + 1 + accept;
      r.draft.clear();
      r.draft_parent.clear();
      r.spec_start = -1;
    }
    FinishReason why = kNotFinished;
    for (int j = 0; j <= accept && why == kNotFinished; ++j) {
      const int32_t tok = (int32_t)y[rows[j]];
      r.tokens.push_back(tok);
      if (r.first_token_step < 0) r.first_token_step = step_;
      const int out = r.num_output();
      const bool may_stop = out >= r.sp.min_tokens;
      if (may_stop && !r.sp.ignore_eos && tok == r.sp.eos_id) why = kStop;
      if (may_stop && why == kNotFinished &&
          std::find(r.sp.stop_ids.begin(), r.sp.stop_ids.end(), tok) != r.sp.stop_ids.end())
        why = kStop;
      if (why == kNotFinished &&
          (out >= r.sp.max_tokens || (int)r.tokens.size() >= cfg_.max_model_len))
        why = kLength;
    }
    if (d > 0) {
      r.num_computed = std::min(r.num_computed, (int)r.tokens.size() - 1);
      if (tree && why == kNotFinished) {
        // accepted node k sits at slot spec_start + 1 + node; its token now has index
        // spec_start + 1 + k (sources never precede destinations, so the copies are ordered)
        const int bs = cfg_.block_size;
        for (int k = 0; k < accept; ++k) {
          const int dst = spec_start + 1 + k, src = spec_start + 1 + r.last_path[k];
          if (src == dst || dst >= r.num_computed) continue;
          kv_moves_.emplace_back((int64_t)r.blocks[src / bs] * bs + src % bs,
                                 (int64_t)r.blocks[dst / bs] * bs + dst % bs);
        }
      }
      register_full_blocks(r);
    }
    if (why != kNotFinished) {
      r.status = kFinished;
      r.reason = why;
      r.finish_step = step_;
      free_request_blocks(r);
      release_slot(r);
      finished.emplace_back(r.id, (int)why);
    }
  }
  if (!finished.empty()) {
    running_.erase(std::remove_if(running_.begin(), running_.end(),
                                  [this](int64_t id) { return reqs_.at(id).status == kFinished; }),
                   running_.end());
  }
  last_sample_ids_.clear();
  last_sample_counts_.clear();
  return finished;
}

std::vector<int32_t> Scheduler::tokens_range(int64_t id, int start, int n) const {
  auto it = reqs_.find(id);
  if (it == reqs_.end()) return {};
  const auto& t = it->second.tokens;
  const int a = std::max(0, std::min(start, (int)t.size()));
  const int b = std::max(a, std::min(start + n, (int)t.size()));
  return std::vector<int32_t>(t.begin() + a, t.begin() + b);
}

int Scheduler::num_tokens(int64_t id) const {
  auto it = reqs_.find(id);
  return it == reqs_.end() ? 0 : (int)it->second.tokens.size();
}

std::vector<int64_t> Scheduler::decode_request_ids() const {
  std::vector<int64_t> out;
  for (int64_t id : running_) {
    const Request& r = reqs_.at(id);
    if ((int)r.tokens.size() - r.num_computed == 1) out.push_back(id);
  }
  return out;
}

void Scheduler::set_draft(int64_t id, const std::vector<int32_t>& draft) {
  auto it = reqs_.find(id);
  if (it == reqs_.end() || it->second.status != kRunning) return;
  it->second.draft = draft;
  it->second.draft_parent.clear();
}

void Scheduler::set_draft_tree(int64_t id, const std::vector<int32_t>& tokens,
                               const std::vector<int32_t>& parents) {
  if (tokens.size() != parents.size())
    throw std::invalid_argument("set_draft_tree: tokens and parents differ in length");
  if ((int)tokens.size() > kMaxTreeDrafts)
    throw std::invalid_argument("set_draft_tree: at most 63 draft nodes");
  for (size_t j = 0; j < parents.size(); ++j)
    if (parents[j] < -1 || parents[j] >= (int)j)
      throw std::invalid_argument("set_draft_tree: every parent must precede its child");
  auto it = reqs_.find(id);
  if (it == reqs_.end() || it->second.status != kRunning) return;
  it->second.draft = tokens;
  it->second.draft_parent = parents;
  // a one-node-per-level tree in order is a chain: verify it without a mask
  bool chain = true;
  for (size_t j = 0; j < parents.size() && chain; ++j) chain = parents[j] == (int)j - 1;
  if (chain) it->second.draft_parent.clear();
}

std::vector<std::pair<int64_t, int64_t>> Scheduler::take_kv_moves() {
  std::vector<std::pair<int64_t, int64_t>> out;
  out.swap(kv_moves_);
  return out;
}

std::vector<int64_t> Scheduler::reserve_slots(int64_t id, int start, int n) {
  std::vector<int64_t> out(std::max(0, n), -1);
  auto it = reqs_.find(id);
  if (it == reqs_.end() || it->second.status != kRunning) return out;
  Request& r = it->second;
  const int bs = cfg_.block_size;
  for (int k = 0; k < n; ++k) {
    const int pos = start + k;
    if (pos < 0 || pos >= cfg_.max_model_len || !ensure_blocks(r, pos + 1)) break;
    out[k] = (int64_t)r.blocks[pos / bs] * bs + pos % bs;
  }
  return out;
}

std::vector<int32_t> Scheduler::block_ids(int64_t id) const {
  auto it = reqs_.find(id);
  return it == reqs_.end() ? std::vector<int32_t>{} : it->second.blocks;
}

std::vector<int32_t> Scheduler::last_path(int64_t id) const {
  auto it = reqs_.find(id);
  return it == reqs_.end() ? std::vector<int32_t>{} : it->second.last_path;
}

int Scheduler::propose_ngram_tree(int k, int n_min, int n_max, int width) {
  k = std::min(k, kMaxTreeDrafts);
  int total = 0;
  for (int64_t id : running_) {
    Request& r = reqs_.at(id);
    r.draft.clear();
    r.draft_parent.clear();
    const int L = (int)r.tokens.size();
    if (L - r.num_computed != 1 || k <= 0 || width <= 0) continue;
    const int32_t* tk = r.tokens.data();
    // continuation starts of the chosen occurrences, distinct as k-token strings
    std::vector<int> from;
    for (int n = std::min(n_max, L - 1); n >= n_min && (int)from.size() < width; --n) {
      for (int st = L - n - 1; st >= 0 && (int)from.size() < width; --st) {
        if (!std::equal(tk + st, tk + st + n, tk + L - n)) continue;
        const int f = st + n, len = std::min(k, L - f);
        bool dup = false;
        for (int g : from) {
          const int lg = std::min(k, L - g);
          if (lg >= len && std::equal(tk + f, tk + f + len, tk + g)) dup = true;
        }
        if (!dup) from.push_back(f);
      }
    }
    if (from.empty()) continue;
    // merge level by level: node of every continuation at the current depth
    std::vector<int> at(from.size(), -1);
    for (int depth = 0; (int)r.draft.size() < k; ++depth) {
      bool grew = false;
      for (size_t c = 0; c < from.size() && (int)r.draft.size() < k; ++c) {
        if (at[c] == -2 || from[c] + depth >= L) continue;
        const int32_t tok = tk[from[c] + depth];
        int node = -1;
        for (int j = 0; j < (int)r.draft.size(); ++j)
          if (r.draft_parent[j] == at[c] && r.draft[j] == tok) {
            node = j;
            break;
          }
        if (node < 0) {
          node = (int)r.draft.size();
          r.draft.push_back(tok);
          r.draft_parent.push_back(at[c]);
        }
        at[c] = node;
        grew = true;
      }
      // continuations that ran out stop; the rest continue at the next depth
      for (size_t c = 0; c < from.size(); ++c)
        if (at[c] != -2 && from[c] + depth + 1 >= L) at[c] = -2;
      if (!grew) break;
    }
    bool chain = true;
    for (size_t j = 0; j < r.draft_parent.size() && chain; ++j)
      chain = r.draft_parent[j] == (int)j - 1;
    if (chain) r.draft_parent.clear();
    total += (int)r.draft.size();
  }
  return total;
}

int Scheduler::propose_ngram(int k, int n_min, int n_max) {
  int total = 0;
  for (int64_t id : running_) {
    Request& r = reqs_.at(id);
    r.draft.clear();
    const int L = (int)r.tokens.size();
    if (L - r.num_computed != 1 || k <= 0) continue;
    const int32_t* tk = r.tokens.data();
    for (int n = std::min(n_max, L - 1); n >= n_min && r.draft.empty(); --n) {
      // latest earlier occurrence of the last n tokens
      for (int st = L - n - 1; st >= 0; --st) {
        if (std::equal(tk + st, tk + st + n, tk + L - n)) {
          const int from = st + n;
          const int cnt = std::min(k, L - from);
          r.draft.assign(tk + from, tk + from + cnt);
          break;
        }
      }
    }
    total += (int)r.draft.size();
  }
  return total;
}

std::vector<int32_t> Scheduler::output_tokens(int64_t id) const {
  auto it = reqs_.find(id);
  if (it == reqs_.end()) return {};
  const Request& r = it->second;
  return std::vector<int32_t>(r.tokens.begin() + r.num_prompt, r.tokens.end());
}

const Request* Scheduler::get(int64_t id) const {
  auto it = reqs_.find(id);
  return it == reqs_.end() ? nullptr : &it->second;
}

void Scheduler::forget(int64_t id) {
  auto it = reqs_.find(id);
  if (it != reqs_.end() && it->second.status == kFinished) reqs_.erase(it);
}

}  // namespace rt
}  // namespace b200
