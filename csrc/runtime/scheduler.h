// Native host runtime of the serving engine: paged-KV block pool with prefix caching and a
// continuous-batching scheduler with chunked prefill and recompute preemption.
//
// The reference inherits these from upstream vLLM's V1 engine (Python scheduler and KV-cache
// manager; the plugin only sizes blocks, vllm_musa/platform.py:616-720).  Here they are C++:
// one call per engine step plans the batch AND writes every per-step input array (token ids,
// positions, slot mapping, query offsets, sequence lengths, block tables, sampling parameters)
// straight into pinned host buffers the model runner copies to the GPU, so host time per step
// stays in the tens of microseconds at hundreds of concurrent requests.
#pragma once
#include <stdint.h>

#include <deque>
#include <list>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

namespace b200 {
namespace rt {

enum Status : int { kWaiting = 0, kRunning = 1, kFinished = 2 };
enum FinishReason : int { kNotFinished = 0, kLength = 1, kStop = 2, kAbort = 3 };

struct SamplingCfg {
  int max_tokens = 16;
  int min_tokens = 0;
  bool ignore_eos = false;
  int eos_id = -1;
  std::vector<int32_t> stop_ids;
  float temperature = 1.f;
  int top_k = 0;
  float top_p = 1.f;
  float min_p = 0.f;
  int64_t seed = 0;
  bool no_prefix_cache = false;  // compute every prompt token (e.g. prompt log-probabilities)
  int priority = 0;              // priority policy: lower values are served first
};

struct Request {
  int64_t id = 0;
  std::vector<int32_t> tokens;  // prompt + generated
  int num_prompt = 0;
  int num_computed = 0;         // tokens whose KV is in the cache (advanced at schedule time)
  int num_cached_prefix = 0;    // tokens served from the prefix cache at admission
  std::vector<int32_t> blocks;  // physical KV blocks
  std::vector<uint64_t> block_hashes;  // hashes of full blocks (prefix caching)
  Status status = kWaiting;
  FinishReason reason = kNotFinished;
  SamplingCfg sp;
  int32_t state_slot = -1;      // per-request recurrent-state slot (hybrid models)
  std::vector<int32_t> draft;   // speculative tokens proposed for the next step
  // Token tree of the drafts: parent index of every draft (-1 = child of the pending token,
  // otherwise an earlier draft).  Empty = the drafts form one chain.
  std::vector<int32_t> draft_parent;
  std::vector<int32_t> last_path;  // drafts accepted by the last verification (tree order)
  int spec_start = -1;          // first position of the in-flight verification step
  int64_t first_token_step = -1;
  int64_t finish_step = -1;
  int num_preemptions = 0;
  int64_t arrival_seq = 0;  // admission order of add_request (ties of equal priority)
  int num_output() const { return (int)tokens.size() - num_prompt; }
};

// Free-list block allocator with reference counts.  A full block carries the hash of its token
// prefix; when its reference count drops to zero it stays in the hash map (reusable) until the
// LRU free list hands it out again.
class BlockPool {
 public:
  explicit BlockPool(int num_blocks);
  int num_free() const { return (int)free_count_; }
  int num_blocks() const { return num_blocks_; }
  int allocate();                  // -1 when empty
  void release(int block);         // refcount--, back to the free list at zero
  void touch(int block);           // refcount++ (cache hit); removes from free list if needed
  int lookup(uint64_t hash) const; // cached block id or -1
  void set_hash(int block, uint64_t hash);
  int refcount(int block) const { return ref_[block]; }
  int64_t cache_hits = 0, cache_queries = 0;

 private:
  int num_blocks_;
  std::vector<int> ref_;
  std::vector<uint64_t> hash_;
  std::list<int> free_;                        // LRU order: front = next to hand out
  std::vector<std::list<int>::iterator> pos_;  // position in free_ (valid when ref == 0)
  std::vector<bool> in_free_;
  size_t free_count_ = 0;
  std::unordered_map<uint64_t, int> cached_;
};

struct SchedulerConfig {
  int block_size = 16;
  int max_num_seqs = 256;
  int max_num_batched_tokens = 8192;
  int max_model_len = 4096;
  int max_blocks_per_seq = 256;  // block-table row width of the step buffers
  bool chunked_prefill = true;
  bool prefix_caching = true;
  int long_prefill_threshold = 0;  // 0 = no per-request cap on one prefill chunk
  // false: first come first served; true: waiting requests are admitted by (priority,
  // arrival) and the preemption victim is the running request that sorts last
  bool priority_policy = false;
};

// Pinned host buffers the scheduler writes each step (capacities fixed at construction).
struct StepBuffers {
  int32_t* input_ids;     // [max_tokens]
  int32_t* positions;     // [max_tokens]
  int32_t* slot_mapping;  // [max_tokens]
  int32_t* cu_q;          // [max_reqs + 1]
  int32_t* seq_lens;      // [max_reqs]
  int32_t* block_tables;  // [max_reqs, max_blocks_per_seq]
  int32_t* logits_idx;    // [max_reqs]  token index of every sampling row
  float* temperature;     // [max_reqs]
  int32_t* top_k;         // [max_reqs]
  float* top_p;           // [max_reqs]
  float* min_p;           // [max_reqs]
  int64_t* seeds;         // [max_reqs]
  int32_t* steps;         // [max_reqs]  output index of the token being drawn
  int32_t* state_slots;   // [max_reqs]  recurrent-state slot of every scheduled request
  // [max_tokens] per-token attention masks of steps that verify a draft tree (null: no tree
  // verification): bit j of a tree request's row lets it see the request's step token j; a
  // zero row is plain causal
  int64_t* tree_mask;
  int max_tokens, max_reqs;
};

struct StepPlan {
  int num_tokens = 0;
  int num_reqs = 0;
  int num_decodes = 0;      // leading requests with exactly one query token
  int num_prefills = 0;     // remaining requests
  int num_prefill_tokens = 0;
  int num_samples = 0;      // sampling rows (decodes + prefills that finish their prompt)
  int max_seq_len = 0;
  int num_preempted = 0;
  bool all_greedy = true;
  bool any_filter = false;  // some row uses top-k / top-p / min-p
  int num_spec_tokens = 0;  // draft tokens under verification this step
  bool tree = false;        // some request verifies a draft tree: tree_mask is filled
  std::vector<int64_t> sample_req_ids;
  std::vector<int32_t> sample_counts;  // sampling rows per request (1 + drafts)
  std::vector<int64_t> req_ids;        // every scheduled request, in step-buffer order
};

class Scheduler {
 public:
  Scheduler(const SchedulerConfig& cfg, int num_blocks, const StepBuffers& buf);
  void add_request(int64_t id, const std::vector<int32_t>& prompt, const SamplingCfg& sp);
  bool abort_request(int64_t id);
  // Plan the next step and fill the step buffers.  Returns an empty plan when idle.
  StepPlan schedule();
  // Append the tokens drawn for the last plan's sampling rows (same order).  A request under
  // speculative verification owns 1 + d consecutive rows (the token drawn at each of its
  // positions); its drafts are accepted while they equal the drawn token, and the first
  // mismatch (or the row after the last draft) contributes the drawn token.  With drafts
  // fixed before sampling this is exact rejection sampling.  Returns the (id, reason) pairs of
  // the requests that finished; their blocks are already released.
  std::vector<std::pair<int64_t, int>> update(const int64_t* sampled, int n);
  // Propose up to k draft tokens per running decode request by prompt lookup: the longest
  // suffix n-gram (n_max down to n_min) that occurred earlier in the request's tokens is
  // followed by its continuation.  Returns the number of drafts set.
  int propose_ngram(int k, int n_min, int n_max);
  void set_draft(int64_t id, const std::vector<int32_t>& draft);
  // Draft tree: tokens in an order where every parent precedes its children (parents[j] in
  // [-1, j); -1 = child of the pending token), at most kMaxTreeDrafts nodes.  A verification
  // step runs the pending token and every node (position = pending + 1 + depth, KV slot =
  // pending + 1 + node index, attention over the context and the node's ancestors); update()
  // follows the drawn tokens down the tree and moves the KV of the accepted path into place.
  void set_draft_tree(int64_t id, const std::vector<int32_t>& tokens,
                      const std::vector<int32_t>& parents);
  // Prompt lookup with several continuations: the continuations of up to ``width`` earlier
  // occurrences of the context's suffix n-gram (longest n first, most recent first, duplicates
  // skipped) merged into a token trie, level by level, of at most k nodes.
  int propose_ngram_tree(int k, int n_min, int n_max, int width);
  // KV copies (source slot, destination slot) that the last update() needs: the accepted path
  // of a draft tree moved to consecutive slots.  Must run before the next step's forward.
  std::vector<std::pair<int64_t, int64_t>> take_kv_moves();
  std::vector<int32_t> last_path(int64_t id) const;
  // KV slots of positions [start, start + n) of a running request, allocating blocks as needed
  // (a model drafter writes its own layer's K/V there while chaining drafts); -1 where the pool
  // has no block left.  block_ids: the request's block table.
  std::vector<int64_t> reserve_slots(int64_t id, int start, int n);
  std::vector<int32_t> block_ids(int64_t id) const;
  static constexpr int kMaxTreeDrafts = 63;  // + the pending token = 64 mask bits
  std::vector<int64_t> decode_request_ids() const;  // running requests with one token pending
  // tokens[start, start + n) of a request (clipped to what exists), and its token count
  std::vector<int32_t> tokens_range(int64_t id, int start, int n) const;
  int num_tokens(int64_t id) const;
  int64_t spec_accepted() const { return spec_accepted_; }
  int64_t spec_proposed() const { return spec_proposed_; }

  bool has_unfinished() const { return !waiting_.empty() || !running_.empty(); }
  int num_waiting() const { return (int)waiting_.size(); }
  int num_running() const { return (int)running_.size(); }
  int num_free_blocks() const { return pool_.num_free(); }
  int64_t step_index() const { return step_; }
  std::vector<int32_t> output_tokens(int64_t id) const;
  const Request* get(int64_t id) const;
  void forget(int64_t id);  // drop a finished request's record
  int64_t prefix_cache_hits() const { return pool_.cache_hits; }
  int64_t prefix_cache_queries() const { return pool_.cache_queries; }

 private:
  bool ensure_blocks(Request& r, int num_tokens);
  void free_request_blocks(Request& r);
  void preempt(Request& r);
  void enqueue_waiting(int64_t id, bool front);
  int64_t pick_victim(size_t from) const;
  void admit_prefix(Request& r);
  void register_full_blocks(Request& r);
  uint64_t block_hash(uint64_t parent, const int32_t* toks, int n) const;

  SchedulerConfig cfg_;
  BlockPool pool_;
  StepBuffers buf_;
  std::unordered_map<int64_t, Request> reqs_;
  std::deque<int64_t> waiting_;
  std::vector<int64_t> running_;
  std::vector<int64_t> last_sample_ids_;
  std::vector<int32_t> last_sample_counts_;
  std::vector<std::pair<int64_t, int64_t>> kv_moves_;
  int64_t spec_accepted_ = 0, spec_proposed_ = 0;
  std::vector<int32_t> free_slots_;
  void release_slot(Request& r);
  int64_t step_ = 0;
  int64_t arrival_seq_ = 0;
};

}  // namespace rt
}  // namespace b200
