// Plain-C++ launcher interface of the vllm_musa_b200 CUDA kernels.
//
// Every kernel translation unit (csrc/**/*.cu) implements one group of these functions and
// includes no torch header; csrc/torch_bindings.cpp validates torch tensors, fills the
// argument structs and registers the ops as torch.ops.b200.*.  All launchers are
// asynchronous on the given stream, allocate nothing, and throw std::runtime_error on bad
// arguments.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace b200 {

// ------------------------------------------------------------------------------- GEMM
namespace gemm {
// kModeStoreT / kModeSiluT ("swap-AB", for decode-sized token counts): A is the WEIGHT [N, K]
// and B the activations [M, K]; the kernel computes C^T tiles and stores C [M, N] (N/2 for
// SiLU) transposed, so the tokens occupy the MMA's N dimension.
enum Mode : int { kModeStore = 0, kModeSiluMul = 1, kModeF32 = 2, kModeScatter = 3,
                  kModeStoreT = 4, kModeSiluT = 5 };
struct GemmArgs {
  const void* A;  // [M, K] bf16, row stride lda
  int64_t lda;
  const void* B;  // [N, K] bf16, row stride ldb
  int64_t ldb;
  void* C;        // [M, N] (or [M, N/2] for SiLU-mul), row stride ldc
  int64_t ldc;
  int M, N, K;
  int mode;
  int bn, splits;  // 0 = automatic
  int mt;          // 128-row halves per CTA (1 or 2); 0 = automatic
  float* workspace;  // split-K partials
  int64_t workspace_numel;
  int* counters;     // split-K per-tile arrival counters (zero-initialised, self-resetting)
  int64_t counters_numel;
  int* err;
  // kModeScatter (GEMM -> reduce-scatter): output row r belongs to rank o = r / rs_rows and is
  // stored (bf16, over NVLink when o is a peer) at peers[o] + (rs_rank * rs_rows + r - o *
  // rs_rows) * ldc: every rank's receive slot holds one rs_rows-row block per source rank.
  void* peers[8] = {};
  int rs_rows = 0, rs_rank = 0, rs_world = 0;
};
struct GemmPlan {
  int bn, splits;
  int64_t workspace_floats;
  int mt;
};
GemmPlan plan_bf16(int M, int N, int K);
void set_katoms(int katoms);  // K atoms per pipeline stage: 0 automatic, else forced (tuning)
void run_bf16(const GemmArgs& a, cudaStream_t s);
struct GroupedGemmArgs {
  const void* A;  // [max_rows, K] expert-sorted rows
  int64_t lda;
  const void* B;  // [num_experts * N, K] stacked expert weights
  int64_t ldb;
  void* C;        // [max_rows, N] (N/2 with SwiGLU)
  int64_t ldc;
  int max_rows, N, K, num_experts, mode, bn;
  const int32_t* tile_expert;
  const int32_t* num_tiles;
  int* err;
};
void run_grouped_bf16(const GroupedGemmArgs& a, cudaStream_t s);
}  // namespace gemm

namespace gemm_fp8 {
// C[M, N] bf16 = sum over 128-wide K blocks of sa[m, kb] * sb[n / 128, kb] * (A . B^T)[kb]
struct Fp8GemmArgs {
  const void* A;  // [M, K] e4m3, row stride lda (elements = bytes)
  int64_t lda;
  const void* B;  // [N, K] e4m3, row stride ldb
  int64_t ldb;
  const float* sa;  // [M, ceil(K/128)] per-token group scales, row stride sa_ld
  int64_t sa_ld;
  const float* sb;  // [ceil(N/128), ceil(K/128)] block scales, row stride sb_ld
  int64_t sb_ld;
  void* C;  // [M, N] bf16, row stride ldc
  int64_t ldc;
  int M, N, K;
  int splits;  // 0 = planner
  float* workspace;
  long workspace_numel;
  int* counters;
  long counters_numel;
  int* err;
  // grouped (MoE) mode: B = [num_experts * N, K], sb = [num_experts * ceil(N/128), K/128]
  const int32_t* tile_expert = nullptr;
  const int32_t* num_tiles = nullptr;
  int num_experts = 0;
};
struct Fp8Plan {
  int splits;
  long workspace_floats;
  int counters;
};
Fp8Plan plan_fp8(int M, int N, int K);
void run_fp8(const Fp8GemmArgs& a, cudaStream_t stream);
}  // namespace gemm_fp8

// ------------------------------------------------------------------------------- GDN
namespace gdn {
void run_causal_conv1d(const void* x, int64_t ldx, const void* w, void* state,
                       const int32_t* cu_q, const int32_t* seq_lens, const int32_t* slots, int R,
                       int T, int C, void* out, int64_t ldo, cudaStream_t s,
                       const void* bias = nullptr);
void run_gdn_recurrent(const void* qkv, int64_t ld_qkv, const void* ba, int64_t ld_ba,
                       const float* A_log, const float* dt_bias, float* state,
                       const int32_t* cu_q, const int32_t* seq_lens, const int32_t* slots, int R,
                       int Hk, int Hv, void* out, int64_t ld_out, cudaStream_t s,
                       bool single_token = false);
void run_sigmoid_gate(void* out, int64_t ldo, const void* gate, int64_t ldg, int T, int W,
                      cudaStream_t s);
// chunked prefill (gdn_chunked.cu): workspace of chunked_workspace_bytes(max_chunks, Hv) with
// max_chunks = ceil(T / 64) + R, chunk_offsets [R + 1] int32, gam_c [max_chunks * Hv] fp32
size_t chunked_workspace_bytes(int max_chunks, int Hv);
void run_gdn_chunked(const void* qkv, int64_t ld_qkv, const void* ba, int64_t ld_ba,
                     const float* A_log, const float* dt_bias, float* state, const int32_t* cu_q,
                     const int32_t* seq_lens, const int32_t* slots, int32_t* chunk_offsets,
                     void* ws, float* gam_c, int R, int T, int Hk, int Hv, void* out,
                     int64_t ld_out, cudaStream_t s);
}  // namespace gdn

// ------------------------------------------------------------------------------- MoE
namespace moe {
void run_topk_softmax(const float* logits, int64_t ld, int T, int E, int k, bool renorm,
                      int32_t* ids, float* w, cudaStream_t s);
void run_grouped_topk(const float* logits, const float* bias, int T, int E, int k, int n_group,
                      int topk_group, bool sigmoid, bool renorm, float scale, int32_t* ids,
                      float* w, cudaStream_t s);
int align_max_rows(int n, int E);
void run_moe_align(const int32_t* ids, int n, int E, int e0, int max_rows, int32_t* sorted_ids,
                   int32_t* tile_expert, int32_t* offsets, int32_t* pos, int32_t* num_tiles,
                   cudaStream_t s);
void run_moe_gather(const void* x, int64_t ldx, const int32_t* sorted_ids, const int32_t* num_tiles,
                    int max_rows, int k, int H, void* out, cudaStream_t s);
void run_moe_combine(const void* y, const int32_t* pos, const float* w, int T, int k, int H,
                     const void* shared, const float* shared_gate, int64_t ld_gate, void* out,
                     int64_t ldo, cudaStream_t s);
// Routed bf16 experts for a few tokens as per-(token, slot) GEMVs: h = SwiGLU(x W_gu_e^T)
// [T*k, I], y = h W_down_e^T [T*k, H], pos [T, k] = pair index or -1 (expert not local);
// combine with run_moe_combine.  w_gu / w_down in the grouped-GEMM layouts.
bool moe_gemv_supported(int H, int I);
void run_moe_gemv(const void* x, int64_t ldx, const int32_t* ids, int T, int k, int E, int e0,
                  const void* w_gu, const void* w_down, int H, int I, void* h, void* y,
                  int32_t* pos, cudaStream_t s);
}  // namespace moe

// ------------------------------------------------------------------------------- norms
namespace norm {
struct RmsNormArgs {
  void* out;
  int64_t ld_out;
  void* x;
  int64_t ld_x;
  void* residual;  // nullptr: plain RMSNorm; else residual += x (in place) first
  int64_t ld_res;
  const void* weight;
  int rows, H;
  float eps;
  bool gemma;
};
void run_rms_norm(const RmsNormArgs& a, cudaStream_t s);
void run_rms_norm_gated(void* out, int64_t ldo, const void* x, int64_t ldx, const void* z,
                        int64_t ldz, const void* w, int rows, int H, int group, float eps,
                        cudaStream_t s);
// (residual += x;) y = RMSNorm(residual or x) * w -> e4m3 [rows, H] + fp32 1x128 scales
// (+ bf16 y when `out` is non-null).
void run_rms_norm_quant_fp8(void* q, int64_t ld_q, float* scales, void* out, int64_t ld_out,
                            const void* x, int64_t ld_x, void* residual, int64_t ld_res,
                            const void* weight, int rows, int H, float eps, cudaStream_t s);
}  // namespace norm

// ------------------------------------------------------------------------------- activations
namespace act {
void run_act_and_mul(void* out, int64_t ld_out, const void* x, int64_t ld_x, int rows, int I,
                     int kind, float limit, cudaStream_t s);
void run_silu_mul_fp8_quant(void* out, float* scales, const void* x, int64_t ld_x, int rows, int I,
                            cudaStream_t s, float limit = 0.f);
void run_group_quant_fp8(void* out, float* scales, const void* x, int64_t ld_x, int rows, int K,
                         cudaStream_t s);
}  // namespace act

// ------------------------------------------------------------------------------- Mamba2
namespace mamba {
struct Mamba2Args {
  const void* xbc;           // bf16 conv output rows: x [H*P] at 0, B [G*N] at b_off, C at c_off
  int64_t ld_xbc;
  int b_off, c_off;
  const void* dt;            // bf16 raw dt [T, >= H] (row stride ld_dt)
  int64_t ld_dt;
  const float* dt_bias;      // [H]
  const float* A_log;        // [H]
  const float* D;            // [H]
  float* state;              // [slots, H, P, N] fp32
  const int32_t* cu_q;
  const int32_t* seq_lens;
  const int32_t* slots;
  void* y;                   // bf16 [T, H*P]
  int64_t ld_y;
  int R, H, G, P, N;
  float dt_min, dt_max;
};
void run_mamba2_scan(const Mamba2Args& a, cudaStream_t s);
// Chunked SSD prefill (64-token chunks, three launches; same contract as run_mamba2_scan).
// T = tokens of the batch; workspaces sized by mamba2_chunked_max_chunks(T, R).
bool mamba2_chunked_supported(int P, int N, int64_t ld_xbc, int b_off, int c_off, int64_t ld_y);
size_t mamba2_chunked_max_chunks(int T, int R);
void run_mamba2_chunked(const Mamba2Args& a, int T, int32_t* chunk_offsets, float* states,
                        void* start_bf16, float* decay, cudaStream_t s);
// out = RMSNorm over groups of `group` channels of (y * silu(z)), times w
void run_gated_rmsnorm(void* out, int64_t ld_o, const void* y, int64_t ld_y, const void* z,
                       int64_t ld_z, const void* w, int T, int C, int group, float eps,
                       cudaStream_t s);
}  // namespace mamba

// ------------------------------------------------------------------------------- W4AFP8 MoE
namespace w4a8 {
// packed int4 [E, N, K/2] x bf16 scales [E, N, K/128] -> bf16 [E * N, K]; experts whose padded
// row range (offsets[e], offsets[e + 1]) is empty are skipped (offsets may be null: expand all).
void run_w4_dequant(void* out, const void* packed, const void* scales, const int32_t* offsets,
                    int E, int N, int K, cudaStream_t s);
// per-row e4m3 quantise -> dequantise round trip (optionally of SwiGLU(+clamp) of [gate | up]);
// rows at or past num_tiles[0] * 128 are skipped when num_tiles is given.
void run_row_fp8_qdq(void* out, const void* x, int64_t ld_x, int rows, int C, bool swiglu,
                     float limit, const int32_t* num_tiles, cudaStream_t s);
}  // namespace w4a8

// ------------------------------------------------------------------------------- rope + kv
namespace rope {
// Multimodal RoPE: mode 0 off, 1 sectioned (s0 | s1 | s2 frequencies), 2 interleaved;
// positions are [3, pos_stride] int32 (temporal, height, width rows).
struct MropeSpec {
  int mode = 0, s0 = 0, s1 = 0, s2 = 0;
  int64_t pos_stride = 0;
};
struct RopeKvArgs {
  void* qkv;
  int64_t ld_qkv;
  const int32_t* positions;
  const float* cos_sin;
  const void* q_norm_w;  // optional
  const void* k_norm_w;  // optional
  void* k_cache;
  void* v_cache;
  const int32_t* slot_mapping;
  int T, Hq, Hkv, D, block_size, rot_dim;
  bool neox;
  float eps;
  int* err;
  MropeSpec mrope;
};
void run_rope_kv(const RopeKvArgs& a, cudaStream_t s);
// Paged cache insert of separate key / value tensors [T, Hkv, D] (row stride *_ld, head stride
// *_hs, in elements); caches [num_blocks, Hkv, block_size, D]; int64 slots, < 0 skipped.
void run_kv_insert(const void* key, int64_t k_ld, int64_t k_hs, const void* value, int64_t v_ld,
                   int64_t v_hs, void* k_cache, void* v_cache, const int64_t* slot_mapping, int T,
                   int Hkv, int D, int block_size, cudaStream_t s);
}  // namespace rope

// ------------------------------------------------------------------------------- attention
namespace attn {
struct DecodeArgs {
  const void* q;
  int64_t ld_q;
  void* o;
  int64_t ld_o;
  void* k_cache;
  void* v_cache;
  int num_blocks;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* seq_lens;
  int B, Hq, Hkv, D, block_size, max_seq_len, num_splits;
  float scale;
  float* ws_o;
  float* ws_lse;
  int* err;
  const float* sinks = nullptr;  // [Hq] per-head sink logits (softmax-only column), or null
};
struct PrefillArgs {
  const void* q;
  int64_t ld_q;
  void* o;
  int64_t ld_o;
  void* k_cache;
  void* v_cache;
  int num_blocks;
  const int32_t* cu_q;
  const int32_t* seq_lens;
  const int32_t* block_tables;
  int64_t bt_stride;
  int32_t* tile_offsets;  // scratch [R+1]
  int T, R, Hq, Hkv, D, block_size, window;
  float scale;
  int* err;
  const float* sinks = nullptr;  // [Hq] per-head sink logits, or null
  bool causal = true;            // false: every query sees its request's whole sequence
  // tree attention (speculative token trees): per query row t, bit j of tree_mask[t] lets it
  // see draft token j of its request (the request's last q_len <= 64 positions); the cached
  // context before them stays visible.  Null: plain causal.
  const uint64_t* tree_mask = nullptr;
};
// head_dim 128 prefill on tcgen05 (prefill_tc.cu); B200_ATTN_TC=0 selects the mma.sync kernel.
bool prefill_tc_enabled(int D);
void set_prefill_tc(bool on);
// two query heads per CTA (even GQA group; prefill_tc2.cu); B200_ATTN_TC2=0 disables
bool prefill_tc2_supported(int D, int Hq, int Hkv);
void set_prefill_tc2(bool on);
void run_prefill_tc2(const PrefillArgs& a, cudaStream_t stream);
void run_prefill_tc(const PrefillArgs& a, cudaStream_t stream);
int decode_num_splits(int B, int Hkv, int max_seq_len);
void run_decode(const DecodeArgs& a, cudaStream_t s);
void run_prefill(const PrefillArgs& a, cudaStream_t s);
}  // namespace attn

// --------------------------------------------------------------- TurboQuant KV cache
// Quantised KV cache: per (token, KV head) one slot of slot_bytes(D, kb, vb) bytes (key codes,
// value codes, three fp16 scales); csrc/attention/turboquant.cu describes the format.
namespace tq {
struct TQStoreArgs {
  const __nv_bfloat16* k;  // [T, >= Hkv*D] rows (row stride ld_k elements)
  const __nv_bfloat16* v;
  int64_t ld_k, ld_v;
  const int* slot_mapping;  // [T]; < 0 skips the token
  uint8_t* cache;           // [num_blocks, Hkv, block_size, slot_bytes]
  int T, Hkv, block_size, num_blocks, slot_bytes;
  bool norm_correction;
  int* err;
};
struct TQDecodeArgs {
  const __nv_bfloat16* q;  // [B, >= Hq*D]
  int64_t ld_q;
  __nv_bfloat16* out;      // [B, >= Hq*D]
  int64_t ld_out;
  const uint8_t* cache;
  const int* block_tables;  // [B, ld_bt]
  int ld_bt;
  const int* seq_lens;      // [B]
  int B, Hq, Hkv, block_size, num_blocks, slot_bytes;
  float scale_log2;         // softmax scale * log2(e)
  int splits;
  float* ws_o;              // [B, Hq, splits, D] when splits > 1
  float* ws_lse;            // [B, Hq, splits]
  int* err;
};
struct TQDequantArgs {
  const uint8_t* cache;
  const int* block_tables;  // [R, ld_bt]
  int ld_bt;
  const int* seq_lens;      // [R]
  __nv_bfloat16* k_out;     // [R * W, Hkv, block_size, D]
  __nv_bfloat16* v_out;
  int R, W, Hkv, block_size, num_blocks, slot_bytes;
  int* err;
};
int slot_bytes(int D, int kb, int vb);
void run_store(const TQStoreArgs& a, int D, int kb, int vb, cudaStream_t stream);
void run_decode(const TQDecodeArgs& a, int D, int kb, int vb, cudaStream_t stream);
void run_dequant(const TQDequantArgs& a, int D, int kb, int vb, cudaStream_t stream);
}  // namespace tq

namespace mla {
// Absorbed multi-head latent attention over a [slots, 576] bf16 latent cache (c_kv | k_pe).
struct MlaArgs {
  const void* q_lat;  // (t, h, c<512) at t*ql_t + h*ql_h + c
  int64_t ql_t, ql_h;
  const void* q_pe;   // (t, h, c<64) at t*qp_t + h*qp_h + c
  int64_t qp_t, qp_h;
  const void* cache;
  const int32_t* block_tables;
  int64_t bt_stride;
  int block_size;
  const int32_t* cu_q;
  const int32_t* seq_lens;
  int R;
  const int32_t* indices;  // [T, topk] token positions (-1 = none) or null for the causal prefix
  int64_t idx_ld;
  int topk;
  void* out;  // (t, h, c<512) bf16 at t*o_t + h*o_h + c
  int64_t o_t, o_h;
  float* ws_o;    // [splits, T, Hq, 512] when splits > 1
  float* ws_lse;  // [splits, T, Hq]
  int T, Hq, splits;
  float scale;
  // decode context parallelism (dense mode): the cache holds tokens p % dcp_size == dcp_rank at
  // local index p / dcp_size; lse_out (optional) [T, Hq] log2-sum-exp of the scaled scores
  int dcp_size = 1, dcp_rank = 0;
  float* lse_out = nullptr;
};
void run_prep(void* q, int64_t ld_q, int Hq, const void* kv, int64_t ld_kv, const void* kv_norm_w,
              float eps, const int32_t* positions, const float* cos_sin, void* cache,
              const int32_t* slots, int T, cudaStream_t s);
void run_attention(const MlaArgs& a, cudaStream_t s);

// DeepSeek-V3.2 lightning indexer.
struct IndexerArgs {
  const void* q;  // [T, 64 * 128] bf16 (RoPE applied), row stride ld_q
  int64_t ld_q;
  const float* w;  // [T, 64] head weights, row stride ld_w
  int64_t ld_w;
  const void* cache;  // [slots, 128] bf16 index keys
  const int32_t* block_tables;
  int64_t bt_stride;
  int block_size;
  const int32_t* cu_q;
  const int32_t* seq_lens;
  int R, T;
  float* scores;  // [T, ld_s]
  int64_t ld_s;
};
void run_indexer_k_prep(const void* k, int64_t ld_k, const void* ln_w, const void* ln_b, float eps,
                        const int32_t* positions, const float* cos_sin, void* cache,
                        const int32_t* slots, int T, cudaStream_t s);
void run_indexer_scores(const IndexerArgs& a, cudaStream_t s);
void run_topk(const float* scores, int64_t ld_s, const int32_t* cu_q, const int32_t* seq_lens,
              int R, int T, int k, int32_t* out, int64_t ld_o, cudaStream_t s);
}  // namespace mla

// ------------------------------------------------------------------------------- sampling
namespace sampling {
struct SampleArgs {
  const float* logits;
  int64_t ld;
  int R, V, vocab_offset;
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const float* min_p;
  const int64_t* seeds;
  const int32_t* steps;
  float* out_val;
  int64_t* out_idx;
};
void run_sample(const SampleArgs& a, cudaStream_t s);
void run_merge_candidates(const float* vals, const int64_t* idx, int S, int R, int64_t* out,
                          cudaStream_t s);
// Vocab-parallel top-k / top-p / min-p sampling (topk_exchange.cu): per-shard candidate rows
// (the <= kCandCap largest scaled logits with their global ids, the shard's max / exp-mass /
// completeness key and its Gumbel-max winner), exchanged over NVLink and merged per row.
constexpr int kCandCap = 128;
struct alignas(16) CandRow {
  float v[kCandCap];
  int32_t id[kCandCap];
  float m, s;        // shard max of l/T and sum exp(l/T - m)
  int32_t n;         // candidates stored
  uint32_t thr;      // every shard token with key >= thr is a candidate (0: all of them)
  float best_v;      // shard Gumbel-max winner (argmax for greedy rows)
  int32_t best_id;
  int32_t pad[2];
};
struct TopkExchangeArgs {
  int rank, world, R, parity, V_total;
  const CandRow* mine;
  CandRow* region[8];   // this call's candidate region of every rank: [world][R] rows
  uint32_t* flags[8];   // communicator flag region of every rank
  uint32_t* epochs;
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const float* min_p;
  const int64_t* seeds;
  const int32_t* steps;
  int64_t* out;         // sampled global ids, -1 where the candidates cannot decide exactly
  int* err;
};
void run_shard_candidates(const float* logits, int64_t ld, int R, int V, int vocab_offset,
                          const float* temperature, const int64_t* seeds, const int32_t* steps,
                          CandRow* out, cudaStream_t s);
void run_merge_candidates_local(const CandRow* cands, int world, int R, const float* temperature,
                                const int32_t* top_k, const float* top_p, const float* min_p,
                                const int64_t* seeds, const int32_t* steps, int V_total,
                                int64_t* out, cudaStream_t s);
void run_topk_exchange(const TopkExchangeArgs& a, cudaStream_t s);
// Repetition / presence / frequency penalties on fp32 logits [R, V_local] (row stride ld) of a
// vocab shard starting at vocab_offset.  entries [n, 3] int32 = (row, global token id, count of
// the token in the row's output so far); every listed token occurs in the prompt or the
// output (rows list each token once).
void run_token_bitmask(float* logits, int64_t ld, const int32_t* bitmask, int words,
                       const int32_t* rows, int R, int V_local, int vocab_offset, cudaStream_t s);
void run_apply_penalties(float* logits, int64_t ld, int V_local, int vocab_offset,
                         const int32_t* entries, int n, const float* rep, const float* pres,
                         const float* freq, cudaStream_t s);
}  // namespace sampling

// ------------------------------------------------------------------------------- misc
namespace misc {
void run_embedding(void* out, const void* table, const int32_t* ids, int T, int H, int64_t vocab,
                   int64_t vocab_start, cudaStream_t s);
void run_gather_rows(void* out, const void* in, int64_t ld_in, const int32_t* idx, int R, int H,
                     int elem_bytes, cudaStream_t s);
}  // namespace misc

namespace ep {
// Expert-parallel all-to-all (csrc/comm/ep_a2a.cu).  Pointer arrays hold every rank's address
// of the same buffer (peer VAs from CUDA IPC).
struct A2AParams {
  int rank, world;
  int Tc, row0;      // this rank's shard: rows [row0, row0 + Tc) of x
  int H, k, E_local;
  int cap;           // receive rows per source rank
  int rs_rows;       // rows per block of the all-reduce staging slot (= ceil(T / world))
  const void* x;     // [T, H] bf16 hidden states (replicated)
  int64_t ldx;
  const int32_t* ids;  // [Tc, k] global expert ids of the shard tokens
  const float* w;      // [Tc, k] routing weights
  int* send_cnt;       // [world] local counters (zero between calls)
  void* recv_x[8];         // [world * cap, H] bf16
  int32_t* recv_ids[8];    // [world * cap, k] local expert ids (-1: not served here)
  float* recv_w[8];        // [world * cap, k]
  int32_t* recv_tok[8];    // [world * cap] shard row of the token at its source
  int32_t* recv_cnt[8];    // [world] rows received from each source
  uint32_t* flags[8];      // [kMaxRanks] arrival epochs
  uint32_t* epoch;         // local call counter
  void* staging[8];        // all-reduce staging slots (this call's parity)
  int* err;
};
void run_dispatch(const A2AParams& p, cudaStream_t s);
void run_return(const A2AParams& p, const void* y, const int32_t* pos, cudaStream_t s);
}  // namespace ep

}  // namespace b200
