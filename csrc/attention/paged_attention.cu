// Paged attention for sm_100a: decode (split-KV, GQA-packed) and chunked prefill (causal,
// optional sliding window), reading K/V straight out of the paged cache with TMA.
//
// Cache layout [num_blocks, Hkv, block_size, D] (written by rope_kv.cu).  Viewed as a 2-D
// tensor [num_blocks*Hkv*block_size, D], a 64-token x 64-column tile is one TMA box with the
// 128-byte swizzle, so a page of one KV head arrives in shared memory in D/64 bulk tensor
// copies, bank-conflict-free for ldmatrix.  Warp roles: warp 4 is the TMA producer (ring of
// STAGES K+V stages, full/empty mbarriers with bounded waits); warps 0..3 compute with
// mma.sync m16n8k16 (bf16 in, fp32 accumulate) and an exp2-domain online softmax.
//
//  decode : CTA = (sequence, kv head, split).  The G = Hq/Hkv query heads of the group are
//           the 16 MMA rows, so each K/V byte is read once per group.  Warp w owns tokens
//           [16w, 16w+16) of every 64-token chunk; the four warp states are merged in shared
//           memory, and splits are merged by attn_combine_kernel (log-sum-exp weights).
//  prefill: CTA = (64-query tile, query head), causal over the request's cached context + its
//           own new tokens (chunked prefill reads earlier chunks back from the cache).
//
// Reference counterparts: the MATE FA3 varlen kernel the reference calls through
// vllm_musa/v1/attention/backends/flash_attn.py:1186-1537 (no source in the reference), split
// metadata from vllm_musa/jit_kernel/fa3_metadata.py:29.
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "../common/mma_sm80.cuh"
#include "../common/tma_host.h"

namespace b200 {
namespace attn {

constexpr int CH = 64;  // KV tokens per stage
constexpr int kComputeWarps = 4;
constexpr int kThreads = (kComputeWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Cfg {
  static constexpr int NH = D / 64;                  // 64-column halves per row
  static constexpr int kHalfBytes = CH * 128;        // one 64x64 bf16 tile
  static constexpr int kKvBytes = NH * kHalfBytes;   // K (or V) of one stage
  static constexpr int kStageBytes = 2 * kKvBytes;
};

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t ld_q;
  __nv_bfloat16* o;
  int64_t ld_o;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* seq_lens;
  int B, Hq, Hkv, block_size, num_splits, chunks_per_split;
  float scale_log2;
  float* ws_o;    // [B, Hq, splits, D]
  float* ws_lse;  // [B, Hq, splits]
  int* err;
  const float* sinks;  // [Hq] natural-log sink logits or null
};

struct PrefillParams {
  __nv_bfloat16* o;
  int64_t ld_o;
  const int32_t* cu_q;
  const int32_t* seq_lens;
  const int32_t* block_tables;
  int64_t bt_stride;
  const int32_t* tile_offsets;  // [R+1]
  int R, max_tiles, Hq, Hkv, block_size, window;
  float scale_log2;
  int* err;
  const float* sinks;  // [Hq] natural-log sink logits or null
  bool causal;
  const uint64_t* tree_mask;  // per query row: visible draft tokens (bit j), or null
};

// A sink is a softmax column with no value: it only adds 2^(sink * log2 e - m) to the row sum.
B200_DEVICE float sink_term(const float* sinks, int head, float m_log2) {
  return sinks == nullptr ? 0.f : exp2f(sinks[head] * kLog2e - m_log2);
}

B200_DEVICE void named_barrier_compute() {
  asm volatile("bar.sync 1, %0;" ::"n"(kComputeWarps * 32) : "memory");
}

// Issue the TMA loads of one 64-token chunk of K and V for kv head `h` into a stage.
template <int D>
B200_DEVICE void load_chunk(const CUtensorMap* tmK, const CUtensorMap* tmV, uint8_t* sK,
                            uint8_t* sV, uint64_t* bar, const int32_t* bt, int chunk, int n_tok,
                            int h, int Hkv, int block_size) {
  using C = Cfg<D>;
  const int box_rows = block_size < CH ? block_size : CH;
  const int sub = CH / box_rows;
  const int last_page = (n_tok - 1) / block_size;
  mbar_arrive_expect_tx(bar, C::kStageBytes);
  for (int j = 0; j < sub; ++j) {
    const int tok = chunk * CH + j * box_rows;
    int page = tok / block_size;
    if (page > last_page) page = last_page;  // beyond the sequence: any valid page (masked)
    const int off = tok % block_size;
    const int blk = bt[page];
    const int row = (blk * Hkv + h) * block_size + off;
#pragma unroll
    for (int hh = 0; hh < C::NH; ++hh) {
      tma_load_2d(sK + hh * C::kHalfBytes + j * box_rows * 128, tmK, bar, hh * 64, row);
      tma_load_2d(sV + hh * C::kHalfBytes + j * box_rows * 128, tmV, bar, hh * 64, row);
    }
  }
}

// S(16 x 16 tokens of this warp) = Q(16 x D) K^T.  qa: A fragments per 16-wide k slice.
template <int D>
B200_DEVICE void qk_16(float (&s)[2][4], const uint32_t (&qa)[D / 16][4], uint32_t sK, int tw,
                       int lane) {
  using C = Cfg<D>;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) s[nt][j] = 0.f;
  const int m = lane >> 3, r = lane & 7;
  const int tok = tw + (m >> 1) * 8 + r;
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
    const int hh = ks / 4, c0 = (ks % 4) * 2;
    uint32_t b0, b1, b2, b3;
    mma::ldsm_x4(mma::sw128(sK + hh * C::kHalfBytes, tok, c0 + (m & 1)), b0, b1, b2, b3);
    mma::mma_bf16(s[0], qa[ks], b0, b1);
    mma::mma_bf16(s[1], qa[ks], b2, b3);
  }
}

template <int D, int STAGES>
__global__ void __launch_bounds__(kThreads)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  DecodeParams p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::kStageBytes);
  uint64_t* empty = full + STAGES;

  pdl_launch_dependents();
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = p.Hq / p.Hkv;
  const int n_tok = p.seq_lens[b];
  const int n_chunks = (n_tok + CH - 1) / CH;
  const int c0 = split * p.chunks_per_split;
  const int c1 = min(n_chunks, c0 + p.chunks_per_split);
  const int nc = c1 > c0 ? c1 - c0 : 0;
  const int32_t* bt = p.block_tables + b * p.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kComputeWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kComputeWarps) {
    if (lane == 0 && nc > 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < nc; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) break;
        uint8_t* st = smem + stage * C::kStageBytes;
        load_chunk<D>(&tmK, &tmV, st, st + C::kKvBytes, &full[stage], bt, c0 + i, n_tok, h,
                      p.Hkv, p.block_size);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    return;  // producer warp takes no part in the merge below
  }

  // ---- compute warps ----
  const int g = lane >> 2, t = lane & 3;
  // Q fragments (rows = heads of this group, zero beyond G).
  uint32_t qa[D / 16][4];
  {
    const __nv_bfloat16* q0 = p.q + b * p.ld_q + (int64_t)(h * G) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int row = g + (j & 1) * 8;
        const int col = ks * 16 + 2 * t + (j >> 1) * 8;
        float x0 = 0.f, x1 = 0.f;
        if (row < G) {
          const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(q0 + row * D + col);
          x0 = __low2float(v);
          x1 = __high2float(v);
        }
        qa[ks][j] = pack_bf16x2(x0, x1);
      }
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int tw = warp * 16;
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int i = 0; i < nc; ++i) {
    if (!mbar_wait(&full[stage], phase, p.err)) {
      ok = false;
      break;
    }
    const uint32_t sK = smem_u32(smem + stage * C::kStageBytes);
    const uint32_t sV = sK + C::kKvBytes;
    float s[2][4];
    qk_16<D>(s, qa, sK, tw, lane);
    // scale into the exp2 domain; mask tokens past the sequence end
    const int tok0 = (c0 + i) * CH + tw;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        s[nt][j] = (tok0 + nt * 8 + 2 * t + (j & 1) >= n_tok) ? -INFINITY : s[nt][j] * p.scale_log2;
    // online softmax on rows g (j=0,1) and g+8 (j=2,3)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      float mx = fmaxf(fmaxf(s[0][2 * rr], s[0][2 * rr + 1]), fmaxf(s[1][2 * rr], s[1][2 * rr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(mrow[rr], mx);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      const float corr = exp2f(mrow[rr] - muse);
      mrow[rr] = mnew;
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][2 * rr] = exp2f(s[nt][2 * rr] - muse);
        s[nt][2 * rr + 1] = exp2f(s[nt][2 * rr + 1] - muse);
        sum += s[nt][2 * rr] + s[nt][2 * rr + 1];
      }
      lrow[rr] = lrow[rr] * corr + sum;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[dt][2 * rr] *= corr;
        o[dt][2 * rr + 1] *= corr;
      }
    }
    uint32_t pa[4];
    pa[0] = pack_bf16x2(s[0][0], s[0][1]);
    pa[1] = pack_bf16x2(s[0][2], s[0][3]);
    pa[2] = pack_bf16x2(s[1][0], s[1][1]);
    pa[3] = pack_bf16x2(s[1][2], s[1][3]);
    {
      const int m = lane >> 3, r = lane & 7;
      const int tok = tw + (m & 1) * 8 + r;
#pragma unroll
      for (int dn = 0; dn < D / 16; ++dn) {
        const int hh = dn / 4, cc = (dn % 4) * 2;
        uint32_t b0, b1, b2, b3;
        mma::ldsm_x4_t(mma::sw128(sV + hh * C::kHalfBytes, tok, cc + (m >> 1)), b0, b1, b2, b3);
        mma::mma_bf16(o[2 * dn], pa, b0, b1);
        mma::mma_bf16(o[2 * dn + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1;
    }
  }
  (void)ok;
  // quad-reduce the row sums
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    lrow[rr] += __shfl_xor_sync(0xffffffffu, lrow[rr], 1);
    lrow[rr] += __shfl_xor_sync(0xffffffffu, lrow[rr], 2);
  }
  // ---- merge the 4 warp states (rows < G only) through shared memory ----
  named_barrier_compute();  // every warp is done reading the stages
  float* sm_o = reinterpret_cast<float*>(smem);                  // [4][16][D]
  float* sm_m = sm_o + kComputeWarps * 16 * D;                    // [4][16]
  float* sm_l = sm_m + kComputeWarps * 16;                        // [4][16]
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int row = g + rr * 8;
    if (row < G) {
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        sm_o[(warp * 16 + row) * D + dt * 8 + 2 * t] = o[dt][2 * rr];
        sm_o[(warp * 16 + row) * D + dt * 8 + 2 * t + 1] = o[dt][2 * rr + 1];
      }
      if (t == 0) {
        sm_m[warp * 16 + row] = mrow[rr];
        sm_l[warp * 16 + row] = lrow[rr];
      }
    }
  }
  named_barrier_compute();
  const int total = G * D;
  for (int e = threadIdx.x; e < total; e += kComputeWarps * 32) {
    const int row = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) M = fmaxf(M, sm_m[w * 16 + row]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) {
      const float f = exp2f(sm_m[w * 16 + row] - Mu);
      L += f * sm_l[w * 16 + row];
      acc += f * sm_o[(w * 16 + row) * D + d];
    }
    const int head = h * G + row;
    const float Ls = (p.num_splits == 1 && L > 0.f) ? L + sink_term(p.sinks, head, Mu) : L;
    const float out = L > 0.f ? acc / Ls : 0.f;
    if (p.num_splits == 1) {
      p.o[b * p.ld_o + (int64_t)head * D + d] = f2bf(out);
    } else {
      const int64_t idx = ((int64_t)b * p.Hq + head) * p.num_splits + split;
      p.ws_o[idx * D + d] = out;
      if (d == 0) p.ws_lse[idx] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

// Merge split-KV partials: O = sum_s 2^(lse_s - M) O_s / sum_s 2^(lse_s - M)
__global__ void attn_combine_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_lse,
                                    __nv_bfloat16* __restrict__ o, int64_t ld_o, int Hq, int S,
                                    int D, const float* __restrict__ sinks) {
  const int b = blockIdx.x, head = blockIdx.y;
  const int64_t base = ((int64_t)b * Hq + head) * S;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, ws_lse[base + s]);
  const float Mu = M == -INFINITY ? 0.f : M;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, acc = 0.f;
    for (int s = 0; s < S; ++s) {
      const float f = exp2f(ws_lse[base + s] - Mu);
      L += f;
      acc += f * ws_o[(base + s) * D + d];
    }
    o[b * ld_o + (int64_t)head * D + d] =
        f2bf(L > 0.f ? acc / (L + sink_term(sinks, head, Mu)) : 0.f);
  }
}

// ------------------------------------------------------------------------------------------
// Prefill
// ------------------------------------------------------------------------------------------
__global__ void tile_offsets_kernel(const int32_t* __restrict__ cu_q, int R, int32_t* __restrict__ out) {
  // single warp-strided prefix sum over R requests (R is small: the prefill batch)
  if (threadIdx.x == 0) {
    int acc = 0;
    out[0] = 0;
    for (int r = 0; r < R; ++r) {
      const int ql = cu_q[r + 1] - cu_q[r];
      acc += (ql + CH - 1) / CH;
      out[r + 1] = acc;
    }
  }
}

template <int D, int STAGES>
__global__ void __launch_bounds__(kThreads)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, PrefillParams p) {
  using C = Cfg<D>;
  constexpr int kQBytes = C::NH * C::kHalfBytes;  // 64 rows x D
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + kQBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sKV + STAGES * C::kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* qbar = empty + STAGES;

  pdl_launch_dependents();
  const int tile = p.max_tiles - 1 - blockIdx.x;  // longest-context tiles first
  const int head = blockIdx.y;
  const int total_tiles = p.tile_offsets[p.R];
  if (tile >= total_tiles) return;
  // request owning this tile
  int lo = 0, hi = p.R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.tile_offsets[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  const int r = lo;
  const int q_begin = p.cu_q[r], q_end = p.cu_q[r + 1];
  const int q0 = q_begin + (tile - p.tile_offsets[r]) * CH;
  const int rows = min(CH, q_end - q0);
  const int seq_len = p.seq_lens[r];
  const int ctx = seq_len - (q_end - q_begin);
  const int pos0 = ctx + (q0 - q_begin);          // position of tile row 0
  const int pos_last = pos0 + rows - 1;
  const int n_chunks = p.causal ? pos_last / CH + 1 : (seq_len + CH - 1) / CH;
  int first_chunk = 0;
  if (p.window > 0) first_chunk = max(0, pos0 - p.window + 1) / CH;
  const int nc = n_chunks - first_chunk;
  const int G = p.Hq / p.Hkv;
  const int h = head / G;
  const int32_t* bt = p.block_tables + r * p.bt_stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kComputeWarps);
    }
    mbar_init(qbar, 1);
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kComputeWarps) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      mbar_arrive_expect_tx(qbar, kQBytes);
#pragma unroll
      for (int hh = 0; hh < C::NH; ++hh)
        tma_load_2d(sQ + hh * C::kHalfBytes, &tmQ, qbar, head * D + hh * 64, q0);
      int stage = 0;
      uint32_t phase = 0;
      for (int i = 0; i < nc; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err)) break;
        uint8_t* st = sKV + stage * C::kStageBytes;
        load_chunk<D>(&tmK, &tmV, st, st + C::kKvBytes, &full[stage], bt, first_chunk + i,
                      seq_len, h, p.Hkv, p.block_size);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    return;
  }

  const int g = lane >> 2, t = lane & 3;
  const int tw = warp * 16;  // this warp's query rows
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  if (!mbar_wait(qbar, 0, p.err)) return;
  const uint32_t sQa = smem_u32(sQ);
  const int my_pos[2] = {pos0 + tw + g, pos0 + tw + g + 8};
  uint64_t tmask[2] = {0, 0};
  if (p.tree_mask != nullptr) {
#pragma unroll
    for (int rr = 0; rr < 2; ++rr)
      if (tw + g + rr * 8 < rows) tmask[rr] = p.tree_mask[q0 + tw + g + rr * 8];
  }
  int stage = 0;
  uint32_t phase = 0;
  for (int i = 0; i < nc; ++i) {
    if (!mbar_wait(&full[stage], phase, p.err)) break;
    const int chunk = first_chunk + i;
    const uint32_t sK = smem_u32(sKV + stage * C::kStageBytes);
    const uint32_t sV = sK + C::kKvBytes;
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[nt][j] = 0.f;
    const int m = lane >> 3, rr8 = lane & 7;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int hh = ks / 4, c0 = (ks % 4) * 2;
      uint32_t qa[4];
      // A fragment: matrices (rows 0-7, c0), (rows 8-15, c0), (rows 0-7, c0+1), (rows 8-15, c0+1)
      mma::ldsm_x4(mma::sw128(sQa + hh * C::kHalfBytes, tw + (m & 1) * 8 + rr8, c0 + (m >> 1)),
                   qa[0], qa[1], qa[2], qa[3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int tok = np * 16 + (m >> 1) * 8 + rr8;
        mma::ldsm_x4(mma::sw128(sK + hh * C::kHalfBytes, tok, c0 + (m & 1)), b0, b1, b2, b3);
        mma::mma_bf16(s[2 * np], qa, b0, b1);
        mma::mma_bf16(s[2 * np + 1], qa, b2, b3);
      }
    }
    // scale + causal / window mask
    const int kv0 = chunk * CH;
    // tree rows mask the step's own tokens; zero tree rows (and causal launches) mask by
    // position
    const bool causal_cut = (kv0 + CH - 1 > pos0 + tw) || (p.window > 0);
    const bool need_mask = p.tree_mask != nullptr ? (kv0 + CH > ctx) || causal_cut
                         : p.causal ? causal_cut
                                    : kv0 + CH > seq_len;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float v = s[nt][j] * p.scale_log2;
        if (need_mask) {
          const int kv = kv0 + nt * 8 + 2 * t + (j & 1);
          const int qp = p.causal ? my_pos[j >> 1] : seq_len - 1;
          if (p.tree_mask != nullptr && tmask[j >> 1] != 0) {
            const int d = kv - ctx;  // draft index; the context before the drafts is visible
            if (kv >= seq_len || (d >= 0 && (d >= 64 || !((tmask[j >> 1] >> d) & 1ull))))
              v = -INFINITY;
          } else if (kv > qp || (p.window > 0 && kv <= qp - p.window)) {
            v = -INFINITY;
          }
        }
        s[nt][j] = v;
      }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) mx = fmaxf(mx, fmaxf(s[nt][2 * rr], s[nt][2 * rr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(mrow[rr], mx);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      const float corr = exp2f(mrow[rr] - muse);
      mrow[rr] = mnew;
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        s[nt][2 * rr] = exp2f(s[nt][2 * rr] - muse);
        s[nt][2 * rr + 1] = exp2f(s[nt][2 * rr + 1] - muse);
        sum += s[nt][2 * rr] + s[nt][2 * rr + 1];
      }
      lrow[rr] = lrow[rr] * corr + sum;
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[dt][2 * rr] *= corr;
        o[dt][2 * rr + 1] *= corr;
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      const int tok = kk * 16 + (m & 1) * 8 + rr8;
#pragma unroll
      for (int dn = 0; dn < D / 16; ++dn) {
        const int hh = dn / 4, cc = (dn % 4) * 2;
        uint32_t b0, b1, b2, b3;
        mma::ldsm_x4_t(mma::sw128(sV + hh * C::kHalfBytes, tok, cc + (m >> 1)), b0, b1, b2, b3);
        mma::mma_bf16(o[2 * dn], pa, b0, b1);
        mma::mma_bf16(o[2 * dn + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1;
    }
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    lrow[rr] += __shfl_xor_sync(0xffffffffu, lrow[rr], 1);
    lrow[rr] += __shfl_xor_sync(0xffffffffu, lrow[rr], 2);
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int row = tw + g + rr * 8;
    if (row >= rows) continue;
    const float mu = mrow[rr] == -INFINITY ? 0.f : mrow[rr];
    const float inv = lrow[rr] > 0.f ? 1.f / (lrow[rr] + sink_term(p.sinks, head, mu)) : 0.f;
    __nv_bfloat16* dst = p.o + (int64_t)(q0 + row) * p.ld_o + (int64_t)head * D;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      *reinterpret_cast<uint32_t*>(dst + dt * 8 + 2 * t) =
          pack_bf16x2(o[dt][2 * rr] * inv, o[dt][2 * rr + 1] * inv);
    }
  }
}

// ------------------------------------------------------------------------------------------
// Host launchers
// ------------------------------------------------------------------------------------------
static CUtensorMap cache_map(void* base, int64_t rows, int D, int box_rows) {
  return make_tma_2d(base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, rows, D, 64, box_rows,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

template <typename K>
static void set_smem(K kern, int bytes) {
  ensure_dynamic_smem(reinterpret_cast<const void*>(kern), bytes);
}

int decode_num_splits(int B, int Hkv, int max_seq_len) {
  const int ctas = B * Hkv;
  const int target = 2 * num_sms();
  if (ctas >= target) return 1;
  const int max_chunks = (max_seq_len + CH - 1) / CH;
  int s = (target + ctas - 1) / ctas;
  s = std::min(s, std::max(1, max_chunks / 2));
  return std::max(1, std::min(s, 64));
}

void run_decode(const DecodeArgs& a, cudaStream_t stream) {
  if (a.B == 0) return;
  B200_REQUIRE(a.Hq % a.Hkv == 0 && a.Hq / a.Hkv <= 16, "decode: GQA group must be <= 16");
  B200_REQUIRE(a.block_size % 16 == 0 && (a.block_size <= 64 || a.block_size % 64 == 0),
               "decode: block_size must be 16, 32, 64 or a multiple of 64");
  const int box_rows = std::min(a.block_size, CH);
  const int64_t cache_rows = (int64_t)a.num_blocks * a.Hkv * a.block_size;
  const CUtensorMap tk = cache_map(a.k_cache, cache_rows, a.D, box_rows);
  const CUtensorMap tv = cache_map(a.v_cache, cache_rows, a.D, box_rows);
  DecodeParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(a.q);
  p.ld_q = a.ld_q;
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.ld_o = a.ld_o;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.seq_lens = a.seq_lens;
  p.B = a.B;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.block_size = a.block_size;
  p.num_splits = std::max(1, a.num_splits);
  const int max_chunks = (a.max_seq_len + CH - 1) / CH;
  p.chunks_per_split = (max_chunks + p.num_splits - 1) / p.num_splits;
  p.scale_log2 = a.scale * kLog2e;
  p.ws_o = a.ws_o;
  p.ws_lse = a.ws_lse;
  p.err = a.err;
  p.sinks = a.sinks;
  if (p.num_splits > 1)
    B200_REQUIRE(a.ws_o && a.ws_lse, "decode: split-KV needs a workspace");
  dim3 grid(a.B, a.Hkv, p.num_splits);
#define B200_DEC(DD)                                                                      \
  {                                                                                       \
    constexpr int ST = 3;                                                                 \
    const int smem = ST * Cfg<DD>::kStageBytes + 1024 + 256;                              \
    B200_REQUIRE(smem >= kComputeWarps * 16 * (DD + 2) * 4 + 1024, "decode smem");        \
    set_smem(decode_kernel<DD, ST>, smem);                                                \
    decode_kernel<DD, ST><<<grid, kThreads, smem, stream>>>(tk, tv, p);                    \
  }
  if (a.D == 64)
    B200_DEC(64)
  else if (a.D == 128)
    B200_DEC(128)
  else if (a.D == 256)
    B200_DEC(256)
  else
    B200_REQUIRE(false, "decode: head_dim must be 64, 128 or 256");
#undef B200_DEC
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
  if (p.num_splits > 1) {
    attn_combine_kernel<<<dim3(a.B, a.Hq), 128, 0, stream>>>(a.ws_o, a.ws_lse, p.o, a.ld_o, a.Hq,
                                                             p.num_splits, a.D, a.sinks);
    B200_CUDA_OK(cudaGetLastError());
  count_launch();
  }
}

void run_prefill(const PrefillArgs& a, cudaStream_t stream) {
  if (a.R == 0 || a.T == 0) return;
  B200_REQUIRE(a.Hq % a.Hkv == 0, "prefill: Hq must be a multiple of Hkv");
  B200_REQUIRE(a.block_size % 16 == 0 && (a.block_size <= 64 || a.block_size % 64 == 0),
               "prefill: block_size must be 16, 32, 64 or a multiple of 64");
  B200_REQUIRE((a.ld_q * 2) % 16 == 0, "prefill: q row stride must be a multiple of 16 bytes");
  B200_REQUIRE(a.causal || a.window == 0, "prefill: a sliding window needs causal attention");
  // the tcgen05 kernels serve the causal, sink-free case; the rest runs on the kernel below
  if (a.causal && a.sinks == nullptr && a.tree_mask == nullptr && prefill_tc_enabled(a.D)) {
    run_prefill_tc(a, stream);
    return;
  }
  const int box_rows = std::min(a.block_size, CH);
  const int64_t cache_rows = (int64_t)a.num_blocks * a.Hkv * a.block_size;
  const CUtensorMap tk = cache_map(a.k_cache, cache_rows, a.D, box_rows);
  const CUtensorMap tv = cache_map(a.v_cache, cache_rows, a.D, box_rows);
  const CUtensorMap tq = make_tma_2d(const_cast<void*>(a.q), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                     (uint64_t)a.Hq * a.D, a.T, a.ld_q, 64, CH,
                                     CU_TENSOR_MAP_SWIZZLE_128B);
  tile_offsets_kernel<<<1, 32, 0, stream>>>(a.cu_q, a.R, a.tile_offsets);
  count_launch();
  PrefillParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.ld_o = a.ld_o;
  p.cu_q = a.cu_q;
  p.seq_lens = a.seq_lens;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.tile_offsets = a.tile_offsets;
  p.R = a.R;
  p.max_tiles = (a.T + CH - 1) / CH + a.R;
  p.Hq = a.Hq;
  p.Hkv = a.Hkv;
  p.block_size = a.block_size;
  p.window = a.window;
  p.scale_log2 = a.scale * kLog2e;
  p.err = a.err;
  p.sinks = a.sinks;
  p.causal = a.causal;
  p.tree_mask = a.tree_mask;
  dim3 grid(p.max_tiles, a.Hq);
#define B200_PRE(DD)                                                                      \
  {                                                                                       \
    constexpr int ST = 2;                                                                 \
    const int smem = Cfg<DD>::NH * Cfg<DD>::kHalfBytes + ST * Cfg<DD>::kStageBytes + 1024 + 256; \
    set_smem(prefill_kernel<DD, ST>, smem);                                               \
    prefill_kernel<DD, ST><<<grid, kThreads, smem, stream>>>(tq, tk, tv, p);               \
  }
  if (a.D == 64)
    B200_PRE(64)
  else if (a.D == 128)
    B200_PRE(128)
  else if (a.D == 256)
    B200_PRE(256)
  else
    B200_REQUIRE(false, "prefill: head_dim must be 64, 128 or 256");
#undef B200_PRE
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace attn
}  // namespace b200
