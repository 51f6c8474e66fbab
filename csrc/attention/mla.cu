// Multi-head latent attention (DeepSeek-V2/V3/V3.2) and the V3.2 lightning indexer, sm_100a.
//
// Cache: one latent row per token, [num_blocks * block_size, 576] bf16 = c_kv (512, RMSNormed)
// | k_pe (64, rotated).  Attention runs in the absorbed (MQA) form for prefill and decode:
//     q_lat[h] = q_nope[h] . W_kb[h]      (512, computed by the caller)
//     s(t, j)  = (q_lat[h] . c_kv[j] + q_pe[h] . k_pe[j]) * scale
//     o_lat[h] = softmax_j(s) . c_kv      (512; the caller applies W_vb and o_proj)
// over either the causal prefix of the token (dense) or an explicit list of token positions
// per query token (DeepSeek sparse attention: the indexer's top-k).
//
//   mla_prep_kernel       q_pe RoPE in place; c_kv RMSNorm + k_pe RoPE + cache insert.
//   mla_attn_kernel       grid (query token, 16-head group, KV split).  8 warps; per 64-key tile
//                         (cp.async gather through the block table or the index list) warp w
//                         scores keys 8w..8w+7 for the 16 heads (mma.sync m16n8k16 over the
//                         576-wide rows), the tile's scores meet in shared memory for the online
//                         softmax, and warp w accumulates output columns 64w..64w+63 over all
//                         64 keys (the 512-wide fp32 row block is split across warps so it stays
//                         in registers).  Split partials are merged by mla_combine_kernel.
//   indexer_k_prep_kernel LayerNorm + RoPE of the indexer key, insert into the index cache.
//   indexer_score_kernel  score(t, j) = sum_h w[t, h] * relu(q[t, h] . k[j]) for 64 heads x 128
//                         dims, 64 keys per step, causal prefix only (others -inf).
//   topk_kernel           per-row top-k positions by a 4-pass radix select on order-preserving
//                         keys (rows with <= k valid keys take all of them).
//
// Reference counterparts: vllm_musa/v1/attention/backends/mla/flashmla.py:47-331 and
// flashmla_sparse.py:109-188 (FlashMLA dense / sparse, MATE library kernels),
// csrc/musa/attention/deepseek_v4_fused_qkv_rmsnorm.mu:74 (latent RMSNorm),
// csrc/musa/attention/deepseek_v4_indexer_topk.mu:86-796 and
// deepseek_v4_sparse_indexer_topk.mu:159 (indexer scoring and radix top-k).
#include <algorithm>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "../common/mma_sm80.cuh"

namespace b200 {
namespace mla {

constexpr int kLat = 512, kPe = 64, kRow = kLat + kPe;  // 576
constexpr int kCB = kRow / 64;                          // 9 column blocks of 64 (128 bytes)
constexpr int kTile = 64;
constexpr int kHeads = 16;  // heads per CTA (one m16 tile)
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCols = kLat / kWarps;  // output columns per warp (64)
constexpr int kQBytes = kCB * kHeads * 128;    // 18 KB
constexpr int kKBytes = kCB * kTile * 128;     // 72 KB per buffer
constexpr int kSStride = kTile + 8;            // padded fp32 score row
constexpr int kSmem = 1024 + kQBytes + 2 * kKBytes + kHeads * kSStride * 4 + 2 * kTile * 8;

// --------------------------------------------------------------------------------- prep
__global__ void mla_prep_kernel(__nv_bfloat16* __restrict__ q, int64_t ld_q, int Hq,
                                const __nv_bfloat16* __restrict__ kv, int64_t ld_kv,
                                const __nv_bfloat16* __restrict__ kv_norm_w, float eps,
                                const int32_t* __restrict__ positions,
                                const float* __restrict__ cos_sin,  // [max_pos, 64]: cos | sin
                                __nv_bfloat16* __restrict__ cache,
                                const int32_t* __restrict__ slots) {
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = positions[t];
  const float* cs = cos_sin + (size_t)pos * kPe;
  // interleaved (GPT-J) pairs: lane rotates dims (2*lane, 2*lane+1) with frequency `lane`
  const float c = cs[lane], s = cs[32 + lane];
  if (warp == 0) {
    const int slot = slots[t];
    const __nv_bfloat16* src = kv + (size_t)t * ld_kv;
    float v[16];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float f[8];
      unpack8(reinterpret_cast<const uint4*>(src)[lane * 2 + j], f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[8 * j + i] = f[i];
        ss += f[i] * f[i];
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / kLat + eps);
    float w[2][8];
#pragma unroll
    for (int j = 0; j < 2; ++j) unpack8(reinterpret_cast<const uint4*>(kv_norm_w)[lane * 2 + j], w[j]);
    const float x0 = bf2f(src[kLat + 2 * lane]), x1 = bf2f(src[kLat + 2 * lane + 1]);
    if (slot >= 0) {
      __nv_bfloat16* dst = cache + (size_t)slot * kRow;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = v[8 * j + i] * r * w[j][i];
        reinterpret_cast<uint4*>(dst)[lane * 2 + j] = pack8(o);
      }
      dst[kLat + 2 * lane] = f2bf(x0 * c - x1 * s);
      dst[kLat + 2 * lane + 1] = f2bf(x1 * c + x0 * s);
    }
  } else {
    for (int h = warp - 1; h < Hq; h += (blockDim.x >> 5) - 1) {
      __nv_bfloat16* qp = q + (size_t)t * ld_q + (size_t)h * (128 + kPe) + 128;
      const float x0 = bf2f(qp[2 * lane]), x1 = bf2f(qp[2 * lane + 1]);
      qp[2 * lane] = f2bf(x0 * c - x1 * s);
      qp[2 * lane + 1] = f2bf(x1 * c + x0 * s);
    }
  }
}

// --------------------------------------------------------------------------------- attention
struct AttnParams {
  const __nv_bfloat16* q_lat;  // (t, h, c<512) at t*ql_t + h*ql_h + c
  int64_t ql_t, ql_h;
  const __nv_bfloat16* q_pe;   // (t, h, c<64) at t*qp_t + h*qp_h + c
  int64_t qp_t, qp_h;
  const __nv_bfloat16* cache;  // [slots, 576]
  const int32_t* block_tables;
  int64_t bt_stride;
  int block_size;
  const int32_t* cu_q;
  const int32_t* seq_lens;
  int R;
  const int32_t* indices;      // [T, topk] token positions (-1 = none) or null (dense)
  int64_t idx_ld;
  int topk;
  __nv_bfloat16* out;          // (t, h, c) at t*o_t + h*o_h + c
  int64_t o_t, o_h;
  float* ws_o;                 // [splits, T, Hq, 512]
  float* ws_lse;               // [splits, T, Hq]
  int T, Hq, splits;
  float scale_log2;
  // decode context parallelism: this rank's cache holds the tokens p with p % dcp_size ==
  // dcp_rank at local index p / dcp_size; lse_out [T, Hq] receives log2-sum-exp of the scores
  int dcp_size, dcp_rank;
  float* lse_out;
};

B200_DEVICE int find_req(const int32_t* cu, int R, int t) {
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kThreads) mla_attn_kernel(AttnParams p) {
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  uint8_t* kbuf = smem + kQBytes;
  float* sS = reinterpret_cast<float*>(kbuf + 2 * kKBytes);
  int64_t* sOff = reinterpret_cast<int64_t*>(sS + kHeads * kSStride);  // [2][64]

  const int t = blockIdx.x, h0 = blockIdx.y * kHeads, split = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = find_req(p.cu_q, p.R, t);
  const int q_len = p.cu_q[r + 1] - p.cu_q[r];
  int count = p.seq_lens[r] - q_len + (t - p.cu_q[r]) + 1;  // causal prefix length
  if (p.dcp_size > 1)  // local tokens among the first `count` (dense mode only)
    count = count > p.dcp_rank ? (count - p.dcp_rank + p.dcp_size - 1) / p.dcp_size : 0;
  // key range of this split (positions in the dense prefix or in the index list)
  // the index list holds min(topk, count) valid positions first (the top-k kernel's layout)
  const int n_keys = max(p.indices ? min(p.topk, count) : count, 0);
  const int tiles = (n_keys + kTile - 1) / kTile;
  const int per = (tiles + p.splits - 1) / p.splits;
  const int tile0 = split * per, tile1 = min(tiles, tile0 + per);
  const int32_t* bt = p.block_tables + (size_t)r * p.bt_stride;
  const int32_t* idx = p.indices ? p.indices + (size_t)t * p.idx_ld : nullptr;

  auto row_offsets = [&](int tile, int buf) {
    if (tid < kTile) {
      const int j = tile * kTile + tid;
      int64_t off = -1;
      if (j < n_keys) {
        const int pos = idx ? idx[j] : j;
        if (pos >= 0 && pos < count) {
          const int blk = bt[pos / p.block_size];
          off = ((int64_t)blk * p.block_size + pos % p.block_size) * kRow;
        }
      }
      sOff[buf * kTile + tid] = off;
    }
  };
  auto issue = [&](int buf) {
    uint8_t* kb = kbuf + buf * kKBytes;
#pragma unroll 4
    for (int i = tid; i < kTile * kCB * 8; i += kThreads) {
      const int row = i / (kCB * 8), w = i - row * (kCB * 8);
      const int cb = w >> 3, c = w & 7;
      const int64_t off = sOff[buf * kTile + row];
      const __nv_bfloat16* src = p.cache + (off >= 0 ? off : 0) + cb * 64 + c * 8;
      cp_async16(kb + cb * (kTile * 128) + row * 128 + ((c ^ (row & 7)) << 4), src, off >= 0);
    }
  };

  // Q tile: 16 heads x 576 (rows >= Hq are zero)
  for (int i = tid; i < kHeads * kCB * 8; i += kThreads) {
    const int row = i / (kCB * 8), w = i - row * (kCB * 8);
    const int cb = w >> 3, c = w & 7;
    const int h = h0 + row;
    const bool ok = h < p.Hq;
    const __nv_bfloat16* src =
        cb < 8 ? p.q_lat + (size_t)t * p.ql_t + (size_t)(ok ? h : 0) * p.ql_h + cb * 64 + c * 8
               : p.q_pe + (size_t)t * p.qp_t + (size_t)(ok ? h : 0) * p.qp_h + c * 8;
    cp_async16(smem + cb * (kHeads * 128) + row * 128 + ((c ^ (row & 7)) << 4), src, ok);
  }
  if (tile0 < tile1) {
    row_offsets(tile0, 0);
    __syncthreads();
    issue(0);
  }
  cp_async_commit();

  float o[kCols / 8][4];
#pragma unroll
  for (int i = 0; i < kCols / 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int g = lane >> 2, tq = lane & 3;
  const int m8 = lane >> 3, r8 = lane & 7;

  for (int tile = tile0; tile < tile1; ++tile) {
    const int buf = (tile - tile0) & 1;
    if (tile + 1 < tile1) row_offsets(tile + 1, buf ^ 1);
    __syncthreads();  // offsets visible; every warp is done with the buffer being refilled
    if (tile + 1 < tile1) issue(buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();  // this tile (and Q) landed

    const uint32_t sK = smem_u32(kbuf + buf * kKBytes);
    // ---- scores of keys 8w .. 8w+7 for the 16 heads
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    {
      // x2: matrices (keys 0-7 of this warp, k chunk c0) and (same keys, chunk c0+1)
      const int tok = warp * 8 + r8;
#pragma unroll 4
      for (int ks = 0; ks < kRow / 16; ++ks) {
        const int cb = ks >> 2, c0 = (ks & 3) * 2;
        uint32_t qa[4];
        mma::ldsm_x4(mma::sw128(sQ + cb * (kHeads * 128), (m8 & 1) * 8 + r8, c0 + (m8 >> 1)),
                     qa[0], qa[1], qa[2], qa[3]);
        uint32_t b0, b1;
        mma::ldsm_x2(mma::sw128(sK + cb * (kTile * 128), tok, c0 + (m8 & 1)), b0, b1);
        mma::mma_bf16(s, qa, b0, b1);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = warp * 8 + 2 * tq + (j & 1);
      const int row = g + (j >> 1) * 8;
      sS[row * kSStride + key] = sOff[buf * kTile + key] >= 0 ? s[j] * p.scale_log2 : -INFINITY;
    }
    __syncthreads();
    // ---- online softmax over the 64-key tile (each warp computes the same row statistics)
    float pv[2][16];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const float* srow = sS + (g + rr * 8) * kSStride;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float2 a = *reinterpret_cast<const float2*>(srow + kk * 16 + 2 * tq);
        const float2 b = *reinterpret_cast<const float2*>(srow + kk * 16 + 8 + 2 * tq);
        pv[rr][4 * kk] = a.x;
        pv[rr][4 * kk + 1] = a.y;
        pv[rr][4 * kk + 2] = b.x;
        pv[rr][4 * kk + 3] = b.y;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 16; ++i) mx = fmaxf(mx, pv[rr][i]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(mrow[rr], mx);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      const float corr = exp2f(mrow[rr] - muse);
      mrow[rr] = mnew;
      float sum = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        pv[rr][i] = exp2f(pv[rr][i] - muse);
        sum += pv[rr][i];
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      lrow[rr] = lrow[rr] * corr + sum;
#pragma unroll
      for (int dt = 0; dt < kCols / 8; ++dt) {
        o[dt][2 * rr] *= corr;
        o[dt][2 * rr + 1] *= corr;
      }
    }
    // ---- O[:, 64w .. 64w+63] += P(16 x 64) . V(64 x 64), V = c_kv columns of the tile
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16x2(pv[0][4 * kk], pv[0][4 * kk + 1]);
      pa[1] = pack_bf16x2(pv[1][4 * kk], pv[1][4 * kk + 1]);
      pa[2] = pack_bf16x2(pv[0][4 * kk + 2], pv[0][4 * kk + 3]);
      pa[3] = pack_bf16x2(pv[1][4 * kk + 2], pv[1][4 * kk + 3]);
      const int tok = kk * 16 + (m8 & 1) * 8 + r8;
#pragma unroll
      for (int dn = 0; dn < kCols / 16; ++dn) {  // 16-wide column slices of this warp's columns
        const int col16 = warp * (kCols / 16) + dn;  // global 16-column slice (0..31)
        const int cb = col16 >> 2, cc = (col16 & 3) * 2;
        uint32_t b0, b1, b2, b3;
        mma::ldsm_x4_t(mma::sw128(sK + cb * (kTile * 128), tok, cc + (m8 >> 1)), b0, b1, b2, b3);
        mma::mma_bf16(o[2 * dn], pa, b0, b1);
        mma::mma_bf16(o[2 * dn + 1], pa, b2, b3);
      }
    }
  }
  cp_async_wait<0>();

  // ---- write out (normalised bf16, or fp32 partial + log2-sum-exp for the combine)
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int h = h0 + g + rr * 8;
    if (h >= p.Hq) continue;
    const float inv = lrow[rr] > 0.f ? 1.f / lrow[rr] : 0.f;
    if (p.splits == 1) {
      __nv_bfloat16* dst = p.out + (size_t)t * p.o_t + (size_t)h * p.o_h + warp * kCols;
#pragma unroll
      for (int dt = 0; dt < kCols / 8; ++dt) {
        const int col = dt * 8 + 2 * tq;
        *reinterpret_cast<uint32_t*>(dst + col) =
            pack_bf16x2(o[dt][2 * rr] * inv, o[dt][2 * rr + 1] * inv);
      }
      if (p.lse_out != nullptr && warp == 0 && tq == 0)
        p.lse_out[(size_t)t * p.Hq + h] = lrow[rr] > 0.f ? mrow[rr] + log2f(lrow[rr]) : -INFINITY;
    } else {
      float* dst = p.ws_o + (((size_t)split * p.T + t) * p.Hq + h) * kLat + warp * kCols;
#pragma unroll
      for (int dt = 0; dt < kCols / 8; ++dt) {
        const int col = dt * 8 + 2 * tq;
        *reinterpret_cast<float2*>(dst + col) =
            make_float2(o[dt][2 * rr] * inv, o[dt][2 * rr + 1] * inv);
      }
      if (warp == 0 && tq == 0)
        p.ws_lse[((size_t)split * p.T + t) * p.Hq + h] =
            lrow[rr] > 0.f ? mrow[rr] + log2f(lrow[rr]) : -INFINITY;
    }
  }
}

__global__ void mla_combine_kernel(const float* __restrict__ ws_o, const float* __restrict__ ws_lse,
                                   int T, int Hq, int splits, __nv_bfloat16* __restrict__ out,
                                   int64_t o_t, int64_t o_h, float* __restrict__ lse_out) {
  const int t = blockIdx.x, h = blockIdx.y;
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, ws_lse[((size_t)s * T + t) * Hq + h]);
  float wsum = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < splits; ++s) {
    const float l = ws_lse[((size_t)s * T + t) * Hq + h];
    const float w = l == -INFINITY ? 0.f : exp2f(l - mx);
    wsum += w;
    if (w == 0.f) continue;
    const float4 v = reinterpret_cast<const float4*>(ws_o + (((size_t)s * T + t) * Hq + h) * kLat)[threadIdx.x];
    acc[0] += w * v.x;
    acc[1] += w * v.y;
    acc[2] += w * v.z;
    acc[3] += w * v.w;
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  if (lse_out != nullptr && threadIdx.x == 0)
    lse_out[(size_t)t * Hq + h] = wsum > 0.f ? mx + log2f(wsum) : -INFINITY;
  __nv_bfloat16* dst = out + (size_t)t * o_t + (size_t)h * o_h + threadIdx.x * 4;
  *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  *reinterpret_cast<uint32_t*>(dst + 2) = pack_bf16x2(acc[2] * inv, acc[3] * inv);
}

// --------------------------------------------------------------------------------- indexer
constexpr int kIdxHeads = 64, kIdxDim = 128, kIdxPe = 64;
constexpr int kIdxThreads = 128;  // 4 warps x 16 heads
constexpr int kIdxChunk = 16;  // key tiles (of 64) per CTA
constexpr int kIdxQBytes = kIdxHeads * kIdxDim * 2;  // 16 KB (2 column blocks)
constexpr int kIdxKBytes = kTile * kIdxDim * 2;      // 16 KB
constexpr int kIdxSmem = 1024 + kIdxQBytes + 2 * kIdxKBytes + 4 * kTile * 4 + kIdxHeads * 4 + 2 * kTile * 8;

__global__ void indexer_k_prep_kernel(const __nv_bfloat16* __restrict__ k, int64_t ld_k,
                                      const __nv_bfloat16* __restrict__ ln_w,
                                      const __nv_bfloat16* __restrict__ ln_b, float eps,
                                      const int32_t* __restrict__ positions,
                                      const float* __restrict__ cos_sin,  // [max_pos, 64]
                                      __nv_bfloat16* __restrict__ cache,  // [slots, 128]
                                      const int32_t* __restrict__ slots, int T) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  const int slot = slots[t];
  if (slot < 0) return;
  const __nv_bfloat16* src = k + (size_t)t * ld_k;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = bf2f(src[lane * 4 + i]);
  float mean = warp_sum(v[0] + v[1] + v[2] + v[3]) / kIdxDim;
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) var += (v[i] - mean) * (v[i] - mean);
  var = warp_sum(var) / kIdxDim;
  const float r = rsqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = (v[i] - mean) * r * bf2f(ln_w[lane * 4 + i]) + bf2f(ln_b[lane * 4 + i]);
  // RoPE (NeoX halves) on the first 64 dims: dim d pairs with d + 32
  const float* cs = cos_sin + (size_t)positions[t] * kIdxPe;
  float out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = lane * 4 + i;
    const float partner = __shfl_xor_sync(0xffffffffu, v[i], 8);  // lanes 0-7 <-> 8-15
    if (d < kIdxPe) {
      const int f = d & 31;
      out[i] = d < 32 ? v[i] * cs[f] - partner * cs[32 + f] : v[i] * cs[f] + partner * cs[32 + f];
    } else {
      out[i] = v[i];
    }
  }
  __nv_bfloat16* dst = cache + (size_t)slot * kIdxDim + lane * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = f2bf(out[i]);
}

struct IdxParams {
  const __nv_bfloat16* q;  // [T, 64*128] (roped), row stride ld_q
  int64_t ld_q;
  const float* w;          // [T, 64] head weights (already scaled), row stride ld_w
  int64_t ld_w;
  const __nv_bfloat16* cache;  // [slots, 128]
  const int32_t* block_tables;
  int64_t bt_stride;
  int block_size;
  const int32_t* cu_q;
  const int32_t* seq_lens;
  int R;
  float* scores;  // [T, ld_s]
  int64_t ld_s;
};

__global__ void __launch_bounds__(kIdxThreads) indexer_score_kernel(IdxParams p) {
  pdl_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sQ = smem_u32(smem);
  uint8_t* kbuf = smem + kIdxQBytes;
  float* sPart = reinterpret_cast<float*>(kbuf + 2 * kIdxKBytes);  // [4 warps][64]
  float* sW = sPart + 4 * kTile;                                   // [64]
  int64_t* sOff = reinterpret_cast<int64_t*>(sW + kIdxHeads);      // [2][64]
  const int t = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = find_req(p.cu_q, p.R, t);
  const int q_len = p.cu_q[r + 1] - p.cu_q[r];
  const int count = p.seq_lens[r] - q_len + (t - p.cu_q[r]) + 1;
  const int tiles = (count + kTile - 1) / kTile;
  const int tile0 = blockIdx.y * kIdxChunk;
  const int tile1 = min(tiles, tile0 + kIdxChunk);
  float* srow = p.scores + (size_t)t * p.ld_s;
  // positions this CTA owns but that are past the prefix read as -inf
  const int own_end = min((int)p.ld_s, (tile0 + kIdxChunk) * kTile);
  for (int j = max(tile0 * kTile, tiles * kTile) + tid; j < own_end; j += kIdxThreads) srow[j] = -INFINITY;
  if (tile0 >= tile1) return;
  const int32_t* bt = p.block_tables + (size_t)r * p.bt_stride;

  for (int i = tid; i < kIdxHeads * 16; i += kIdxThreads) {
    const int row = i >> 4, w = i & 15, cb = w >> 3, c = w & 7;
    cp_async16(smem + cb * (kIdxHeads * 128) + row * 128 + ((c ^ (row & 7)) << 4),
               p.q + (size_t)t * p.ld_q + row * kIdxDim + cb * 64 + c * 8);
  }
  if (tid < kIdxHeads) sW[tid] = p.w[(size_t)t * p.ld_w + tid];
  auto offsets = [&](int tile, int buf) {
    if (tid < kTile) {
      const int pos = tile * kTile + tid;
      sOff[buf * kTile + tid] =
          pos < count ? ((int64_t)bt[pos / p.block_size] * p.block_size + pos % p.block_size) * kIdxDim
                      : -1;
    }
  };
  auto issue = [&](int buf) {
    uint8_t* kb = kbuf + buf * kIdxKBytes;
    for (int i = tid; i < kTile * 16; i += kIdxThreads) {
      const int row = i >> 4, w = i & 15, cb = w >> 3, c = w & 7;
      const int64_t off = sOff[buf * kTile + row];
      cp_async16(kb + cb * (kTile * 128) + row * 128 + ((c ^ (row & 7)) << 4),
                 p.cache + (off >= 0 ? off : 0) + cb * 64 + c * 8, off >= 0);
    }
  };
  offsets(tile0, 0);
  __syncthreads();
  issue(0);
  cp_async_commit();
  const int g = lane >> 2, tq = lane & 3, m8 = lane >> 3, r8 = lane & 7;
  for (int tile = tile0; tile < tile1; ++tile) {
    const int buf = (tile - tile0) & 1;
    if (tile + 1 < tile1) offsets(tile + 1, buf ^ 1);
    __syncthreads();
    if (tile + 1 < tile1) issue(buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t sK = smem_u32(kbuf + buf * kIdxKBytes);
    // warp w: heads 16w..16w+15 against the 64 keys
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[nt][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kIdxDim / 16; ++ks) {
      const int cb = ks >> 2, c0 = (ks & 3) * 2;
      uint32_t qa[4];
      mma::ldsm_x4(mma::sw128(sQ + cb * (kIdxHeads * 128), warp * 16 + (m8 & 1) * 8 + r8, c0 + (m8 >> 1)),
                   qa[0], qa[1], qa[2], qa[3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        const int tok = np * 16 + (m8 >> 1) * 8 + r8;
        mma::ldsm_x4(mma::sw128(sK + cb * (kTile * 128), tok, c0 + (m8 & 1)), b0, b1, b2, b3);
        mma::mma_bf16(s[2 * np], qa, b0, b1);
        mma::mma_bf16(s[2 * np + 1], qa, b2, b3);
      }
    }
    // relu, head weights, sum over this warp's 16 heads (rows g and g+8 of each quad column)
    const float w0 = sW[warp * 16 + g], w1 = sW[warp * 16 + g + 8];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float v = w0 * fmaxf(s[nt][j], 0.f) + w1 * fmaxf(s[nt][2 + j], 0.f);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        if (g == 0) sPart[warp * kTile + nt * 8 + 2 * tq + j] = v;
      }
    }
    __syncthreads();
    if (tid < kTile) {
      const int pos = tile * kTile + tid;
      const float v = sPart[tid] + sPart[kTile + tid] + sPart[2 * kTile + tid] + sPart[3 * kTile + tid];
      if (pos < p.ld_s) srow[pos] = pos < count ? v : -INFINITY;
    }
  }
  cp_async_wait<0>();
}

// Order-preserving map of fp32 to uint32 (larger float -> larger key; -inf smallest finite).
B200_DEVICE uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One CTA per row: top-k positions among the row's first `count` scores.
__global__ void __launch_bounds__(1024) topk_kernel(const float* __restrict__ scores, int64_t ld_s,
                                                    const int32_t* __restrict__ cu_q,
                                                    const int32_t* __restrict__ seq_lens, int R,
                                                    int k, int32_t* __restrict__ out, int64_t ld_o) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_need, s_cnt_gt, s_cnt_eq;
  const int t = blockIdx.x;
  const int r = find_req(cu_q, R, t);
  const int q_len = cu_q[r + 1] - cu_q[r];
  const int count = seq_lens[r] - q_len + (t - cu_q[r]) + 1;
  int32_t* o = out + (size_t)t * ld_o;
  const float* s = scores + (size_t)t * ld_s;
  if (count <= k) {
    for (int j = threadIdx.x; j < k; j += blockDim.x) o[j] = j < count ? j : -1;
    return;
  }
  // radix select the k-th largest key, 8 bits at a time from the top
  uint32_t prefix = 0, need = k;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t mask_hi = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    for (int j = threadIdx.x; j < count; j += blockDim.x) {
      const uint32_t key = fkey(s[j]);
      if ((key & mask_hi) == prefix) atomicAdd(&hist[(key >> shift) & 255], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t acc = 0;
      int b = 255;
      for (; b > 0; --b) {
        if (acc + hist[b] >= need) break;
        acc += hist[b];
      }
      s_prefix = prefix | ((uint32_t)b << shift);
      s_need = need - acc;
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_need;
    __syncthreads();
  }
  // prefix = the k-th largest key; take every key above it and `need` keys equal to it
  if (threadIdx.x == 0) {
    s_cnt_gt = 0;
    s_cnt_eq = 0;
  }
  __syncthreads();
  const uint32_t n_gt = k - need;
  for (int j = threadIdx.x; j < count; j += blockDim.x) {
    const uint32_t key = fkey(s[j]);
    if (key > prefix) {
      o[atomicAdd(&s_cnt_gt, 1u)] = j;
    } else if (key == prefix) {
      const uint32_t e = atomicAdd(&s_cnt_eq, 1u);
      if (e < need) o[n_gt + e] = j;
    }
  }
}

// --------------------------------------------------------------------------------- launchers
void run_prep(void* q, int64_t ld_q, int Hq, const void* kv, int64_t ld_kv, const void* kv_norm_w,
              float eps, const int32_t* positions, const float* cos_sin, void* cache,
              const int32_t* slots, int T, cudaStream_t s) {
  if (T == 0) return;
  mla_prep_kernel<<<T, 256, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(q), ld_q, Hq,
                                    reinterpret_cast<const __nv_bfloat16*>(kv), ld_kv,
                                    reinterpret_cast<const __nv_bfloat16*>(kv_norm_w), eps,
                                    positions, cos_sin, reinterpret_cast<__nv_bfloat16*>(cache),
                                    slots);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_attention(const MlaArgs& a, cudaStream_t s) {
  if (a.T == 0) return;
  B200_REQUIRE(a.splits >= 1 && a.splits <= 64, "mla: 1..64 splits");
  B200_REQUIRE(a.indices == nullptr || a.topk % kTile == 0, "mla: topk must be a multiple of 64");
  B200_REQUIRE(a.splits == 1 || (a.ws_o && a.ws_lse), "mla: split workspace missing");
  AttnParams p;
  p.q_lat = reinterpret_cast<const __nv_bfloat16*>(a.q_lat);
  p.ql_t = a.ql_t;
  p.ql_h = a.ql_h;
  p.q_pe = reinterpret_cast<const __nv_bfloat16*>(a.q_pe);
  p.qp_t = a.qp_t;
  p.qp_h = a.qp_h;
  p.cache = reinterpret_cast<const __nv_bfloat16*>(a.cache);
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.block_size = a.block_size;
  p.cu_q = a.cu_q;
  p.seq_lens = a.seq_lens;
  p.R = a.R;
  p.indices = a.indices;
  p.idx_ld = a.idx_ld;
  p.topk = a.topk;
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.o_t = a.o_t;
  p.o_h = a.o_h;
  p.ws_o = a.ws_o;
  p.ws_lse = a.ws_lse;
  p.T = a.T;
  p.Hq = a.Hq;
  p.splits = a.splits;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.dcp_size = a.dcp_size > 0 ? a.dcp_size : 1;
  p.dcp_rank = a.dcp_rank;
  p.lse_out = a.lse_out;
  B200_REQUIRE(p.dcp_size == 1 || a.indices == nullptr,
               "mla: decode context parallelism covers the dense (causal prefix) mode only");
  B200_REQUIRE(p.dcp_rank >= 0 && p.dcp_rank < p.dcp_size, "mla: dcp rank");
  ensure_dynamic_smem(reinterpret_cast<const void*>(mla_attn_kernel), kSmem);
  mla_attn_kernel<<<dim3(a.T, (a.Hq + kHeads - 1) / kHeads, a.splits), kThreads, kSmem, s>>>(p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
  if (a.splits > 1) {
    mla_combine_kernel<<<dim3(a.T, a.Hq), kLat / 4, 0, s>>>(a.ws_o, a.ws_lse, a.T, a.Hq, a.splits,
                                                           p.out, a.o_t, a.o_h, a.lse_out);
    B200_CUDA_OK(cudaGetLastError());
    count_launch();
  }
}

void run_indexer_k_prep(const void* k, int64_t ld_k, const void* ln_w, const void* ln_b, float eps,
                        const int32_t* positions, const float* cos_sin, void* cache,
                        const int32_t* slots, int T, cudaStream_t s) {
  if (T == 0) return;
  indexer_k_prep_kernel<<<(T + 7) / 8, 256, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(k), ld_k, reinterpret_cast<const __nv_bfloat16*>(ln_w),
      reinterpret_cast<const __nv_bfloat16*>(ln_b), eps, positions, cos_sin,
      reinterpret_cast<__nv_bfloat16*>(cache), slots, T);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_indexer_scores(const IndexerArgs& a, cudaStream_t s) {
  if (a.T == 0) return;
  IdxParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(a.q);
  p.ld_q = a.ld_q;
  p.w = a.w;
  p.ld_w = a.ld_w;
  p.cache = reinterpret_cast<const __nv_bfloat16*>(a.cache);
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.block_size = a.block_size;
  p.cu_q = a.cu_q;
  p.seq_lens = a.seq_lens;
  p.R = a.R;
  p.scores = a.scores;
  p.ld_s = a.ld_s;
  const int chunks = (int)((a.ld_s + kTile * kIdxChunk - 1) / (kTile * kIdxChunk));
  ensure_dynamic_smem(reinterpret_cast<const void*>(indexer_score_kernel), kIdxSmem);
  indexer_score_kernel<<<dim3(a.T, chunks), kIdxThreads, kIdxSmem, s>>>(p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_topk(const float* scores, int64_t ld_s, const int32_t* cu_q, const int32_t* seq_lens,
              int R, int T, int k, int32_t* out, int64_t ld_o, cudaStream_t s) {
  if (T == 0) return;
  topk_kernel<<<T, 1024, 0, s>>>(scores, ld_s, cu_q, seq_lens, R, k, out, ld_o);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace mla
}  // namespace b200
