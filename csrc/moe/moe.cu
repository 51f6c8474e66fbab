// Mixture-of-experts routing and data movement for sm_100a.
//
//  topk_softmax   router logits [T, E] -> softmax -> top-k (optionally renormalised):
//                 one warp per token, E/32 logits per lane, k rounds of warp arg-max.
//  grouped_topk   DeepSeek-style: sigmoid (or softmax) scores + correction bias, experts in
//                 n_group groups, keep the topk_group best groups (by the sum of each group's
//                 top-2 biased scores), then top-k inside them; weights are the unbiased
//                 scores, renormalised and scaled by routed_scaling_factor.
//  moe_align      sort the T*k (token, slot) assignments by expert and pad every expert's
//                 segment to a multiple of 128 rows: sorted_ids[P] (assignment index or -1),
//                 tile_expert[P/128], the padded offsets and the live tile count, all on
//                 the device (CUDA-graph safe: no host round trip).
//  moe_gather     A rows of the grouped GEMM: x[sorted_ids[i] / k] (zeros for padding).
//  moe_combine    out[t] = sum_j w[t, j] * y[pos(t, j)] (+ shared-expert output if given).
//
// Reference counterparts: vllm_musa/jit_kernel/csrc/topk/topk_gating.mu:858-981 (top-k
// softmax / sigmoid, shared slot), vllm_musa/model_executor/layers/fused_moe/router/
// grouped_topk_router.py:59-388, vllm_musa/jit_kernel/tilelang/deep_gemm_contig_preprocess.py
// (expert-contiguous layout), vllm_musa/jit_kernel/csrc/moe/moe_sum_reduce.mu:53-374.
#include <algorithm>

#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace moe {

constexpr int kTile = 128;

// ------------------------------------------------------------------------------ top-k softmax
template <int EPL>  // experts per lane
__global__ void topk_softmax_kernel(const float* __restrict__ logits, int64_t ld, int T, int E,
                                    int k, bool renorm, int32_t* __restrict__ ids,
                                    float* __restrict__ w) {
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  float v[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane * EPL + i;
    v[i] = e < E ? logits[(size_t)t * ld + e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    v[i] = lane * EPL + i < E ? __expf(v[i] - mx) : 0.f;
    s += v[i];
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
  float picked_sum = 0.f;
  for (int j = 0; j < k; ++j) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane * EPL + i;
      if (e < E && v[i] > bv) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      ids[(size_t)t * k + j] = bi;
      w[(size_t)t * k + j] = bv * inv;
    }
    picked_sum += bv * inv;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane * EPL + i == bi) v[i] = -2.f;  // remove from further rounds
  }
  __syncwarp();
  if (renorm && lane < k) w[(size_t)t * k + lane] /= picked_sum;
}

// ------------------------------------------------------------------------------ grouped top-k
// One warp per token; up to 512 experts (EPL <= 16), up to 32 groups.
template <int EPL>
__global__ void grouped_topk_kernel(const float* __restrict__ logits,
                                    const float* __restrict__ bias, int T, int E, int k,
                                    int n_group, int topk_group, bool sigmoid, bool renorm,
                                    float scale, int32_t* __restrict__ ids,
                                    float* __restrict__ w) {
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  float sc[EPL], bsc[EPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane * EPL + i;
    const float l = e < E ? logits[(size_t)t * E + e] : -INFINITY;
    sc[i] = l;
    mx = fmaxf(mx, l);
  }
  if (!sigmoid) {
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      sc[i] = lane * EPL + i < E ? __expf(sc[i] - mx) : 0.f;
      s += sc[i];
    }
    s = warp_sum(s);
#pragma unroll
    for (int i = 0; i < EPL; ++i) sc[i] /= s;
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) sc[i] = 1.f / (1.f + __expf(-sc[i]));
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane * EPL + i;
    bsc[i] = e < E ? sc[i] + (bias ? bias[e] : 0.f) : -INFINITY;
  }
  // group scores: sum of the two best biased scores of each group (groups are contiguous)
  const int gsize = E / n_group;
  __shared__ float gscore[8][32];
  float* gs = gscore[(threadIdx.x / 32) & 7];
  for (int g = 0; g < n_group; ++g) {
    float b1 = -INFINITY, b2 = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane * EPL + i;
      if (e >= g * gsize && e < (g + 1) * gsize) {
        const float x = bsc[i];
        if (x > b1) {
          b2 = b1;
          b1 = x;
        } else if (x > b2) {
          b2 = x;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float o1 = __shfl_xor_sync(0xffffffffu, b1, o);
      const float o2 = __shfl_xor_sync(0xffffffffu, b2, o);
      // merge two sorted pairs
      const float n1 = fmaxf(b1, o1);
      const float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
      b1 = n1;
      b2 = n2;
    }
    if (lane == 0) gs[g] = gsize >= 2 ? b1 + b2 : b1;
  }
  __syncwarp();
  // keep the topk_group best groups
  unsigned keep = 0;
  if (lane == 0) {
    for (int r = 0; r < topk_group; ++r) {
      int bg = -1;
      float bv = -INFINITY;
      for (int g = 0; g < n_group; ++g)
        if (!(keep >> g & 1) && gs[g] > bv) {
          bv = gs[g];
          bg = g;
        }
      if (bg >= 0) keep |= 1u << bg;
    }
  }
  keep = __shfl_sync(0xffffffffu, keep, 0);
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane * EPL + i;
    if (e < E && !(keep >> (e / gsize) & 1)) bsc[i] = -INFINITY;
  }
  float picked = 0.f;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane * EPL + i;
      if (e < E && bsc[i] > bv) {
        bv = bsc[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    float s_unb = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane * EPL + i == bi) {
        s_unb = sc[i];
        bsc[i] = -INFINITY;
      }
    s_unb = __shfl_sync(0xffffffffu, s_unb, (bi / EPL) & 31);
    if (lane == 0) {
      ids[(size_t)t * k + j] = bi;
      w[(size_t)t * k + j] = s_unb;
    }
    picked += s_unb;
  }
  __syncwarp();
  if (lane < k) {
    float x = w[(size_t)t * k + lane];
    if (renorm) x /= picked;
    w[(size_t)t * k + lane] = x * scale;
  }
}

// ------------------------------------------------------------------------------ align / sort
// Single CTA of 1024 threads: histogram, padded exclusive scan, stable placement.
__global__ void __launch_bounds__(1024)
    moe_align_kernel(const int32_t* __restrict__ ids, int n, int E, int e0, int max_rows,
                     int32_t* __restrict__ sorted_ids, int32_t* __restrict__ tile_expert,
                     int32_t* __restrict__ offsets, int32_t* __restrict__ pos,
                     int32_t* __restrict__ num_tiles) {
  extern __shared__ int32_t sh[];
  int32_t* cnt = sh;           // [E]
  int32_t* start = sh + E;     // [E + 1]
  int32_t* cursor = sh + 2 * E + 1;  // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = ids[i] - e0;  // local expert index (expert parallelism)
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      start[e] = acc;
      acc += (cnt[e] + kTile - 1) / kTile * kTile;
    }
    start[E] = acc;
    *num_tiles = acc / kTile;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = start[e];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = 0;
  const int total = start[E];
  for (int r = threadIdx.x; r < max_rows; r += blockDim.x) sorted_ids[r] = -1;
  __syncthreads();
  for (int tI = threadIdx.x; tI < total / kTile; tI += blockDim.x) {
    // expert owning tile tI: binary search over start[]
    int lo = 0, hi = E - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (start[mid] <= tI * kTile) lo = mid; else hi = mid - 1;
    }
    tile_expert[tI] = lo;
  }
  __syncthreads();
  // placement: the slot inside an expert's segment is taken with an atomic; rows are
  // computed independently, so the order inside a segment does not change any result.
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = ids[i] - e0;
    if (e >= 0 && e < E) {
      const int p = start[e] + atomicAdd(&cursor[e], 1);
      sorted_ids[p] = i;
      pos[i] = p;
    } else {
      pos[i] = -1;
    }
  }
}

__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                  const int32_t* __restrict__ sorted_ids,
                                  const int32_t* __restrict__ num_tiles, int k, int H,
                                  __nv_bfloat16* __restrict__ out) {
  const int r = blockIdx.x;
  if (r >= *num_tiles * kTile) return;
  const int a = sorted_ids[r];
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)r * H);
  const uint4* src = a >= 0 ? reinterpret_cast<const uint4*>(x + (size_t)(a / k) * ldx) : nullptr;
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x)
    dst[c] = src ? src[c] : make_uint4(0, 0, 0, 0);
}

__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ pos,
                                   const float* __restrict__ w, int T, int k, int H,
                                   const __nv_bfloat16* __restrict__ shared,
                                   const float* __restrict__ shared_gate, int64_t ld_gate,
                                   __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int t = blockIdx.x;
  // sigmoid-gated shared expert (Qwen2/3-MoE style): the gate logit rides in the router GEMM
  const float sg = shared_gate ? 1.f / (1.f + __expf(-shared_gate[(size_t)t * ld_gate])) : 1.f;
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    float acc[8];
    if (shared) {
      unpack8(reinterpret_cast<const uint4*>(shared + (size_t)t * H)[c], acc);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] *= sg;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
    for (int j = 0; j < k; ++j) {
      const int p = pos[(size_t)t * k + j];
      if (p < 0) continue;
      const float wt = w[(size_t)t * k + j];
      float f[8];
      unpack8(reinterpret_cast<const uint4*>(y + (size_t)p * H)[c], f);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += wt * f[q];
    }
    reinterpret_cast<uint4*>(out + (size_t)t * ldo)[c] = pack8(acc);
  }
}

// ------------------------------------------------------------------------------ launchers
void run_topk_softmax(const float* logits, int64_t ld, int T, int E, int k, bool renorm,
                      int32_t* ids, float* w, cudaStream_t s) {
  B200_REQUIRE(E <= 512 && k <= 32 && k <= E, "topk_softmax: E <= 512, k <= 32");
  if (T == 0) return;
  const int warps = 8, blocks = (T + warps - 1) / warps;
  const int epl = (E + 31) / 32;
#define B200_TK(N) \
  topk_softmax_kernel<N><<<blocks, warps * 32, 0, s>>>(logits, ld, T, E, k, renorm, ids, w)
  if (epl <= 2) B200_TK(2);
  else if (epl <= 4) B200_TK(4);
  else if (epl <= 8) B200_TK(8);
  else B200_TK(16);
#undef B200_TK
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_grouped_topk(const float* logits, const float* bias, int T, int E, int k, int n_group,
                      int topk_group, bool sigmoid, bool renorm, float scale, int32_t* ids,
                      float* w, cudaStream_t s) {
  B200_REQUIRE(E <= 512 && k <= 32 && n_group <= 32 && E % n_group == 0,
               "grouped_topk: E <= 512, n_group <= 32 dividing E");
  if (T == 0) return;
  const int warps = 8, blocks = (T + warps - 1) / warps;
  const int epl = (E + 31) / 32;
#define B200_GT(N)                                                                            \
  grouped_topk_kernel<N><<<blocks, warps * 32, 0, s>>>(logits, bias, T, E, k, n_group,       \
                                                       topk_group, sigmoid, renorm, scale, ids, w)
  if (epl <= 2) B200_GT(2);
  else if (epl <= 4) B200_GT(4);
  else if (epl <= 8) B200_GT(8);
  else B200_GT(16);
#undef B200_GT
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

int align_max_rows(int n, int E) { return ((n + E * (kTile - 1)) + kTile - 1) / kTile * kTile; }

void run_moe_align(const int32_t* ids, int n, int E, int e0, int max_rows, int32_t* sorted_ids,
                   int32_t* tile_expert, int32_t* offsets, int32_t* pos, int32_t* num_tiles,
                   cudaStream_t s) {
  B200_REQUIRE(max_rows >= align_max_rows(n, E), "moe_align: max_rows too small");
  const int smem = (3 * E + 1) * sizeof(int32_t);
  moe_align_kernel<<<1, 1024, smem, s>>>(ids, n, E, e0, max_rows, sorted_ids, tile_expert, offsets,
                                         pos, num_tiles);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_moe_gather(const void* x, int64_t ldx, const int32_t* sorted_ids, const int32_t* num_tiles,
                    int max_rows, int k, int H, void* out, cudaStream_t s) {
  B200_REQUIRE(H % 8 == 0, "moe_gather: H % 8");
  if (max_rows == 0) return;
  moe_gather_kernel<<<max_rows, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx,
                                             sorted_ids, num_tiles, k, H,
                                             reinterpret_cast<__nv_bfloat16*>(out));
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_moe_combine(const void* y, const int32_t* pos, const float* w, int T, int k, int H,
                     const void* shared, const float* shared_gate, int64_t ld_gate, void* out,
                     int64_t ldo, cudaStream_t s) {
  B200_REQUIRE(H % 8 == 0, "moe_combine: H % 8");
  if (T == 0) return;
  moe_combine_kernel<<<T, 128, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(y), pos, w, T, k, H,
                                       reinterpret_cast<const __nv_bfloat16*>(shared),
                                       shared_gate, ld_gate,
                                       reinterpret_cast<__nv_bfloat16*>(out), ldo);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace moe
}  // namespace b200
