// Token sampling for sm_100a.
//
// One CTA (1024 threads) per row of logits [R, V] (fp32).  Per row the kernel applies
// temperature, optional top-k, top-p and min-p filtering, and then draws the token:
//   temperature == 0 : argmax (greedy)
//   otherwise        : Gumbel-max  argmax_i(l_i / T + G_i),  G_i = -log(-log(u_i))
// which samples exactly from softmax(l / T) restricted to the kept set, with no softmax /
// normalisation pass and no sort.  u_i comes from the Philox-4x32-10 counter-based generator
// (Salmon et al., SC'11) keyed by the request seed with counter (vocab index, step), so the
// same token is drawn whichever rank (vocab shard) evaluates an index: vocab-parallel ranks
// each reduce their shard to one (score, index) candidate and the global choice is the max.
//
// Top-k and top-p thresholds are found with a 4-pass 8-bit radix select on order-preserving
// float keys: counts for top-k, exp-mass for top-p (no sort, no materialised probabilities).
// Ties at a threshold are kept.
//
// Reference counterparts: csrc/musa/sampler.mu:124 (top-k/top-p sampling from probs),
// csrc/musa/top_k_mask_logits.mu:91 and top_p_mask_logits.mu:149 (radix select on logits),
// csrc/musa/min_p_sampler.mu:98-207 (min-p), vllm_musa/v1/sample/topk_topp_sampler.py:351.
#include <algorithm>
#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "sampling_common.cuh"

namespace b200 {
namespace sampling {

__global__ void __launch_bounds__(kThreads)
    sample_kernel(const float* __restrict__ logits, int64_t ld, int V, int vocab_offset,
                  const float* __restrict__ temperature, const int32_t* __restrict__ top_k,
                  const float* __restrict__ top_p, const float* __restrict__ min_p,
                  const int64_t* __restrict__ seeds, const int32_t* __restrict__ steps,
                  float* __restrict__ out_val, int64_t* __restrict__ out_idx) {
  __shared__ float red[32];
  __shared__ int hc[256];
  __shared__ float hm[256];
  __shared__ uint32_t sprefix;
  __shared__ float starget;
  __shared__ Cand cand[32];
  const int row = blockIdx.x;
  const float* x = logits + row * ld;
  const float T = temperature ? temperature[row] : 0.f;
  const bool greedy = !(T > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / T;
  const int k = (top_k && !greedy) ? top_k[row] : 0;
  const float p = (top_p && !greedy) ? top_p[row] : 1.f;
  const float mp = (min_p && !greedy) ? min_p[row] : 0.f;

  uint32_t floor_key = 0;
  if (!greedy && ((k > 0 && k < V) || p < 1.f || mp > 0.f)) {
    float m = -INFINITY;
    for (int i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, x[i] * inv_t);
    m = block_max(m, red);
    if (k > 0 && k < V)
      floor_key = radix_select<false>(x, V, inv_t, m, 0u, (float)k, hc, hm, &sprefix, &starget);
    if (mp > 0.f) floor_key = max(floor_key, fkey(m + logf(mp)));
    if (p < 1.f) {
      float s = 0.f;
      for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float l = x[i] * inv_t;
        if (fkey(l) >= floor_key) s += __expf(l - m);
      }
      s = block_sum(s, red);
      const uint32_t tp =
          radix_select<true>(x, V, inv_t, m, floor_key, p * s, hc, hm, &sprefix, &starget);
      floor_key = max(floor_key, tp);
    }
  }
  const uint64_t seed = seeds ? (uint64_t)seeds[row] : 0ull;
  const uint32_t step = steps ? (uint32_t)steps[row] : 0u;
  Cand best{-INFINITY, 0x7fffffff};
  const bool vec = ((vocab_offset | V) & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  if (vec) {
    // four consecutive tokens per thread: one 16-byte load and one Philox block per group
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const uint32_t g0 = (uint32_t)vocab_offset >> 2;
    for (int j = threadIdx.x; j < V / 4; j += blockDim.x) {
      const float4 v = x4[j];
      const float l[4] = {v.x * inv_t, v.y * inv_t, v.z * inv_t, v.w * inv_t};
      const int gi = vocab_offset + 4 * j;
      if (greedy) {
#pragma unroll
        for (int e = 0; e < 4; ++e) best = better(best, Cand{l[e], gi + e});
      } else {
        const U4 r = philox_group(seed, step, g0 + j);
        const uint32_t bits[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (fkey(l[e]) >= floor_key)
            best = better(best, Cand{l[e] + gumbel_from_bits(bits[e]), gi + e});
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float l = x[i] * inv_t;
      if (fkey(l) < floor_key) continue;
      const int gi = vocab_offset + i;
      const float sc = greedy ? l : l + gumbel(seed, step, (uint32_t)gi);
      best = better(best, Cand{sc, gi});
    }
  }
  // block argmax
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Cand other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
    best = better(best, other);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) cand[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = lane < (blockDim.x >> 5) ? cand[lane] : Cand{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      Cand other{__shfl_xor_sync(0xffffffffu, best.v, o),
                 __shfl_xor_sync(0xffffffffu, best.i, o)};
      best = better(best, other);
    }
    if (lane == 0) {
      if (out_val) out_val[row] = best.v;
      out_idx[row] = best.i == 0x7fffffff ? vocab_offset : best.i;
    }
  }
}

// Merge per-shard candidates [S, R] (value, index) -> [R] index (max value, lowest index).
__global__ void merge_candidates_kernel(const float* __restrict__ vals,
                                        const int64_t* __restrict__ idx, int S, int R,
                                        int64_t* __restrict__ out) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  float bv = -INFINITY;
  int64_t bi = idx[r];
  for (int s = 0; s < S; ++s) {
    const float v = vals[s * R + r];
    const int64_t i = idx[s * R + r];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
    }
  }
  out[r] = bi;
}

void run_sample(const SampleArgs& a, cudaStream_t s) {
  if (a.R == 0) return;
  sample_kernel<<<a.R, kThreads, 0, s>>>(a.logits, a.ld, a.V, a.vocab_offset, a.temperature,
                                          a.top_k, a.top_p, a.min_p, a.seeds, a.steps, a.out_val,
                                          a.out_idx);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_merge_candidates(const float* vals, const int64_t* idx, int S, int R, int64_t* out,
                          cudaStream_t s) {
  if (R == 0) return;
  merge_candidates_kernel<<<(R + 255) / 256, 256, 0, s>>>(vals, idx, S, R, out);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

// ------------------------------------------------------------------------------ penalties
// vLLM's logits-processor semantics (the reference inherits them from upstream vLLM): a token
// seen in the prompt or the output has its logit divided by the repetition penalty when
// positive and multiplied by it otherwise; each output occurrence subtracts the frequency
// penalty, and any output occurrence subtracts the presence penalty once.
__global__ void apply_penalties_kernel(float* __restrict__ logits, int64_t ld, int V_local,
                                       int vocab_offset, const int32_t* __restrict__ entries,
                                       int n, const float* __restrict__ rep,
                                       const float* __restrict__ pres,
                                       const float* __restrict__ freq) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int row = entries[3 * i], tok = entries[3 * i + 1] - vocab_offset;
  const int cnt = entries[3 * i + 2];
  if (tok < 0 || tok >= V_local) return;  // another rank's vocab shard
  float* p = logits + (size_t)row * ld + tok;
  float v = *p;
  const float r = rep[row];
  if (r != 1.f) v = v > 0.f ? v / r : v * r;
  v -= freq[row] * (float)cnt;
  if (cnt > 0) v -= pres[row];
  *p = v;
}

void run_apply_penalties(float* logits, int64_t ld, int V_local, int vocab_offset,
                         const int32_t* entries, int n, const float* rep, const float* pres,
                         const float* freq, cudaStream_t s) {
  if (n == 0) return;
  apply_penalties_kernel<<<(n + 255) / 256, 256, 0, s>>>(logits, ld, V_local, vocab_offset,
                                                         entries, n, rep, pres, freq);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

// Constrained decoding: logits[rows[r]][j] = -inf where bit (vocab_offset + j) of bitmask row r
// is clear (bit t of 32-bit word t / 32 allows token t; tokens past the bitmask are masked).
__global__ void token_bitmask_kernel(float* __restrict__ logits, int64_t ld,
                                     const int32_t* __restrict__ bitmask, int words,
                                     const int32_t* __restrict__ rows, int V_local,
                                     int vocab_offset) {
  const int r = blockIdx.y;
  const int row = rows[r];
  const int32_t* bm = bitmask + (int64_t)r * words;
  float* out = logits + (int64_t)row * ld;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < V_local; j += gridDim.x * blockDim.x) {
    const int t = vocab_offset + j;
    const int w = t >> 5;
    if (w >= words || ((bm[w] >> (t & 31)) & 1) == 0) out[j] = -INFINITY;
  }
}

void run_token_bitmask(float* logits, int64_t ld, const int32_t* bitmask, int words,
                       const int32_t* rows, int R, int V_local, int vocab_offset,
                       cudaStream_t s) {
  if (R == 0 || V_local == 0) return;
  const dim3 grid(std::min(64, (V_local + 1023) / 1024), R);
  token_bitmask_kernel<<<grid, 256, 0, s>>>(logits, ld, bitmask, words, rows, V_local,
                                            vocab_offset);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace sampling
}  // namespace b200
