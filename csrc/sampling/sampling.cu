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
#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace sampling {

constexpr int kThreads = 1024;

// ---- Philox-4x32-10 (Salmon, Moraes, Dror, Shaw 2011) ----
struct U4 {
  uint32_t x, y, z, w;
};
B200_DEVICE U4 philox(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += W0;
    k1 += W1;
  }
  return c;
}

B200_DEVICE float uniform_open(uint32_t bits) {
  return ((float)(bits >> 8) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
}

// Gumbel(0,1) from 32 random bits: G = -log(E), E = -log(u) ~ Exp(1).  The inner log is the
// accurate one (u near 1 gives the largest G, which decides the argmax); the outer log's
// argument E is away from the ill-conditioned point, so the fast log is accurate enough.
B200_DEVICE float gumbel_from_bits(uint32_t b) { return -__logf(-logf(uniform_open(b))); }

B200_DEVICE U4 philox_group(uint64_t seed, uint32_t step, uint32_t group) {
  return philox(U4{group, step, 0x5a4d5153u, 0u}, (uint32_t)seed, (uint32_t)(seed >> 32));
}

// Noise of global token `idx`: component (idx & 3) of the Philox block of group idx >> 2.
B200_DEVICE float gumbel(uint64_t seed, uint32_t step, uint32_t idx) {
  const U4 r = philox_group(seed, step, idx >> 2);
  const uint32_t sel = idx & 3;
  const uint32_t b = sel == 0 ? r.x : sel == 1 ? r.y : sel == 2 ? r.z : r.w;
  return gumbel_from_bits(b);
}

B200_DEVICE uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct Cand {
  float v;
  int i;
};
B200_DEVICE Cand better(Cand a, Cand b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

// Radix select over the row: returns the largest threshold key t such that the measure
// (count or exp-mass) of {key >= t} is >= target.  Elements with key < floor_key are ignored.
template <bool kMass>
B200_DEVICE uint32_t radix_select(const float* x, int V, float inv_t, float m, uint32_t floor_key,
                                  float target, int* hc, float* hm, uint32_t* shared_prefix,
                                  float* shared_target) {
  uint32_t prefix = 0, mask = 0;
  if (threadIdx.x == 0) *shared_target = target;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += blockDim.x) {
      hc[b] = 0;
      hm[b] = 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
      const float l = x[i] * inv_t;
      const uint32_t k = fkey(l);
      if (k < floor_key || (k & mask) != prefix) continue;
      const int d = (k >> shift) & 255;
      if (kMass)
        atomicAdd(&hm[d], __expf(l - m));
      else
        atomicAdd(&hc[d], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      // lane owns bins [lane*8, lane*8+8); suffix sums from the top bin down
      float s[8];
      float tot = 0.f;
#pragma unroll
      for (int j = 7; j >= 0; --j) {
        const float val = kMass ? hm[lane * 8 + j] : (float)hc[lane * 8 + j];
        tot += val;
        s[j] = tot;  // sum of this lane's bins >= j
      }
      // exclusive suffix over higher lanes
      float above = 0.f;
      float run = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_down_sync(0xffffffffu, run, o);
        if (lane + o < 32) run += t;
      }
      above = run - tot;  // sum over lanes > lane
      const float tgt = *shared_target;
      int found = -1;
      float above_d = 0.f;
#pragma unroll
      for (int j = 7; j >= 0; --j) {
        const float ge = above + s[j];                           // measure of digits >= d
        const float gt = above + (j < 7 ? s[j + 1] : 0.f);       // measure of digits > d
        if (found < 0 && gt < tgt && ge >= tgt) {
          found = lane * 8 + j;
          above_d = gt;
        }
      }
      // the highest lane with a hit wins (there is exactly one crossing; fall back to 0)
      const unsigned hit = __ballot_sync(0xffffffffu, found >= 0);
      if (lane == 0) {
        *shared_prefix = 0xFFFFFFFFu;
      }
      __syncwarp();
      if (hit) {
        const int src = 31 - __clz(hit);
        const int d = __shfl_sync(0xffffffffu, found, src);
        const float ad = __shfl_sync(0xffffffffu, above_d, src);
        if (lane == 0) {
          *shared_prefix = (uint32_t)d;
          *shared_target = tgt - ad;
        }
      }
      // no crossing (rounding left the total just under the target): keep every element
      // that matches the prefix so far, i.e. stop with the lower digits at zero.
    }
    __syncthreads();
    const uint32_t d = *shared_prefix;
    __syncthreads();
    if (d == 0xFFFFFFFFu) break;
    prefix |= d << shift;
    mask |= 255u << shift;
  }
  return prefix < floor_key ? floor_key : prefix;
}

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

}  // namespace sampling
}  // namespace b200
