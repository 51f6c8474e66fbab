// Device helpers shared by the sampling kernels (sampling.cu) and the vocab-parallel top-k /
// top-p exchange (topk_exchange.cu): the Philox-4x32-10 counter-based generator (Salmon et
// al., SC'11) keyed by (seed, step, global token id), Gumbel noise from its bits,
// order-preserving float keys and the 8-bit radix select over a row.
#pragma once
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

}  // namespace sampling
}  // namespace b200
