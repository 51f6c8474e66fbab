// Vocab-parallel top-k / top-p / min-p sampling without gathering the logits.
//
// With tensor parallelism every rank holds the logits of its vocab shard.  Instead of an
// all-gather of the [R, V] logits (what the reference does before its top-k / top-p masks:
// vllm_musa/distributed/device_communicators/musa_jit_custom_all_reduce.py:1404-1447,1941-1956
// and vllm_musa/v1/sample/topk_topp_sampler.py:216-351), each rank reduces its shard to a
// fixed-size candidate row and the ranks exchange only those:
//
//   shard_candidates_kernel (one CTA per row, this rank's shard):
//     m = max l/T, s = sum exp(l/T - m) over the shard; thr = the radix-select key of the
//     shard's 128th largest scaled logit; the <= 128 candidates with key >= thr (value, global
//     id); and the shard's Gumbel-max winner over every token (for rows without a filter).
//   topk_exchange_kernel (NVLink):
//     every block stores its rows' candidate rows into every peer's region (plain 16-byte
//     stores to peer memory), runs a per-block epoch barrier with the peers (the communicator's
//     flag protocol, bounded spin), then merges each row from local memory:
//       sort the world x 128 candidates (value desc, id asc); floor key F from top-k (the k-th
//       candidate, ties kept), min-p (M + log min_p, M the global max) and top-p (the sorted
//       prefix whose exp-mass reaches p x the kept mass: the kept candidates' mass when top-k or
//       min-p is set, else the full-vocab mass sum_r s_r e^{m_r - M}); then Gumbel-max over the
//       candidates with key >= F, with the same Philox noise as the full-vocab sampler.
//     The result is exact (the same token as sampling the gathered logits) when every rank that
//     dropped tokens dropped only keys below F (F >= thr_r); otherwise the row's output is -1 and
//     the caller falls back to the gathered path for that step.  Rows without any filter take
//     the max of the ranks' Gumbel winners (exact).
//
// One rank's exchange traffic is R x 1056 bytes per peer (vs R x V/world x 4 for a logits
// all-gather: 60x less at V = 128256, world 8).  No TMA; peer memory is touched by plain
// loads / stores only.
#include <float.h>

#include "../b200_kernels.h"
#include "../comm/custom_ar.h"
#include "../common/common.cuh"
#include "sampling_common.cuh"

namespace b200 {
namespace sampling {

namespace {

B200_DEVICE void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
B200_DEVICE uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------------- per-shard candidates
__global__ void __launch_bounds__(kThreads)
    shard_candidates_kernel(const float* __restrict__ logits, int64_t ld, int V, int vocab_offset,
                            const float* __restrict__ temperature,
                            const int64_t* __restrict__ seeds, const int32_t* __restrict__ steps,
                            CandRow* __restrict__ out) {
  __shared__ float red[32];
  __shared__ int hc[256];
  __shared__ float hm[256];
  __shared__ uint32_t sprefix;
  __shared__ float starget;
  __shared__ int count;
  __shared__ Cand cand[32];
  const int row = blockIdx.x;
  const float* x = logits + row * ld;
  const float T = temperature ? temperature[row] : 0.f;
  const bool greedy = !(T > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / T;
  CandRow* o = out + row;
  if (threadIdx.x == 0) count = 0;
  float m = -INFINITY;
  for (int i = threadIdx.x; i < V; i += blockDim.x) m = fmaxf(m, x[i] * inv_t);
  m = block_max(m, red);
  float s = 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) s += __expf(x[i] * inv_t - m);
  s = block_sum(s, red);
  uint32_t thr = 0;
  if (V > kCandCap)
    thr = radix_select<false>(x, V, inv_t, m, 0u, (float)kCandCap, hc, hm, &sprefix, &starget);
  __syncthreads();
  // gather the candidates and the shard's Gumbel-max winner in one pass
  const uint64_t seed = seeds ? (uint64_t)seeds[row] : 0ull;
  const uint32_t step = steps ? (uint32_t)steps[row] : 0u;
  Cand best{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float l = x[i] * inv_t;
    const int gi = vocab_offset + i;
    if (fkey(l) >= thr) {
      const int pos = atomicAdd(&count, 1);
      if (pos < kCandCap) {
        o->v[pos] = l;
        o->id[pos] = gi;
      }
    }
    best = better(best, Cand{greedy ? l : l + gumbel(seed, step, (uint32_t)gi), gi});
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    Cand other{__shfl_xor_sync(0xffffffffu, best.v, d), __shfl_xor_sync(0xffffffffu, best.i, d)};
    best = better(best, other);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) cand[warp] = best;
  __syncthreads();
  if (warp == 0) {
    best = lane < (blockDim.x >> 5) ? cand[lane] : Cand{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
      Cand other{__shfl_xor_sync(0xffffffffu, best.v, d),
                 __shfl_xor_sync(0xffffffffu, best.i, d)};
      best = better(best, other);
    }
    if (lane == 0) {
      o->m = m;
      o->s = s;
      o->n = min(count, kCandCap);
      // thr 0: the shard sent every token; overflow (ties past the cap): never complete
      o->thr = count > kCandCap ? 0xFFFFFFFFu : thr;
      o->best_v = best.v;
      o->best_id = best.i == 0x7fffffff ? vocab_offset : best.i;
    }
  }
}

// ---------------------------------------------------------------------- merge of one row
constexpr int kMergeThreads = 512;
constexpr int kMergeMax = comm::kMaxRanks * kCandCap;  // 1024

struct MergeSmem {
  float v[kMergeMax];
  int32_t id[kMergeMax];
  float scan[kMergeMax];
  float wsum[kMergeThreads / 32];
  Cand cand[kMergeThreads / 32];
  uint32_t F;
};

// Descending by value, ascending id on ties (the order the full-vocab sampler breaks ties in).
B200_DEVICE bool before(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// Returns the sampled token, or -1 when the candidates cannot decide the row exactly.
B200_DEVICE int64_t merge_row(const CandRow* const* rows, int world, float T, int k, float p,
                              float mp, uint64_t seed, uint32_t step, int V_total, MergeSmem& sm) {
  const bool greedy = !(T > 0.f);
  const int N = world * kCandCap;
  int Np = 1;
  while (Np < N) Np <<= 1;
  // global max, full-vocab mass, completeness thresholds
  float M = -INFINITY;
  for (int r = 0; r < world; ++r) M = fmaxf(M, rows[r]->m);
  float Z = 0.f;
  int total = 0;
  for (int r = 0; r < world; ++r) {
    Z += rows[r]->s * __expf(rows[r]->m - M);
    total += rows[r]->n;
  }
  const bool has_k = !greedy && k > 0 && k < V_total;
  const bool has_p = !greedy && p < 1.f;
  const bool has_mp = !greedy && mp > 0.f;
  if (greedy || (!has_k && !has_p && !has_mp)) {
    // no filter: the max of the shards' winners (Gumbel-max or argmax over every token)
    float bv = -INFINITY;
    int64_t bi = 0x7fffffff;
    for (int r = 0; r < world; ++r) {
      const float v = rows[r]->best_v;
      const int i = rows[r]->best_id;
      if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
      }
    }
    return bi;
  }
  for (int i = threadIdx.x; i < Np; i += blockDim.x) {
    const int r = i / kCandCap, j = i - r * kCandCap;
    const bool ok = i < N && j < rows[r]->n;
    sm.v[i] = ok ? rows[r]->v[j] : -INFINITY;
    sm.id[i] = ok ? rows[r]->id[j] : 0x7fffffff;
  }
  __syncthreads();
  // bitonic sort (descending)
  for (int size = 2; size <= Np; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < Np; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float vi = sm.v[i], vj = sm.v[j];
          const int ii = sm.id[i], ij = sm.id[j];
          const bool swap = desc ? before(vj, ij, vi, ii) : before(vi, ii, vj, ij);
          if (swap) {
            sm.v[i] = vj;
            sm.v[j] = vi;
            sm.id[i] = ij;
            sm.id[j] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  uint32_t F = 0;
  if (has_k) {
    if (k > total) return -1;  // fewer candidates than k (a shard smaller than k sent all)
    F = fkey(sm.v[k - 1]);
  }
  if (has_mp) F = max(F, fkey(M + logf(mp)));
  if (has_p) {
    // mass of the kept set, then the sorted prefix reaching p of it (ties at the cut kept)
    for (int i = threadIdx.x; i < Np; i += blockDim.x)
      sm.scan[i] = (sm.v[i] > -INFINITY && fkey(sm.v[i]) >= F) ? __expf(sm.v[i] - M) : 0.f;
    __syncthreads();
    // inclusive scan: each thread sums a contiguous chunk, then the chunk totals
    const int per = Np / blockDim.x > 0 ? Np / blockDim.x : 1;
    const int b0 = threadIdx.x * per;
    float run = 0.f;
    if (b0 < Np)
      for (int i = b0; i < b0 + per; ++i) {
        run += sm.scan[i];
        sm.scan[i] = run;
      }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float incl = run;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += t;
    }
    if (lane == 31) sm.wsum[warp] = incl;
    __syncthreads();
    float wbase = 0.f;
    for (int w = 0; w < warp; ++w) wbase += sm.wsum[w];
    const float excl = wbase + incl - run;
    if (b0 < Np)
      for (int i = b0; i < b0 + per; ++i) sm.scan[i] += excl;
    __syncthreads();
    const float kept_mass = (has_k || has_mp) ? sm.scan[Np - 1] : Z;
    const float target = p * kept_mass;
    if (threadIdx.x == 0) sm.F = F;
    __syncthreads();
    // first sorted index whose prefix mass reaches the target
    for (int i = threadIdx.x; i < Np; i += blockDim.x) {
      const bool hit = sm.scan[i] >= target && (i == 0 || sm.scan[i - 1] < target) &&
                       sm.v[i] > -INFINITY;
      if (hit) sm.F = max(F, fkey(sm.v[i]));
    }
    __syncthreads();
    F = sm.F;
    __syncthreads();
  }
  // exact only if no shard dropped a token with key >= F
  for (int r = 0; r < world; ++r)
    if (rows[r]->thr != 0u && F < rows[r]->thr) return -1;
  // Gumbel-max over the kept candidates
  Cand best{-INFINITY, 0x7fffffff};
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    if (!(sm.v[i] > -INFINITY) || fkey(sm.v[i]) < F) continue;
    best = better(best, Cand{sm.v[i] + gumbel(seed, step, (uint32_t)sm.id[i]), sm.id[i]});
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    Cand other{__shfl_xor_sync(0xffffffffu, best.v, d), __shfl_xor_sync(0xffffffffu, best.i, d)};
    best = better(best, other);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sm.cand[warp] = best;
  __syncthreads();
  best = Cand{-INFINITY, 0x7fffffff};
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) best = better(best, sm.cand[w]);
  __syncthreads();
  return best.i == 0x7fffffff ? -1 : best.i;
}

struct RowParams {
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const float* min_p;
  const int64_t* seeds;
  const int32_t* steps;
};

B200_DEVICE int64_t merge_one(const CandRow* const* rows, int world, const RowParams& rp, int r,
                              int V_total, MergeSmem& sm) {
  const float T = rp.temperature ? rp.temperature[r] : 0.f;
  return merge_row(rows, world, T, rp.top_k ? rp.top_k[r] : 0, rp.top_p ? rp.top_p[r] : 1.f,
                   rp.min_p ? rp.min_p[r] : 0.f, rp.seeds ? (uint64_t)rp.seeds[r] : 0ull,
                   rp.steps ? (uint32_t)rp.steps[r] : 0u, V_total, sm);
}

// Single-GPU form: every shard's candidate rows are already in local memory [world][R].
__global__ void __launch_bounds__(kMergeThreads)
    merge_local_kernel(const CandRow* __restrict__ cands, int world, int R, RowParams rp,
                       int V_total, int64_t* __restrict__ out) {
  __shared__ MergeSmem sm;
  const CandRow* rows[comm::kMaxRanks];
  for (int r = blockIdx.x; r < R; r += gridDim.x) {
    for (int w = 0; w < world; ++w) rows[w] = cands + (size_t)w * R + r;
    const int64_t t = merge_one(rows, world, rp, r, V_total, sm);
    if (threadIdx.x == 0) out[r] = t;
    __syncthreads();
  }
}

struct ExchangeParams {
  int rank, world, R, parity, V_total;
  const CandRow* mine;                   // [R] this rank's candidate rows (local)
  CandRow* region[comm::kMaxRanks];      // this call's candidate region of every rank [world][R]
  uint32_t* flags[comm::kMaxRanks];      // flag region of every rank (phases 4 / 5)
  uint32_t* epochs;                      // local per-block epoch counters
  RowParams rp;
  int64_t* out;
  int* err;
};

__global__ void __launch_bounds__(kMergeThreads) topk_exchange_kernel(ExchangeParams a) {
  __shared__ MergeSmem sm;
  __shared__ uint32_t epoch_s;
  __shared__ int ok_all;
  constexpr int kVecs = (int)(sizeof(CandRow) / 16);
  // 1. store this rank's candidate rows of this block into every rank's region [rank][row]
  for (int r = blockIdx.x; r < a.R; r += gridDim.x) {
    const uint4* src = reinterpret_cast<const uint4*>(a.mine + r);
    for (int i = threadIdx.x; i < a.world * kVecs; i += blockDim.x) {
      const int p = i / kVecs, c = i - p * kVecs;
      uint4* dst = reinterpret_cast<uint4*>(a.region[p] + (size_t)a.rank * a.R + r);
      dst[c] = src[c];
    }
  }
  __syncthreads();
  __threadfence_system();
  if (threadIdx.x == 0) {
    epoch_s = a.epochs[blockIdx.x] + 1;
    a.epochs[blockIdx.x] = epoch_s;
    ok_all = 1;
  }
  __syncthreads();
  // 2. per-block epoch barrier with every peer (bounded)
  if (threadIdx.x < a.world) {
    const int p = threadIdx.x;
    const size_t phase = 4 + a.parity;
    uint32_t* peer_slot =
        a.flags[p] + (phase * comm::kMaxBlocks + blockIdx.x) * comm::kMaxRanks + a.rank;
    st_release_sys_u32(peer_slot, epoch_s);
    const uint32_t* my_slot =
        a.flags[a.rank] + (phase * comm::kMaxBlocks + blockIdx.x) * comm::kMaxRanks + p;
    const long long t0 = clock64();
    for (uint32_t spin = 1; (int32_t)(ld_acquire_sys_u32(my_slot) - epoch_s) < 0; ++spin) {
      if ((spin & 31) != 0) continue;  // error word / clock every 32nd poll
      if (clock64() - t0 > kWaitBudgetCycles) {
        record_error(a.err, kErrPeerTimeout);
        ok_all = 0;
        break;
      }
      if (error_raised(a.err)) {
        ok_all = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (!ok_all) return;
  // 3. merge every row of this block from local memory
  const CandRow* local = a.region[a.rank];
  const CandRow* rows[comm::kMaxRanks];
  for (int r = blockIdx.x; r < a.R; r += gridDim.x) {
    for (int w = 0; w < a.world; ++w) rows[w] = local + (size_t)w * a.R + r;
    const int64_t t = merge_one(rows, a.world, a.rp, r, a.V_total, sm);
    if (threadIdx.x == 0) a.out[r] = t;
    __syncthreads();
  }
}

}  // namespace

void run_shard_candidates(const float* logits, int64_t ld, int R, int V, int vocab_offset,
                          const float* temperature, const int64_t* seeds, const int32_t* steps,
                          CandRow* out, cudaStream_t s) {
  if (R == 0) return;
  shard_candidates_kernel<<<R, kThreads, 0, s>>>(logits, ld, V, vocab_offset, temperature, seeds,
                                                  steps, out);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_merge_candidates_local(const CandRow* cands, int world, int R, const float* temperature,
                                const int32_t* top_k, const float* top_p, const float* min_p,
                                const int64_t* seeds, const int32_t* steps, int V_total,
                                int64_t* out, cudaStream_t s) {
  B200_REQUIRE(world >= 1 && world <= comm::kMaxRanks, "merge candidates: world size");
  if (R == 0) return;
  RowParams rp{temperature, top_k, top_p, min_p, seeds, steps};
  merge_local_kernel<<<std::min(R, 1024), kMergeThreads, 0, s>>>(cands, world, R, rp, V_total,
                                                                 out);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_topk_exchange(const TopkExchangeArgs& x, cudaStream_t s) {
  B200_REQUIRE(x.world >= 2 && x.world <= comm::kMaxRanks, "top-k exchange: world size");
  if (x.R == 0) return;
  ExchangeParams a{};
  a.rank = x.rank;
  a.world = x.world;
  a.R = x.R;
  a.parity = x.parity;
  a.V_total = x.V_total;
  a.mine = x.mine;
  for (int p = 0; p < x.world; ++p) {
    a.region[p] = x.region[p];
    a.flags[p] = x.flags[p];
  }
  a.epochs = x.epochs;
  a.rp = RowParams{x.temperature, x.top_k, x.top_p, x.min_p, x.seeds, x.steps};
  a.out = x.out;
  a.err = x.err;
  const int blocks = std::min(x.R, comm::kMaxBlocks);
  topk_exchange_kernel<<<blocks, kMergeThreads, 0, s>>>(a);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace sampling
}  // namespace b200
