// TurboQuant-style quantised KV cache for sm_100a: store, paged decode and prefill dequant.
//
// Reference behaviour: the reference's MUSATurboQuantAttentionBackend
// (vllm_musa/v1/attention/backends/turboquant.py:37-114) serves the four cache dtypes
// turboquant_k8v4 / turboquant_4bit_nc / turboquant_k3v4_nc / turboquant_3bit_nc through the
// upstream TurboQuant attention implementation.  This file is this framework's own design of
// that cache for Blackwell:
//
//   key, MSE mode (3 or 4 bits): randomised Walsh-Hadamard rotation y = H (s . k) / sqrt(D)
//     (s = +-1 signs from a murmur3 fmix32 hash of the dimension index, H the Sylvester
//     Hadamard matrix), every coordinate of sqrt(D) * y / |k| snapped to the nearest
//     Lloyd-Max level of the standard normal (Max, 1960), one fp16 scale per vector.  With
//     norm correction the scale is |k| / |levels| (the dequantised vector keeps the exact
//     norm), otherwise |k| / sqrt(D).  Scores are taken in the rotated space: the decode
//     kernel rotates q once per warp, so keys are never rotated back on the decode path.
//   key, fp8 mode (8 bits): e4m3 with one fp16 scale (amax / 448) per vector, not rotated.
//   value (3 or 4 bits): uniform levels between the vector's min and max (fp16 scale, zero).
//   value, fp8 mode (8 bits): e4m3 with one fp16 scale (amax / 448) per vector (zero unused);
//     with fp8 keys this is the "fp8" KV cache (e4m3 with per-vector scales).
//
// Slot of one (token, KV head), bytes: [key codes D*kb/8 | value codes D*vb/8 | key scale f16 |
// value scale f16 | value zero f16 | pad to 16].  Codes are a little-endian bit stream: the
// code of dimension i occupies bits [i*b, i*b + b).  The cache is [num_blocks, Hkv,
// block_size, slot] bytes, the geometry of the bf16 caches with the slot as the last dim.
//
// One warp owns one (token, head) vector: lane l holds dimensions [E*l, E*l + E), E = D / 32,
// so the Hadamard transform is E-wide butterflies in registers plus five shuffle stages.
#include <stdexcept>
#include <string>

#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "../common/host_check.h"

namespace b200 {
namespace tq {

// Lloyd-Max reconstruction levels of N(0, 1), ascending (Lloyd iteration to convergence:
// boundaries at midpoints, levels at the conditional means of the normal density).
__constant__ float c_lv3[8] = {-2.1519457f, -1.3439093f, -0.7560053f, -0.2450942f,
                               0.2450942f,  0.7560053f,  1.3439093f,  2.1519457f};
__constant__ float c_lv4[16] = {-2.7325896f, -2.0690172f, -1.6180464f, -1.2562312f,
                                -0.9423405f, -0.6567591f, -0.3880483f, -0.1283950f,
                                0.1283950f,  0.3880483f,  0.6567591f,  0.9423405f,
                                1.2562312f,  1.6180464f,  2.0690172f,  2.7325896f};

constexpr int kMaxGroup = 8;   // query heads per KV head handled by one decode CTA
constexpr int kDecodeWarps = 4;

template <int B>
B200_DEVICE float level(int i) {
  if constexpr (B == 3) return c_lv3[i];
  else return c_lv4[i];
}

// Index of the nearest level: the number of midpoints strictly below z.
template <int B>
B200_DEVICE int nearest_level(float z) {
  int idx = 0;
#pragma unroll
  for (int i = 0; i < (1 << B) - 1; ++i) idx += z > 0.5f * (level<B>(i) + level<B>(i + 1));
  return idx;
}

B200_DEVICE uint32_t fmix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85ebca6bu;
  h ^= h >> 13;
  h *= 0xc2b2ae35u;
  h ^= h >> 16;
  return h;
}

B200_DEVICE float rot_sign(int i) {
  return (fmix32(uint32_t(i) + 0x9e3779b9u) & 1u) ? -1.f : 1.f;
}

// In-place natural-order Walsh-Hadamard transform of the warp's D = 32 * E values.
template <int E>
B200_DEVICE void warp_fwht(float (&x)[E], int lane) {
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int i = 0; i < E; ++i) {
      if ((i & h) == 0) {
        const float a = x[i], b = x[i + h];
        x[i] = a + b;
        x[i + h] = a - b;
      }
    }
  }
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float o = __shfl_xor_sync(0xffffffffu, x[i], m);
      x[i] = upper ? (o - x[i]) : (x[i] + o);
    }
  }
}

// OR `nbits` (<= 8) bits of `val` into the bit stream at `pos` (shared-memory words).
B200_DEVICE void put_bits(uint32_t* w, int pos, uint32_t val, int nbits) {
  const int word = pos >> 5, sh = pos & 31;
  atomicOr(&w[word], val << sh);
  if (sh + nbits > 32) atomicOr(&w[word + 1], val >> (32 - sh));
}

// Read `nbits` (<= 32, plus shift <= 31) bits at `pos` of a slot's word stream.
B200_DEVICE uint32_t get_bits(const uint32_t* w, int pos, int nbits) {
  const int word = pos >> 5, sh = pos & 31;
  uint64_t v = w[word];
  if (sh + nbits > 32) v |= uint64_t(w[word + 1]) << 32;
  return uint32_t(v >> sh) & (nbits >= 32 ? 0xffffffffu : ((1u << nbits) - 1u));
}

B200_DEVICE float half_at(const uint32_t* w, int byte_off) {
  const uint32_t word = w[byte_off >> 2];
  const unsigned short bits = (byte_off & 2) ? (word >> 16) : (word & 0xffffu);
  return __half2float(__ushort_as_half(bits));
}

B200_DEVICE float fp8_to_float(uint32_t byte) {
  __nv_fp8_e4m3 f;
  f.__x = static_cast<__nv_fp8_storage_t>(byte);
  return static_cast<float>(f);
}

// Dequantise this lane's E key coordinates.  MSE keys come back in the ROTATED space.
// Per-lane level indices differ, so the table is read from shared memory (`lv`): divergent
// __constant__ reads would serialise across the warp.
template <int E, int KB>
B200_DEVICE void load_key(const uint32_t* sw, int lane, float ksc, const float* lv, float (&k)[E]) {
  if constexpr (KB == 8) {
#pragma unroll
    for (int c = 0; c < E; c += 4) {
      const uint32_t word = sw[(E * lane + c) >> 2];
#pragma unroll
      for (int e = 0; e < 4 && c + e < E; ++e) {
        const int byte = (E * lane + c + e) & 3;  // E = 2 puts odd lanes in the upper half
        k[c + e] = fp8_to_float((word >> (8 * byte)) & 0xffu) * ksc;
      }
    }
  } else {
    const uint32_t bits = get_bits(sw, E * lane * KB, E * KB);
#pragma unroll
    for (int e = 0; e < E; ++e) k[e] = lv[(bits >> (e * KB)) & ((1u << KB) - 1u)] * ksc;
  }
}

template <int E, int VB>
B200_DEVICE void load_value(const uint32_t* sw, int key_bytes, int lane, float vsc, float vz,
                            float (&v)[E]) {
  if constexpr (VB == 8) {  // e4m3 codes, byte-aligned after the key codes
    const uint8_t* bytes = reinterpret_cast<const uint8_t*>(sw) + key_bytes + E * lane;
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = fp8_to_float(bytes[e]) * vsc;
  } else {
    const uint32_t bits = get_bits(sw, key_bytes * 8 + E * lane * VB, E * VB);
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = float((bits >> (e * VB)) & ((1u << VB) - 1u)) * vsc + vz;
  }
}

// ------------------------------------------------------------------------------------ store
template <int D, int KB, int VB>
__global__ void __launch_bounds__(256) tq_store_kernel(TQStoreArgs a) {
  constexpr int E = D / 32;
  constexpr int L = (1 << VB) - 1;
  __shared__ float s_lv[16];
  if constexpr (KB != 8) {
    if (threadIdx.x < (1 << KB)) s_lv[threadIdx.x] = level<KB>(threadIdx.x);
    __syncthreads();
  }
  extern __shared__ uint32_t tq_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int t = blockIdx.x;
  const int slot = a.slot_mapping[t];
  if (slot < 0) return;
  const int blk = slot / a.block_size, off = slot % a.block_size;
  if (blk >= a.num_blocks) {
    if (lane == 0 && warp == 0) record_error(a.err, kErrBadIndex);
    return;
  }
  const int words = a.slot_bytes >> 2;
  uint32_t* w = tq_smem + warp * words;
  const int key_bytes = D * KB / 8, meta = key_bytes + D * VB / 8;
  const float rs = rsqrtf(float(D));
  for (int h = warp; h < a.Hkv; h += nw) {
    float kx[E], vx[E];
    const __nv_bfloat16* kp = a.k + int64_t(t) * a.ld_k + h * D + E * lane;
    const __nv_bfloat16* vp = a.v + int64_t(t) * a.ld_v + h * D + E * lane;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      kx[e] = __bfloat162float(kp[e]);
      vx[e] = __bfloat162float(vp[e]);
    }
    for (int i = lane; i < words; i += 32) w[i] = 0u;
    __syncwarp();
    float ksc;
    if constexpr (KB == 8) {
      float am = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) am = fmaxf(am, fabsf(kx[e]));
      am = warp_max(am);
      ksc = __half2float(__float2half_rn(am / 448.f));
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float x = ksc > 0.f ? kx[e] / ksc : 0.f;
        const uint32_t b = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
        put_bits(w, (E * lane + e) * 8, b, 8);
      }
    } else {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        ss += kx[e] * kx[e];
        kx[e] *= rot_sign(E * lane + e);
      }
      const float norm = sqrtf(warp_sum(ss));
      warp_fwht<E>(kx, lane);
      const float zmul = norm > 0.f ? sqrtf(float(D)) / norm : 0.f;
      float cs = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int c = nearest_level<KB>(kx[e] * rs * zmul);
        const float lv = s_lv[c];
        cs += lv * lv;
        put_bits(w, (E * lane + e) * KB, uint32_t(c), KB);
      }
      cs = warp_sum(cs);
      ksc = a.norm_correction ? (cs > 0.f ? norm / sqrtf(cs) : 0.f) : norm * rs;
      ksc = __half2float(__float2half_rn(ksc));
    }
    __half hsc, hz;
    if constexpr (VB == 8) {
      float am = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) am = fmaxf(am, fabsf(vx[e]));
      am = warp_max(am);
      hsc = __float2half_rn(am / 448.f);
      hz = __float2half_rn(0.f);
      const float vsc = __half2float(hsc);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float x = vsc > 0.f ? vx[e] / vsc : 0.f;
        const uint32_t b = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
        put_bits(w, key_bytes * 8 + (E * lane + e) * 8, b, 8);
      }
    } else {
      float vmin = vx[0], vmax = vx[0];
#pragma unroll
      for (int e = 1; e < E; ++e) {
        vmin = fminf(vmin, vx[e]);
        vmax = fmaxf(vmax, vx[e]);
      }
      vmin = -warp_max(-vmin);
      vmax = warp_max(vmax);
      hsc = __float2half_rn((vmax - vmin) / float(L));
      hz = __float2half_rn(vmin);
      const float vsc = __half2float(hsc), vz = __half2float(hz);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        int c = 0;
        if (vsc > 0.f) c = min(L, max(0, __float2int_rn((vx[e] - vz) / vsc)));
        put_bits(w, key_bytes * 8 + (E * lane + e) * VB, uint32_t(c), VB);
      }
    }
    if (lane == 0) {
      const uint32_t kb16 = __half_as_ushort(__float2half_rn(ksc));
      atomicOr(&w[meta >> 2], kb16 | (uint32_t(__half_as_ushort(hsc)) << 16));
      atomicOr(&w[(meta >> 2) + 1], uint32_t(__half_as_ushort(hz)));
    }
    __syncwarp();
    uint32_t* dst = reinterpret_cast<uint32_t*>(
        a.cache + ((int64_t(blk) * a.Hkv + h) * a.block_size + off) * a.slot_bytes);
    for (int i = lane; i < words; i += 32) dst[i] = w[i];
    __syncwarp();
  }
}

// ----------------------------------------------------------------------------------- decode
template <int D, int KB, int VB>
__global__ void __launch_bounds__(kDecodeWarps * 32) tq_decode_kernel(TQDecodeArgs a) {
  constexpr int E = D / 32;
  __shared__ float s_m[kDecodeWarps][kMaxGroup], s_l[kDecodeWarps][kMaxGroup];
  __shared__ float s_acc[kDecodeWarps][kMaxGroup][D];
  __shared__ float s_lv[16];
  if constexpr (KB != 8) {
    if (threadIdx.x < (1 << KB)) s_lv[threadIdx.x] = level<KB>(threadIdx.x);
    __syncthreads();
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
  const int G = a.Hq / a.Hkv;
  const int S = a.seq_lens[b];
  const int chunk = (S + a.splits - 1) / a.splits;
  const int t0 = sp * chunk, t1 = min(S, t0 + chunk);
  const int key_bytes = D * KB / 8, meta = key_bytes + D * VB / 8;
  const float rs = rsqrtf(float(D));

  float q[kMaxGroup][E], acc[kMaxGroup][E], m[kMaxGroup], l[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[g][e] = 0.f;
    if (g < G) {
      const __nv_bfloat16* qp = a.q + int64_t(b) * a.ld_q + (h * G + g) * D + E * lane;
#pragma unroll
      for (int e = 0; e < E; ++e) q[g][e] = __bfloat162float(qp[e]) * a.scale_log2;
      if constexpr (KB != 8) {
#pragma unroll
        for (int e = 0; e < E; ++e) q[g][e] *= rot_sign(E * lane + e);
        warp_fwht<E>(q[g], lane);
#pragma unroll
        for (int e = 0; e < E; ++e) q[g][e] *= rs;
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) q[g][e] = 0.f;
    }
  }

  const int* bt = a.block_tables + int64_t(b) * a.ld_bt;
  for (int t = t0 + warp; t < t1; t += kDecodeWarps) {
    const int blk = bt[t / a.block_size];
    if (blk < 0 || blk >= a.num_blocks) {
      if (lane == 0) record_error(a.err, kErrBadIndex);
      continue;
    }
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(
        a.cache + ((int64_t(blk) * a.Hkv + h) * a.block_size + (t % a.block_size)) * a.slot_bytes);
    const float ksc = half_at(sw, meta), vsc = half_at(sw, meta + 2), vz = half_at(sw, meta + 4);
    float k[E], v[E];
    load_key<E, KB>(sw, lane, ksc, s_lv, k);
    load_value<E, VB>(sw, key_bytes, lane, vsc, vz, v);
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g < G) {
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) s = fmaf(q[g][e], k[e], s);
        s = warp_sum(s);
        const float mn = fmaxf(m[g], s);
        const float corr = exp2f(m[g] - mn), p = exp2f(s - mn);
        m[g] = mn;
        l[g] = l[g] * corr + p;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[g][e] = fmaf(acc[g][e], corr, p * v[e]);
      }
    }
  }

#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g < G) {
      if (lane == 0) {
        s_m[warp][g] = m[g];
        s_l[warp][g] = l[g];
      }
#pragma unroll
      for (int e = 0; e < E; ++e) s_acc[warp][g][E * lane + e] = acc[g][e];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int g = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < kDecodeWarps; ++w2) M = fmaxf(M, s_m[w2][g]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w2 = 0; w2 < kDecodeWarps; ++w2) {
        const float wt = s_m[w2][g] == -INFINITY ? 0.f : exp2f(s_m[w2][g] - M);
        Ls += s_l[w2][g] * wt;
        O += s_acc[w2][g][d] * wt;
      }
    }
    const int hq = h * G + g;
    const float o = Ls > 0.f ? O / Ls : 0.f;
    if (a.splits == 1) {
      a.out[int64_t(b) * a.ld_out + hq * D + d] = __float2bfloat16(o);
    } else {
      const int64_t row = (int64_t(b) * a.Hq + hq) * a.splits + sp;
      a.ws_o[row * D + d] = o;
      if (d == 0) a.ws_lse[row] = Ls > 0.f ? M + log2f(Ls) : -INFINITY;
    }
  }
}

// Merge the split partials of one (sequence, query head): weights 2^(lse_s - max lse).
__global__ void tq_combine_kernel(TQDecodeArgs a, int D) {
  const int b = blockIdx.x, hq = blockIdx.y;
  const int64_t row0 = (int64_t(b) * a.Hq + hq) * a.splits;
  float M = -INFINITY;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.ws_lse[row0 + s]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float O = 0.f, W = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < a.splits; ++s) {
        const float lse = a.ws_lse[row0 + s];
        if (lse == -INFINITY) continue;
        const float wt = exp2f(lse - M);
        W += wt;
        O += wt * a.ws_o[(row0 + s) * D + d];
      }
    }
    a.out[int64_t(b) * a.ld_out + hq * D + d] = __float2bfloat16(W > 0.f ? O / W : 0.f);
  }
}

// ------------------------------------------------------------------------- prefill dequant
// One CTA per (request, block-table entry): dequantises the entry's page into bf16 caches laid
// out [R * W, Hkv, block_size, D] (page r * W + w), keys back in the original space.
template <int D, int KB, int VB>
__global__ void __launch_bounds__(256) tq_dequant_kernel(TQDequantArgs a) {
  constexpr int E = D / 32;
  __shared__ float s_lv[16];
  if constexpr (KB != 8) {
    if (threadIdx.x < (1 << KB)) s_lv[threadIdx.x] = level<KB>(threadIdx.x);
    __syncthreads();
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int r = blockIdx.x / a.W, wi = blockIdx.x % a.W;
  const int S = a.seq_lens[r];
  if (wi * a.block_size >= S) return;
  const int blk = a.block_tables[int64_t(r) * a.ld_bt + wi];
  if (blk < 0 || blk >= a.num_blocks) {
    if (threadIdx.x == 0) record_error(a.err, kErrBadIndex);
    return;
  }
  const int key_bytes = D * KB / 8, meta = key_bytes + D * VB / 8;
  const float rs = rsqrtf(float(D));
  const int n = a.Hkv * a.block_size;
  for (int i = warp; i < n; i += nw) {
    const int h = i / a.block_size, off = i % a.block_size;
    if (wi * a.block_size + off >= S) continue;
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(
        a.cache + ((int64_t(blk) * a.Hkv + h) * a.block_size + off) * a.slot_bytes);
    const float ksc = half_at(sw, meta), vsc = half_at(sw, meta + 2), vz = half_at(sw, meta + 4);
    float k[E], v[E];
    load_key<E, KB>(sw, lane, ksc, s_lv, k);
    load_value<E, VB>(sw, key_bytes, lane, vsc, vz, v);
    if constexpr (KB != 8) {
      warp_fwht<E>(k, lane);
#pragma unroll
      for (int e = 0; e < E; ++e) k[e] *= rs * rot_sign(E * lane + e);
    }
    const int64_t o = ((int64_t(blockIdx.x) * a.Hkv + h) * a.block_size + off) * D + E * lane;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      a.k_out[o + e] = __float2bfloat16(k[e]);
      a.v_out[o + e] = __float2bfloat16(v[e]);
    }
  }
}

// ------------------------------------------------------------------------------- launchers
namespace {

template <template <int, int, int> class F, typename... Args>
void dispatch(int D, int kb, int vb, Args&&... args) {
  auto by_bits = [&](auto dtag) {
    constexpr int DD = decltype(dtag)::value;
    if (kb == 8 && vb == 8) return F<DD, 8, 8>::run(args...);
    if (kb == 8 && vb == 4) return F<DD, 8, 4>::run(args...);
    if (kb == 4 && vb == 4) return F<DD, 4, 4>::run(args...);
    if (kb == 3 && vb == 4) return F<DD, 3, 4>::run(args...);
    if (kb == 3 && vb == 3) return F<DD, 3, 3>::run(args...);
    throw std::runtime_error("turboquant: unsupported key/value bits " + std::to_string(kb) +
                             "/" + std::to_string(vb));
  };
  if (D == 64) return by_bits(std::integral_constant<int, 64>{});
  if (D == 128) return by_bits(std::integral_constant<int, 128>{});
  if (D == 256) return by_bits(std::integral_constant<int, 256>{});
  throw std::runtime_error("turboquant: head_dim must be 64, 128 or 256");
}

template <int D, int KB, int VB>
struct StoreL {
  static void run(const TQStoreArgs& a, cudaStream_t st) {
    const int warps = std::min(8, std::max(1, a.Hkv));
    const size_t smem = size_t(warps) * a.slot_bytes;
    tq_store_kernel<D, KB, VB><<<a.T, warps * 32, smem, st>>>(a);
    count_launch();
  }
};

template <int D, int KB, int VB>
struct DecodeL {
  static void run(const TQDecodeArgs& a, cudaStream_t st) {
    dim3 grid(a.B, a.Hkv, a.splits);
    tq_decode_kernel<D, KB, VB><<<grid, kDecodeWarps * 32, 0, st>>>(a);
    count_launch();
    if (a.splits > 1) {
      tq_combine_kernel<<<dim3(a.B, a.Hq), std::min(D, 256), 0, st>>>(a, D);
      count_launch();
    }
  }
};

template <int D, int KB, int VB>
struct DequantL {
  static void run(const TQDequantArgs& a, cudaStream_t st) {
    tq_dequant_kernel<D, KB, VB><<<a.R * a.W, 256, 0, st>>>(a);
    count_launch();
  }
};

}  // namespace

int slot_bytes(int D, int kb, int vb) { return ((D * kb / 8 + D * vb / 8 + 6) + 15) / 16 * 16; }

void run_store(const TQStoreArgs& a, int D, int kb, int vb, cudaStream_t st) {
  if (a.T == 0) return;
  if (a.slot_bytes != slot_bytes(D, kb, vb)) throw std::runtime_error("turboquant: slot size");
  dispatch<StoreL>(D, kb, vb, a, st);
}

void run_decode(const TQDecodeArgs& a, int D, int kb, int vb, cudaStream_t st) {
  if (a.B == 0) return;
  if (a.Hq % a.Hkv != 0 || a.Hq / a.Hkv > kMaxGroup)
    throw std::runtime_error("turboquant decode: at most 8 query heads per KV head");
  if (a.splits < 1 || (a.splits > 1 && (!a.ws_o || !a.ws_lse)))
    throw std::runtime_error("turboquant decode: split workspace");
  dispatch<DecodeL>(D, kb, vb, a, st);
}

void run_dequant(const TQDequantArgs& a, int D, int kb, int vb, cudaStream_t st) {
  if (a.R == 0 || a.W == 0) return;
  dispatch<DequantL>(D, kb, vb, a, st);
}

}  // namespace tq
}  // namespace b200
