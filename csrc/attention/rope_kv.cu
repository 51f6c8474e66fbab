// Fused (optional per-head Q/K RMSNorm) + rotary embedding + paged KV-cache insert.
//
// Input is the packed QKV projection output [T, (Hq + 2*Hkv) * D].  Per token:
//   q heads: [RMSNorm] -> RoPE -> written back in place (attention reads q from the buffer)
//   k heads: [RMSNorm] -> RoPE -> written to k_cache at slot_mapping[t]
//   v heads: copied to v_cache at slot_mapping[t]
// With no cache (k_cache == nullptr) it only rotates: q and k are written back in place.
// Cache layout is [num_blocks, Hkv, block_size, D] so that one page of one KV head is a
// contiguous block_size*D run (a single bulk copy for the attention kernels).  RoPE supports
// NeoX (rotate halves) and GPT-J (rotate pairs) styles and partial rotary (rot_dim < D); the
// cos/sin cache is [max_pos, rot_dim] fp32 = [cos(rot_dim/2) | sin(rot_dim/2)].  Multimodal
// RoPE (M-RoPE) takes positions [3, T] and picks each frequency's row by section.
//
// Reference counterparts: vllm_musa/jit_kernel/csrc/norm/qk_mrope.mu:168-1311 (Qwen3 fused
// QK-norm + RoPE + cache), vllm_musa/jit_kernel/csrc/rope/rotary_embedding.mu:124-708 (RoPE),
// csrc/musa/cache_kernels.mu:16 (reshape_and_cache_flash NHD).  One warp per (token, head);
// the head vector is staged in shared memory so any rot_dim / style pairs are one load away.
#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace rope {

constexpr int kWarps = 4;

// Which position row (0 temporal, 1 height, 2 width) rotary frequency f uses.  Sectioned
// (Qwen2-VL style): the first s0 frequencies temporal, the next s1 height, the rest width.
// Interleaved (Qwen3-VL style): f % 3 == 1 height while f < 3 * s1, f % 3 == 2 width while
// f < 3 * s2, otherwise temporal.
B200_DEVICE int mrope_component(const MropeSpec& mr, int f) {
  if (mr.mode == 1) return f < mr.s0 ? 0 : (f < mr.s0 + mr.s1 ? 1 : 2);
  const int r = f % 3;
  if (r == 1 && f < 3 * mr.s1) return 1;
  if (r == 2 && f < 3 * mr.s2) return 2;
  return 0;
}

template <int D>
__global__ void __launch_bounds__(kWarps * 32)
    rope_kv_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld_qkv,
                   const int32_t* __restrict__ positions, const float* __restrict__ cos_sin,
                   const __nv_bfloat16* __restrict__ q_norm_w,
                   const __nv_bfloat16* __restrict__ k_norm_w, __nv_bfloat16* __restrict__ k_cache,
                   __nv_bfloat16* __restrict__ v_cache, const int32_t* __restrict__ slot_mapping,
                   int T, int Hq, int Hkv, int block_size, int rot_dim, int neox, float eps,
                   int* err, MropeSpec mr) {
  constexpr int E = D / 32;  // elements per lane
  __shared__ float stage[kWarps][D];
  pdl_launch_dependents();
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  const int64_t gid = (int64_t)blockIdx.x * kWarps + warp;
  if (gid >= (int64_t)T * heads) return;
  const int t = gid / heads, h = gid % heads;
  __nv_bfloat16* src = qkv + t * ld_qkv + (int64_t)h * D + lane * E;

  float v[E];
#pragma unroll
  for (int j = 0; j < E; ++j) v[j] = bf2f(src[j]);

  const bool is_q = h < Hq, is_k = !is_q && h < Hq + Hkv, is_v = h >= Hq + Hkv;
  const int32_t slot = slot_mapping ? slot_mapping[t] : -1;

  if (!is_v) {
    const __nv_bfloat16* nw = is_q ? q_norm_w : k_norm_w;
    if (nw) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) ss += v[j] * v[j];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / D + eps);
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = v[j] * inv * bf2f(nw[lane * E + j]);
    }
    if (rot_dim > 0) {
#pragma unroll
      for (int j = 0; j < E; ++j) stage[warp][lane * E + j] = v[j];
      __syncwarp();
      const int half = rot_dim / 2;
      const float* cs = cos_sin + (int64_t)positions[t] * rot_dim;
#pragma unroll
      for (int j = 0; j < E; ++j) {
        const int i = lane * E + j;
        if (i < rot_dim) {
          if (mr.mode != 0) {
            // multimodal RoPE: frequency f takes its position from the temporal / height /
            // width row of `positions` ([3, pos_stride])
            const int f = neox ? (i < half ? i : i - half) : i / 2;
            const int comp = mrope_component(mr, f);
            cs = cos_sin + (int64_t)positions[comp * mr.pos_stride + t] * rot_dim;
          }
          if (neox) {
            const int f = i < half ? i : i - half;
            const float c = cs[f], s = cs[half + f];
            const float other = stage[warp][i < half ? i + half : i - half];
            v[j] = i < half ? v[j] * c - other * s : v[j] * c + other * s;
          } else {
            const int f = i / 2;
            const float c = cs[f], s = cs[half + f];
            const float other = stage[warp][i ^ 1];
            v[j] = (i & 1) ? v[j] * c + other * s : v[j] * c - other * s;
          }
        }
      }
    }
  }

  if (is_q || (is_k && k_cache == nullptr)) {  // rotate-only mode keeps k in place too
#pragma unroll
    for (int j = 0; j < E; ++j) src[j] = f2bf(v[j]);
    return;
  }
  if (k_cache == nullptr) return;
  if (slot < 0) return;  // padding token: nothing to cache
  const int kvh = is_k ? h - Hq : h - Hq - Hkv;
  const int64_t blk = slot / block_size, off = slot % block_size;
  __nv_bfloat16* dst = (is_k ? k_cache : v_cache) + ((blk * Hkv + kvh) * block_size + off) * D +
                       lane * E;
#pragma unroll
  for (int j = 0; j < E; ++j) dst[j] = f2bf(v[j]);
}

// Vectorised form for the common layouts (no M-RoPE): lane l owns the E = D / 32 consecutive
// elements [E l, E l + E) of the head, loaded and stored as one 4 / 8 / 16-byte vector; NeoX
// pairs (i, i + rot_dim / 2) sit in lanes l and l ^ (rot_dim / 2E) and are exchanged with one
// warp shuffle per element (rot_dim / 2E is a power of two for every supported rot_dim), GPT-J
// pairs (i, i ^ 1) sit in the same lane; cos / sin come in as vectors of E (NeoX) or E / 2
// (GPT-J) floats.  Same results as rope_kv_kernel.
template <int E>
struct BfVec;
template <>
struct BfVec<2> { using T = uint32_t; };
template <>
struct BfVec<4> { using T = uint2; };
template <>
struct BfVec<8> { using T = uint4; };

template <int E>
B200_DEVICE void load_bf(const __nv_bfloat16* p, float (&v)[E]) {
  const typename BfVec<E>::T raw = *reinterpret_cast<const typename BfVec<E>::T*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < E / 2; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    v[2 * j] = f.x;
    v[2 * j + 1] = f.y;
  }
}

template <int E>
B200_DEVICE void store_bf(__nv_bfloat16* p, const float (&v)[E]) {
  typename BfVec<E>::T raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int j = 0; j < E / 2; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<typename BfVec<E>::T*>(p) = raw;
}

template <int D>
__global__ void __launch_bounds__(kWarps * 32)
    rope_kv_vec_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld_qkv,
                       const int32_t* __restrict__ positions, const float* __restrict__ cos_sin,
                       const __nv_bfloat16* __restrict__ q_norm_w,
                       const __nv_bfloat16* __restrict__ k_norm_w,
                       __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                       const int32_t* __restrict__ slot_mapping, int T, int Hq, int Hkv,
                       int block_size, int rot_dim, int neox, float eps) {
  constexpr int E = D / 32;
  pdl_launch_dependents();
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int heads = Hq + 2 * Hkv;
  const int64_t gid = (int64_t)blockIdx.x * kWarps + warp;
  if (gid >= (int64_t)T * heads) return;
  const int t = gid / heads, h = gid % heads;
  __nv_bfloat16* src = qkv + t * ld_qkv + (int64_t)h * D + lane * E;
  float v[E];
  load_bf<E>(src, v);
  const bool is_q = h < Hq, is_k = !is_q && h < Hq + Hkv, is_v = h >= Hq + Hkv;
  if (!is_v) {
    const __nv_bfloat16* nw = is_q ? q_norm_w : k_norm_w;
    if (nw) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < E; ++j) ss += v[j] * v[j];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / D + eps);
      float w[E];
      load_bf<E>(nw + lane * E, w);
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = v[j] * inv * w[j];
    }
    if (rot_dim > 0) {
      const int half = rot_dim / 2;
      const float* cs = cos_sin + (int64_t)positions[t] * rot_dim;
      if (neox) {
        const int P = half / E;  // partner lane distance (power of two)
        float o[E];
#pragma unroll
        for (int j = 0; j < E; ++j) o[j] = __shfl_xor_sync(0xffffffffu, v[j], P);
        if (lane < 2 * P) {
          const int f0 = E * (lane & (P - 1));
          const bool lo = lane < P;
#pragma unroll
          for (int j = 0; j < E; ++j) {
            const float c = cs[f0 + j], sn = cs[half + f0 + j];
            v[j] = lo ? v[j] * c - o[j] * sn : v[j] * c + o[j] * sn;
          }
        }
      } else if (lane * E < rot_dim) {
#pragma unroll
        for (int j = 0; j < E; j += 2) {
          const int f = (lane * E + j) / 2;
          const float c = cs[f], sn = cs[half + f];
          const float a = v[j], b = v[j + 1];
          v[j] = a * c - b * sn;
          v[j + 1] = b * c + a * sn;
        }
      }
    }
  }
  if (is_q || (is_k && k_cache == nullptr)) {
    store_bf<E>(src, v);
    return;
  }
  if (k_cache == nullptr) return;
  const int32_t slot = slot_mapping ? slot_mapping[t] : -1;
  if (slot < 0) return;
  const int kvh = is_k ? h - Hq : h - Hq - Hkv;
  const int64_t blk = slot / block_size, off = slot % block_size;
  __nv_bfloat16* dst = (is_k ? k_cache : v_cache) + ((blk * Hkv + kvh) * block_size + off) * D +
                       lane * E;
  store_bf<E>(dst, v);
}

// Paged KV-cache insert of separate key / value tensors ([T, Hkv, D] with row and head
// strides, as an attention layer hands them over after its own RoPE): one warp per (token,
// KV head), 16-byte vectors, slot < 0 skips the token.  Same cache layout as above.
template <int D>
__global__ void __launch_bounds__(kWarps * 32)
    kv_insert_kernel(const __nv_bfloat16* __restrict__ key, int64_t k_ld, int64_t k_hs,
                     const __nv_bfloat16* __restrict__ value, int64_t v_ld, int64_t v_hs,
                     __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                     const int64_t* __restrict__ slot_mapping, int T, int Hkv, int block_size) {
  constexpr int V = D / 8;  // 16-byte vectors per head row
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int64_t gid = (int64_t)blockIdx.x * kWarps + warp;
  if (gid >= (int64_t)T * Hkv) return;
  const int t = gid / Hkv, h = gid % Hkv;
  const int64_t slot = slot_mapping[t];
  if (slot < 0) return;
  const int64_t blk = slot / block_size, off = slot % block_size;
  const int64_t dst = ((blk * Hkv + h) * block_size + off) * D;
  const uint4* ks = reinterpret_cast<const uint4*>(key + t * k_ld + h * k_hs);
  const uint4* vs = reinterpret_cast<const uint4*>(value + t * v_ld + h * v_hs);
  for (int i = lane; i < V; i += 32) {
    reinterpret_cast<uint4*>(k_cache + dst)[i] = ks[i];
    reinterpret_cast<uint4*>(v_cache + dst)[i] = vs[i];
  }
}

void run_kv_insert(const void* key, int64_t k_ld, int64_t k_hs, const void* value, int64_t v_ld,
                   int64_t v_hs, void* k_cache, void* v_cache, const int64_t* slot_mapping, int T,
                   int Hkv, int D, int block_size, cudaStream_t s) {
  if (T == 0) return;
  B200_REQUIRE(k_ld % 8 == 0 && k_hs % 8 == 0 && v_ld % 8 == 0 && v_hs % 8 == 0,
               "kv_insert: 16-byte aligned rows");
  const int64_t warps = (int64_t)T * Hkv;
  const int blocks = (int)((warps + kWarps - 1) / kWarps);
#define B200_KVI(DD)                                                                           \
  kv_insert_kernel<DD><<<blocks, kWarps * 32, 0, s>>>(                                         \
      reinterpret_cast<const __nv_bfloat16*>(key), k_ld, k_hs,                                 \
      reinterpret_cast<const __nv_bfloat16*>(value), v_ld, v_hs,                               \
      reinterpret_cast<__nv_bfloat16*>(k_cache), reinterpret_cast<__nv_bfloat16*>(v_cache),   \
      slot_mapping, T, Hkv, block_size)
  switch (D) {
    case 64: B200_KVI(64); break;
    case 128: B200_KVI(128); break;
    case 256: B200_KVI(256); break;
    default: B200_REQUIRE(false, "kv_insert: head_dim must be 64, 128 or 256");
  }
#undef B200_KVI
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_rope_kv(const RopeKvArgs& a, cudaStream_t s) {
  if (a.T == 0) return;
  B200_REQUIRE(a.rot_dim % 2 == 0 && a.rot_dim <= a.D, "rope_kv: rot_dim");
  B200_REQUIRE(a.mrope.mode == 0 ||
                   (a.mrope.mode == 1 && a.mrope.s0 + a.mrope.s1 + a.mrope.s2 == a.rot_dim / 2) ||
                   (a.mrope.mode == 2 && a.mrope.pos_stride >= a.T),
               "rope_kv: M-RoPE sections must cover rot_dim / 2 frequencies");
  B200_REQUIRE(a.mrope.mode == 0 || a.mrope.pos_stride >= a.T, "rope_kv: M-RoPE position rows");
  const int64_t warps = (int64_t)a.T * (a.Hq + 2 * a.Hkv);
  const int blocks = (int)((warps + kWarps - 1) / kWarps);
  // vectorised kernel: no M-RoPE, 4-byte aligned rows, and for NeoX a partner-lane distance
  // rot_dim / (2E) that is a power of two
  const int E = a.D / 32;
  const int P = a.rot_dim / 2 / (E > 0 ? E : 1);
  const bool vec = a.mrope.mode == 0 && (a.ld_qkv % E) == 0 && a.D % 64 == 0 &&
                   (a.rot_dim == 0 || (a.neox ? (a.rot_dim % (2 * E) == 0 && P > 0 &&
                                                 (P & (P - 1)) == 0)
                                               : a.rot_dim % E == 0)) &&
                   (reinterpret_cast<uintptr_t>(a.qkv) % (2 * E)) == 0;
  if (vec) {
#define B200_ROPE_VEC(DD)                                                                        \
  rope_kv_vec_kernel<DD><<<blocks, kWarps * 32, 0, s>>>(                                         \
      reinterpret_cast<__nv_bfloat16*>(a.qkv), a.ld_qkv, a.positions, a.cos_sin,                 \
      reinterpret_cast<const __nv_bfloat16*>(a.q_norm_w),                                        \
      reinterpret_cast<const __nv_bfloat16*>(a.k_norm_w),                                        \
      reinterpret_cast<__nv_bfloat16*>(a.k_cache), reinterpret_cast<__nv_bfloat16*>(a.v_cache), \
      a.slot_mapping, a.T, a.Hq, a.Hkv, a.block_size, a.rot_dim, a.neox ? 1 : 0, a.eps)
    switch (a.D) {
      case 64:
        B200_ROPE_VEC(64);
        break;
      case 128:
        B200_ROPE_VEC(128);
        break;
      case 256:
        B200_ROPE_VEC(256);
        break;
      default:
        B200_REQUIRE(false, "rope_kv: head_dim must be 64, 128 or 256");
    }
#undef B200_ROPE_VEC
    B200_CUDA_OK(cudaGetLastError());
    count_launch();
    return;
  }
#define B200_ROPE_LAUNCH(DD)                                                                     \
  rope_kv_kernel<DD><<<blocks, kWarps * 32, 0, s>>>(                                             \
      reinterpret_cast<__nv_bfloat16*>(a.qkv), a.ld_qkv, a.positions, a.cos_sin,                 \
      reinterpret_cast<const __nv_bfloat16*>(a.q_norm_w),                                        \
      reinterpret_cast<const __nv_bfloat16*>(a.k_norm_w),                                        \
      reinterpret_cast<__nv_bfloat16*>(a.k_cache), reinterpret_cast<__nv_bfloat16*>(a.v_cache), \
      a.slot_mapping, a.T, a.Hq, a.Hkv, a.block_size, a.rot_dim, a.neox ? 1 : 0, a.eps, a.err, \
      a.mrope)
  switch (a.D) {
    case 64:
      B200_ROPE_LAUNCH(64);
      break;
    case 128:
      B200_ROPE_LAUNCH(128);
      break;
    case 256:
      B200_ROPE_LAUNCH(256);
      break;
    default:
      B200_REQUIRE(false, "rope_kv: head_dim must be 64, 128 or 256");
  }
#undef B200_ROPE_LAUNCH
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace rope
}  // namespace b200
