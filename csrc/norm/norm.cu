// RMSNorm family for sm_100a: plain RMSNorm, fused residual-add + RMSNorm (in place), the
// Gemma (1 + w) variant, and gated RMSNorm (RMSNorm(x) * silu(z), grouped) used by
// Gated-DeltaNet output projections.
//
// Reference counterparts: csrc/musa/fused_add_rmsnorm.mu:54 (fused add, in place),
// vllm_musa/jit_kernel/csrc/norm/rmsnorm.mu:163-433 (vec8 / small-H / fused-add variants),
// vllm_musa/jit_kernel/tilelang/layernorm_gated.py:42 (gated).  Design here: one CTA per row,
// rows held in registers as 128-bit vectors (VPT vectors of 8 bf16 per thread), a single pass
// over HBM for read and write, fp32 statistics.
#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace norm {

template <int VPT, bool kAdd, bool kGemma>
__global__ void rmsnorm_kernel(__nv_bfloat16* __restrict__ out, int64_t ld_out,
                               __nv_bfloat16* __restrict__ x, int64_t ld_x,
                               __nv_bfloat16* __restrict__ residual, int64_t ld_res,
                               const __nv_bfloat16* __restrict__ w, int H, float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int nvec = H / 8;
  uint4* xr = reinterpret_cast<uint4*>(x + row * ld_x);
  uint4* rr = kAdd ? reinterpret_cast<uint4*>(residual + row * ld_res) : nullptr;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      unpack8(xr[c], v[i]);
      if constexpr (kAdd) {
        float r[8];
        unpack8(rr[c], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        // residual is stored rounded to bf16; normalise the rounded value like the
        // unfused add-then-norm sequence would.
        uint4 packed = pack8(v[i]);
        rr[c] = packed;
        unpack8(packed, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / H + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* orow = reinterpret_cast<uint4*>(out + row * ld_out);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nvec) {
      float wf[8];
      unpack8(wr[c], wf);
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * (kGemma ? (1.f + wf[j]) : wf[j]);
      orow[c] = pack8(o);
    }
  }
}

// Gated RMSNorm: out = RMSNorm_group(x) * w * silu(z), statistics per group of `group` elems.
// One warp per (row, group) when group <= 256 elements; generic loop otherwise.
__global__ void rmsnorm_gated_kernel(__nv_bfloat16* __restrict__ out, int64_t ldo,
                                     const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                     const __nv_bfloat16* __restrict__ z, int64_t ldz,
                                     const __nv_bfloat16* __restrict__ w, int rows, int H,
                                     int group, float eps) {
  const int warps = blockDim.x / 32;
  const int gid = blockIdx.x * warps + threadIdx.x / 32;
  const int groups_per_row = H / group;
  if (gid >= rows * groups_per_row) return;
  const int row = gid / groups_per_row, g = gid % groups_per_row;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* xp = x + (size_t)row * ldx + g * group;
  const __nv_bfloat16* zp = z + (size_t)row * ldz + g * group;
  __nv_bfloat16* op = out + (size_t)row * ldo + g * group;
  float ss = 0.f;
  for (int i = lane; i < group; i += 32) {
    const float t = bf2f(xp[i]);
    ss += t * t;
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / group + eps);
  for (int i = lane; i < group; i += 32) {
    const float zv = bf2f(zp[i]);
    const float s = zv / (1.f + __expf(-zv));
    op[i] = f2bf(bf2f(xp[i]) * inv * bf2f(w[i % group]) * s);
  }
}

// (residual add +) RMSNorm + per-token 1x128 e4m3 quantisation in one pass: the normalised
// row stays in registers; each 128-element group is 16 consecutive 8-element vectors held by
// 16 consecutive lanes (blockDim is a multiple of 16), so the group amax is a half-warp
// shuffle reduction.  Writes e4m3 [rows, H] + fp32 scales [rows, H/128] (scale = amax / 448)
// and, when `out` is non-null, the bf16 normalised row as well (consumers that need both).
// Reference counterpart: csrc/musa/quantization/fused_add_rms_norm_per_token_group_fp8_quant.cu:59
// (hidden fixed at 4096 there; any multiple of 128 here).
template <int VPT, bool kAdd>
__global__ void rmsnorm_quant_kernel(__nv_fp8_e4m3* __restrict__ q, int64_t ld_q,
                                     float* __restrict__ scales, __nv_bfloat16* __restrict__ out,
                                     int64_t ld_out, const __nv_bfloat16* __restrict__ x,
                                     int64_t ld_x, __nv_bfloat16* __restrict__ residual,
                                     int64_t ld_res, const __nv_bfloat16* __restrict__ w, int H,
                                     float eps) {
  __shared__ float red[32];
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int nvec = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ld_x);
  uint4* rr = kAdd ? reinterpret_cast<uint4*>(residual + row * ld_res) : nullptr;
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    if (c < nvec) {
      unpack8(xr[c], v[i]);
      if constexpr (kAdd) {
        float r[8];
        unpack8(rr[c], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[j];
        const uint4 packed = pack8(v[i]);
        rr[c] = packed;
        unpack8(packed, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / H + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  const int groups = H / 128;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    const bool live = c < nvec;
    float o[8];
    float amax = 0.f;
    if (live) {
      float wf[8];
      unpack8(wr[c], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * inv * wf[j];
      const uint4 ob = pack8(o);
      if (out != nullptr) reinterpret_cast<uint4*>(out + row * ld_out)[c] = ob;
      unpack8(ob, o);  // quantise the bf16-rounded value, like norm-then-quant would
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(o[j]));
    }
#pragma unroll
    for (int off = 8; off >= 1; off >>= 1)
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (!live) continue;
    const float scale = fmaxf(amax, 1e-10f) / 448.f;
    const float qi = 1.f / scale;
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __nv_fp8_e4m3 a(o[j] * qi), b(o[4 + j] * qi);
      lo |= (uint32_t)(*reinterpret_cast<const uint8_t*>(&a)) << (8 * j);
      hi |= (uint32_t)(*reinterpret_cast<const uint8_t*>(&b)) << (8 * j);
    }
    reinterpret_cast<uint2*>(q + row * ld_q)[c] = make_uint2(lo, hi);
    if ((c & 15) == 0) scales[(size_t)row * groups + c / 16] = scale;
  }
}

void run_rms_norm_quant_fp8(void* q, int64_t ld_q, float* scales, void* out, int64_t ld_out,
                            const void* x, int64_t ld_x, void* residual, int64_t ld_res,
                            const void* weight, int rows, int H, float eps, cudaStream_t s) {
  B200_REQUIRE(H % 128 == 0, "rms_norm_quant_fp8: hidden size must be a multiple of 128");
  B200_REQUIRE(ld_q % 8 == 0, "rms_norm_quant_fp8: fp8 row stride must be a multiple of 8");
  if (rows == 0) return;
  const int nvec = H / 8;
  int threads = 128;
  while (threads < 1024 && (nvec + threads - 1) / threads > 4) threads *= 2;
  const int vpt = (nvec + threads - 1) / threads;
#define B200_NQ(V, ADD)                                                                         \
  rmsnorm_quant_kernel<V, ADD><<<rows, threads, 0, s>>>(                                         \
      reinterpret_cast<__nv_fp8_e4m3*>(q), ld_q, scales, reinterpret_cast<__nv_bfloat16*>(out), \
      ld_out, reinterpret_cast<const __nv_bfloat16*>(x), ld_x,                                   \
      reinterpret_cast<__nv_bfloat16*>(residual), ld_res,                                        \
      reinterpret_cast<const __nv_bfloat16*>(weight), H, eps)
#define B200_NQV(ADD)            \
  if (vpt <= 1)                  \
    B200_NQ(1, ADD);             \
  else if (vpt <= 2)             \
    B200_NQ(2, ADD);             \
  else if (vpt <= 4)             \
    B200_NQ(4, ADD);             \
  else                           \
    B200_NQ(8, ADD);
  B200_REQUIRE(vpt <= 8, "rms_norm_quant_fp8: hidden size too large");
  if (residual) {
    B200_NQV(true)
  } else {
    B200_NQV(false)
  }
#undef B200_NQV
#undef B200_NQ
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

template <bool kAdd, bool kGemma>
static void launch_vpt(const RmsNormArgs& a, cudaStream_t s) {
  const int nvec = a.H / 8;
  int threads = 128;
  while (threads < 1024 && (nvec + threads - 1) / threads > 4) threads *= 2;
  const int vpt = (nvec + threads - 1) / threads;
  dim3 grid(a.rows);
#define B200_NORM_LAUNCH(V)                                                                \
  rmsnorm_kernel<V, kAdd, kGemma><<<grid, threads, 0, s>>>(                                \
      reinterpret_cast<__nv_bfloat16*>(a.out), a.ld_out, reinterpret_cast<__nv_bfloat16*>(a.x), \
      a.ld_x, reinterpret_cast<__nv_bfloat16*>(a.residual), a.ld_res,                      \
      reinterpret_cast<const __nv_bfloat16*>(a.weight), a.H, a.eps)
  if (vpt <= 1)
    B200_NORM_LAUNCH(1);
  else if (vpt <= 2)
    B200_NORM_LAUNCH(2);
  else if (vpt <= 4)
    B200_NORM_LAUNCH(4);
  else if (vpt <= 8)
    B200_NORM_LAUNCH(8);
  else
    B200_REQUIRE(false, "rms_norm: hidden size too large");
#undef B200_NORM_LAUNCH
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_rms_norm(const RmsNormArgs& a, cudaStream_t s) {
  B200_REQUIRE(a.H % 8 == 0, "rms_norm: hidden size must be a multiple of 8");
  if (a.rows == 0) return;
  if (a.residual) {
    if (a.gemma)
      launch_vpt<true, true>(a, s);
    else
      launch_vpt<true, false>(a, s);
  } else {
    if (a.gemma)
      launch_vpt<false, true>(a, s);
    else
      launch_vpt<false, false>(a, s);
  }
}

void run_rms_norm_gated(void* out, int64_t ldo, const void* x, int64_t ldx, const void* z,
                        int64_t ldz, const void* w, int rows, int H, int group, float eps,
                        cudaStream_t s) {
  B200_REQUIRE(H % group == 0, "rms_norm_gated: H must be a multiple of the group size");
  const int total = rows * (H / group);
  if (total == 0) return;
  const int threads = 256;
  rmsnorm_gated_kernel<<<(total + 7) / 8, threads, 0, s>>>(
      reinterpret_cast<__nv_bfloat16*>(out), ldo, reinterpret_cast<const __nv_bfloat16*>(x), ldx,
      reinterpret_cast<const __nv_bfloat16*>(z), ldz, reinterpret_cast<const __nv_bfloat16*>(w),
      rows, H, group, eps);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace norm
}  // namespace b200
