// Gated activations (SwiGLU / GeGLU) over [rows, 2*I] -> [rows, I], optional clamp, and the
// fused SwiGLU + per-token-group FP8 (e4m3, 1x128) quantisation used before block-scaled FP8
// GEMMs.
//
// Reference counterparts: vllm_musa/model_executor/layers/activation.py:11-53 (SiluAndMul,
// clamp variant), csrc/musa/quantization/silu_and_mul_per_token_group_fp8_quant.cu:37.  The
// dense-model hot path does not use these: the gate/up GEMM applies SwiGLU in its epilogue
// (csrc/gemm/gemm_bf16.cu, kSiluMul).  These serve MoE experts and FP8 models.
#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace act {

B200_DEVICE float silu(float x) { return x / (1.f + __expf(-x)); }
B200_DEVICE float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  return 0.5f * x * (1.f + tanhf(k0 * (x + 0.044715f * x * x * x)));
}

template <int KIND>
__global__ void act_and_mul_kernel(__nv_bfloat16* __restrict__ out, int64_t ld_out,
                                   const __nv_bfloat16* __restrict__ x, int64_t ld_x, int I,
                                   float limit) {
  const int row = blockIdx.y;
  const int nvec = I / 8;
  const uint4* g = reinterpret_cast<const uint4*>(x + row * ld_x);
  const uint4* u = reinterpret_cast<const uint4*>(x + row * ld_x + I);
  uint4* o = reinterpret_cast<uint4*>(out + row * ld_out);
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < nvec; c += gridDim.x * blockDim.x) {
    float gf[8], uf[8], of[8];
    unpack8(g[c], gf);
    unpack8(u[c], uf);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float gv = gf[j], uv = uf[j];
      if (limit > 0.f) {
        gv = fminf(gv, limit);
        uv = fmaxf(fminf(uv, limit), -limit);
      }
      of[j] = (KIND == 0 ? silu(gv) : gelu_tanh(gv)) * uv;
    }
    o[c] = pack8(of);
  }
}

// SwiGLU + FP8 quant with 1x128 groups.  One warp per (row, group of 128): each lane holds 4
// values; scale = amax / 448 (e4m3 max), stored fp32 row-major [rows, I/128].
__global__ void silu_mul_fp8_quant_kernel(__nv_fp8_e4m3* __restrict__ out,
                                          float* __restrict__ scales,
                                          const __nv_bfloat16* __restrict__ x, int64_t ld_x,
                                          int rows, int I, float limit) {
  const int groups = I / 128;
  const int gid = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (gid >= rows * groups) return;
  const int row = gid / groups, g = gid % groups, lane = threadIdx.x & 31;
  const __nv_bfloat16* gp = x + row * ld_x + g * 128 + lane * 4;
  const __nv_bfloat16* up = gp + I;
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float gv = bf2f(gp[j]), uv = bf2f(up[j]);
    if (limit > 0.f) {  // clamped SwiGLU: gate <= limit, |up| <= limit
      gv = fminf(gv, limit);
      uv = fmaxf(fminf(uv, limit), -limit);
    }
    v[j] = silu(gv) * uv;
    amax = fmaxf(amax, fabsf(v[j]));
  }
  amax = warp_max(amax);
  const float scale = fmaxf(amax, 1e-10f) / 448.f;
  const float inv = 1.f / scale;
  __nv_fp8_e4m3* op = out + (size_t)row * I + g * 128 + lane * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) op[j] = __nv_fp8_e4m3(v[j] * inv);
  if (lane == 0) scales[(size_t)row * groups + g] = scale;
}

// Per-token-group FP8 quantisation of a bf16 activation (group 128).
__global__ void group_quant_fp8_kernel(__nv_fp8_e4m3* __restrict__ out, float* __restrict__ scales,
                                       const __nv_bfloat16* __restrict__ x, int64_t ld_x, int rows,
                                       int K) {
  const int groups = K / 128;
  const int gid = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (gid >= rows * groups) return;
  const int row = gid / groups, g = gid % groups, lane = threadIdx.x & 31;
  const __nv_bfloat16* xp = x + row * ld_x + g * 128 + lane * 4;
  float v[4];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = bf2f(xp[j]);
    amax = fmaxf(amax, fabsf(v[j]));
  }
  amax = warp_max(amax);
  const float scale = fmaxf(amax, 1e-10f) / 448.f;
  const float inv = 1.f / scale;
  __nv_fp8_e4m3* op = out + (size_t)row * K + g * 128 + lane * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) op[j] = __nv_fp8_e4m3(v[j] * inv);
  if (lane == 0) scales[(size_t)row * groups + g] = scale;
}

void run_act_and_mul(void* out, int64_t ld_out, const void* x, int64_t ld_x, int rows, int I,
                     int kind, float limit, cudaStream_t s) {
  B200_REQUIRE(I % 8 == 0, "act_and_mul: I must be a multiple of 8");
  if (rows == 0) return;
  const int nvec = I / 8;
  const int threads = 128;
  dim3 grid((nvec + threads - 1) / threads, rows);
  if (kind == 0)
    act_and_mul_kernel<0><<<grid, threads, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out), ld_out,
                                                   reinterpret_cast<const __nv_bfloat16*>(x), ld_x,
                                                   I, limit);
  else
    act_and_mul_kernel<1><<<grid, threads, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(out), ld_out,
                                                   reinterpret_cast<const __nv_bfloat16*>(x), ld_x,
                                                   I, limit);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_silu_mul_fp8_quant(void* out, float* scales, const void* x, int64_t ld_x, int rows, int I,
                            cudaStream_t s, float limit) {
  B200_REQUIRE(I % 128 == 0, "silu_mul_fp8_quant: I must be a multiple of 128");
  const int total = rows * (I / 128);
  if (total == 0) return;
  silu_mul_fp8_quant_kernel<<<(total + 7) / 8, 256, 0, s>>>(
      reinterpret_cast<__nv_fp8_e4m3*>(out), scales, reinterpret_cast<const __nv_bfloat16*>(x),
      ld_x, rows, I, limit);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_group_quant_fp8(void* out, float* scales, const void* x, int64_t ld_x, int rows, int K,
                         cudaStream_t s) {
  B200_REQUIRE(K % 128 == 0, "group_quant_fp8: K must be a multiple of 128");
  const int total = rows * (K / 128);
  if (total == 0) return;
  group_quant_fp8_kernel<<<(total + 7) / 8, 256, 0, s>>>(
      reinterpret_cast<__nv_fp8_e4m3*>(out), scales, reinterpret_cast<const __nv_bfloat16*>(x),
      ld_x, rows, K);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace act
}  // namespace b200
