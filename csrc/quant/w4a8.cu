// W4AFP8 routed experts: packed signed INT4 weights with bf16 per-(row, 128-column) scales,
// activations quantised per token to e4m3 with one dynamic scale per row.
//
//   w4_dequant_kernel   packed int4 [E, N, K/2] (element 2j in the low nibble, 2j+1 in the
//                       high one) x scales [E, N, K/128] -> bf16 [E * N, K], only for experts
//                       that received rows (the padded offsets from moe_align), so a decode step
//                       expands the handful of live experts, not all of them
//   row_fp8_qdq_kernel  per-row e4m3 round trip: scale = max(amax, 1e-4) / 448, q =
//                       e4m3(clamp(v / scale, +-448)), out = q * scale in bf16.  kSwiGLU first
//                       forms v = bf16(silu(min(g, L)) * clamp(u, -L, L)) from [gate | up] rows
//
// The expert GEMMs are the tcgen05 grouped bf16 GEMM over the expanded weights: both operand
// values (an e4m3 code times its row scale, an int4 times its group scale) reach the tensor core
// rounded once to bf16 and the products accumulate in fp32 in TMEM.
//
// Reference counterparts: vllm_musa/kernels/w4afp8_moe.py:8-337 (assign / scatter-quantise /
// SwiGLU-quantise / combine around the mixed-dtype grouped GEMM),
// vllm_musa/model_executor/layers/quantization/w4afp8.py:26-170 (checkpoint layout).
#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace w4a8 {

// 8 packed bytes (16 int4) -> 16 bf16 values times one group scale.
__global__ void __launch_bounds__(256)
w4_dequant_kernel(__nv_bfloat16* __restrict__ out, const uint8_t* __restrict__ packed,
                  const __nv_bfloat16* __restrict__ scales, const int32_t* __restrict__ offsets,
                  int N, int K) {
  const int e = blockIdx.y;
  if (offsets != nullptr && offsets[e + 1] <= offsets[e]) return;  // expert got no rows
  const int64_t vec_per_row = K / 16;
  const int64_t nvec = (int64_t)N * vec_per_row;
  const uint2* src = reinterpret_cast<const uint2*>(packed + (size_t)e * N * (K / 2));
  const __nv_bfloat16* sc = scales + (size_t)e * N * (K / 128);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)e * N * K);
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nvec;
       v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = v / vec_per_row, c = v % vec_per_row;  // 16-element column chunk
    const float s = bf2f(sc[n * (K / 128) + c / 8]);
    const uint2 b = src[v];
    float f[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t byte = ((j < 4 ? b.x : b.y) >> ((j & 3) * 8)) & 0xffu;
      f[2 * j] = (float)((int)((byte & 15u) ^ 8u) - 8) * s;
      f[2 * j + 1] = (float)((int)((byte >> 4) ^ 8u) - 8) * s;
    }
    float lo[8], hi[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      lo[j] = f[j];
      hi[j] = f[8 + j];
    }
    dst[2 * v] = pack8(lo);
    dst[2 * v + 1] = pack8(hi);
  }
}

template <bool kSwiGLU>
__global__ void __launch_bounds__(256)
row_fp8_qdq_kernel(__nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ x,
                   int64_t ld_x, int C, float limit, const int32_t* __restrict__ num_tiles) {
  extern __shared__ float vals[];  // C floats
  __shared__ float red[32];
  const int row = blockIdx.x;
  if (num_tiles != nullptr && row >= num_tiles[0] * 128) return;
  const __nv_bfloat16* xr = x + (size_t)row * ld_x;
  float amax = 0.f;
  for (int c8 = threadIdx.x; c8 < C / 8; c8 += blockDim.x) {
    float v[8];
    unpack8(reinterpret_cast<const uint4*>(xr)[c8], v);
    if constexpr (kSwiGLU) {
      float u[8];
      unpack8(reinterpret_cast<const uint4*>(xr + C)[c8], u);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float g = v[j], uu = u[j];
        if (limit > 0.f) {
          g = fminf(g, limit);
          uu = fmaxf(fminf(uu, limit), -limit);
        }
        v[j] = bf2f(f2bf(g / (1.f + __expf(-g)) * uu));
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      vals[c8 * 8 + j] = v[j];
      amax = fmaxf(amax, fabsf(v[j]));
    }
  }
  amax = block_max(amax, red);
  const float scale = fmaxf(amax, 1e-4f) / 448.f;
  __nv_bfloat16* orow = out + (size_t)row * C;
  for (int c8 = threadIdx.x; c8 < C / 8; c8 += blockDim.x) {
    float q[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float t = fminf(fmaxf(vals[c8 * 8 + j] / scale, -448.f), 448.f);
      q[j] = float(__nv_fp8_e4m3(t)) * scale;
    }
    reinterpret_cast<uint4*>(orow)[c8] = pack8(q);
  }
}

void run_w4_dequant(void* out, const void* packed, const void* scales, const int32_t* offsets,
                    int E, int N, int K, cudaStream_t s) {
  const int64_t nvec = (int64_t)N * (K / 16);
  const int blocks = (int)std::min<int64_t>((nvec + 255) / 256, 1184);
  w4_dequant_kernel<<<dim3(blocks, E), 256, 0, s>>>(
      reinterpret_cast<__nv_bfloat16*>(out), reinterpret_cast<const uint8_t*>(packed),
      reinterpret_cast<const __nv_bfloat16*>(scales), offsets, N, K);
  B200_CUDA_OK(cudaGetLastError());
}

void run_row_fp8_qdq(void* out, const void* x, int64_t ld_x, int rows, int C, bool swiglu,
                     float limit, const int32_t* num_tiles, cudaStream_t s) {
  const size_t smem = (size_t)C * sizeof(float);
  if (swiglu) {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(row_fp8_qdq_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
    row_fp8_qdq_kernel<true><<<rows, 256, smem, s>>>(
        reinterpret_cast<__nv_bfloat16*>(out), reinterpret_cast<const __nv_bfloat16*>(x), ld_x, C,
        limit, num_tiles);
  } else {
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(row_fp8_qdq_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem);
    row_fp8_qdq_kernel<false><<<rows, 256, smem, s>>>(
        reinterpret_cast<__nv_bfloat16*>(out), reinterpret_cast<const __nv_bfloat16*>(x), ld_x, C,
        limit, num_tiles);
  }
  B200_CUDA_OK(cudaGetLastError());
}

}  // namespace w4a8
}  // namespace b200
