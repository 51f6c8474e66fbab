// Routed bf16 experts for a few tokens (decode): one GEMV per (token, slot) pair instead of
// align -> gather -> two grouped GEMMs.  With a handful of routed rows every grouped-GEMM tile
// holds one or two real rows and only the live experts' N-tiles run; here every pair spreads
// its expert's weight rows over many CTAs, so the weight stream (the whole cost at this size)
// runs at HBM rate.
//
//   moe_gemv_gate_up_kernel  grid (pairs, I / 32), 8 warps x 4 channels: the gate and up rows of
//                            the pair's expert (interleaved in groups of 8 rows) dotted with
//                            the token's row, h = silu(gate) * up  -> h [pairs, I] bf16.  Also
//                            writes pos[pair] = pair (or -1 when the expert lives elsewhere).
//   moe_gemv_down_kernel     grid (pairs, H / 32): w_down rows of the expert dotted with h ->
//                            y [pairs, H] bf16.
// The weighted sum over a token's slots (plus the shared expert) is the existing moe_combine
// kernel, reading y through pos.
//
// Every lane streams 16-byte weight vectors (8 rows in flight per warp), the activation row
// sits in shared memory, fp32 accumulation, warp-shuffle reduction.
//
// Reference counterpart: the GEMV backend of the reference's fused-MoE dispatch policy
// (vllm_musa/model_executor/layers/fused_moe/dispatch_policy.py:690-743), which it picks below
// a per-shape token threshold.
#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace moe {
namespace {

constexpr int kThreads = 256;
constexpr int kCh = 32;  // output channels per CTA (4 per warp)

B200_DEVICE uint4 ldg_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

B200_DEVICE float dot8(const float (&x)[8], const uint4& w) {
  float f[8];
  unpack8(w, f);
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) s = fmaf(x[q], f[q], s);
  return s;
}

__global__ void __launch_bounds__(kThreads)
moe_gemv_gate_up_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                        const int32_t* __restrict__ ids, int k, int E, int e0,
                        const __nv_bfloat16* __restrict__ w_gu, int H, int I,
                        __nv_bfloat16* __restrict__ h, int32_t* __restrict__ pos) {
  extern __shared__ uint4 sx[];  // the token's row, H / 8 vectors
  const int p = blockIdx.x, t = p / k;
  const int e = ids[p] - e0;
  const bool local = e >= 0 && e < E;
  if (blockIdx.y == 0 && threadIdx.x == 0) pos[p] = local ? p : -1;
  if (!local) return;
  const int nv = H / 8;
  for (int v = threadIdx.x; v < nv; v += kThreads)
    sx[v] = reinterpret_cast<const uint4*>(x + (size_t)t * ldx)[v];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.y * kCh + warp * 4;  // this warp's 4 channels (one group of 8 rows)
  // rows of channel c: gate = 16 (c / 8) + c % 8, up = gate + 8 (expert-local)
  const __nv_bfloat16* base = w_gu + (size_t)e * 2 * I * H;
  const __nv_bfloat16* rows[8];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int c = c0 + q;
    const size_t g = (size_t)(16 * (c >> 3) + (c & 7));
    rows[q] = base + g * H;
    rows[4 + q] = base + (g + 8) * H;
  }
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int v = lane; v < nv; v += 32) {
    float xv[8];
    unpack8(sx[v], xv);
    uint4 wv[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) wv[r] = ldg_nc(rows[r] + (size_t)v * 8);
#pragma unroll
    for (int r = 0; r < 8; ++r) acc[r] += dot8(xv, wv[r]);
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) acc[r] = warp_sum(acc[r]);
  if (lane < 4) {
    float gv = acc[0], uv = acc[4];
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (lane == q) {
        gv = acc[q];
        uv = acc[4 + q];
      }
    h[(size_t)p * I + c0 + lane] = f2bf(gv / (1.f + __expf(-gv)) * uv);
  }
}

__global__ void __launch_bounds__(kThreads)
moe_gemv_down_kernel(const __nv_bfloat16* __restrict__ h, const int32_t* __restrict__ ids,
                     int E, int e0, const __nv_bfloat16* __restrict__ w_down, int H, int I,
                     __nv_bfloat16* __restrict__ y) {
  extern __shared__ uint4 sh[];  // the pair's h row, I / 8 vectors
  const int p = blockIdx.x;
  const int e = ids[p] - e0;
  if (e < 0 || e >= E) return;
  const int nv = I / 8;
  for (int v = threadIdx.x; v < nv; v += kThreads)
    sh[v] = reinterpret_cast<const uint4*>(h + (size_t)p * I)[v];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.y * kCh + warp * 4;
  const __nv_bfloat16* base = w_down + ((size_t)e * H + c0) * I;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int v = lane; v < nv; v += 32) {
    float hv[8];
    unpack8(sh[v], hv);
    uint4 wv[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) wv[r] = ldg_nc(base + (size_t)r * I + (size_t)v * 8);
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r] += dot8(hv, wv[r]);
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) acc[r] = warp_sum(acc[r]);
  if (lane < 4) {
    float o = acc[0];
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (lane == q) o = acc[q];
    y[(size_t)p * H + c0 + lane] = f2bf(o);
  }
}

}  // namespace

bool moe_gemv_supported(int H, int I) { return H % kCh == 0 && I % kCh == 0 && H <= 16384 && I <= 16384; }

void run_moe_gemv(const void* x, int64_t ldx, const int32_t* ids, int T, int k, int E, int e0,
                  const void* w_gu, const void* w_down, int H, int I, void* h, void* y,
                  int32_t* pos, cudaStream_t s) {
  if (T == 0) return;
  B200_REQUIRE(moe_gemv_supported(H, I), "moe_gemv: H and I multiples of 32, at most 16384");
  B200_REQUIRE(ldx % 8 == 0, "moe_gemv: x rows 16-byte aligned");
  const int pairs = T * k;
  moe_gemv_gate_up_kernel<<<dim3(pairs, I / kCh), kThreads, H * 2, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, ids, k, E, e0,
      reinterpret_cast<const __nv_bfloat16*>(w_gu), H, I, reinterpret_cast<__nv_bfloat16*>(h),
      pos);
  moe_gemv_down_kernel<<<dim3(pairs, H / kCh), kThreads, I * 2, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(h), ids, E, e0,
      reinterpret_cast<const __nv_bfloat16*>(w_down), H, I, reinterpret_cast<__nv_bfloat16*>(y));
  B200_CUDA_OK(cudaGetLastError());
  count_launch(2);
}

}  // namespace moe
}  // namespace b200
