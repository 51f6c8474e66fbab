// Mamba2 selective state-space scan (SSD recurrence) with per-request state slots, and the
// gate-then-normalise RMSNorm of the Mamba2 mixer output.
//
//   dt_t = clamp(softplus(dt_raw_t + dt_bias_h), lo, hi),  dA_t = exp(dt_t * A_h),  A_h = -exp(A_log_h)
//   S_t  = dA_t S_{t-1} + dt_t x_t B_t^T           S: [P, N] per head (fp32, kept in registers)
//   y_t  = S_t C_t + D_h x_t
//
// CTA = (request, head), P x 4 threads: thread (p, q) owns state row p, columns n = 4k + q
// (the four threads of a quad read four consecutive shared-memory words, the other quads of
// the warp the same words: broadcast, no bank conflicts).  Tokens are staged 16 at a time
// (x, B, C, dt, dA in shared memory), then the recurrence walks them; y needs a 4-lane
// reduction per token.  Decode (one token) and prefill (many) use the same kernel.
//
//   gated_rmsnorm_kernel  out = RMSNorm_group(y * silu(z)) * w   (Mamba2's norm_before_gate =
//                         False; groups of C / n_groups channels)
//
// Reference counterparts: the vLLM Mamba2 mixer and selective-scan kernels the reference
// patches in (vllm-patches 0038, 0117-0119, 0132, 0200; Mamba2 SSD as published by Dao & Gu,
// "Transformers are SSMs", 2024).
#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace mamba {

constexpr int kTok = 16;   // tokens staged per round
constexpr int kMaxP = 64;  // head dim (threads = 4 * P)

template <int N>
__global__ void __launch_bounds__(256) mamba2_scan_kernel(Mamba2Args p) {
  constexpr int NPT = N / 4;
  __shared__ float sx[kTok][kMaxP];
  __shared__ float sB[kTok][N];
  __shared__ float sC[kTok][N];
  __shared__ float sdt[kTok], sdA[kTok];
  const int r = blockIdx.x, h = blockIdx.y;
  const int P = p.P;
  const int tid = threadIdx.x, pi = tid >> 2, q = tid & 3;
  const int q0 = p.cu_q[r], L = p.cu_q[r + 1] - q0;
  if (L <= 0) return;
  const bool hist = p.seq_lens[r] - L > 0;
  float* st = p.state + (((size_t)p.slots[r] * p.H + h) * P + pi) * N;
  float s[NPT];
#pragma unroll
  for (int k = 0; k < NPT; ++k) s[k] = hist ? st[4 * k + q] : 0.f;
  const int g = h / (p.H / p.G);
  const float A = -expf(p.A_log[h]);
  const float dtb = p.dt_bias[h], Dh = p.D[h];
  const int nthr = blockDim.x;
  const __nv_bfloat16* xbc = reinterpret_cast<const __nv_bfloat16*>(p.xbc);
  const __nv_bfloat16* dtp = reinterpret_cast<const __nv_bfloat16*>(p.dt);
  __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(p.y);
  for (int t0 = 0; t0 < L; t0 += kTok) {
    const int n = min(kTok, L - t0);
    for (int e = tid; e < n * P; e += nthr) {
      const int i = e / P, j = e % P;
      sx[i][j] = bf2f(xbc[(size_t)(q0 + t0 + i) * p.ld_xbc + h * P + j]);
    }
    for (int e = tid; e < n * N; e += nthr) {
      const int i = e / N, j = e % N;
      const __nv_bfloat16* row = xbc + (size_t)(q0 + t0 + i) * p.ld_xbc;
      sB[i][j] = bf2f(row[p.b_off + g * N + j]);
      sC[i][j] = bf2f(row[p.c_off + g * N + j]);
    }
    if (tid < n) {
      const float raw = bf2f(dtp[(size_t)(q0 + t0 + tid) * p.ld_dt + h]) + dtb;
      float dt = raw > 20.f ? raw : log1pf(expf(raw));
      dt = fminf(fmaxf(dt, p.dt_min), p.dt_max);
      sdt[tid] = dt;
      sdA[tid] = expf(dt * A);
    }
    __syncthreads();
    if (pi < P) {
      for (int i = 0; i < n; ++i) {
        const float xv = sx[i][pi];
        const float coef = sdt[i] * xv, dA = sdA[i];
        float y = 0.f;
#pragma unroll
        for (int k = 0; k < NPT; ++k) {
          s[k] = fmaf(s[k], dA, coef * sB[i][4 * k + q]);
          y = fmaf(s[k], sC[i][4 * k + q], y);
        }
        y += __shfl_xor_sync(0xffffffffu, y, 1);
        y += __shfl_xor_sync(0xffffffffu, y, 2);
        if (q == 0) yp[(size_t)(q0 + t0 + i) * p.ld_y + h * P + pi] = f2bf(fmaf(Dh, xv, y));
      }
    }
    __syncthreads();
  }
  if (pi < P) {
#pragma unroll
    for (int k = 0; k < NPT; ++k) st[4 * k + q] = s[k];
  }
}

// One CTA per (token, group): two passes over the group's channels (the second hits L1).
__global__ void __launch_bounds__(256)
gated_rmsnorm_kernel(__nv_bfloat16* __restrict__ out, int64_t ld_o,
                     const __nv_bfloat16* __restrict__ y, int64_t ld_y,
                     const __nv_bfloat16* __restrict__ z, int64_t ld_z,
                     const __nv_bfloat16* __restrict__ w, int group, float eps) {
  __shared__ float red[32];
  const int t = blockIdx.x, g0 = blockIdx.y * group;
  const __nv_bfloat16* yr = y + (size_t)t * ld_y + g0;
  const __nv_bfloat16* zr = z + (size_t)t * ld_z + g0;
  float ss = 0.f;
  for (int c8 = threadIdx.x; c8 < group / 8; c8 += blockDim.x) {
    float a[8], b[8];
    unpack8(reinterpret_cast<const uint4*>(yr)[c8], a);
    unpack8(reinterpret_cast<const uint4*>(zr)[c8], b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = a[j] * (b[j] / (1.f + __expf(-b[j])));
      ss = fmaf(v, v, ss);
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / group + eps);
  __nv_bfloat16* orow = out + (size_t)t * ld_o + g0;
  for (int c8 = threadIdx.x; c8 < group / 8; c8 += blockDim.x) {
    float a[8], b[8], ww[8], o[8];
    unpack8(reinterpret_cast<const uint4*>(yr)[c8], a);
    unpack8(reinterpret_cast<const uint4*>(zr)[c8], b);
    unpack8(reinterpret_cast<const uint4*>(w + g0)[c8], ww);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = a[j] * (b[j] / (1.f + __expf(-b[j]))) * inv * ww[j];
    reinterpret_cast<uint4*>(orow)[c8] = pack8(o);
  }
}

void run_mamba2_scan(const Mamba2Args& a, cudaStream_t s) {
  if (a.R == 0) return;
  B200_REQUIRE(a.P > 0 && a.P <= kMaxP && a.P % 8 == 0, "mamba2: head_dim must be 8..64");
  B200_REQUIRE(a.H % a.G == 0, "mamba2: heads must be a multiple of groups");
  const dim3 grid(a.R, a.H);
  const int threads = a.P * 4;
  if (a.N == 128)
    mamba2_scan_kernel<128><<<grid, threads, 0, s>>>(a);
  else if (a.N == 64)
    mamba2_scan_kernel<64><<<grid, threads, 0, s>>>(a);
  else if (a.N == 16)
    mamba2_scan_kernel<16><<<grid, threads, 0, s>>>(a);
  else
    B200_REQUIRE(false, "mamba2: state size must be 16, 64 or 128");
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_gated_rmsnorm(void* out, int64_t ld_o, const void* y, int64_t ld_y, const void* z,
                       int64_t ld_z, const void* w, int T, int C, int group, float eps,
                       cudaStream_t s) {
  if (T == 0) return;
  B200_REQUIRE(group % 8 == 0 && C % group == 0, "gated rmsnorm: group must divide C, % 8");
  gated_rmsnorm_kernel<<<dim3(T, C / group), 256, 0, s>>>(
      reinterpret_cast<__nv_bfloat16*>(out), ld_o, reinterpret_cast<const __nv_bfloat16*>(y),
      ld_y, reinterpret_cast<const __nv_bfloat16*>(z), ld_z,
      reinterpret_cast<const __nv_bfloat16*>(w), group, eps);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace mamba
}  // namespace b200
