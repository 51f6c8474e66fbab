// Chunked (matrix-form) Mamba2 SSD prefill for sm_100a.
//
// Per head h (A = -exp(A_log_h) < 0) and token t: dt_t = clamp(softplus(dt_raw + dt_bias)),
//     S_t = e^{dt_t A} S_{t-1} + dt_t x_t B_t^T        S: [P, N]
//     y_t = S_t C_t + D x_t
// Over a chunk of Q = 64 tokens with a_i = cumsum(dt A) (a_i <= 0, non-increasing) and S0 the
// state at the chunk start, everything is a product of small matrices:
//     y_i  = e^{a_i} S0 C_i + sum_{j<=i} e^{a_i - a_j} dt_j (C_i . B_j) x_j + D x_i
//     S_Q  = e^{a_Q} S0 + Sc,    Sc = sum_j e^{a_Q - a_j} dt_j x_j B_j^T
// which splits the scan into three launches:
//   ssd_chunk_state_kernel  one CTA per (chunk, head), all chunks in parallel: Sc as an mma.sync
//                           product (x^T scaled by the decay weights) x B, [P, N] fp32 to the
//                           workspace, and the chunk's total decay e^{a_Q}.
//   ssd_state_pass_kernel   one CTA per (request, head, 1024 state elements): walks the
//                           request's chunks in order (elementwise S = e^{a_Q} S + Sc in fp32),
//                           writes each chunk's start state in bf16 (the scan's operand) and
//                           the final state to the request's slot.
//   ssd_chunk_scan_kernel   one CTA per (chunk, head), all chunks in parallel: three tensor-core
//                           products per warp (16 rows of the chunk): C S0^T (scaled by e^{a_i}),
//                           G = C B^T masked to j <= i and weighted by e^{a_i - a_j} dt_j in
//                           registers, then G x reusing G's accumulators as the A operand; plus
//                           D x, stored as bf16.
// The token-recurrent kernel (mamba2.cu) keeps decode and short requests; the state layout
// [slots, H, P, N] fp32 is shared.  Operands are bf16 (x, B, C as produced; the chunk-start state
// and the decay-weighted G are rounded to bf16) with fp32 accumulation; the state carried across
// chunks stays fp32.
//
// Reference counterpart: the Mamba2 SSD chunk-scan kernels vLLM runs for the reference's Mamba
// layers (vllm-patches 0038, 0117-0119; algorithm of Dao & Gu, "Transformers are SSMs", 2024).
#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "../common/mma_sm80.cuh"

namespace b200 {
namespace mamba {
namespace {

constexpr int kQ = 64;          // chunk length (tokens)
constexpr int kThreads = 128;   // chunk kernels: 4 warps of 16 rows

struct SsdParams {
  Mamba2Args a;
  int32_t* chunk_offsets;  // [R+1] first chunk of every request
  float* states;           // [max_chunks, H, P, N] fp32 chunk contributions Sc
  __nv_bfloat16* start_bf16;  // [max_chunks, H, P, N] chunk-start states (the scan's operand)
  float* decay;            // [max_chunks, H]: e^{a_Q} of every chunk
  int max_chunks;
};

__global__ void ssd_chunk_offsets_kernel(const int32_t* __restrict__ cu_q, int R,
                                         int32_t* __restrict__ out) {
  if (threadIdx.x == 0) {
    int acc = 0;
    out[0] = 0;
    for (int r = 0; r < R; ++r) {
      acc += (cu_q[r + 1] - cu_q[r] + kQ - 1) / kQ;
      out[r + 1] = acc;
    }
  }
}

B200_DEVICE int chunk_request(const int32_t* off, int R, int c) {
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (off[mid] <= c) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Address of element (row, col) of a bf16 tile stored with 128-byte rows and the 128-byte swizzle.
B200_DEVICE uint32_t sw_elem(uint32_t base, int row, int col) {
  return mma::sw128(base, row, col >> 3) + ((col & 7) << 1);
}

B200_DEVICE float ld_bf16(uint32_t addr) {
  uint16_t u;
  asm volatile("ld.shared.b16 %0, [%1];" : "=h"(u) : "r"(addr));
  return __bfloat162float(*reinterpret_cast<__nv_bfloat16*>(&u));
}

// cp_async16 takes a generic pointer to the shared destination
B200_DEVICE void* smem_ptr(uint32_t addr) { return __cvta_shared_to_generic(addr); }

B200_DEVICE void st_16(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w));
}

// The chunk's gates: sdt[i] = dt_i (0 past the chunk's n tokens), sac[i] = a_i (inclusive cumsum
// of dt A).  Threads 0-63 (two warps) take one token each.
B200_DEVICE void chunk_gates(const Mamba2Args& a, int t0, int n, int h, float A, float dtb,
                             float* sdt, float* sac, float* wtot) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid < kQ) {
    float dt = 0.f;
    if (tid < n) {
      const __nv_bfloat16* dtp = reinterpret_cast<const __nv_bfloat16*>(a.dt);
      const float raw = bf2f(dtp[(size_t)(t0 + tid) * a.ld_dt + h]) + dtb;
      dt = raw > 20.f ? raw : log1pf(expf(raw));
      dt = fminf(fmaxf(dt, a.dt_min), a.dt_max);
    }
    sdt[tid] = dt;
    float v = dt * A;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    if (tid == 31) *wtot = v;
    sac[tid] = v;
  }
  __syncthreads();
  if (tid >= 32 && tid < kQ) sac[tid] += *wtot;
  __syncthreads();
}

// ------------------------------------------------------------------------------ chunk states
// Staging: every global row goes to shared memory with cp.async (16-byte pieces, the token-major
// rows as they are: x [j][p], B [j][n]; rows past the chunk zero-filled), all issued before the
// gates are computed so the loads overlap them.  The MMA reads both operands K-major (k = token)
// through transposing ldmatrix.
template <int P, int N>
__global__ void __launch_bounds__(kThreads) ssd_chunk_state_kernel(SsdParams p) {
  __shared__ __align__(1024) __nv_bfloat16 sX[kQ * 64];       // [j][p] (128-byte rows)
  __shared__ __align__(1024) __nv_bfloat16 sB[kQ * N];        // [j][n], N / 64 halves
  __shared__ float sdt[kQ], sac[kQ], wtot;
  const Mamba2Args& a = p.a;
  const int chunk = blockIdx.x, h = blockIdx.y;
  if (chunk >= p.chunk_offsets[a.R]) return;
  const int r = chunk_request(p.chunk_offsets, a.R, chunk);
  const int t0 = a.cu_q[r] + (chunk - p.chunk_offsets[r]) * kQ;
  const int n = min(kQ, a.cu_q[r + 1] - t0);
  const int g = h / (a.H / a.G);
  const __nv_bfloat16* xbc = reinterpret_cast<const __nv_bfloat16*>(a.xbc);
  const uint32_t bX = smem_u32(sX), bB = smem_u32(sB);
  constexpr int kHalf = kQ * 128;
  const int tid = threadIdx.x;
  for (int e = tid; e < kQ * (P / 8); e += kThreads) {
    const int j = e / (P / 8), c = e % (P / 8);
    const __nv_bfloat16* src = xbc + (size_t)(t0 + (j < n ? j : 0)) * a.ld_xbc + h * P + c * 8;
    cp_async16(smem_ptr(mma::sw128(bX, j, c)), src, j < n);
  }
  for (int e = tid; e < kQ * (N / 8); e += kThreads) {
    const int j = e / (N / 8), c = e % (N / 8);
    const __nv_bfloat16* src =
        xbc + (size_t)(t0 + (j < n ? j : 0)) * a.ld_xbc + a.b_off + g * N + c * 8;
    cp_async16(smem_ptr(mma::sw128(bB + (c >> 3) * kHalf, j, c & 7)), src, j < n);
  }
  cp_async_commit();
  const float A = -expf(a.A_log[h]);
  chunk_gates(a, t0, n, h, A, a.dt_bias[h], sdt, sac, &wtot);
  const float last = sac[kQ - 1];
  cp_async_wait<0>();
  __syncthreads();
  // x_j *= e^{a_Q - a_j} dt_j (zero past the chunk), in place
  for (int e = tid; e < kQ * (P / 8); e += kThreads) {
    const int j = e / (P / 8), c = e % (P / 8);
    const uint32_t ad = mma::sw128(bX, j, c);
    const float w = expf(last - sac[j]) * sdt[j];
    uint4 u;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                 : "r"(ad));
    float v[8];
    unpack8(u, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] *= w;
    st_16(ad, pack8(v));
  }
  __syncthreads();
  // Sc [P][N] = Xw^T B: warp -> 16 rows (p) x NT n-tiles; A = Xw^T and B both K-major (k = j)
  constexpr int MT = P / 16, WPM = 4 / MT, NT = (N / 8) / WPM;
  const int warp = tid >> 5, lane = tid & 31, gq = lane >> 2, t = lane & 3;
  const int mt = warp % MT, nt0 = (warp / MT) * NT;
  const int m = lane >> 3, rr8 = lane & 7;
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[i][k] = 0.f;
#pragma unroll
  for (int ks = 0; ks < kQ / 16; ++ks) {
    uint32_t af[4];
    mma::ldsm_x4_t(mma::sw128(bX, ks * 16 + (m >> 1) * 8 + rr8, mt * 2 + (m & 1)), af[0],
                   af[1], af[2], af[3]);
    const int tok = ks * 16 + (m & 1) * 8 + rr8;
#pragma unroll
    for (int np = 0; np < NT / 2; ++np) {
      const int ng = nt0 / 2 + np;  // 16-column group of n
      uint32_t b0, b1, b2, b3;
      mma::ldsm_x4_t(mma::sw128(bB + (ng >> 2) * kHalf, tok, (ng & 3) * 2 + (m >> 1)), b0, b1,
                     b2, b3);
      mma::mma_bf16(acc[2 * np], af, b0, b1);
      mma::mma_bf16(acc[2 * np + 1], af, b2, b3);
    }
  }
  float* out = p.states + ((size_t)chunk * a.H + h) * P * N;
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int row = mt * 16 + gq + rr * 8, col = (nt0 + i) * 8 + 2 * t;
      *reinterpret_cast<float2*>(out + (size_t)row * N + col) =
          make_float2(acc[i][2 * rr], acc[i][2 * rr + 1]);
    }
  if (tid == 0) p.decay[(size_t)chunk * a.H + h] = expf(last);
}

// ------------------------------------------------------------------------------- state pass
// CTA = (request, head, slice of 1024 state elements); thread = 8 consecutive elements.  The
// next chunk's contribution and decay are loaded before the current chunk's start state is
// stored, so one load latency per chunk is in flight instead of one per element.
constexpr int kPassThreads = 128;
constexpr int kPassSlice = kPassThreads * 8;

template <int P, int N>
__global__ void __launch_bounds__(kPassThreads) ssd_state_pass_kernel(SsdParams p) {
  const Mamba2Args& a = p.a;
  const int r = blockIdx.x, h = blockIdx.y;
  const int c0 = p.chunk_offsets[r], c1 = p.chunk_offsets[r + 1];
  if (c1 <= c0) return;
  const int e0 = (blockIdx.z * kPassThreads + threadIdx.x) * 8;
  const int L = a.cu_q[r + 1] - a.cu_q[r];
  const bool hist = a.seq_lens[r] - L > 0;
  float* st = a.state + ((size_t)a.slots[r] * a.H + h) * P * N + e0;
  float s[8];
  if (hist) {
    const float4 lo = *reinterpret_cast<const float4*>(st), hi = *reinterpret_cast<const float4*>(st + 4);
    s[0] = lo.x; s[1] = lo.y; s[2] = lo.z; s[3] = lo.w;
    s[4] = hi.x; s[5] = hi.y; s[6] = hi.z; s[7] = hi.w;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) s[k] = 0.f;
  }
  const size_t stride = (size_t)a.H * P * N;
  const float* src = p.states + ((size_t)c0 * a.H + h) * P * N + e0;
  __nv_bfloat16* dst = p.start_bf16 + ((size_t)c0 * a.H + h) * P * N + e0;
  float4 lo = *reinterpret_cast<const float4*>(src), hi = *reinterpret_cast<const float4*>(src + 4);
  float d = p.decay[(size_t)c0 * a.H + h];
  for (int c = c0; c < c1; ++c) {
    const float f[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    const float dc = d;
    if (c + 1 < c1) {
      src += stride;
      lo = *reinterpret_cast<const float4*>(src);
      hi = *reinterpret_cast<const float4*>(src + 4);
      d = p.decay[(size_t)(c + 1) * a.H + h];
    }
    *reinterpret_cast<uint4*>(dst) = pack8(s);
    dst += stride;
#pragma unroll
    for (int k = 0; k < 8; ++k) s[k] = fmaf(s[k], dc, f[k]);
  }
  *reinterpret_cast<float4*>(st) = make_float4(s[0], s[1], s[2], s[3]);
  *reinterpret_cast<float4*>(st + 4) = make_float4(s[4], s[5], s[6], s[7]);
}

// ------------------------------------------------------------------------------- chunk scan
template <int P, int N>
struct ScanSmem {
  static constexpr int kHalfC = kQ * 128;        // 64 rows of 64 bf16 (one 64-column half)
  static constexpr int kHalfS = P * 128;
  static constexpr int kC = 0;                   // C  [i][n], N/64 halves
  static constexpr int kB = kC + (N / 64) * kHalfC;   // B  [j][n]
  static constexpr int kS = kB + (N / 64) * kHalfC;   // S0 [p][n] (bf16)
  static constexpr int kX = kS + (N / 64) * kHalfS;   // x [j][p] (128-byte rows)
  static constexpr int kF = kX + kHalfC;              // fp32 dt, a, scratch
  static constexpr int kBytes = kF + (2 * kQ + 4) * 4;
};

template <int P, int N>
__global__ void __launch_bounds__(kThreads) ssd_chunk_scan_kernel(SsdParams p) {
  using L = ScanSmem<P, N>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const Mamba2Args& a = p.a;
  const int chunk = blockIdx.x, h = blockIdx.y;
  if (chunk >= p.chunk_offsets[a.R]) return;
  const int r = chunk_request(p.chunk_offsets, a.R, chunk);
  const int t0 = a.cu_q[r] + (chunk - p.chunk_offsets[r]) * kQ;
  const int n = min(kQ, a.cu_q[r + 1] - t0);
  const int g = h / (a.H / a.G);
  float* sdt = reinterpret_cast<float*>(smem + L::kF);
  float* sac = sdt + kQ;
  const uint32_t base = smem_u32(smem);
  const uint32_t bC = base + L::kC, bB = base + L::kB, bS = base + L::kS, bX = base + L::kX;
  const __nv_bfloat16* xbc = reinterpret_cast<const __nv_bfloat16*>(a.xbc);
  const int tid = threadIdx.x;
  // cp.async staging of C, B [i][n], the bf16 chunk-start state [p][n] and x [j][p], issued
  // before the gates so the loads overlap them; rows past the chunk are zero-filled
  for (int e = tid; e < kQ * (N / 8); e += kThreads) {
    const int i = e / (N / 8), c = e % (N / 8);
    const __nv_bfloat16* row = xbc + (size_t)(t0 + (i < n ? i : 0)) * a.ld_xbc + g * N + c * 8;
    const uint32_t off = (c >> 3) * L::kHalfC;
    cp_async16(smem_ptr(mma::sw128(bC + off, i, c & 7)), row + a.c_off, i < n);
    cp_async16(smem_ptr(mma::sw128(bB + off, i, c & 7)), row + a.b_off, i < n);
  }
  const __nv_bfloat16* s0 = p.start_bf16 + ((size_t)chunk * a.H + h) * P * N;
  for (int e = tid; e < P * (N / 8); e += kThreads) {
    const int pr = e / (N / 8), c = e % (N / 8);
    cp_async16(smem_ptr(mma::sw128(bS + (c >> 3) * L::kHalfS, pr, c & 7)),
               s0 + (size_t)pr * N + c * 8);
  }
  for (int e = tid; e < kQ * (P / 8); e += kThreads) {
    const int j = e / (P / 8), c = e % (P / 8);
    const __nv_bfloat16* src = xbc + (size_t)(t0 + (j < n ? j : 0)) * a.ld_xbc + h * P + c * 8;
    cp_async16(smem_ptr(mma::sw128(bX, j, c)), src, j < n);
  }
  cp_async_commit();
  const float A = -expf(a.A_log[h]);
  chunk_gates(a, t0, n, h, A, a.dt_bias[h], sdt, sac, sac + kQ);
  cp_async_wait<0>();
  __syncthreads();

  const int warp = tid >> 5, lane = tid & 31, gq = lane >> 2, t = lane & 3;
  const int m = lane >> 3, rr8 = lane & 7;
  const int i0 = warp * 16;
  float acc[P / 8][4], gacc[kQ / 8][4];
#pragma unroll
  for (int i = 0; i < P / 8; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[i][k] = 0.f;
#pragma unroll
  for (int i = 0; i < kQ / 8; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) gacc[i][k] = 0.f;
  // C S0^T and G = C B^T share the A fragments of C
#pragma unroll
  for (int ks = 0; ks < N / 16; ++ks) {
    const int hh = ks >> 2, c0 = (ks & 3) * 2;
    uint32_t af[4];
    mma::ldsm_x4(mma::sw128(bC + hh * L::kHalfC, i0 + (m & 1) * 8 + rr8, c0 + (m >> 1)), af[0],
                 af[1], af[2], af[3]);
#pragma unroll
    for (int np = 0; np < P / 16; ++np) {
      uint32_t b0, b1, b2, b3;
      mma::ldsm_x4(mma::sw128(bS + hh * L::kHalfS, np * 16 + (m >> 1) * 8 + rr8, c0 + (m & 1)),
                   b0, b1, b2, b3);
      mma::mma_bf16(acc[2 * np], af, b0, b1);
      mma::mma_bf16(acc[2 * np + 1], af, b2, b3);
    }
#pragma unroll
    for (int np = 0; np < kQ / 16; ++np) {
      uint32_t b0, b1, b2, b3;
      mma::ldsm_x4(mma::sw128(bB + hh * L::kHalfC, np * 16 + (m >> 1) * 8 + rr8, c0 + (m & 1)),
                   b0, b1, b2, b3);
      mma::mma_bf16(gacc[2 * np], af, b0, b1);
      mma::mma_bf16(gacc[2 * np + 1], af, b2, b3);
    }
  }
  const int ia = i0 + gq, ib = ia + 8;
  const float aa = sac[ia], ab = sac[ib];
  const float ea = expf(aa), eb = expf(ab);
#pragma unroll
  for (int i = 0; i < P / 8; ++i) {
    acc[i][0] *= ea;
    acc[i][1] *= ea;
    acc[i][2] *= eb;
    acc[i][3] *= eb;
  }
  // decay-weighted causal mask of G, in the accumulators
#pragma unroll
  for (int nt = 0; nt < kQ / 8; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = nt * 8 + 2 * t + (e & 1);
      const int i = e < 2 ? ia : ib;
      const float ai = e < 2 ? aa : ab;
      gacc[nt][e] = j <= i ? gacc[nt][e] * expf(ai - sac[j]) * sdt[j] : 0.f;
    }
  // + G x: G's accumulators are the A fragments (k = j)
#pragma unroll
  for (int kk = 0; kk < kQ / 16; ++kk) {
    uint32_t pa[4];
    pa[0] = pack_bf16x2(gacc[2 * kk][0], gacc[2 * kk][1]);
    pa[1] = pack_bf16x2(gacc[2 * kk][2], gacc[2 * kk][3]);
    pa[2] = pack_bf16x2(gacc[2 * kk + 1][0], gacc[2 * kk + 1][1]);
    pa[3] = pack_bf16x2(gacc[2 * kk + 1][2], gacc[2 * kk + 1][3]);
    const int tok = kk * 16 + (m & 1) * 8 + rr8;
#pragma unroll
    for (int np = 0; np < P / 16; ++np) {
      uint32_t b0, b1, b2, b3;
      mma::ldsm_x4_t(mma::sw128(bX, tok, np * 2 + (m >> 1)), b0, b1, b2, b3);
      mma::mma_bf16(acc[2 * np], pa, b0, b1);
      mma::mma_bf16(acc[2 * np + 1], pa, b2, b3);
    }
  }
  const float Dh = a.D[h];
  __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(a.y);
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int i = rr ? ib : ia;
    if (i >= n) continue;
    __nv_bfloat16* dst = yp + (size_t)(t0 + i) * a.ld_y + h * P;
#pragma unroll
    for (int nt = 0; nt < P / 8; ++nt) {
      const int pc = nt * 8 + 2 * t;
      const float x0 = ld_bf16(sw_elem(bX, i, pc)), x1 = ld_bf16(sw_elem(bX, i, pc + 1));
      *reinterpret_cast<uint32_t*>(dst + pc) =
          pack_bf16x2(fmaf(Dh, x0, acc[nt][2 * rr]), fmaf(Dh, x1, acc[nt][2 * rr + 1]));
    }
  }
}

template <int P, int N>
void launch(const SsdParams& p, cudaStream_t s) {
  const dim3 grid(p.max_chunks, p.a.H);
  ssd_chunk_state_kernel<P, N><<<grid, kThreads, 0, s>>>(p);
  static_assert((P * N) % kPassSlice == 0, "state pass slices");
  ssd_state_pass_kernel<P, N><<<dim3(p.a.R, p.a.H, P * N / kPassSlice), kPassThreads, 0, s>>>(p);
  const int smem = ScanSmem<P, N>::kBytes;
  ensure_dynamic_smem(reinterpret_cast<const void*>(ssd_chunk_scan_kernel<P, N>), smem);
  ssd_chunk_scan_kernel<P, N><<<grid, kThreads, smem, s>>>(p);
}

}  // namespace

bool mamba2_chunked_supported(int P, int N, int64_t ld_xbc, int b_off, int c_off, int64_t ld_y) {
  return (P == 64 || P == 32) && (N == 128 || N == 64) && ld_xbc % 8 == 0 && b_off % 8 == 0 &&
         c_off % 8 == 0 && ld_y % 2 == 0;
}

size_t mamba2_chunked_max_chunks(int T, int R) { return (size_t)(T + kQ - 1) / kQ + R; }

void run_mamba2_chunked(const Mamba2Args& a, int T, int32_t* chunk_offsets, float* states,
                        void* start_bf16, float* decay, cudaStream_t s) {
  if (a.R == 0 || T == 0) return;
  B200_REQUIRE(mamba2_chunked_supported(a.P, a.N, a.ld_xbc, a.b_off, a.c_off, a.ld_y),
               "mamba2 chunked: head_dim 32/64, state 64/128, 16-byte aligned rows");
  B200_REQUIRE(a.H % a.G == 0, "mamba2: heads must be a multiple of groups");
  SsdParams p{};
  p.a = a;
  p.chunk_offsets = chunk_offsets;
  p.states = states;
  p.start_bf16 = reinterpret_cast<__nv_bfloat16*>(start_bf16);
  p.decay = decay;
  p.max_chunks = (int)mamba2_chunked_max_chunks(T, a.R);
  ssd_chunk_offsets_kernel<<<1, 32, 0, s>>>(a.cu_q, a.R, chunk_offsets);
  if (a.P == 64 && a.N == 128) launch<64, 128>(p, s);
  else if (a.P == 64 && a.N == 64) launch<64, 64>(p, s);
  else if (a.P == 32 && a.N == 128) launch<32, 128>(p, s);
  else launch<32, 64>(p, s);
  B200_CUDA_OK(cudaGetLastError());
  count_launch(4);
}

}  // namespace mamba
}  // namespace b200
