// Gated DeltaNet (Qwen3-Next linear-attention layers) for sm_100a.
//
//  causal_conv1d   depthwise causal convolution (kernel 4) + SiLU over the packed [q | k | v]
//                  channels of a varlen batch.  Token t of request r reads inputs t-3..t; the
//                  ones before the request's first new token come from its conv state slot
//                  (the last 3 inputs of its previous chunk; zeros for a fresh request).
//  conv_state_update  writes each request's last 3 inputs back into its slot.
//  gdn_recurrent   the gated delta rule, token by token:
//                      S <- exp(g_t) S;  u = beta_t (v_t - S^T k_t);  S <- S + k_t u^T;
//                      o_t = S^T q_t
//                  with q, k L2-normalised (q also scaled by 1/sqrt(dk)), g_t =
//                  -exp(A_log) softplus(a_t + dt_bias), beta_t = sigmoid(b_t).  The rows of S
//                  for different value columns evolve independently, so one CTA owns 32 value
//                  columns of one (request, value head): four CTAs per head keep several CTAs
//                  resident per SM (the decode step is a load-update-store of 64 KB of state
//                  per head).  The state slice lives in registers (4 threads per value column,
//                  32 key rows each) for the whole chunk; tokens are staged through shared
//                  memory 16 at a time.  Prefill chunks and decode steps
//                  use the same kernel; the state slot carries across engine steps.
// State layout: [slots, Hv, dv, dk] fp32 (value-major, so each thread's 32 key rows are one
// contiguous 128-byte run).
//
// Reference counterparts: vllm_musa/model_executor/layers/mamba/gdn/qwen_gdn_linear_attn.py
// :296-557 (MATE gated_delta_rule_decode / chunk_gated_delta_rule, no source in the
// reference), vllm_musa/jit_kernel/tilelang/causal_conv1d.py:101-989,
// vllm_musa/jit_kernel/fused_gdn_gating.py:22.
#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace gdn {

constexpr int kDK = 128, kDV = 128;
constexpr int kVSplit = 4;                   // CTAs per (request, head): 32 value columns each
constexpr int kThreads = 128;                // 32 value columns x 4 key quarters
constexpr int kTok = 16;       // tokens staged per round (24 KB of shared memory)

B200_DEVICE int find_req(const int32_t* cu, int R, int t) {
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ------------------------------------------------------------------------------ conv1d
__global__ void causal_conv1d_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                     const __nv_bfloat16* __restrict__ w,  // [C, 4]
                                     const __nv_bfloat16* __restrict__ state,  // [slots, C, 3]
                                     const int32_t* __restrict__ cu_q,
                                     const int32_t* __restrict__ seq_lens,
                                     const int32_t* __restrict__ slots, int R, int C,
                                     __nv_bfloat16* __restrict__ out, int64_t ldo,
                                     const __nv_bfloat16* __restrict__ bias) {
  pdl_launch_dependents();
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int r = find_req(cu_q, R, t);
  const int q0 = cu_q[r];
  const int q_len = cu_q[r + 1] - q0;
  const bool hist = seq_lens[r] - q_len > 0;
  const __nv_bfloat16* st = state + ((size_t)slots[r] * C + c) * 3;
  float acc = bias != nullptr ? bf2f(bias[c]) : 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int tau = t - 3 + j;  // absolute token index in the batch
    float xin;
    if (tau >= q0) {
      xin = bf2f(x[(size_t)tau * ldx + c]);
    } else {
      const int back = q0 - tau;  // 1..3 tokens before the chunk
      xin = hist ? bf2f(st[3 - back]) : 0.f;
    }
    acc += xin * bf2f(w[c * 4 + j]);
  }
  out[(size_t)t * ldo + c] = f2bf(acc / (1.f + __expf(-acc)));
}

// Vectorised form: a thread owns 8 consecutive channels (one 16-byte vector) of kConvTok
// consecutive tokens and walks them with a rolling window of the 4 input rows a token needs
// (packed bf16, 4 registers a row), the next two rows already in flight, so each input element
// is loaded (kConvTok + 3) / kConvTok times and every access is a 16-byte vector.  (Holding all
// kConvTok + 3 rows unpacked took 212 registers a thread and 2 CTAs per SM.)  Tokens keep
// their own request's history rule (inputs before the request's first new token come from its
// conv state slot, or zeros).  Same results as causal_conv1d_kernel.
constexpr int kConvTok = 32;

__global__ void __launch_bounds__(128)
    causal_conv1d_vec_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                             const __nv_bfloat16* __restrict__ w,  // [C, 4]
                             const __nv_bfloat16* __restrict__ state,  // [slots, C, 3]
                             const int32_t* __restrict__ cu_q, const int32_t* __restrict__ seq_lens,
                             const int32_t* __restrict__ slots, int R, int T, int C,
                             __nv_bfloat16* __restrict__ out, int64_t ldo,
                             const __nv_bfloat16* __restrict__ bias) {
  pdl_launch_dependents();
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= C) return;
  const int t0 = blockIdx.y * kConvTok;
  const int t1 = min(T, t0 + kConvTok);
  float wt[8][4], b[8];
  {
    const uint4* wp = reinterpret_cast<const uint4*>(w + (size_t)c0 * 4);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float f[8];
      unpack8(wp[q], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) wt[q * 2 + j / 4][j % 4] = f[j];
    }
    if (bias != nullptr)
      unpack8(*reinterpret_cast<const uint4*>(bias + c0), b);
    else
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) b[ch] = 0.f;
  }
  auto row = [&](int tau) -> uint4 {  // input row tau of these channels (zeros outside [0, t1))
    return tau >= 0 && tau < t1 ? *reinterpret_cast<const uint4*>(x + (size_t)tau * ldx + c0)
                                : make_uint4(0, 0, 0, 0);
  };
  // window w0..w2 = rows t-3..t-1; n1, n2 = rows t, t+1 (in flight)
  uint4 w0 = row(t0 - 3), w1 = row(t0 - 2), w2 = row(t0 - 1);
  uint4 n1 = row(t0), n2 = row(t0 + 1);
  int r = find_req(cu_q, R, t0);
#pragma unroll 1
  for (int t = t0; t < t1; ++t) {
    const uint4 w3 = n1;
    n1 = n2;
    n2 = row(t + 2);
    while (r + 1 < R && t >= cu_q[r + 1]) ++r;
    const int q0 = cu_q[r];
    const bool hist = seq_lens[r] - (cu_q[r + 1] - q0) > 0;
    float acc[8];
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) acc[ch] = b[ch];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int tau = t - 3 + j;
      if (tau >= q0) {
        float xv[8];
        unpack8(j == 0 ? w0 : j == 1 ? w1 : j == 2 ? w2 : w3, xv);
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) acc[ch] += xv[ch] * wt[ch][j];
      } else if (hist) {
        const int back = q0 - tau;  // 1..3 tokens before the chunk
        const __nv_bfloat16* st = state + ((size_t)slots[r] * C + c0) * 3 + (3 - back);
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) acc[ch] += bf2f(st[ch * 3]) * wt[ch][j];
      }
    }
    float o[8];
#pragma unroll
    for (int ch = 0; ch < 8; ++ch) o[ch] = acc[ch] / (1.f + __expf(-acc[ch]));
    *reinterpret_cast<uint4*>(out + (size_t)t * ldo + c0) = pack8(o);
    w0 = w1;
    w1 = w2;
    w2 = w3;
  }
}

__global__ void conv_state_update_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                         __nv_bfloat16* __restrict__ state,
                                         const int32_t* __restrict__ cu_q,
                                         const int32_t* __restrict__ seq_lens,
                                         const int32_t* __restrict__ slots, int R, int C) {
  const int r = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C || r >= R) return;
  const int q0 = cu_q[r], L = cu_q[r + 1] - q0;
  const bool hist = seq_lens[r] - L > 0;
  __nv_bfloat16* st = state + ((size_t)slots[r] * C + c) * 3;
  float old[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) old[j] = hist ? bf2f(st[j]) : 0.f;
  float nw[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int rel = L - 3 + j;  // index into this chunk (negative: from the old state)
    nw[j] = rel >= 0 ? bf2f(x[(size_t)(q0 + rel) * ldx + c]) : old[3 + rel];
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) st[j] = f2bf(nw[j]);
}

// ------------------------------------------------------------------------------ recurrence
struct RecParams {
  const __nv_bfloat16* qkv;  // [T, >= 2*Hk*dk + Hv*dv] conv output
  int64_t ld_qkv;
  const __nv_bfloat16* ba;   // [T, >= 2*Hv]: b then a
  int64_t ld_ba;
  const float* A_log;        // [Hv]
  const float* dt_bias;      // [Hv]
  float* state;              // [slots, Hv, dv, dk]
  const int32_t* cu_q;
  const int32_t* seq_lens;
  const int32_t* slots;
  __nv_bfloat16* out;        // [T, Hv*dv]
  int64_t ld_out;
  int R, Hk, Hv;
};

__global__ void __launch_bounds__(kThreads, 4) gdn_recurrent_kernel(RecParams p) {
  pdl_launch_dependents();
  __shared__ float sq[kTok][kDK], sk[kTok][kDK], sv[kTok][kDV / kVSplit];
  __shared__ float sg[kTok], sb[kTok];
  const int r = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x;
  const int vloc = tid >> 2, kq = tid & 3;
  const int vcol = blockIdx.z * (kDV / kVSplit) + vloc;
  const int warp = tid >> 5, lane = tid & 31;
  const int q0 = p.cu_q[r];
  const int L = p.cu_q[r + 1] - q0;
  const bool hist = p.seq_lens[r] - L > 0;
  const int hk = h / (p.Hv / p.Hk);
  float* gstate = p.state + (((size_t)p.slots[r] * p.Hv + h) * kDV + vcol) * kDK + kq * 32;
  float S[32];
  if (hist) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v4 = reinterpret_cast<const float4*>(gstate)[i];
      S[4 * i] = v4.x;
      S[4 * i + 1] = v4.y;
      S[4 * i + 2] = v4.z;
      S[4 * i + 3] = v4.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) S[i] = 0.f;
  }
  const float A = -__expf(p.A_log[h]);
  const float dtb = p.dt_bias[h];
  const float qscale = rsqrtf((float)kDK);
  const int qoff = hk * kDK, koff = p.Hk * kDK + hk * kDK, voff = 2 * p.Hk * kDK + h * kDV;
  for (int base = 0; base < L; base += kTok) {
    const int nt = min(kTok, L - base);
    __syncthreads();  // previous round done with the staging buffers
    // stage + L2-normalise q and k (one warp per token), v, gates
    for (int j = warp; j < nt; j += kThreads / 32) {
      const __nv_bfloat16* row = p.qkv + (size_t)(q0 + base + j) * p.ld_qkv;
      float qv[4], kv[4];
      float sqq = 0.f, skk = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qv[e] = bf2f(row[qoff + lane * 4 + e]);
        kv[e] = bf2f(row[koff + lane * 4 + e]);
        sqq += qv[e] * qv[e];
        skk += kv[e] * kv[e];
      }
      sqq = warp_sum(sqq);
      skk = warp_sum(skk);
      const float iq = rsqrtf(sqq + 1e-6f) * qscale, ik = rsqrtf(skk + 1e-6f);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sq[j][lane * 4 + e] = qv[e] * iq;
        sk[j][lane * 4 + e] = kv[e] * ik;
      }
      sv[j][lane] = bf2f(row[voff + blockIdx.z * (kDV / kVSplit) + lane]);
      if (lane == 0) {
        const __nv_bfloat16* ba = p.ba + (size_t)(q0 + base + j) * p.ld_ba;
        const float b = bf2f(ba[h]), a = bf2f(ba[p.Hv + h]);
        const float x = a + dtb;
        const float sp = x > 20.f ? x : log1pf(__expf(x));  // softplus
        sg[j] = __expf(A * sp);
        sb[j] = 1.f / (1.f + __expf(-b));
      }
    }
    __syncthreads();
    for (int j = 0; j < nt; ++j) {
      const float decay = sg[j], beta = sb[j];
      const float* kk = &sk[j][kq * 32];
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        S[i] *= decay;
        dot += S[i] * kk[i];
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      const float u = (sv[j][vloc] - dot) * beta;
      const float* qq = &sq[j][kq * 32];
      float o = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        S[i] += kk[i] * u;
        o += S[i] * qq[i];
      }
      o += __shfl_xor_sync(0xffffffffu, o, 1);
      o += __shfl_xor_sync(0xffffffffu, o, 2);
      if (kq == 0) p.out[(size_t)(q0 + base + j) * p.ld_out + h * kDV + vcol] = f2bf(o);
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
    reinterpret_cast<float4*>(gstate)[i] = make_float4(S[4 * i], S[4 * i + 1], S[4 * i + 2], S[4 * i + 3]);
}

// Decode form (every request has exactly one new token): one CTA per (request, value head),
// 8 warps x 16 value rows.  A lane owns key dims [4 lane, 4 lane + 4) of its warp's 16 state
// rows, so each warp issues 16 independent 16-byte loads per lane before any arithmetic and
// the whole 64 KB state of the head is in flight at once (the step is a load-update-store of
// the state: HBM-bound).  Per row: s = e^g S_v; u = beta (v_v - s.k); s += u k; o_v = s.q, with
// the two dot products as warp reductions.  Same math and state layout as gdn_recurrent_kernel.
constexpr int kDecThreads = 256;
constexpr int kDecRowsPerWarp = kDV / (kDecThreads / 32);  // 16

__global__ void __launch_bounds__(kDecThreads, 2) gdn_decode_kernel(RecParams p) {
  pdl_launch_dependents();
  const int r = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = p.cu_q[r];
  const bool hist = p.seq_lens[r] - 1 > 0;
  const int hk = h / (p.Hv / p.Hk);
  const int v0 = warp * kDecRowsPerWarp;
  float* gstate = p.state + (((size_t)p.slots[r] * p.Hv + h) * kDV + v0) * kDK + lane * 4;
  float4 S[kDecRowsPerWarp];
  if (hist) {
#pragma unroll
    for (int j = 0; j < kDecRowsPerWarp; ++j)
      S[j] = *reinterpret_cast<const float4*>(gstate + (size_t)j * kDK);
  } else {
#pragma unroll
    for (int j = 0; j < kDecRowsPerWarp; ++j) S[j] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const __nv_bfloat16* row = p.qkv + (size_t)t * p.ld_qkv;
  const int qoff = hk * kDK, koff = p.Hk * kDK + hk * kDK, voff = 2 * p.Hk * kDK + h * kDV;
  const uint2 qr = *reinterpret_cast<const uint2*>(row + qoff + lane * 4);
  const uint2 kr = *reinterpret_cast<const uint2*>(row + koff + lane * 4);
  const float vv = lane < kDecRowsPerWarp ? bf2f(row[voff + v0 + lane]) : 0.f;
  const __nv_bfloat16* ba = p.ba + (size_t)t * p.ld_ba;
  const float b = bf2f(ba[h]), a = bf2f(ba[p.Hv + h]);
  float q[4], k[4];
  {
    const __nv_bfloat162* q2 = reinterpret_cast<const __nv_bfloat162*>(&qr);
    const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kr);
    const float2 q01 = __bfloat1622float2(q2[0]), q23 = __bfloat1622float2(q2[1]);
    const float2 k01 = __bfloat1622float2(k2[0]), k23 = __bfloat1622float2(k2[1]);
    q[0] = q01.x; q[1] = q01.y; q[2] = q23.x; q[3] = q23.y;
    k[0] = k01.x; k[1] = k01.y; k[2] = k23.x; k[3] = k23.y;
  }
  const float sqq = warp_sum(q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3]);
  const float skk = warp_sum(k[0] * k[0] + k[1] * k[1] + k[2] * k[2] + k[3] * k[3]);
  const float iq = rsqrtf(sqq + 1e-6f) * rsqrtf((float)kDK), ik = rsqrtf(skk + 1e-6f);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    q[e] *= iq;
    k[e] *= ik;
  }
  const float x = a + p.dt_bias[h];
  const float sp = x > 20.f ? x : log1pf(__expf(x));  // softplus
  const float decay = __expf(-__expf(p.A_log[h]) * sp);
  const float beta = 1.f / (1.f + __expf(-b));
  float mine = 0.f;  // lane j < 16 keeps the output of row v0 + j
#pragma unroll
  for (int j = 0; j < kDecRowsPerWarp; ++j) {
    float4 s4 = S[j];
    s4.x *= decay;
    s4.y *= decay;
    s4.z *= decay;
    s4.w *= decay;
    const float dot = warp_sum(s4.x * k[0] + s4.y * k[1] + s4.z * k[2] + s4.w * k[3]);
    const float u = (__shfl_sync(0xffffffffu, vv, j) - dot) * beta;
    s4.x += k[0] * u;
    s4.y += k[1] * u;
    s4.z += k[2] * u;
    s4.w += k[3] * u;
    const float o = warp_sum(s4.x * q[0] + s4.y * q[1] + s4.z * q[2] + s4.w * q[3]);
    if (lane == j) mine = o;
    S[j] = s4;
  }
#pragma unroll
  for (int j = 0; j < kDecRowsPerWarp; ++j)
    *reinterpret_cast<float4*>(gstate + (size_t)j * kDK) = S[j];
  if (lane < kDecRowsPerWarp)
    p.out[(size_t)t * p.ld_out + h * kDV + v0 + lane] = f2bf(mine);
}

// Attention output gate (Qwen3-Next gated attention): out *= sigmoid(gate), both [T, W].
__global__ void sigmoid_gate_kernel(__nv_bfloat16* __restrict__ out, int64_t ldo,
                                    const __nv_bfloat16* __restrict__ gate, int64_t ldg, int W) {
  pdl_launch_dependents();
  const int t = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= W) return;
  float o[8], g[8];
  uint4* op = reinterpret_cast<uint4*>(out + (size_t)t * ldo + c);
  unpack8(*op, o);
  unpack8(*reinterpret_cast<const uint4*>(gate + (size_t)t * ldg + c), g);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = o[j] / (1.f + __expf(-g[j]));
  *op = pack8(o);
}

// ------------------------------------------------------------------------------ launchers
void run_causal_conv1d(const void* x, int64_t ldx, const void* w, void* state,
                       const int32_t* cu_q, const int32_t* seq_lens, const int32_t* slots, int R,
                       int T, int C, void* out, int64_t ldo, cudaStream_t s,
                       const void* bias) {
  if (T == 0 || R == 0) return;
  const int threads = 128;
  const bool vec = C % 8 == 0 && ldx % 8 == 0 && ldo % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                     reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(bias)) % 16) == 0;
  if (vec)
    causal_conv1d_vec_kernel<<<dim3((C / 8 + threads - 1) / threads,
                                    (T + kConvTok - 1) / kConvTok), threads, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<const __nv_bfloat16*>(w),
        reinterpret_cast<const __nv_bfloat16*>(state), cu_q, seq_lens, slots, R, T, C,
        reinterpret_cast<__nv_bfloat16*>(out), ldo, reinterpret_cast<const __nv_bfloat16*>(bias));
  else
    causal_conv1d_kernel<<<dim3((C + threads - 1) / threads, T), threads, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<const __nv_bfloat16*>(w),
        reinterpret_cast<const __nv_bfloat16*>(state), cu_q, seq_lens, slots, R, C,
        reinterpret_cast<__nv_bfloat16*>(out), ldo, reinterpret_cast<const __nv_bfloat16*>(bias));
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
  conv_state_update_kernel<<<dim3((C + threads - 1) / threads, R), threads, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), ldx, reinterpret_cast<__nv_bfloat16*>(state),
      cu_q, seq_lens, slots, R, C);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_gdn_recurrent(const void* qkv, int64_t ld_qkv, const void* ba, int64_t ld_ba,
                       const float* A_log, const float* dt_bias, float* state,
                       const int32_t* cu_q, const int32_t* seq_lens, const int32_t* slots, int R,
                       int Hk, int Hv, void* out, int64_t ld_out, cudaStream_t s,
                       bool single_token) {
  B200_REQUIRE(Hv % Hk == 0, "gdn: value heads must be a multiple of key heads");
  if (R == 0) return;
  RecParams p;
  p.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv);
  p.ld_qkv = ld_qkv;
  p.ba = reinterpret_cast<const __nv_bfloat16*>(ba);
  p.ld_ba = ld_ba;
  p.A_log = A_log;
  p.dt_bias = dt_bias;
  p.state = state;
  p.cu_q = cu_q;
  p.seq_lens = seq_lens;
  p.slots = slots;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.R = R;
  p.Hk = Hk;
  p.Hv = Hv;
  if (single_token)
    gdn_decode_kernel<<<dim3(R, Hv), kDecThreads, 0, s>>>(p);
  else
    gdn_recurrent_kernel<<<dim3(R, Hv, kVSplit), kThreads, 0, s>>>(p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_sigmoid_gate(void* out, int64_t ldo, const void* gate, int64_t ldg, int T, int W,
                      cudaStream_t s) {
  B200_REQUIRE(W % 8 == 0, "sigmoid_gate: width % 8");
  if (T == 0) return;
  const int threads = 128;
  sigmoid_gate_kernel<<<dim3((W / 8 + threads - 1) / threads, T), threads, 0, s>>>(
      reinterpret_cast<__nv_bfloat16*>(out), ldo, reinterpret_cast<const __nv_bfloat16*>(gate),
      ldg, W);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace gdn
}  // namespace b200
