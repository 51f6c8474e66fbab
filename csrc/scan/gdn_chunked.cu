// Chunked gated delta rule (Qwen3-Next linear-attention prefill) for sm_100a.
//
// Token recurrence (per value head; S [dv, dk], q/k L2-normalised, q scaled by 1/sqrt(dk)):
//     S <- e^{g_t} S;  u_t = beta_t (v_t - S k_t);  S <- S + u_t k_t^T;  o_t = S q_t
// Over a chunk of C <= 64 tokens with G = cumsum(g), Gam = e^G and S0 the state at the chunk
// start, the updates U = [u_t] solve a unit lower-triangular system and everything else is a
// product of small matrices:
//     (I + diag(beta) L) [W | U0] = diag(beta) [diag(Gam) K | V],  L_ti = e^{G_t-G_i} k_t.k_i (i<t)
//     U  = U0 - W S0^T
//     O  = diag(Gam) Q S0^T + Mq U,  Mq_ti = e^{G_t-G_i} q_t.k_i (i<=t)
//     S' = e^{G_C} S0 + U^T diag(e^{G_C-G}) K
//
//   gdn_chunk_prep_kernel   one CTA per (chunk, value head), all chunks in parallel: stages
//                           normalised q, k and v, the gates, builds K K^T / Q K^T with the
//                           decay factors, and solves for [W | U0] by forward substitution
//                           (one thread per column, the 64 rows in registers).  Writes W, Qg =
//                           diag(Gam) Q, Kt = diag(e^{G_C-G}) K, Mq (bf16), U0 (fp32), e^{G_C}.
//   gdn_chunk_scan_kernel   one CTA per (request, value head, 32 value columns), sequential over
//                           the request's chunks: the state slice [32, 128] stays in mma.sync
//                           accumulator registers; per chunk three tensor-core products
//                           (U = U0 - W S^T, O = Qg S^T + Mq U, S = e^{G_C} S + U^T Kt) on
//                           bf16 operands with fp32 accumulation.
// The prep kernel's work (the O(C^2 d) part) is fully parallel; the sequential scan does
// O(C d^2) tensor-core work per chunk instead of C dependent token steps.  Short requests
// (decode) keep the token-recurrent kernel (gdn.cu); the state layout is shared.
//
// Reference counterpart: MATE chunk_gated_delta_rule called from vllm_musa/model_executor/
// layers/mamba/gdn/qwen_gdn_linear_attn.py:296-557 (no kernel source in the reference).
#include "../b200_kernels.h"
#include "../common/common.cuh"
#include "../common/mma_sm80.cuh"

namespace b200 {
namespace gdn {

namespace {

constexpr int kC = 64;       // chunk length
constexpr int kD = 128;      // dk = dv
constexpr int kPrepThreads = 256;
constexpr int kScanThreads = 128;
constexpr int kCols = 32;    // value columns per scan CTA
constexpr int kPadK = kD + 1;
constexpr int kLdP = kD + 8;  // bf16 row stride (272 B) of the prep kernel's tensor-core copies

// workspace block per (chunk, head)
constexpr size_t kWBytes = kC * kD * 2, kQgBytes = kC * kD * 2, kKtBytes = kC * kD * 2;
constexpr size_t kMqBytes = kC * kC * 2, kU0Bytes = kC * kD * 4;
constexpr size_t kBlockBytes = kWBytes + kQgBytes + kKtBytes + kMqBytes + kU0Bytes;

struct ChunkParams {
  const __nv_bfloat16* qkv;
  int64_t ld_qkv;
  const __nv_bfloat16* ba;
  int64_t ld_ba;
  const float* A_log;
  const float* dt_bias;
  float* state;
  const int32_t* cu_q;
  const int32_t* seq_lens;
  const int32_t* slots;
  int32_t* chunk_offsets;  // [R+1]
  uint8_t* ws;             // [max_chunks * Hv] blocks of kBlockBytes
  float* gam_c;            // [max_chunks * Hv]
  __nv_bfloat16* out;
  int64_t ld_out;
  int R, Hk, Hv, max_chunks;
};

__global__ void chunk_offsets_kernel(const int32_t* __restrict__ cu_q, int R,
                                     int32_t* __restrict__ out) {
  if (threadIdx.x == 0) {
    int acc = 0;
    out[0] = 0;
    for (int r = 0; r < R; ++r) {
      acc += (cu_q[r + 1] - cu_q[r] + kC - 1) / kC;
      out[r + 1] = acc;
    }
  }
}

B200_DEVICE int find_chunk_req(const int32_t* off, int R, int c) {
  int lo = 0, hi = R - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (off[mid] <= c) lo = mid; else hi = mid - 1;
  }
  return lo;
}

B200_DEVICE uint8_t* block_of(const ChunkParams& p, int chunk, int h) {
  return p.ws + ((size_t)chunk * p.Hv + h) * kBlockBytes;
}

B200_DEVICE uint32_t s_addr(const void* p) { return smem_u32(p); }

// A fragment (16 x 16 at (row0, k0)) of a row-major bf16 matrix with row stride ld elements
B200_DEVICE void load_a(const __nv_bfloat16* base, int ld, int row0, int k0, int lane,
                        uint32_t (&a)[4]) {
  const __nv_bfloat16* p = base + (row0 + (lane & 15)) * ld + k0 + ((lane >> 4) << 3);
  mma::ldsm_x4(s_addr(p), a[0], a[1], a[2], a[3]);
}
// B fragments of two n8 tiles (n0, n0+8) x k16 at k0 from an [n][k] (k contiguous) matrix
B200_DEVICE void load_b_nk(const __nv_bfloat16* base, int ld, int n0, int k0, int lane,
                           uint32_t& b0, uint32_t& b1, uint32_t& b2, uint32_t& b3) {
  const __nv_bfloat16* p =
      base + (n0 + (lane & 7) + ((lane >> 4) << 3)) * ld + k0 + (((lane >> 3) & 1) << 3);
  mma::ldsm_x4(s_addr(p), b0, b1, b2, b3);
}
// B fragments of two n8 tiles x k16 from a [k][n] (n contiguous) matrix (transposing load)
B200_DEVICE void load_b_kn(const __nv_bfloat16* base, int ld, int n0, int k0, int lane,
                           uint32_t& b0, uint32_t& b1, uint32_t& b2, uint32_t& b3) {
  const __nv_bfloat16* p =
      base + (k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * ld + n0 + ((lane >> 4) << 3);
  mma::ldsm_x4_t(s_addr(p), b0, b1, b2, b3);
}

// ------------------------------------------------------------------------------------ prep
__global__ void __launch_bounds__(kPrepThreads) gdn_chunk_prep_kernel(ChunkParams p) {
  extern __shared__ float smf[];
  float* sK = smf;                      // [64][129] normalised k
  float* sQ = sK + kC * kPadK;          // [64][129] normalised, scaled q
  float* sV = sQ + kC * kPadK;          // [64][129] v
  float* sL = sV + kC * kPadK;          // [64][65] beta_t e^{G_t-G_i} k_t.k_i (i<t)
  float* sG = sL + kC * (kC + 1);       // [64] cumulative log decay
  float* sB = sG + kC;                  // [64] beta
  __nv_bfloat16* sKb = reinterpret_cast<__nv_bfloat16*>(sB + kC);  // [64][136] bf16 k
  __nv_bfloat16* sQb = sKb + kC * kLdP;                              // [64][136] bf16 q

  const int chunk = blockIdx.x, h = blockIdx.y;
  const int total = p.chunk_offsets[p.R];
  if (chunk >= total) return;
  const int r = find_chunk_req(p.chunk_offsets, p.R, chunk);
  const int t0 = p.cu_q[r] + (chunk - p.chunk_offsets[r]) * kC;
  const int C = min(kC, p.cu_q[r + 1] - t0);
  const int hk = h / (p.Hv / p.Hk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float qscale = rsqrtf((float)kD);

  // stage q, k (L2-normalised) and v; one warp per token, 4 elements per lane
  for (int t = warp; t < kC; t += kPrepThreads / 32) {
    float qv[4] = {0.f, 0.f, 0.f, 0.f}, kv[4] = {0.f, 0.f, 0.f, 0.f}, vv[4] = {0.f, 0.f, 0.f, 0.f};
    if (t < C) {
      const __nv_bfloat16* row = p.qkv + (size_t)(t0 + t) * p.ld_qkv;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qv[e] = bf2f(row[hk * kD + lane * 4 + e]);
        kv[e] = bf2f(row[p.Hk * kD + hk * kD + lane * 4 + e]);
        vv[e] = bf2f(row[2 * p.Hk * kD + h * kD + lane * 4 + e]);
      }
    }
    float sq = 0.f, sk = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sq += qv[e] * qv[e];
      sk += kv[e] * kv[e];
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    const float iq = t < C ? rsqrtf(sq + 1e-6f) * qscale : 0.f;
    const float ik = t < C ? rsqrtf(sk + 1e-6f) : 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sQ[t * kPadK + lane * 4 + e] = qv[e] * iq;
      sK[t * kPadK + lane * 4 + e] = kv[e] * ik;
      sV[t * kPadK + lane * 4 + e] = vv[e];
      sQb[t * kLdP + lane * 4 + e] = f2bf(qv[e] * iq);
      sKb[t * kLdP + lane * 4 + e] = f2bf(kv[e] * ik);
    }
  }
  // gates and the cumulative log decay (warp 0: two tokens per lane, then a scan)
  if (warp == 0) {
    const float A = -__expf(p.A_log[h]);
    const float dtb = p.dt_bias[h];
    float g[2], b[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int t = lane + 32 * k;
      g[k] = 0.f;
      b[k] = 0.f;
      if (t < C) {
        const __nv_bfloat16* bar = p.ba + (size_t)(t0 + t) * p.ld_ba;
        const float x = bf2f(bar[p.Hv + h]) + dtb;
        const float sp = x > 20.f ? x : log1pf(__expf(x));  // softplus
        g[k] = A * sp;
        b[k] = 1.f / (1.f + __expf(-bf2f(bar[h])));
      }
    }
    // inclusive scan of g over the 64 tokens
#pragma unroll
    for (int k = 0; k < 2; ++k) {
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, g[k], off);
        if (lane >= off) g[k] += y;
      }
    }
    const float carry = __shfl_sync(0xffffffffu, g[0], 31);
    sG[lane] = g[0];
    sG[lane + 32] = g[1] + carry;
    sB[lane] = b[0];
    sB[lane + 32] = b[1];
  }
  __syncthreads();

  uint8_t* blk = block_of(p, chunk, h);
  __nv_bfloat16* gW = reinterpret_cast<__nv_bfloat16*>(blk);
  __nv_bfloat16* gQg = reinterpret_cast<__nv_bfloat16*>(blk + kWBytes);
  __nv_bfloat16* gKt = reinterpret_cast<__nv_bfloat16*>(blk + kWBytes + kQgBytes);
  __nv_bfloat16* gMq = reinterpret_cast<__nv_bfloat16*>(blk + kWBytes + kQgBytes + kKtBytes);
  float* gU0 = reinterpret_cast<float*>(blk + kWBytes + kQgBytes + kKtBytes + kMqBytes);
  const float Gc = sG[C - 1];

  // decayed K K^T (strictly lower, times beta_t) and Q K^T (lower incl. diagonal) on the
  // tensor cores (bf16 operands, fp32 accumulation): warp w owns rows [16 (w&3), +16) and
  // columns [32 (w>>2), +32) of both 64 x 64 products
  {
    const int mt = warp & 3, nh = warp >> 2;
    const int g = lane >> 2, tq = lane & 3;
    float kk[4][4], qk[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) kk[nt][e] = qk[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kD / 16; ++ks) {
      uint32_t ak[4], aq[4];
      load_a(sKb, kLdP, mt * 16, ks * 16, lane, ak);
      load_a(sQb, kLdP, mt * 16, ks * 16, lane, aq);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b0, b1, b2, b3;
        load_b_nk(sKb, kLdP, nh * 32 + np * 16, ks * 16, lane, b0, b1, b2, b3);
        mma::mma_bf16(kk[2 * np], ak, b0, b1);
        mma::mma_bf16(kk[2 * np + 1], ak, b2, b3);
        mma::mma_bf16(qk[2 * np], aq, b0, b1);
        mma::mma_bf16(qk[2 * np + 1], aq, b2, b3);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = mt * 16 + g + ((e >> 1) << 3);
        const int i = nh * 32 + nt * 8 + 2 * tq + (e & 1);
        float kv = 0.f, qv = 0.f;
        if (i <= t) {
          const float dec = __expf(sG[t] - sG[i]);
          kv = kk[nt][e] * dec * sB[t];
          qv = qk[nt][e] * dec;
        }
        sL[t * (kC + 1) + i] = i < t ? kv : 0.f;
        gMq[t * kC + i] = f2bf(qv);
      }
  }
  __syncthreads();

  // forward substitution for [W | U0]: one column per thread, rows in registers
  {
    const int col = tid;  // 0..127 -> W (Gam-scaled K), 128..255 -> U0 (V)
    float x[kC];
#pragma unroll
    for (int t = 0; t < kC; ++t) {
      float rhs = col < kD ? __expf(sG[t]) * sK[t * kPadK + col] : sV[t * kPadK + col - kD];
      rhs *= sB[t];
#pragma unroll
      for (int i = 0; i < t; ++i) rhs -= sL[t * (kC + 1) + i] * x[i];
      x[t] = rhs;
    }
    if (col < kD) {
#pragma unroll
      for (int t = 0; t < kC; ++t) gW[t * kD + col] = f2bf(x[t]);
    } else {
#pragma unroll
      for (int t = 0; t < kC; ++t) gU0[t * kD + col - kD] = x[t];
    }
  }
  // Qg = diag(Gam) Q, Kt = diag(e^{G_C - G}) K
  for (int e = tid; e < kC * kD; e += kPrepThreads) {
    const int t = e / kD, d = e % kD;
    gQg[e] = f2bf(__expf(sG[t]) * sQ[t * kPadK + d]);
    gKt[e] = f2bf(t < C ? __expf(Gc - sG[t]) * sK[t * kPadK + d] : 0.f);
  }
  if (tid == 0) p.gam_c[(size_t)chunk * p.Hv + h] = __expf(Gc);
}

// ------------------------------------------------------------------------------------ scan
constexpr int kLdA = kD + 8;   // bf16 row stride (272 B) of the 128-wide staged operands
constexpr int kLdM = kC + 8;   // 64-wide (144 B)
constexpr int kLdS = kD + 8;   // state slice rows
constexpr int kLdU = kC + 8;   // U^T rows

struct ScanSmem {
  __nv_bfloat16 W[kC * kLdA];
  __nv_bfloat16 Qg[kC * kLdA];
  __nv_bfloat16 Kt[kC * kLdA];
  __nv_bfloat16 Mq[kC * kLdM];
  float U0[kC * kCols];
  __nv_bfloat16 S[kCols * kLdS];   // state slice [v][k] (bf16 copy for the products)
  __nv_bfloat16 Ut[kCols * kLdU];  // U^T [v][t]
};

__global__ void __launch_bounds__(kScanThreads) gdn_chunk_scan_kernel(ChunkParams p) {
  extern __shared__ uint8_t sm_raw[];
  ScanSmem& sm = *reinterpret_cast<ScanSmem*>(
      (reinterpret_cast<uintptr_t>(sm_raw) + 127) & ~uintptr_t(127));
  const int r = blockIdx.x, h = blockIdx.y;
  const int c0 = blockIdx.z * kCols;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int q0 = p.cu_q[r];
  const int L = p.cu_q[r + 1] - q0;
  if (L <= 0) return;
  const bool hist = p.seq_lens[r] - L > 0;
  float* gstate = p.state + (((size_t)p.slots[r] * p.Hv + h) * kD + c0) * kD;

  // state slice S[v][k] (v < 32, k < 128) as accumulators of the S update product:
  // warp w owns k columns [32w, 32w+32): 2 m16 tiles (v) x 4 n8 tiles (k)
  float acc[2][4][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int v = mt * 16 + g + ((e >> 1) << 3);
        const int k = warp * 32 + nt * 8 + 2 * tq + (e & 1);
        acc[mt][nt][e] = hist ? gstate[(size_t)v * kD + k] : 0.f;
      }

  const int cfirst = p.chunk_offsets[r], nch = p.chunk_offsets[r + 1] - cfirst;
  for (int ci = 0; ci < nch; ++ci) {
    const int chunk = cfirst + ci;
    const int C = min(kC, L - ci * kC);
    const uint8_t* blk = p.ws + ((size_t)chunk * p.Hv + h) * kBlockBytes;
    __syncthreads();  // previous chunk done with the staging buffers
    // stage this chunk's operands (16-byte async copies) and the bf16 state slice
    {
      const uint4* src[3] = {reinterpret_cast<const uint4*>(blk),
                             reinterpret_cast<const uint4*>(blk + kWBytes),
                             reinterpret_cast<const uint4*>(blk + kWBytes + kQgBytes)};
      __nv_bfloat16* dst[3] = {sm.W, sm.Qg, sm.Kt};
#pragma unroll
      for (int m = 0; m < 3; ++m)
        for (int i = tid; i < kC * kD / 8; i += kScanThreads) {
          const int t = i / (kD / 8), c = i % (kD / 8);
          cp_async16(dst[m] + t * kLdA + c * 8, src[m] + i);
        }
      const uint4* mq = reinterpret_cast<const uint4*>(blk + kWBytes + kQgBytes + kKtBytes);
      for (int i = tid; i < kC * kC / 8; i += kScanThreads) {
        const int t = i / (kC / 8), c = i % (kC / 8);
        cp_async16(sm.Mq + t * kLdM + c * 8, mq + i);
      }
      const float* u0 =
          reinterpret_cast<const float*>(blk + kWBytes + kQgBytes + kKtBytes + kMqBytes);
      for (int i = tid; i < kC * kCols / 4; i += kScanThreads) {
        const int t = i / (kCols / 4), c = i % (kCols / 4);
        cp_async16(sm.U0 + t * kCols + c * 4, u0 + (size_t)t * kD + c0 + c * 4);
      }
      cp_async_commit();
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int v = mt * 16 + g, k = warp * 32 + nt * 8 + 2 * tq;
        *reinterpret_cast<uint32_t*>(&sm.S[v * kLdS + k]) =
            pack_bf16x2(acc[mt][nt][0], acc[mt][nt][1]);
        *reinterpret_cast<uint32_t*>(&sm.S[(v + 8) * kLdS + k]) =
            pack_bf16x2(acc[mt][nt][2], acc[mt][nt][3]);
      }
    cp_async_wait<0>();
    __syncthreads();

    // U = U0 - W S^T and P1 = Qg S^T : warp w owns token rows [16w, 16w+16), N = 32 (v)
    float u[4][4], o[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) u[nt][e] = o[nt][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kD / 16; ++ks) {
      uint32_t aw[4], aq[4];
      load_a(sm.W, kLdA, warp * 16, ks * 16, lane, aw);
      load_a(sm.Qg, kLdA, warp * 16, ks * 16, lane, aq);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b0, b1, b2, b3;
        load_b_nk(sm.S, kLdS, np * 16, ks * 16, lane, b0, b1, b2, b3);
        mma::mma_bf16(u[2 * np], aw, b0, b1);
        mma::mma_bf16(u[2 * np + 1], aw, b2, b3);
        mma::mma_bf16(o[2 * np], aq, b0, b1);
        mma::mma_bf16(o[2 * np + 1], aq, b2, b3);
      }
    }
    // U = U0 - W S^T  -> U^T in shared memory (bf16) for the two products that consume it
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = warp * 16 + g + ((e >> 1) << 3);
        const int v = nt * 8 + 2 * tq + (e & 1);
        u[nt][e] = sm.U0[t * kCols + v] - u[nt][e];
        sm.Ut[v * kLdU + t] = f2bf(u[nt][e]);
      }
    __syncthreads();
    // O = Qg S^T + Mq U  (Mq rows of this warp, U as [v][t])
#pragma unroll
    for (int ks = 0; ks < kC / 16; ++ks) {
      uint32_t am[4];
      load_a(sm.Mq, kLdM, warp * 16, ks * 16, lane, am);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b0, b1, b2, b3;
        load_b_nk(sm.Ut, kLdU, np * 16, ks * 16, lane, b0, b1, b2, b3);
        mma::mma_bf16(o[2 * np], am, b0, b1);
        mma::mma_bf16(o[2 * np + 1], am, b2, b3);
      }
    }
    const int tbase = q0 + ci * kC;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int t = warp * 16 + g + hh * 8;
        if (t < C) {
          const int v = c0 + nt * 8 + 2 * tq;
          *reinterpret_cast<uint32_t*>(p.out + (size_t)(tbase + t) * p.ld_out + h * kD + v) =
              pack_bf16x2(o[nt][2 * hh], o[nt][2 * hh + 1]);
        }
      }
    // S = e^{G_C} S + U^T Kt : A = U^T [v][t] (2 m16 tiles), B = Kt [t][k] (transposing load)
    const float gc = p.gam_c[(size_t)chunk * p.Hv + h];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[mt][nt][e] *= gc;
#pragma unroll
    for (int ks = 0; ks < kC / 16; ++ks) {
      uint32_t a0[4], a1[4];
      load_a(sm.Ut, kLdU, 0, ks * 16, lane, a0);
      load_a(sm.Ut, kLdU, 16, ks * 16, lane, a1);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b0, b1, b2, b3;
        load_b_kn(sm.Kt, kLdA, warp * 32 + np * 16, ks * 16, lane, b0, b1, b2, b3);
        mma::mma_bf16(acc[0][2 * np], a0, b0, b1);
        mma::mma_bf16(acc[0][2 * np + 1], a0, b2, b3);
        mma::mma_bf16(acc[1][2 * np], a1, b0, b1);
        mma::mma_bf16(acc[1][2 * np + 1], a1, b2, b3);
      }
    }
  }
  // state slice back to its slot
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int v = mt * 16 + g + ((e >> 1) << 3);
        const int k = warp * 32 + nt * 8 + 2 * tq + (e & 1);
        gstate[(size_t)v * kD + k] = acc[mt][nt][e];
      }
}

}  // namespace

size_t chunked_workspace_bytes(int max_chunks, int Hv) {
  return (size_t)max_chunks * Hv * kBlockBytes;
}

void run_gdn_chunked(const void* qkv, int64_t ld_qkv, const void* ba, int64_t ld_ba,
                     const float* A_log, const float* dt_bias, float* state, const int32_t* cu_q,
                     const int32_t* seq_lens, const int32_t* slots, int32_t* chunk_offsets,
                     void* ws, float* gam_c, int R, int T, int Hk, int Hv, void* out,
                     int64_t ld_out, cudaStream_t s) {
  if (R == 0 || T == 0) return;
  B200_REQUIRE(Hv % Hk == 0, "gdn chunked: Hv must be a multiple of Hk");
  ChunkParams p;
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
  p.chunk_offsets = chunk_offsets;
  p.ws = reinterpret_cast<uint8_t*>(ws);
  p.gam_c = gam_c;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.R = R;
  p.Hk = Hk;
  p.Hv = Hv;
  p.max_chunks = (T + kC - 1) / kC + R;
  chunk_offsets_kernel<<<1, 32, 0, s>>>(cu_q, R, chunk_offsets);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
  const int prep_smem = (3 * kC * kPadK + kC * (kC + 1) + 2 * kC) * (int)sizeof(float) +
                        2 * kC * kLdP * (int)sizeof(__nv_bfloat16);
  ensure_dynamic_smem(reinterpret_cast<const void*>(gdn_chunk_prep_kernel), prep_smem);
  gdn_chunk_prep_kernel<<<dim3(p.max_chunks, Hv), kPrepThreads, prep_smem, s>>>(p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
  const int scan_smem = (int)sizeof(ScanSmem) + 128;
  ensure_dynamic_smem(reinterpret_cast<const void*>(gdn_chunk_scan_kernel), scan_smem);
  gdn_chunk_scan_kernel<<<dim3(R, Hv, kD / kCols), kScanThreads, scan_smem, s>>>(p);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace gdn
}  // namespace b200
