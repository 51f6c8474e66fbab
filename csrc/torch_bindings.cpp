// torch.ops.b200.* registration for the sm_100a kernels, plus pybind11 helpers.
//
// This is the only translation unit that includes torch headers next to the kernel launchers:
// it checks devices, dtypes, shapes, strides and alignment, then calls the plain-C++ launchers
// declared in b200_kernels.h on the current CUDA stream.  Mirrors the role of the reference's
// csrc/musa/torch_bindings.cpp:9-275 (`_C_musa_ops` schemas); the op set is this framework's.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <torch/library.h>

#include <mutex>

#include "b200_kernels.h"
#include "common/host_check.h"
#include "comm/custom_ar.h"

namespace {

using at::Tensor;

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bf16")
#define CHECK_ROWMAJOR(x) TORCH_CHECK((x).dim() == 2 && (x).stride(1) == 1, #x " must be 2-D, rows contiguous")

cudaStream_t stream_of(const Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()); }

// ---- per-device error word (bounded waits record timeouts here) ----
std::mutex g_err_mu;
Tensor g_err[64];

Tensor error_word_for(const at::Device& dev) {
  std::lock_guard<std::mutex> lk(g_err_mu);
  const int i = dev.index();
  TORCH_CHECK(i >= 0 && i < 64, "device index out of range");
  if (!g_err[i].defined())
    g_err[i] = at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(dev));
  return g_err[i];
}
int* err_ptr(const Tensor& t) { return error_word_for(t.device()).data_ptr<int>(); }

template <typename F>
void guarded(F&& f) {
  try {
    f();
  } catch (const std::runtime_error& e) {
    TORCH_CHECK(false, e.what());
  }
}

// ------------------------------------------------------------------------------------- GEMM
void gemm_bf16(const Tensor& A, const Tensor& B, Tensor& C, int64_t mode, int64_t bn,
               int64_t splits, const c10::optional<Tensor>& workspace, int64_t mt,
               const c10::optional<Tensor>& counters) {
  CHECK_CUDA(A);
  CHECK_CUDA(B);
  CHECK_CUDA(C);
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_ROWMAJOR(A);
  CHECK_ROWMAJOR(B);
  CHECK_ROWMAJOR(C);
  TORCH_CHECK(A.size(1) == B.size(1), "gemm_bf16: K mismatch");
  const int M = A.size(0), N = B.size(0), K = A.size(1);
  if (mode == 4 || mode == 5) {  // swapped: A = weight [features, K], B = activations [tokens, K]
    TORCH_CHECK(C.size(0) == N && C.size(1) == (mode == 5 ? M / 2 : M), "gemm_bf16: C^T shape");
    TORCH_CHECK(C.stride(1) == 1, "gemm_bf16: C row-major");
  } else {
    TORCH_CHECK(C.size(0) == M && C.size(1) == (mode == 1 ? N / 2 : N), "gemm_bf16: C shape");
  }
  TORCH_CHECK(C.scalar_type() == (mode == 2 ? at::kFloat : at::kBFloat16), "gemm_bf16: C dtype");
  const c10::cuda::CUDAGuard g(A.device());
  b200::gemm::GemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.M = M;
  a.N = N;
  a.K = K;
  a.mode = mode;
  a.bn = bn;
  a.splits = splits;
  a.mt = mt;
  if (workspace.has_value()) {
    TORCH_CHECK(workspace->scalar_type() == at::kFloat && workspace->is_cuda(), "workspace");
    a.workspace = workspace->data_ptr<float>();
    a.workspace_numel = workspace->numel();
  }
  if (counters.has_value()) {
    TORCH_CHECK(counters->scalar_type() == at::kInt && counters->is_cuda(), "counters");
    a.counters = counters->data_ptr<int>();
    a.counters_numel = counters->numel();
  }
  a.err = err_ptr(A);
  guarded([&] { b200::gemm::run_bf16(a, stream_of(A)); });
}

std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K) {
  const auto p = b200::gemm::plan_bf16(M, N, K);
  return {p.bn, p.splits, p.workspace_floats, p.mt};
}

void gemm_fp8(const Tensor& A, const Tensor& sa, const Tensor& B, const Tensor& sb, Tensor& C,
              int64_t splits, const c10::optional<Tensor>& workspace,
              const c10::optional<Tensor>& counters, const c10::optional<Tensor>& tile_expert,
              const c10::optional<Tensor>& num_tiles, int64_t num_experts) {
  CHECK_CUDA(A);
  CHECK_CUDA(B);
  TORCH_CHECK(A.scalar_type() == at::kFloat8_e4m3fn && B.scalar_type() == at::kFloat8_e4m3fn,
              "gemm_fp8: e4m3 operands");
  CHECK_ROWMAJOR(A);
  CHECK_ROWMAJOR(B);
  CHECK_ROWMAJOR(C);
  TORCH_CHECK(C.scalar_type() == at::kBFloat16, "gemm_fp8: bf16 output");
  TORCH_CHECK(sa.scalar_type() == at::kFloat && sb.scalar_type() == at::kFloat &&
                  sa.stride(1) == 1 && sb.stride(1) == 1,
              "gemm_fp8: fp32 row-major scales");
  const bool grouped = tile_expert.has_value();
  const int E = grouped ? num_experts : 1;
  TORCH_CHECK(!grouped || (num_tiles.has_value() && E > 0 && B.size(0) % E == 0),
              "gemm_fp8: grouped mode needs num_tiles and B rows = E * N");
  const int M = A.size(0), N = B.size(0) / E, K = A.size(1);
  const int kb = (K + 127) / 128;
  TORCH_CHECK(B.size(1) == K && C.size(0) == M && C.size(1) == N, "gemm_fp8: shapes");
  TORCH_CHECK(sa.size(0) >= M && sa.size(1) >= kb, "gemm_fp8: activation scales [M, K/128]");
  TORCH_CHECK(sb.size(0) >= E * ((N + 127) / 128) && sb.size(1) >= kb,
              "gemm_fp8: weight scales [E * N/128, K/128]");
  const c10::cuda::CUDAGuard g(A.device());
  b200::gemm_fp8::Fp8GemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.sa = sa.data_ptr<float>();
  a.sa_ld = sa.stride(0);
  a.sb = sb.data_ptr<float>();
  a.sb_ld = sb.stride(0);
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.M = M;
  a.N = N;
  a.K = K;
  a.splits = splits;
  if (workspace.has_value()) {
    TORCH_CHECK(workspace->scalar_type() == at::kFloat && workspace->is_cuda(), "workspace");
    a.workspace = workspace->data_ptr<float>();
    a.workspace_numel = workspace->numel();
  }
  if (counters.has_value()) {
    TORCH_CHECK(counters->scalar_type() == at::kInt && counters->is_cuda(), "counters");
    a.counters = counters->data_ptr<int>();
    a.counters_numel = counters->numel();
  }
  if (grouped) {
    TORCH_CHECK(tile_expert->scalar_type() == at::kInt && num_tiles->scalar_type() == at::kInt,
                "gemm_fp8: int32 tile metadata");
    a.tile_expert = tile_expert->data_ptr<int32_t>();
    a.num_tiles = num_tiles->data_ptr<int32_t>();
    a.num_experts = E;
  }
  a.err = err_ptr(A);
  guarded([&] { b200::gemm_fp8::run_fp8(a, stream_of(A)); });
}

std::vector<int64_t> gemm_fp8_plan(int64_t M, int64_t N, int64_t K) {
  const auto p = b200::gemm_fp8::plan_fp8(M, N, K);
  return {p.splits, p.workspace_floats, p.counters};
}

// ------------------------------------------------------------------------------------- norms
void rms_norm(Tensor& out, const Tensor& x, const Tensor& w, double eps, bool gemma) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_ROWMAJOR(x);
  CHECK_ROWMAJOR(out);
  TORCH_CHECK(w.is_contiguous() && w.numel() == x.size(1), "rms_norm: weight");
  const c10::cuda::CUDAGuard g(x.device());
  b200::norm::RmsNormArgs a{};
  a.out = out.data_ptr();
  a.ld_out = out.stride(0);
  a.x = const_cast<void*>(x.data_ptr());
  a.ld_x = x.stride(0);
  a.residual = nullptr;
  a.weight = w.data_ptr();
  a.rows = x.size(0);
  a.H = x.size(1);
  a.eps = eps;
  a.gemma = gemma;
  guarded([&] { b200::norm::run_rms_norm(a, stream_of(x)); });
}

void fused_add_rms_norm(Tensor& x, Tensor& residual, const Tensor& w, double eps, bool gemma) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(residual);
  CHECK_BF16(w);
  CHECK_ROWMAJOR(x);
  CHECK_ROWMAJOR(residual);
  TORCH_CHECK(x.sizes() == residual.sizes(), "fused_add_rms_norm: shape mismatch");
  TORCH_CHECK(w.is_contiguous() && w.numel() == x.size(1), "fused_add_rms_norm: weight");
  const c10::cuda::CUDAGuard g(x.device());
  b200::norm::RmsNormArgs a{};
  a.out = x.data_ptr();
  a.ld_out = x.stride(0);
  a.x = x.data_ptr();
  a.ld_x = x.stride(0);
  a.residual = residual.data_ptr();
  a.ld_res = residual.stride(0);
  a.weight = w.data_ptr();
  a.rows = x.size(0);
  a.H = x.size(1);
  a.eps = eps;
  a.gemma = gemma;
  guarded([&] { b200::norm::run_rms_norm(a, stream_of(x)); });
}

void rms_norm_quant_fp8(Tensor& q, Tensor& scales, std::optional<Tensor> out, Tensor& x,
                       std::optional<Tensor> residual, const Tensor& w, double eps) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_ROWMAJOR(x);
  CHECK_ROWMAJOR(q);
  TORCH_CHECK(q.scalar_type() == at::kFloat8_e4m3fn, "rms_norm_quant_fp8: q must be e4m3");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.is_contiguous(),
              "rms_norm_quant_fp8: scales must be contiguous fp32");
  const int64_t rows = x.size(0), H = x.size(1);
  TORCH_CHECK(q.size(0) == rows && q.size(1) == H, "rms_norm_quant_fp8: q shape");
  TORCH_CHECK(scales.numel() >= rows * (H / 128), "rms_norm_quant_fp8: scales too small");
  TORCH_CHECK(w.is_contiguous() && w.numel() == H, "rms_norm_quant_fp8: weight");
  if (out) {
    CHECK_BF16(*out);
    CHECK_ROWMAJOR(*out);
    TORCH_CHECK(out->size(0) == rows && out->size(1) == H, "rms_norm_quant_fp8: out shape");
  }
  if (residual) {
    CHECK_BF16(*residual);
    CHECK_ROWMAJOR(*residual);
    TORCH_CHECK(residual->sizes() == x.sizes(), "rms_norm_quant_fp8: residual shape");
  }
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::norm::run_rms_norm_quant_fp8(
        q.data_ptr(), q.stride(0), scales.data_ptr<float>(), out ? out->data_ptr() : nullptr,
        out ? out->stride(0) : 0, x.data_ptr(), x.stride(0),
        residual ? residual->data_ptr() : nullptr, residual ? residual->stride(0) : 0,
        w.data_ptr(), (int)rows, (int)H, (float)eps, stream_of(x));
  });
}

void rms_norm_gated(Tensor& out, const Tensor& x, const Tensor& z, const Tensor& w, int64_t group,
                    double eps) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(z);
  CHECK_BF16(w);
  CHECK_ROWMAJOR(x);
  CHECK_ROWMAJOR(z);
  CHECK_ROWMAJOR(out);
  TORCH_CHECK(w.numel() == group, "rms_norm_gated: weight must have `group` elements");
  const c10::cuda::CUDAGuard g(x.device());
  const int H = x.size(1);
  const int rows = x.size(0);
  TORCH_CHECK(z.size(1) == H && out.size(1) == H && z.size(0) == rows, "rms_norm_gated: shapes");
  guarded([&] {
    b200::norm::run_rms_norm_gated(out.data_ptr(), out.stride(0), x.data_ptr(), x.stride(0),
                                   z.data_ptr(), z.stride(0), w.data_ptr(), rows, H, group, eps,
                                   stream_of(x));
  });
}

// ------------------------------------------------------------------------------------- act
void act_and_mul(Tensor& out, const Tensor& x, int64_t kind, double limit) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_ROWMAJOR(x);
  CHECK_ROWMAJOR(out);
  const int I = x.size(1) / 2;
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) == I, "act_and_mul: out shape");
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::act::run_act_and_mul(out.data_ptr(), out.stride(0), x.data_ptr(), x.stride(0), x.size(0),
                               I, kind, limit, stream_of(x));
  });
}

void silu_mul_fp8_quant(Tensor& out, Tensor& scales, const Tensor& x, double limit) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_ROWMAJOR(x);
  const int I = x.size(1) / 2;
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && out.is_contiguous() &&
                  out.size(0) == x.size(0) && out.size(1) == I,
              "silu_mul_fp8_quant: out");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.is_contiguous() &&
                  scales.numel() == x.size(0) * (I / 128),
              "silu_mul_fp8_quant: scales");
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::act::run_silu_mul_fp8_quant(out.data_ptr(), scales.data_ptr<float>(), x.data_ptr(),
                                      x.stride(0), x.size(0), I, stream_of(x), (float)limit);
  });
}

void group_quant_fp8(Tensor& out, Tensor& scales, const Tensor& x) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_ROWMAJOR(x);
  const int K = x.size(1);
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && out.is_contiguous() &&
                  out.sizes() == x.sizes(),
              "group_quant_fp8: out");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.numel() == x.size(0) * (K / 128),
              "group_quant_fp8: scales");
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::act::run_group_quant_fp8(out.data_ptr(), scales.data_ptr<float>(), x.data_ptr(),
                                   x.stride(0), x.size(0), K, stream_of(x));
  });
}

// ------------------------------------------------------------------------------------- rope+kv
void kv_insert(const Tensor& key, const Tensor& value, Tensor& k_cache, Tensor& v_cache,
               const Tensor& slot_mapping) {
  CHECK_CUDA(key);
  CHECK_BF16(key);
  CHECK_BF16(value);
  TORCH_CHECK(key.dim() == 3 && value.dim() == 3 && key.stride(2) == 1 && value.stride(2) == 1,
              "kv_insert: key / value [T, Hkv, D] with unit inner stride");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  k_cache.size(1) == key.size(1) && k_cache.size(3) == key.size(2),
              "kv_insert: caches [num_blocks, Hkv, block_size, D]");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kLong && slot_mapping.is_contiguous(),
              "kv_insert: int64 slot_mapping");
  const int T = std::min<int64_t>(slot_mapping.numel(), key.size(0));
  const c10::cuda::CUDAGuard g(key.device());
  guarded([&] {
    b200::rope::run_kv_insert(key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(),
                              value.stride(0), value.stride(1), k_cache.data_ptr(),
                              v_cache.data_ptr(), slot_mapping.data_ptr<int64_t>(), T,
                              key.size(1), key.size(2), k_cache.size(2), stream_of(key));
  });
}

void rope_kv(Tensor& qkv, const Tensor& positions, const Tensor& cos_sin,
             const c10::optional<Tensor>& q_norm_w, const c10::optional<Tensor>& k_norm_w,
             const c10::optional<Tensor>& k_cache_opt, const c10::optional<Tensor>& v_cache_opt,
             const Tensor& slot_mapping, int64_t Hq, int64_t Hkv, int64_t rot_dim, bool neox,
             double eps, int64_t head_dim, c10::optional<at::IntArrayRef> mrope_section,
             bool mrope_interleaved) {
  CHECK_CUDA(qkv);
  CHECK_BF16(qkv);
  CHECK_ROWMAJOR(qkv);
  const bool cached = k_cache_opt.has_value();
  TORCH_CHECK(cached == v_cache_opt.has_value(), "rope_kv: pass both caches or neither");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.is_contiguous(), "positions int32");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kInt && slot_mapping.is_contiguous(),
              "slot_mapping int32");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.is_contiguous() &&
                  cos_sin.size(1) == rot_dim,
              "cos_sin must be fp32 [max_pos, rot_dim]");
  if (cached) {
    const Tensor& k_cache = *k_cache_opt;
    const Tensor& v_cache = *v_cache_opt;
    CHECK_BF16(k_cache);
    CHECK_BF16(v_cache);
    TORCH_CHECK(k_cache.dim() == 4 && k_cache.is_contiguous() && v_cache.is_contiguous(),
                "kv cache must be contiguous [blocks, Hkv, block_size, D]");
    TORCH_CHECK(k_cache.size(1) == Hkv, "rope_kv: cache heads");
  }
  const int T = qkv.size(0);
  const int D = cached ? k_cache_opt->size(3) : (int)head_dim;
  TORCH_CHECK(D > 0, "rope_kv: head_dim required without a cache");
  TORCH_CHECK(qkv.size(1) >= (Hq + 2 * Hkv) * D, "rope_kv: qkv width");
  const c10::cuda::CUDAGuard g(qkv.device());
  b200::rope::RopeKvArgs a{};
  a.qkv = qkv.data_ptr();
  a.ld_qkv = qkv.stride(0);
  a.positions = positions.data_ptr<int32_t>();
  a.cos_sin = cos_sin.data_ptr<float>();
  a.q_norm_w = q_norm_w.has_value() ? q_norm_w->data_ptr() : nullptr;
  a.k_norm_w = k_norm_w.has_value() ? k_norm_w->data_ptr() : nullptr;
  a.k_cache = cached ? k_cache_opt->data_ptr() : nullptr;
  a.v_cache = cached ? v_cache_opt->data_ptr() : nullptr;
  a.slot_mapping = slot_mapping.data_ptr<int32_t>();
  a.T = T;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = D;
  a.block_size = cached ? k_cache_opt->size(2) : 1;
  a.rot_dim = rot_dim;
  a.neox = neox;
  a.eps = eps;
  a.err = err_ptr(qkv);
  if (mrope_section.has_value()) {
    const auto sec = *mrope_section;
    TORCH_CHECK(sec.size() == 3, "rope_kv: mrope_section needs 3 entries");
    TORCH_CHECK(positions.dim() == 2 && positions.size(0) == 3 && positions.size(1) >= T,
                "rope_kv: M-RoPE positions must be [3, >= T]");
    a.mrope.mode = mrope_interleaved ? 2 : 1;
    a.mrope.s0 = sec[0];
    a.mrope.s1 = sec[1];
    a.mrope.s2 = sec[2];
    a.mrope.pos_stride = positions.size(1);
  }
  guarded([&] { b200::rope::run_rope_kv(a, stream_of(qkv)); });
}

// ------------------------------------------------------------------------------------- MLA
void mla_prep(Tensor& q, const Tensor& kv, const Tensor& kv_norm_w, double eps,
              const Tensor& positions, const Tensor& cos_sin, Tensor& cache,
              const Tensor& slot_mapping, int64_t Hq) {
  CHECK_CUDA(q);
  CHECK_BF16(q);
  CHECK_BF16(kv);
  TORCH_CHECK(q.stride(1) == 1 && kv.stride(1) == 1 && q.size(1) >= Hq * 192 && kv.size(1) >= 576,
              "mla_prep: q [T, Hq*192], kv [T, 576] row-major");
  TORCH_CHECK(cache.is_contiguous() && cache.size(-1) == 576 && cache.scalar_type() == at::kBFloat16,
              "mla_prep: bf16 latent cache [..., 576]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == 64, "mla_prep: cos_sin [P, 64]");
  TORCH_CHECK(positions.scalar_type() == at::kInt && slot_mapping.scalar_type() == at::kInt,
              "mla_prep: int32 positions / slots");
  const c10::cuda::CUDAGuard g(q.device());
  guarded([&] {
    b200::mla::run_prep(q.data_ptr(), q.stride(0), Hq, kv.data_ptr(), kv.stride(0),
                        kv_norm_w.data_ptr(), eps, positions.data_ptr<int32_t>(),
                        cos_sin.data_ptr<float>(), cache.data_ptr(), slot_mapping.data_ptr<int32_t>(),
                        q.size(0), stream_of(q));
  });
}

void mla_attention(const Tensor& q_lat, const Tensor& q_pe, const Tensor& cache,
                   const Tensor& block_tables, const Tensor& cu_q, const Tensor& seq_lens,
                   const c10::optional<Tensor>& indices, Tensor& out, double scale, int64_t splits,
                   const c10::optional<Tensor>& ws_o, const c10::optional<Tensor>& ws_lse,
                   int64_t dcp_size, int64_t dcp_rank, const c10::optional<Tensor>& lse_out) {
  CHECK_CUDA(q_lat);
  TORCH_CHECK(q_lat.dim() == 3 && q_pe.dim() == 3 && out.dim() == 3, "mla_attention: [T, H, C] views");
  TORCH_CHECK(q_lat.stride(2) == 1 && q_pe.stride(2) == 1 && out.stride(2) == 1 &&
                  q_lat.size(2) == 512 && q_pe.size(2) == 64 && out.size(2) == 512,
              "mla_attention: inner dims 512 / 64 contiguous");
  TORCH_CHECK(q_lat.scalar_type() == at::kBFloat16 && q_pe.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16 && cache.scalar_type() == at::kBFloat16,
              "mla_attention: bf16");
  TORCH_CHECK(cache.is_contiguous() && cache.size(-1) == 576, "mla_attention: cache [..., 576]");
  TORCH_CHECK(block_tables.dim() == 2 && block_tables.stride(1) == 1, "mla_attention: block tables");
  const int bs = cache.dim() == 3 ? cache.size(1) : cache.size(-2);
  b200::mla::MlaArgs a{};
  a.q_lat = q_lat.data_ptr();
  a.ql_t = q_lat.stride(0);
  a.ql_h = q_lat.stride(1);
  a.q_pe = q_pe.data_ptr();
  a.qp_t = q_pe.stride(0);
  a.qp_h = q_pe.stride(1);
  a.cache = cache.data_ptr();
  a.block_tables = block_tables.data_ptr<int32_t>();
  a.bt_stride = block_tables.stride(0);
  a.block_size = bs;
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.R = seq_lens.size(0);
  if (indices.has_value()) {
    TORCH_CHECK(indices->scalar_type() == at::kInt && indices->stride(1) == 1, "mla: int32 indices");
    a.indices = indices->data_ptr<int32_t>();
    a.idx_ld = indices->stride(0);
    a.topk = indices->size(1);
  }
  a.out = out.data_ptr();
  a.o_t = out.stride(0);
  a.o_h = out.stride(1);
  a.T = q_lat.size(0);
  a.Hq = q_lat.size(1);
  a.splits = splits;
  a.scale = scale;
  if (splits > 1) {
    TORCH_CHECK(ws_o.has_value() && ws_lse.has_value() &&
                    ws_o->numel() >= splits * a.T * a.Hq * 512 && ws_lse->numel() >= splits * a.T * a.Hq,
                "mla_attention: split workspace too small");
    a.ws_o = ws_o->data_ptr<float>();
    a.ws_lse = ws_lse->data_ptr<float>();
  }
  a.dcp_size = (int)dcp_size;
  a.dcp_rank = (int)dcp_rank;
  if (lse_out.has_value()) {
    TORCH_CHECK(lse_out->scalar_type() == at::kFloat && lse_out->is_contiguous() &&
                    lse_out->numel() >= (int64_t)a.T * a.Hq,
                "mla_attention: lse_out [T, H] fp32");
    a.lse_out = lse_out->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard g(q_lat.device());
  guarded([&] { b200::mla::run_attention(a, stream_of(q_lat)); });
}

void indexer_k_prep(const Tensor& k, const Tensor& ln_w, const Tensor& ln_b, double eps,
                    const Tensor& positions, const Tensor& cos_sin, Tensor& cache,
                    const Tensor& slot_mapping) {
  CHECK_CUDA(k);
  CHECK_BF16(k);
  TORCH_CHECK(k.stride(1) == 1 && k.size(1) >= 128, "indexer_k_prep: k [T, 128]");
  TORCH_CHECK(cache.is_contiguous() && cache.size(-1) == 128, "indexer_k_prep: cache [..., 128]");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == 64, "indexer: cos_sin [P, 64]");
  const c10::cuda::CUDAGuard g(k.device());
  guarded([&] {
    b200::mla::run_indexer_k_prep(k.data_ptr(), k.stride(0), ln_w.data_ptr(), ln_b.data_ptr(), eps,
                                  positions.data_ptr<int32_t>(), cos_sin.data_ptr<float>(),
                                  cache.data_ptr(), slot_mapping.data_ptr<int32_t>(), k.size(0),
                                  stream_of(k));
  });
}

void indexer_scores(const Tensor& q, const Tensor& w, const Tensor& cache,
                    const Tensor& block_tables, const Tensor& cu_q, const Tensor& seq_lens,
                    Tensor& scores) {
  CHECK_CUDA(q);
  CHECK_BF16(q);
  TORCH_CHECK(q.stride(1) == 1 && q.size(1) >= 64 * 128, "indexer_scores: q [T, 64*128]");
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.stride(1) == 1 && w.size(1) >= 64,
              "indexer_scores: fp32 weights [T, 64]");
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.stride(1) == 1, "indexer_scores: fp32 out");
  TORCH_CHECK(cache.is_contiguous() && cache.size(-1) == 128, "indexer_scores: cache [..., 128]");
  b200::mla::IndexerArgs a{};
  a.q = q.data_ptr();
  a.ld_q = q.stride(0);
  a.w = w.data_ptr<float>();
  a.ld_w = w.stride(0);
  a.cache = cache.data_ptr();
  a.block_tables = block_tables.data_ptr<int32_t>();
  a.bt_stride = block_tables.stride(0);
  a.block_size = cache.dim() == 3 ? cache.size(1) : cache.size(-2);
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.R = seq_lens.size(0);
  a.T = q.size(0);
  a.scores = scores.data_ptr<float>();
  a.ld_s = scores.size(1);
  TORCH_CHECK(scores.stride(0) == scores.size(1), "indexer_scores: contiguous scores");
  const c10::cuda::CUDAGuard g(q.device());
  guarded([&] { b200::mla::run_indexer_scores(a, stream_of(q)); });
}

void mla_topk(const Tensor& scores, const Tensor& cu_q, const Tensor& seq_lens, Tensor& out) {
  CHECK_CUDA(scores);
  TORCH_CHECK(scores.scalar_type() == at::kFloat && scores.stride(1) == 1, "topk: fp32 scores");
  TORCH_CHECK(out.scalar_type() == at::kInt && out.stride(1) == 1, "topk: int32 out");
  const c10::cuda::CUDAGuard g(scores.device());
  guarded([&] {
    b200::mla::run_topk(scores.data_ptr<float>(), scores.stride(0), cu_q.data_ptr<int32_t>(),
                        seq_lens.data_ptr<int32_t>(), seq_lens.size(0), scores.size(0), out.size(1),
                        out.data_ptr<int32_t>(), out.stride(0), stream_of(scores));
  });
}

// ------------------------------------------------------------------------------------- attention
static const float* sink_ptr(const c10::optional<Tensor>& sinks, int64_t Hq) {
  if (!sinks.has_value()) return nullptr;
  TORCH_CHECK(sinks->scalar_type() == at::kFloat && sinks->is_contiguous() && sinks->numel() == Hq,
              "attention sinks: fp32 [num_q_heads]");
  return sinks->data_ptr<float>();
}

void paged_decode(const Tensor& q, Tensor& out, const Tensor& k_cache, const Tensor& v_cache,
                  const Tensor& block_tables, const Tensor& seq_lens, int64_t Hq, int64_t Hkv,
                  int64_t max_seq_len, double scale, int64_t num_splits,
                  const c10::optional<Tensor>& ws_o, const c10::optional<Tensor>& ws_lse,
                  const c10::optional<Tensor>& sinks) {
  CHECK_CUDA(q);
  CHECK_BF16(q);
  CHECK_ROWMAJOR(q);
  CHECK_ROWMAJOR(out);
  CHECK_BF16(k_cache);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4,
              "kv cache layout");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.stride(1) == 1, "block_tables");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.is_contiguous(), "seq_lens");
  const int D = k_cache.size(3);
  const int B = q.size(0);
  TORCH_CHECK(seq_lens.numel() >= B && block_tables.size(0) >= B, "decode: batch");
  TORCH_CHECK(q.size(1) >= Hq * D && out.size(1) >= Hq * D, "decode: widths");
  const c10::cuda::CUDAGuard g(q.device());
  b200::attn::DecodeArgs a{};
  a.q = q.data_ptr();
  a.ld_q = q.stride(0);
  a.o = out.data_ptr();
  a.ld_o = out.stride(0);
  a.k_cache = const_cast<void*>(k_cache.data_ptr());
  a.v_cache = const_cast<void*>(v_cache.data_ptr());
  a.num_blocks = k_cache.size(0);
  a.block_tables = block_tables.data_ptr<int32_t>();
  a.bt_stride = block_tables.stride(0);
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = D;
  a.block_size = k_cache.size(2);
  a.max_seq_len = max_seq_len;
  a.num_splits = num_splits;
  a.scale = scale;
  if (num_splits > 1) {
    TORCH_CHECK(ws_o.has_value() && ws_lse.has_value(), "decode: split workspace required");
    TORCH_CHECK(ws_o->numel() >= (int64_t)B * Hq * num_splits * D &&
                    ws_lse->numel() >= (int64_t)B * Hq * num_splits,
                "decode: split workspace too small");
    a.ws_o = ws_o->data_ptr<float>();
    a.ws_lse = ws_lse->data_ptr<float>();
  }
  a.sinks = sink_ptr(sinks, Hq);
  a.err = err_ptr(q);
  guarded([&] { b200::attn::run_decode(a, stream_of(q)); });
}

void paged_prefill(const Tensor& q, Tensor& out, const Tensor& k_cache, const Tensor& v_cache,
                   const Tensor& cu_q, const Tensor& seq_lens, const Tensor& block_tables,
                   Tensor& tile_offsets, int64_t Hq, int64_t Hkv, double scale, int64_t window,
                   const c10::optional<Tensor>& sinks, bool causal,
                   const c10::optional<Tensor>& tree_mask) {
  CHECK_CUDA(q);
  CHECK_BF16(q);
  CHECK_ROWMAJOR(q);
  CHECK_ROWMAJOR(out);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.dim() == 4,
              "kv cache layout");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  block_tables.scalar_type() == at::kInt && tile_offsets.scalar_type() == at::kInt,
              "prefill: int32 metadata");
  const int R = seq_lens.numel();
  TORCH_CHECK(cu_q.numel() >= R + 1 && tile_offsets.numel() >= R + 1, "prefill: metadata sizes");
  const c10::cuda::CUDAGuard g(q.device());
  b200::attn::PrefillArgs a{};
  a.q = q.data_ptr();
  a.ld_q = q.stride(0);
  a.o = out.data_ptr();
  a.ld_o = out.stride(0);
  a.k_cache = const_cast<void*>(k_cache.data_ptr());
  a.v_cache = const_cast<void*>(v_cache.data_ptr());
  a.num_blocks = k_cache.size(0);
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.block_tables = block_tables.data_ptr<int32_t>();
  a.bt_stride = block_tables.stride(0);
  a.tile_offsets = tile_offsets.data_ptr<int32_t>();
  a.T = q.size(0);
  a.R = R;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.D = k_cache.size(3);
  a.block_size = k_cache.size(2);
  a.window = window;
  a.scale = scale;
  a.sinks = sink_ptr(sinks, Hq);
  a.causal = causal;
  if (tree_mask.has_value()) {
    TORCH_CHECK(tree_mask->scalar_type() == at::kLong && tree_mask->is_contiguous() &&
                    tree_mask->numel() >= q.size(0) && causal,
                "tree attention: int64 mask per query row (causal mode)");
    a.tree_mask = reinterpret_cast<const uint64_t*>(tree_mask->data_ptr<int64_t>());
  }
  a.err = err_ptr(q);
  guarded([&] { b200::attn::run_prefill(a, stream_of(q)); });
}


// ---- TurboQuant KV cache ----
void tq_store(const Tensor& k, const Tensor& v, Tensor& cache, const Tensor& slot_mapping,
              int64_t key_bits, int64_t value_bits, bool norm_correction) {
  CHECK_CUDA(k);
  CHECK_BF16(k);
  CHECK_BF16(v);
  CHECK_ROWMAJOR(k);
  CHECK_ROWMAJOR(v);
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.is_contiguous() && cache.dim() == 4,
              "tq_store: cache must be contiguous uint8 [blocks, Hkv, block_size, slot]");
  TORCH_CHECK(slot_mapping.scalar_type() == at::kInt && slot_mapping.is_contiguous(),
              "tq_store: slot_mapping");
  const int T = k.size(0), Hkv = cache.size(1);
  TORCH_CHECK(v.size(0) == T && slot_mapping.numel() >= T, "tq_store: token count");
  TORCH_CHECK(k.size(1) % Hkv == 0, "tq_store: k width");
  const int D = k.size(1) / Hkv;
  TORCH_CHECK(v.size(1) >= Hkv * D, "tq_store: v width");
  c10::cuda::CUDAGuard g(k.device());
  b200::tq::TQStoreArgs a{};
  a.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  a.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  a.ld_k = k.stride(0);
  a.ld_v = v.stride(0);
  a.slot_mapping = slot_mapping.data_ptr<int>();
  a.cache = cache.data_ptr<uint8_t>();
  a.T = T;
  a.Hkv = Hkv;
  a.block_size = cache.size(2);
  a.num_blocks = cache.size(0);
  a.slot_bytes = cache.size(3);
  a.norm_correction = norm_correction;
  a.err = err_ptr(k);
  guarded([&] { b200::tq::run_store(a, D, key_bits, value_bits, stream_of(k)); });
}

void tq_decode(const Tensor& q, Tensor& out, const Tensor& cache, const Tensor& block_tables,
               const Tensor& seq_lens, int64_t Hq, int64_t head_dim, double scale,
               int64_t key_bits, int64_t value_bits, int64_t num_splits,
               const c10::optional<Tensor>& ws_o, const c10::optional<Tensor>& ws_lse) {
  CHECK_CUDA(q);
  CHECK_BF16(q);
  CHECK_BF16(out);
  CHECK_ROWMAJOR(q);
  CHECK_ROWMAJOR(out);
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.is_contiguous() && cache.dim() == 4,
              "tq_decode: cache");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.stride(1) == 1,
              "tq_decode: block_tables");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.is_contiguous(), "tq_decode: seq_lens");
  const int B = q.size(0), D = head_dim;
  TORCH_CHECK(seq_lens.numel() >= B && block_tables.size(0) >= B, "tq_decode: batch");
  TORCH_CHECK(q.size(1) >= Hq * D && out.size(1) >= Hq * D, "tq_decode: widths");
  c10::cuda::CUDAGuard g(q.device());
  b200::tq::TQDecodeArgs a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.ld_q = q.stride(0);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.ld_out = out.stride(0);
  a.cache = cache.data_ptr<uint8_t>();
  a.block_tables = block_tables.data_ptr<int>();
  a.ld_bt = block_tables.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.B = B;
  a.Hq = Hq;
  a.Hkv = cache.size(1);
  a.block_size = cache.size(2);
  a.num_blocks = cache.size(0);
  a.slot_bytes = cache.size(3);
  a.scale_log2 = float(scale * 1.4426950408889634);
  a.splits = num_splits;
  if (num_splits > 1) {
    TORCH_CHECK(ws_o.has_value() && ws_lse.has_value(), "tq_decode: split workspace");
    TORCH_CHECK(ws_o->scalar_type() == at::kFloat && ws_o->numel() >= int64_t(B) * Hq * num_splits * D,
                "tq_decode: ws_o too small");
    TORCH_CHECK(ws_lse->scalar_type() == at::kFloat && ws_lse->numel() >= int64_t(B) * Hq * num_splits,
                "tq_decode: ws_lse too small");
    a.ws_o = ws_o->data_ptr<float>();
    a.ws_lse = ws_lse->data_ptr<float>();
  }
  a.err = err_ptr(q);
  TORCH_CHECK(a.slot_bytes == b200::tq::slot_bytes(D, key_bits, value_bits), "tq_decode: slot size");
  guarded([&] { b200::tq::run_decode(a, D, key_bits, value_bits, stream_of(q)); });
}

void tq_dequant(const Tensor& cache, const Tensor& block_tables, const Tensor& seq_lens,
                Tensor& k_out, Tensor& v_out, int64_t head_dim, int64_t key_bits,
                int64_t value_bits) {
  CHECK_CUDA(cache);
  TORCH_CHECK(cache.scalar_type() == at::kByte && cache.is_contiguous() && cache.dim() == 4,
              "tq_dequant: cache");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && block_tables.stride(1) == 1,
              "tq_dequant: block_tables");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.is_contiguous(), "tq_dequant: seq_lens");
  CHECK_BF16(k_out);
  CHECK_BF16(v_out);
  const int R = block_tables.size(0), Hkv = cache.size(1), bs = cache.size(2), D = head_dim;
  TORCH_CHECK(k_out.is_contiguous() && v_out.is_contiguous() && k_out.dim() == 4 &&
                  k_out.size(0) % std::max(R, 1) == 0 && k_out.size(1) == Hkv &&
                  k_out.size(2) == bs && k_out.size(3) == D && v_out.sizes() == k_out.sizes(),
              "tq_dequant: outputs must be [R * W, Hkv, block_size, D]");
  c10::cuda::CUDAGuard g(cache.device());
  b200::tq::TQDequantArgs a{};
  a.cache = cache.data_ptr<uint8_t>();
  a.block_tables = block_tables.data_ptr<int>();
  a.ld_bt = block_tables.stride(0);
  a.seq_lens = seq_lens.data_ptr<int>();
  a.k_out = reinterpret_cast<__nv_bfloat16*>(k_out.data_ptr());
  a.v_out = reinterpret_cast<__nv_bfloat16*>(v_out.data_ptr());
  a.R = R;
  a.W = R ? k_out.size(0) / R : 0;
  TORCH_CHECK(a.W <= block_tables.size(1), "tq_dequant: more pages than block-table columns");
  a.Hkv = Hkv;
  a.block_size = bs;
  a.num_blocks = cache.size(0);
  a.slot_bytes = cache.size(3);
  a.err = err_ptr(cache);
  TORCH_CHECK(a.slot_bytes == b200::tq::slot_bytes(D, key_bits, value_bits), "tq_dequant: slot size");
  guarded([&] { b200::tq::run_dequant(a, D, key_bits, value_bits, stream_of(cache)); });
}

int64_t tq_slot_bytes(int64_t D, int64_t kb, int64_t vb) { return b200::tq::slot_bytes(D, kb, vb); }

int64_t decode_num_splits(int64_t B, int64_t Hkv, int64_t max_seq_len) {
  return b200::attn::decode_num_splits(B, Hkv, max_seq_len);
}

// ------------------------------------------------------------------------------------- sampling
void sample(const Tensor& logits, const c10::optional<Tensor>& temperature,
            const c10::optional<Tensor>& top_k, const c10::optional<Tensor>& top_p,
            const c10::optional<Tensor>& min_p, const c10::optional<Tensor>& seeds,
            const c10::optional<Tensor>& steps, int64_t vocab_offset, Tensor& out_idx,
            const c10::optional<Tensor>& out_val) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat, "sample: fp32 logits");
  CHECK_ROWMAJOR(logits);
  TORCH_CHECK(out_idx.scalar_type() == at::kLong && out_idx.numel() >= logits.size(0), "out_idx");
  const c10::cuda::CUDAGuard g(logits.device());
  b200::sampling::SampleArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.R = logits.size(0);
  a.V = logits.size(1);
  a.vocab_offset = vocab_offset;
  a.temperature = temperature.has_value() ? temperature->data_ptr<float>() : nullptr;
  a.top_k = top_k.has_value() ? top_k->data_ptr<int32_t>() : nullptr;
  a.top_p = top_p.has_value() ? top_p->data_ptr<float>() : nullptr;
  a.min_p = min_p.has_value() ? min_p->data_ptr<float>() : nullptr;
  a.seeds = seeds.has_value() ? seeds->data_ptr<int64_t>() : nullptr;
  a.steps = steps.has_value() ? steps->data_ptr<int32_t>() : nullptr;
  a.out_idx = out_idx.data_ptr<int64_t>();
  a.out_val = out_val.has_value() ? out_val->data_ptr<float>() : nullptr;
  guarded([&] { b200::sampling::run_sample(a, stream_of(logits)); });
}

void merge_candidates(const Tensor& vals, const Tensor& idx, Tensor& out) {
  CHECK_CUDA(vals);
  TORCH_CHECK(vals.scalar_type() == at::kFloat && idx.scalar_type() == at::kLong &&
                  vals.is_contiguous() && idx.is_contiguous() && vals.dim() == 2,
              "merge_candidates: [S, R] fp32 / int64");
  const c10::cuda::CUDAGuard g(vals.device());
  guarded([&] {
    b200::sampling::run_merge_candidates(vals.data_ptr<float>(), idx.data_ptr<int64_t>(),
                                         vals.size(0), vals.size(1), out.data_ptr<int64_t>(),
                                         stream_of(vals));
  });
}

void apply_penalties(Tensor& logits, const Tensor& entries, const Tensor& rep, const Tensor& pres,
                     const Tensor& freq, int64_t vocab_offset) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "apply_penalties: fp32 [R, V] logits");
  TORCH_CHECK(entries.scalar_type() == at::kInt && entries.is_contiguous() &&
                  entries.dim() == 2 && entries.size(1) == 3,
              "apply_penalties: int32 [n, 3] entries");
  for (const Tensor* t : {&rep, &pres, &freq})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() >= logits.size(0),
                "apply_penalties: fp32 per-row penalties");
  const c10::cuda::CUDAGuard g(logits.device());
  guarded([&] {
    b200::sampling::run_apply_penalties(logits.data_ptr<float>(), logits.stride(0),
                                        logits.size(1), vocab_offset, entries.data_ptr<int32_t>(),
                                        entries.size(0), rep.data_ptr<float>(),
                                        pres.data_ptr<float>(), freq.data_ptr<float>(),
                                        stream_of(logits));
  });
}

void apply_token_bitmask(Tensor& logits, const Tensor& bitmask, const Tensor& rows,
                         int64_t vocab_offset) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "apply_token_bitmask: fp32 [S, V] logits");
  TORCH_CHECK(bitmask.scalar_type() == at::kInt && bitmask.dim() == 2 && bitmask.is_contiguous(),
              "apply_token_bitmask: int32 [R, words] bitmask");
  TORCH_CHECK(rows.scalar_type() == at::kInt && rows.is_contiguous() &&
                  rows.numel() == bitmask.size(0),
              "apply_token_bitmask: int32 [R] logits rows");
  TORCH_CHECK(bitmask.device() == logits.device() && rows.device() == logits.device(),
              "apply_token_bitmask: tensors on the logits' device");
  const c10::cuda::CUDAGuard g(logits.device());
  guarded([&] {
    b200::sampling::run_token_bitmask(logits.data_ptr<float>(), logits.stride(0),
                                      bitmask.data_ptr<int32_t>(), bitmask.size(1),
                                      rows.data_ptr<int32_t>(), rows.numel(), logits.size(1),
                                      vocab_offset, stream_of(logits));
  });
}

// ------------------------------------------------------------------------------------- misc
void embedding(Tensor& out, const Tensor& table, const Tensor& ids, int64_t vocab_start) {
  CHECK_CUDA(table);
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && ids.scalar_type() == at::kInt &&
                  ids.is_contiguous(),
              "embedding: contiguous table/out, int32 ids");
  TORCH_CHECK(table.element_size() == 2, "embedding: 16-bit table");
  const c10::cuda::CUDAGuard g(table.device());
  guarded([&] {
    b200::misc::run_embedding(out.data_ptr(), table.data_ptr(), ids.data_ptr<int32_t>(),
                              ids.numel(), table.size(1), table.size(0), vocab_start,
                              stream_of(table));
  });
}

void gather_rows(Tensor& out, const Tensor& x, const Tensor& idx) {
  CHECK_CUDA(x);
  CHECK_ROWMAJOR(x);
  TORCH_CHECK(out.is_contiguous() && idx.scalar_type() == at::kInt && idx.is_contiguous(),
              "gather_rows: int32 idx");
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::misc::run_gather_rows(out.data_ptr(), x.data_ptr(), x.stride(0), idx.data_ptr<int32_t>(),
                                idx.numel(), x.size(1), x.element_size(), stream_of(x));
  });
}

Tensor error_word(const Tensor& like) { return error_word_for(like.device()); }

// ------------------------------------------------------------------------------------- GDN
void causal_conv1d(const Tensor& x, const Tensor& w, Tensor& state, const Tensor& cu_q,
                   const Tensor& seq_lens, const Tensor& slots, Tensor& out,
                   const c10::optional<Tensor>& bias) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_ROWMAJOR(x);
  CHECK_ROWMAJOR(out);
  TORCH_CHECK(w.is_contiguous() && w.dim() == 2 && w.size(1) == 4, "conv weight [C, 4]");
  TORCH_CHECK(state.is_contiguous() && state.dim() == 3 && state.size(2) == 3 &&
                  state.scalar_type() == at::kBFloat16,
              "conv state [slots, C, 3] bf16");
  const int C = w.size(0);
  TORCH_CHECK(state.size(1) == C && x.size(1) >= C && out.size(1) >= C, "conv widths");
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::gdn::run_causal_conv1d(x.data_ptr(), x.stride(0), w.data_ptr(), state.data_ptr(),
                                 cu_q.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(),
                                 slots.data_ptr<int32_t>(), seq_lens.numel(), x.size(0), C,
                                 out.data_ptr(), out.stride(0), stream_of(x),
                                 bias.has_value() ? bias->data_ptr() : nullptr);
  });
}

static b200::mamba::Mamba2Args mamba2_args(const Tensor& xbc, int64_t b_off, int64_t c_off,
                                           const Tensor& dt, const Tensor& dt_bias,
                                           const Tensor& A_log, const Tensor& D, Tensor& state,
                                           const Tensor& cu_q, const Tensor& seq_lens,
                                           const Tensor& slots, Tensor& y, int64_t H, int64_t G,
                                           int64_t P, int64_t N, double dt_min, double dt_max) {
  CHECK_CUDA(xbc);
  CHECK_BF16(xbc);
  CHECK_ROWMAJOR(xbc);
  CHECK_BF16(dt);
  CHECK_ROWMAJOR(dt);
  CHECK_BF16(y);
  CHECK_ROWMAJOR(y);
  for (const Tensor* t : {&dt_bias, &A_log, &D})
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == H,
                "mamba2: fp32 [H] dt_bias / A_log / D");
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.dim() == 4 &&
                  state.size(1) == H && state.size(2) == P && state.size(3) == N,
              "mamba2: state [slots, H, P, N] fp32");
  TORCH_CHECK(xbc.size(1) >= c_off + G * N && b_off >= H * P && dt.size(1) >= H &&
                  y.size(1) >= H * P && xbc.size(0) == y.size(0) && dt.size(0) == y.size(0),
              "mamba2: widths");
  TORCH_CHECK(cu_q.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt &&
                  slots.scalar_type() == at::kInt,
              "mamba2: int32 metadata");
  b200::mamba::Mamba2Args a{};
  a.xbc = xbc.data_ptr();
  a.ld_xbc = xbc.stride(0);
  a.b_off = b_off;
  a.c_off = c_off;
  a.dt = dt.data_ptr();
  a.ld_dt = dt.stride(0);
  a.dt_bias = dt_bias.data_ptr<float>();
  a.A_log = A_log.data_ptr<float>();
  a.D = D.data_ptr<float>();
  a.state = state.data_ptr<float>();
  a.cu_q = cu_q.data_ptr<int32_t>();
  a.seq_lens = seq_lens.data_ptr<int32_t>();
  a.slots = slots.data_ptr<int32_t>();
  a.y = y.data_ptr();
  a.ld_y = y.stride(0);
  a.R = seq_lens.numel();
  a.H = H;
  a.G = G;
  a.P = P;
  a.N = N;
  a.dt_min = dt_min;
  a.dt_max = dt_max;
  return a;
}

void mamba2_scan(const Tensor& xbc, int64_t b_off, int64_t c_off, const Tensor& dt,
                 const Tensor& dt_bias, const Tensor& A_log, const Tensor& D, Tensor& state,
                 const Tensor& cu_q, const Tensor& seq_lens, const Tensor& slots, Tensor& y,
                 int64_t H, int64_t G, int64_t P, int64_t N, double dt_min, double dt_max) {
  const c10::cuda::CUDAGuard g(xbc.device());
  const auto a = mamba2_args(xbc, b_off, c_off, dt, dt_bias, A_log, D, state, cu_q, seq_lens,
                             slots, y, H, G, P, N, dt_min, dt_max);
  guarded([&] { b200::mamba::run_mamba2_scan(a, stream_of(xbc)); });
}

// Chunked SSD prefill (csrc/scan/mamba2_chunked.cu): ``num_tokens`` = cu_q[R] - cu_q[0];
// workspaces chunk_offsets int32 [R+1], states fp32 and start_bf16 bf16 [max_chunks * H * P * N],
// decay fp32 [max_chunks * H] with max_chunks = ceil(num_tokens / 64) + R.
void mamba2_chunked(const Tensor& xbc, int64_t b_off, int64_t c_off, const Tensor& dt,
                    const Tensor& dt_bias, const Tensor& A_log, const Tensor& D, Tensor& state,
                    const Tensor& cu_q, const Tensor& seq_lens, const Tensor& slots, Tensor& y,
                    int64_t H, int64_t G, int64_t P, int64_t N, double dt_min, double dt_max,
                    Tensor& chunk_offsets, Tensor& states, Tensor& start_bf16, Tensor& decay,
                    int64_t num_tokens) {
  const c10::cuda::CUDAGuard g(xbc.device());
  const auto a = mamba2_args(xbc, b_off, c_off, dt, dt_bias, A_log, D, state, cu_q, seq_lens,
                             slots, y, H, G, P, N, dt_min, dt_max);
  const size_t mc = b200::mamba::mamba2_chunked_max_chunks((int)num_tokens, a.R);
  TORCH_CHECK(chunk_offsets.scalar_type() == at::kInt && chunk_offsets.numel() >= a.R + 1,
              "mamba2_chunked: chunk_offsets [R+1] int32");
  TORCH_CHECK(states.scalar_type() == at::kFloat && states.is_contiguous() &&
                  (size_t)states.numel() >= mc * H * P * N,
              "mamba2_chunked: states workspace too small");
  TORCH_CHECK(start_bf16.scalar_type() == at::kBFloat16 && start_bf16.is_contiguous() &&
                  (size_t)start_bf16.numel() >= mc * H * P * N &&
                  reinterpret_cast<uintptr_t>(start_bf16.data_ptr()) % 16 == 0,
              "mamba2_chunked: bf16 chunk-start state workspace");
  TORCH_CHECK(decay.scalar_type() == at::kFloat && (size_t)decay.numel() >= mc * H,
              "mamba2_chunked: decay workspace too small");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(xbc.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(states.data_ptr()) % 16 == 0,
              "mamba2_chunked: 16-byte aligned xbc / states");
  TORCH_CHECK(b200::mamba::mamba2_chunked_supported((int)P, (int)N, a.ld_xbc, a.b_off, a.c_off,
                                                    a.ld_y),
              "mamba2_chunked: head_dim 32/64, state 64/128, rows of multiples of 8 elements");
  guarded([&] {
    b200::mamba::run_mamba2_chunked(a, (int)num_tokens, chunk_offsets.data_ptr<int32_t>(),
                                    states.data_ptr<float>(), start_bf16.data_ptr(),
                                    decay.data_ptr<float>(),
                                    stream_of(xbc));
  });
}

void gated_rmsnorm(Tensor& out, const Tensor& y, const Tensor& z, const Tensor& w, int64_t group,
                   double eps) {
  CHECK_CUDA(y);
  CHECK_BF16(y);
  CHECK_BF16(z);
  CHECK_BF16(w);
  CHECK_ROWMAJOR(y);
  CHECK_ROWMAJOR(z);
  CHECK_ROWMAJOR(out);
  const int C = w.numel();
  TORCH_CHECK(y.size(1) >= C && z.size(1) >= C && out.size(1) >= C && w.is_contiguous(),
              "gated rmsnorm: widths");
  TORCH_CHECK((y.stride(0) * 2) % 16 == 0 && (z.stride(0) * 2) % 16 == 0 &&
                  (out.stride(0) * 2) % 16 == 0 && (z.storage_offset() * 2) % 16 == 0 &&
                  (y.storage_offset() * 2) % 16 == 0,
              "gated rmsnorm: 16-byte aligned rows");
  const c10::cuda::CUDAGuard g(y.device());
  guarded([&] {
    b200::mamba::run_gated_rmsnorm(out.data_ptr(), out.stride(0), y.data_ptr(), y.stride(0),
                                   z.data_ptr(), z.stride(0), w.data_ptr(), y.size(0), C, group,
                                   eps, stream_of(y));
  });
}

void gdn_chunked(const Tensor& qkv, const Tensor& ba, const Tensor& A_log, const Tensor& dt_bias,
                 Tensor& state, const Tensor& cu_q, const Tensor& seq_lens, const Tensor& slots,
                 int64_t Hk, int64_t Hv, Tensor& out, Tensor& ws, Tensor& chunk_offsets,
                 Tensor& gam_c) {
  CHECK_CUDA(qkv);
  CHECK_BF16(qkv);
  CHECK_ROWMAJOR(qkv);
  CHECK_ROWMAJOR(ba);
  CHECK_ROWMAJOR(out);
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.dim() == 4 &&
                  state.size(1) == Hv && state.size(2) == 128 && state.size(3) == 128,
              "gdn state [slots, Hv, 128, 128] fp32");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat,
              "A_log / dt_bias fp32");
  const int R = seq_lens.numel(), T = qkv.size(0);
  const int max_chunks = (T + 63) / 64 + R;
  TORCH_CHECK(ws.is_contiguous() &&
                  (size_t)ws.numel() * ws.element_size() >=
                      b200::gdn::chunked_workspace_bytes(max_chunks, Hv),
              "gdn_chunked: workspace too small");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ws.data_ptr()) % 16 == 0, "gdn_chunked: workspace alignment");
  TORCH_CHECK(chunk_offsets.scalar_type() == at::kInt && chunk_offsets.numel() >= R + 1,
              "gdn_chunked: chunk_offsets [R+1] int32");
  TORCH_CHECK(gam_c.scalar_type() == at::kFloat && gam_c.numel() >= (int64_t)max_chunks * Hv,
              "gdn_chunked: gam_c too small");
  const c10::cuda::CUDAGuard g(qkv.device());
  guarded([&] {
    b200::gdn::run_gdn_chunked(qkv.data_ptr(), qkv.stride(0), ba.data_ptr(), ba.stride(0),
                               A_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
                               state.data_ptr<float>(), cu_q.data_ptr<int32_t>(),
                               seq_lens.data_ptr<int32_t>(), slots.data_ptr<int32_t>(),
                               chunk_offsets.data_ptr<int32_t>(), ws.data_ptr(),
                               gam_c.data_ptr<float>(), R, T, Hk, Hv, out.data_ptr(),
                               out.stride(0), stream_of(qkv));
  });
}

void gdn_recurrent(const Tensor& qkv, const Tensor& ba, const Tensor& A_log, const Tensor& dt_bias,
                   Tensor& state, const Tensor& cu_q, const Tensor& seq_lens, const Tensor& slots,
                   int64_t Hk, int64_t Hv, Tensor& out, bool single_token) {
  CHECK_CUDA(qkv);
  CHECK_BF16(qkv);
  CHECK_ROWMAJOR(qkv);
  CHECK_ROWMAJOR(ba);
  CHECK_ROWMAJOR(out);
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.is_contiguous() && state.dim() == 4 &&
                  state.size(1) == Hv && state.size(2) == 128 && state.size(3) == 128,
              "gdn state [slots, Hv, 128, 128] fp32");
  TORCH_CHECK(A_log.scalar_type() == at::kFloat && dt_bias.scalar_type() == at::kFloat,
              "A_log / dt_bias fp32");
  const c10::cuda::CUDAGuard g(qkv.device());
  guarded([&] {
    b200::gdn::run_gdn_recurrent(qkv.data_ptr(), qkv.stride(0), ba.data_ptr(), ba.stride(0),
                                 A_log.data_ptr<float>(), dt_bias.data_ptr<float>(),
                                 state.data_ptr<float>(), cu_q.data_ptr<int32_t>(),
                                 seq_lens.data_ptr<int32_t>(), slots.data_ptr<int32_t>(),
                                 seq_lens.numel(), Hk, Hv, out.data_ptr(), out.stride(0),
                                 stream_of(qkv), single_token);
  });
}

void sigmoid_gate(Tensor& out, const Tensor& gate) {
  CHECK_CUDA(out);
  CHECK_ROWMAJOR(out);
  CHECK_ROWMAJOR(gate);
  const c10::cuda::CUDAGuard g(out.device());
  guarded([&] {
    b200::gdn::run_sigmoid_gate(out.data_ptr(), out.stride(0), gate.data_ptr(), gate.stride(0),
                                out.size(0), out.size(1), stream_of(out));
  });
}

// ------------------------------------------------------------------------------------- MoE
void gemm_grouped_bf16(const Tensor& A, const Tensor& B, Tensor& C, const Tensor& tile_expert,
                       const Tensor& num_tiles, int64_t num_experts, int64_t mode, int64_t bn) {
  CHECK_CUDA(A);
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_ROWMAJOR(A);
  CHECK_ROWMAJOR(B);
  CHECK_ROWMAJOR(C);
  TORCH_CHECK(B.size(0) % num_experts == 0, "grouped gemm: B rows must be E * N");
  const int N = B.size(0) / num_experts;
  TORCH_CHECK(A.size(1) == B.size(1), "grouped gemm: K mismatch");
  TORCH_CHECK(C.size(0) == A.size(0) && C.size(1) == (mode == 1 ? N / 2 : N), "grouped gemm: C");
  TORCH_CHECK(tile_expert.scalar_type() == at::kInt && num_tiles.scalar_type() == at::kInt,
              "grouped gemm: int32 tile metadata");
  const c10::cuda::CUDAGuard g(A.device());
  b200::gemm::GroupedGemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.max_rows = A.size(0);
  a.N = N;
  a.K = A.size(1);
  a.num_experts = num_experts;
  a.mode = mode;
  a.bn = bn;
  a.tile_expert = tile_expert.data_ptr<int32_t>();
  a.num_tiles = num_tiles.data_ptr<int32_t>();
  a.err = err_ptr(A);
  guarded([&] { b200::gemm::run_grouped_bf16(a, stream_of(A)); });
}

void w4_dequant(Tensor& out, const Tensor& packed, const Tensor& scales,
                const c10::optional<Tensor>& offsets) {
  CHECK_CUDA(packed);
  TORCH_CHECK(packed.dim() == 3 && packed.is_contiguous() && packed.scalar_type() == at::kChar,
              "w4_dequant: packed int4 [E, N, K/2] int8");
  const int E = packed.size(0), N = packed.size(1), K = packed.size(2) * 2;
  TORCH_CHECK(K % 128 == 0, "w4_dequant: K must be a multiple of 128");
  TORCH_CHECK(scales.is_contiguous() && scales.scalar_type() == at::kBFloat16 &&
                  scales.numel() == (int64_t)E * N * (K / 128),
              "w4_dequant: bf16 scales [E, N, K/128]");
  CHECK_BF16(out);
  TORCH_CHECK(out.is_contiguous() && out.numel() == (int64_t)E * N * K, "w4_dequant: out [E*N, K]");
  if (offsets.has_value())
    TORCH_CHECK(offsets->scalar_type() == at::kInt && offsets->numel() >= E + 1,
                "w4_dequant: int32 offsets [E + 1]");
  const c10::cuda::CUDAGuard g(packed.device());
  guarded([&] {
    b200::w4a8::run_w4_dequant(out.data_ptr(), packed.data_ptr(), scales.data_ptr(),
                               offsets.has_value() ? offsets->data_ptr<int32_t>() : nullptr, E, N,
                               K, stream_of(packed));
  });
}

void row_fp8_qdq(Tensor& out, const Tensor& x, bool swiglu, double limit,
                 const c10::optional<Tensor>& num_tiles) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_ROWMAJOR(x);
  CHECK_BF16(out);
  TORCH_CHECK(out.is_contiguous(), "row_fp8_qdq: contiguous out");
  const int C = out.size(1);
  TORCH_CHECK(C % 8 == 0 && x.size(1) == (swiglu ? 2 * C : C) && x.size(0) == out.size(0),
              "row_fp8_qdq: shapes");
  TORCH_CHECK((int64_t)C * 4 <= 200 * 1024, "row_fp8_qdq: row too long");
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::w4a8::run_row_fp8_qdq(out.data_ptr(), x.data_ptr(), x.stride(0), x.size(0), C, swiglu,
                                (float)limit,
                                num_tiles.has_value() ? num_tiles->data_ptr<int32_t>() : nullptr,
                                stream_of(x));
  });
}

void topk_softmax(const Tensor& logits, Tensor& ids, Tensor& w, bool renorm) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(1) == 1, "router logits fp32");
  TORCH_CHECK(ids.scalar_type() == at::kInt && w.scalar_type() == at::kFloat, "ids/w dtypes");
  const c10::cuda::CUDAGuard g(logits.device());
  guarded([&] {
    b200::moe::run_topk_softmax(logits.data_ptr<float>(), logits.stride(0), logits.size(0),
                                logits.size(1), ids.size(1), renorm, ids.data_ptr<int32_t>(),
                                w.data_ptr<float>(), stream_of(logits));
  });
}

void grouped_topk(const Tensor& logits, const c10::optional<Tensor>& bias, Tensor& ids, Tensor& w,
                  int64_t n_group, int64_t topk_group, bool sigmoid, bool renorm, double scale) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.is_contiguous(), "router logits fp32");
  const c10::cuda::CUDAGuard g(logits.device());
  guarded([&] {
    b200::moe::run_grouped_topk(logits.data_ptr<float>(),
                                bias.has_value() ? bias->data_ptr<float>() : nullptr,
                                logits.size(0), logits.size(1), ids.size(1), n_group, topk_group,
                                sigmoid, renorm, scale, ids.data_ptr<int32_t>(),
                                w.data_ptr<float>(), stream_of(logits));
  });
}

void moe_align(const Tensor& ids, int64_t E, Tensor& sorted_ids, Tensor& tile_expert,
               Tensor& offsets, Tensor& pos, Tensor& num_tiles, int64_t expert_offset) {
  CHECK_CUDA(ids);
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous(), "moe_align: int32 ids");
  const c10::cuda::CUDAGuard g(ids.device());
  guarded([&] {
    b200::moe::run_moe_align(ids.data_ptr<int32_t>(), ids.numel(), E, expert_offset,
                             sorted_ids.numel(),
                             sorted_ids.data_ptr<int32_t>(), tile_expert.data_ptr<int32_t>(),
                             offsets.data_ptr<int32_t>(), pos.data_ptr<int32_t>(),
                             num_tiles.data_ptr<int32_t>(), stream_of(ids));
  });
}

void moe_gather(const Tensor& x, const Tensor& sorted_ids, const Tensor& num_tiles, int64_t k,
                Tensor& out) {
  CHECK_CUDA(x);
  CHECK_ROWMAJOR(x);
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::moe::run_moe_gather(x.data_ptr(), x.stride(0), sorted_ids.data_ptr<int32_t>(),
                              num_tiles.data_ptr<int32_t>(), out.size(0), k, x.size(1),
                              out.data_ptr(), stream_of(x));
  });
}

void moe_combine(const Tensor& y, const Tensor& pos, const Tensor& w,
                 const c10::optional<Tensor>& shared, Tensor& out,
                 const c10::optional<Tensor>& shared_gate) {
  CHECK_CUDA(y);
  TORCH_CHECK(y.is_contiguous() && pos.is_contiguous() && w.is_contiguous(), "moe_combine");
  CHECK_ROWMAJOR(out);
  if (shared.has_value()) TORCH_CHECK(shared->is_contiguous(), "moe_combine: shared contiguous");
  if (shared_gate.has_value())
    TORCH_CHECK(shared_gate->scalar_type() == at::kFloat && shared.has_value(),
                "moe_combine: fp32 shared gate needs a shared output");
  const c10::cuda::CUDAGuard g(y.device());
  guarded([&] {
    b200::moe::run_moe_combine(y.data_ptr(), pos.data_ptr<int32_t>(), w.data_ptr<float>(),
                               pos.size(0), pos.size(1), y.size(1),
                               shared.has_value() ? shared->data_ptr() : nullptr,
                               shared_gate.has_value() ? shared_gate->data_ptr<float>() : nullptr,
                               shared_gate.has_value() ? shared_gate->stride(0) : 0,
                               out.data_ptr(), out.stride(0), stream_of(y));
  });
}

void moe_gemv(const Tensor& x, const Tensor& ids, int64_t E, int64_t expert_offset,
              const Tensor& w_gu, const Tensor& w_down, Tensor& h, Tensor& y, Tensor& pos) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_ROWMAJOR(x);
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && ids.dim() == 2,
              "moe_gemv: int32 ids [T, k]");
  const int64_t T = ids.size(0), k = ids.size(1), H = x.size(1);
  TORCH_CHECK(x.size(0) == T, "moe_gemv: x rows");
  TORCH_CHECK(w_gu.is_contiguous() && w_down.is_contiguous() && w_gu.size(1) == H &&
                  w_gu.size(0) % (2 * E) == 0,
              "moe_gemv: w_gu [E * 2I, H], w_down [E * H, I]");
  const int64_t I = w_gu.size(0) / E / 2;
  TORCH_CHECK(w_down.size(0) == E * H && w_down.size(1) == I, "moe_gemv: w_down [E * H, I]");
  TORCH_CHECK(h.is_contiguous() && h.numel() >= T * k * I && y.is_contiguous() &&
                  y.numel() >= T * k * H && pos.scalar_type() == at::kInt &&
                  pos.is_contiguous() && pos.numel() >= T * k,
              "moe_gemv: h [T*k, I], y [T*k, H], pos [T, k] int32");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(w_gu.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(w_down.data_ptr()) % 16 == 0 &&
                  reinterpret_cast<uintptr_t>(h.data_ptr()) % 16 == 0,
              "moe_gemv: 16-byte aligned operands");
  TORCH_CHECK(b200::moe::moe_gemv_supported((int)H, (int)I), "moe_gemv: H, I % 32");
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] {
    b200::moe::run_moe_gemv(x.data_ptr(), x.stride(0), ids.data_ptr<int32_t>(), (int)T, (int)k,
                            (int)E, (int)expert_offset, w_gu.data_ptr(), w_down.data_ptr(),
                            (int)H, (int)I, h.data_ptr(), y.data_ptr(), pos.data_ptr<int32_t>(),
                            stream_of(x));
  });
}

// ------------------------------------------------------------------------------------- comm
// Fused all-reduce: `bufs` holds per-rank device addresses as int64:
//   [0:W) staging slot, [W:2W) output slot, [2W:3W) flag region (this call's parity).
void fused_allreduce(const Tensor& like, const std::vector<int64_t>& bufs, int64_t epochs_ptr,
                     int64_t rank, int64_t world, int64_t T, int64_t H, int64_t blocks,
                     int64_t parity, bool two_shot, const c10::optional<Tensor>& residual,
                     const c10::optional<Tensor>& weight, double eps, int64_t rs_rows,
                     bool end_barrier) {
  TORCH_CHECK((int64_t)bufs.size() == 3 * world, "fused_allreduce: buffer table size");
  const c10::cuda::CUDAGuard g(like.device());
  b200::comm::ArParams a{};
  a.rank = rank;
  a.world = world;
  a.T = T;
  a.H = H;
  a.blocks = blocks;
  a.parity = parity;
  a.two_shot = two_shot;
  for (int p = 0; p < world; ++p) {
    a.staging[p] = reinterpret_cast<const void*>(bufs[p]);
    a.out[p] = reinterpret_cast<void*>(bufs[world + p]);
    a.flags[p] = reinterpret_cast<uint32_t*>(bufs[2 * world + p]);
  }
  a.epochs = reinterpret_cast<uint32_t*>(epochs_ptr);
  if (residual.has_value()) {
    TORCH_CHECK(residual->is_contiguous() && residual->scalar_type() == at::kBFloat16 &&
                    residual->size(0) >= T && residual->size(1) == H,
                "fused_allreduce: residual");
    a.residual = residual->data_ptr();
  }
  if (weight.has_value()) {
    TORCH_CHECK(weight->numel() == H && weight->scalar_type() == at::kBFloat16, "weight");
    a.weight = weight->data_ptr();
  }
  a.eps = eps;
  a.rs_rows = rs_rows;
  a.end_barrier = end_barrier;
  a.err = err_ptr(like);
  guarded([&] { b200::comm::run_fused_allreduce(a, stream_of(like)); });
}

// NVLS fused all-reduce.  `ptrs` = [mc_staging, mc_out, out_local, mc_flags, flags, epochs,
// mc_q, q_local, mc_s, s_local] (0 = absent).
void nvls_allreduce(const Tensor& like, const std::vector<int64_t>& ptrs, int64_t rank,
                    int64_t world, int64_t T, int64_t H, bool two_shot,
                    const c10::optional<Tensor>& residual, const c10::optional<Tensor>& weight,
                    double eps, int64_t rows_per_warp) {
  TORCH_CHECK(ptrs.size() == 10, "nvls_allreduce: pointer table size");
  const c10::cuda::CUDAGuard g(like.device());
  b200::comm::NvlsParams a{};
  a.rank = rank;
  a.world = world;
  a.T = T;
  a.H = H;
  a.two_shot = two_shot;
  a.blocks = b200::comm::nvls_blocks(T, world, two_shot, (int)rows_per_warp);
  a.mc_staging = reinterpret_cast<const void*>(ptrs[0]);
  a.mc_out = reinterpret_cast<void*>(ptrs[1]);
  a.out_local = reinterpret_cast<void*>(ptrs[2]);
  a.mc_flags = reinterpret_cast<uint32_t*>(ptrs[3]);
  a.flags = reinterpret_cast<uint32_t*>(ptrs[4]);
  a.epochs = reinterpret_cast<uint32_t*>(ptrs[5]);
  a.mc_q = reinterpret_cast<void*>(ptrs[6]);
  a.q_local = reinterpret_cast<void*>(ptrs[7]);
  a.mc_s = reinterpret_cast<float*>(ptrs[8]);
  a.s_local = reinterpret_cast<float*>(ptrs[9]);
  if (residual.has_value()) {
    TORCH_CHECK(residual->is_contiguous() && residual->scalar_type() == at::kBFloat16 &&
                    residual->size(0) >= T && residual->size(1) == H,
                "nvls_allreduce: residual");
    a.residual = residual->data_ptr();
  }
  if (weight.has_value()) {
    TORCH_CHECK(weight->numel() == H && weight->scalar_type() == at::kBFloat16, "weight");
    a.weight = weight->data_ptr();
  }
  a.eps = eps;
  a.err = err_ptr(like);
  guarded([&] { b200::comm::run_nvls_allreduce(a, stream_of(like)); });
}

// Expert-parallel all-to-all: `ints` = [rank, world, Tc, row0, H, k, E_local, cap, rs_rows];
// `ptrs` = [send_cnt, epoch, then per rank (world entries each): recv_x, recv_ids, recv_w,
// recv_tok, recv_cnt, flags, staging].
static b200::ep::A2AParams a2a_params(const Tensor& like, const std::vector<int64_t>& ints,
                                      const std::vector<int64_t>& ptrs) {
  TORCH_CHECK(ints.size() == 9, "ep a2a: 9 integer parameters");
  b200::ep::A2AParams p{};
  p.rank = ints[0];
  p.world = ints[1];
  p.Tc = ints[2];
  p.row0 = ints[3];
  p.H = ints[4];
  p.k = ints[5];
  p.E_local = ints[6];
  p.cap = ints[7];
  p.rs_rows = ints[8];
  TORCH_CHECK(p.world >= 1 && p.world <= 8 && (int64_t)ptrs.size() == 2 + 7 * p.world,
              "ep a2a: pointer table size");
  p.send_cnt = reinterpret_cast<int*>(ptrs[0]);
  p.epoch = reinterpret_cast<uint32_t*>(ptrs[1]);
  for (int r = 0; r < p.world; ++r) {
    p.recv_x[r] = reinterpret_cast<void*>(ptrs[2 + r]);
    p.recv_ids[r] = reinterpret_cast<int32_t*>(ptrs[2 + p.world + r]);
    p.recv_w[r] = reinterpret_cast<float*>(ptrs[2 + 2 * p.world + r]);
    p.recv_tok[r] = reinterpret_cast<int32_t*>(ptrs[2 + 3 * p.world + r]);
    p.recv_cnt[r] = reinterpret_cast<int32_t*>(ptrs[2 + 4 * p.world + r]);
    p.flags[r] = reinterpret_cast<uint32_t*>(ptrs[2 + 5 * p.world + r]);
    p.staging[r] = reinterpret_cast<void*>(ptrs[2 + 6 * p.world + r]);
  }
  p.err = err_ptr(like);
  return p;
}

void ep_dispatch(const Tensor& x, const Tensor& ids, const Tensor& w,
                 const std::vector<int64_t>& ints, const std::vector<int64_t>& ptrs) {
  CHECK_CUDA(x);
  CHECK_BF16(x);
  TORCH_CHECK(x.stride(1) == 1, "ep_dispatch: row-major x");
  TORCH_CHECK(ids.scalar_type() == at::kInt && ids.is_contiguous() && w.scalar_type() == at::kFloat &&
                  w.is_contiguous(),
              "ep_dispatch: int32 ids / fp32 weights [Tc, k]");
  auto p = a2a_params(x, ints, ptrs);
  TORCH_CHECK(ids.size(0) >= p.Tc && ids.size(1) == p.k && x.size(1) == p.H, "ep_dispatch: shapes");
  p.x = x.data_ptr();
  p.ldx = x.stride(0);
  p.ids = ids.data_ptr<int32_t>();
  p.w = w.data_ptr<float>();
  const c10::cuda::CUDAGuard g(x.device());
  guarded([&] { b200::ep::run_dispatch(p, stream_of(x)); });
}

void ep_return(const Tensor& y, const Tensor& pos, const std::vector<int64_t>& ints,
               const std::vector<int64_t>& ptrs) {
  CHECK_CUDA(y);
  CHECK_BF16(y);
  TORCH_CHECK(y.is_contiguous() && pos.scalar_type() == at::kInt && pos.is_contiguous(),
              "ep_return: contiguous y, int32 pos");
  auto p = a2a_params(y, ints, ptrs);
  TORCH_CHECK(y.size(1) == p.H && pos.size(0) == (int64_t)p.world * p.cap && pos.size(1) == p.k,
              "ep_return: shapes");
  const c10::cuda::CUDAGuard g(y.device());
  guarded([&] { b200::ep::run_return(p, y.data_ptr(), pos.data_ptr<int32_t>(), stream_of(y)); });
}

// Vocab-parallel sampling: exchange per-row candidates over NVLink and merge.
// ptrs = [vals of every rank (world), ids of every rank (world), flags of every rank (world)]
void exchange_candidates(const Tensor& vals, const Tensor& ids, Tensor& out,
                         const std::vector<int64_t>& ptrs, int64_t epochs_ptr, int64_t rank,
                         int64_t world, int64_t parity) {
  CHECK_CUDA(vals);
  TORCH_CHECK(vals.scalar_type() == at::kFloat && ids.scalar_type() == at::kLong &&
                  out.scalar_type() == at::kLong && vals.is_contiguous() && ids.is_contiguous(),
              "exchange_candidates: fp32 scores, int64 ids");
  TORCH_CHECK((int64_t)ptrs.size() == 3 * world, "exchange_candidates: pointer table");
  b200::comm::CandParams a{};
  a.rank = rank;
  a.world = world;
  a.R = vals.size(0);
  a.parity = parity;
  for (int p = 0; p < world; ++p) {
    a.vals[p] = reinterpret_cast<float*>(ptrs[p]);
    a.ids[p] = reinterpret_cast<int64_t*>(ptrs[world + p]);
    a.flags[p] = reinterpret_cast<uint32_t*>(ptrs[2 * world + p]);
  }
  a.epochs = reinterpret_cast<uint32_t*>(epochs_ptr);
  a.my_vals = vals.data_ptr<float>();
  a.my_ids = ids.data_ptr<int64_t>();
  a.out = out.data_ptr<int64_t>();
  a.err = err_ptr(vals);
  const c10::cuda::CUDAGuard g(vals.device());
  guarded([&] { b200::comm::run_exchange_candidates(a, stream_of(vals)); });
}

// ---- vocab-parallel top-k / top-p: per-shard candidate rows, local merge, NVLink exchange
static const float* opt_f32(const c10::optional<Tensor>& t) {
  return t.has_value() ? t->data_ptr<float>() : nullptr;
}
static const int32_t* opt_i32(const c10::optional<Tensor>& t) {
  return t.has_value() ? t->data_ptr<int32_t>() : nullptr;
}
static const int64_t* opt_i64(const c10::optional<Tensor>& t) {
  return t.has_value() ? t->data_ptr<int64_t>() : nullptr;
}

int64_t cand_row_bytes() { return (int64_t)sizeof(b200::sampling::CandRow); }

void shard_candidates(const Tensor& logits, const c10::optional<Tensor>& temperature,
                      const c10::optional<Tensor>& seeds, const c10::optional<Tensor>& steps,
                      int64_t vocab_offset, Tensor& out) {
  CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2 && logits.stride(1) == 1,
              "shard_candidates: fp32 [R, V] logits");
  TORCH_CHECK(out.is_contiguous() &&
                  out.numel() * out.element_size() >=
                      logits.size(0) * (int64_t)sizeof(b200::sampling::CandRow) &&
                  reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "shard_candidates: output rows");
  const c10::cuda::CUDAGuard g(logits.device());
  guarded([&] {
    b200::sampling::run_shard_candidates(
        logits.data_ptr<float>(), logits.stride(0), logits.size(0), logits.size(1), vocab_offset,
        opt_f32(temperature), opt_i64(seeds), opt_i32(steps),
        reinterpret_cast<b200::sampling::CandRow*>(out.data_ptr()), stream_of(logits));
  });
}

void merge_candidates_local(const Tensor& cands, int64_t world, int64_t R,
                            const c10::optional<Tensor>& temperature,
                            const c10::optional<Tensor>& top_k, const c10::optional<Tensor>& top_p,
                            const c10::optional<Tensor>& min_p, const c10::optional<Tensor>& seeds,
                            const c10::optional<Tensor>& steps, int64_t V_total, Tensor& out) {
  CHECK_CUDA(cands);
  TORCH_CHECK(cands.numel() * cands.element_size() >=
                  world * R * (int64_t)sizeof(b200::sampling::CandRow) &&
                  out.scalar_type() == at::kLong && out.numel() >= R,
              "merge_candidates_local: shapes");
  const c10::cuda::CUDAGuard g(cands.device());
  guarded([&] {
    b200::sampling::run_merge_candidates_local(
        reinterpret_cast<const b200::sampling::CandRow*>(cands.data_ptr()), world, R,
        opt_f32(temperature), opt_i32(top_k), opt_f32(top_p), opt_f32(min_p), opt_i64(seeds),
        opt_i32(steps), V_total, out.data_ptr<int64_t>(), stream_of(cands));
  });
}

// ptrs = [candidate region of every rank (world), flag region of every rank (world)]
void topk_exchange(const Tensor& mine, const std::vector<int64_t>& ptrs, int64_t epochs_ptr,
                   int64_t rank, int64_t world, int64_t parity, int64_t V_total,
                   const c10::optional<Tensor>& temperature, const c10::optional<Tensor>& top_k,
                   const c10::optional<Tensor>& top_p, const c10::optional<Tensor>& min_p,
                   const c10::optional<Tensor>& seeds, const c10::optional<Tensor>& steps,
                   Tensor& out) {
  CHECK_CUDA(mine);
  TORCH_CHECK((int64_t)ptrs.size() == 2 * world && world <= 8, "topk_exchange: pointer table");
  TORCH_CHECK(out.scalar_type() == at::kLong, "topk_exchange: int64 out");
  b200::sampling::TopkExchangeArgs a{};
  a.rank = rank;
  a.world = world;
  a.R = out.size(0);
  a.parity = parity;
  a.V_total = V_total;
  a.mine = reinterpret_cast<const b200::sampling::CandRow*>(mine.data_ptr());
  for (int p = 0; p < world; ++p) {
    a.region[p] = reinterpret_cast<b200::sampling::CandRow*>(ptrs[p]);
    a.flags[p] = reinterpret_cast<uint32_t*>(ptrs[world + p]);
  }
  a.epochs = reinterpret_cast<uint32_t*>(epochs_ptr);
  a.temperature = opt_f32(temperature);
  a.top_k = opt_i32(top_k);
  a.top_p = opt_f32(top_p);
  a.min_p = opt_f32(min_p);
  a.seeds = opt_i64(seeds);
  a.steps = opt_i32(steps);
  a.out = out.data_ptr<int64_t>();
  a.err = err_ptr(mine);
  const c10::cuda::CUDAGuard g(mine.device());
  guarded([&] { b200::sampling::run_topk_exchange(a, stream_of(mine)); });
}

// Row-parallel GEMM whose epilogue performs the reduce-scatter: C rows go to their owner
// rank's receive slot (`recv` = every rank's slot address, peers included).
void gemm_bf16_rs(const Tensor& A, const Tensor& B, const std::vector<int64_t>& recv,
                  int64_t rs_rows, int64_t rank, int64_t bn, int64_t splits, int64_t mt,
                  const c10::optional<Tensor>& workspace, const c10::optional<Tensor>& counters) {
  CHECK_CUDA(A);
  CHECK_BF16(A);
  CHECK_BF16(B);
  CHECK_ROWMAJOR(A);
  CHECK_ROWMAJOR(B);
  TORCH_CHECK(A.size(1) == B.size(1), "gemm_bf16_rs: K mismatch");
  TORCH_CHECK(recv.size() >= 1 && recv.size() <= 8, "gemm_bf16_rs: 1..8 ranks");
  const c10::cuda::CUDAGuard g(A.device());
  b200::gemm::GemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.C = reinterpret_cast<void*>(recv[rank]);
  a.ldc = B.size(0);
  a.M = A.size(0);
  a.N = B.size(0);
  a.K = A.size(1);
  a.mode = b200::gemm::kModeScatter;
  a.bn = bn;
  a.splits = splits;
  a.mt = mt;
  for (size_t i = 0; i < recv.size(); ++i) a.peers[i] = reinterpret_cast<void*>(recv[i]);
  a.rs_rows = rs_rows;
  a.rs_rank = rank;
  a.rs_world = recv.size();
  if (workspace.has_value()) {
    a.workspace = workspace->data_ptr<float>();
    a.workspace_numel = workspace->numel();
  }
  if (counters.has_value()) {
    a.counters = counters->data_ptr<int>();
    a.counters_numel = counters->numel();
  }
  a.err = err_ptr(A);
  guarded([&] { b200::gemm::run_bf16(a, stream_of(A)); });
}

}  // namespace

TORCH_LIBRARY(b200, m) {
  m.def(
      "gemm_bf16(Tensor A, Tensor B, Tensor(a!) C, int mode=0, int bn=0, int splits=0, "
      "Tensor? workspace=None, int mt=0, Tensor(b!)? counters=None) -> ()");
  m.def("rms_norm(Tensor(a!) out, Tensor x, Tensor weight, float eps, bool gemma=False) -> ()");
  m.def(
      "tq_store(Tensor k, Tensor v, Tensor(a!) cache, Tensor slot_mapping, int key_bits, "
      "int value_bits, bool norm_correction) -> ()");
  m.def(
      "tq_decode(Tensor q, Tensor(a!) out, Tensor cache, Tensor block_tables, Tensor seq_lens, "
      "int Hq, int head_dim, float scale, int key_bits, int value_bits, int num_splits, "
      "Tensor(b!)? ws_o, Tensor(c!)? ws_lse) -> ()");
  m.def(
      "tq_dequant(Tensor cache, Tensor block_tables, Tensor seq_lens, Tensor(a!) k_out, "
      "Tensor(b!) v_out, int head_dim, int key_bits, int value_bits) -> ()");
  m.def(
      "fused_add_rms_norm(Tensor(a!) x, Tensor(b!) residual, Tensor weight, float eps, "
      "bool gemma=False) -> ()");
  m.def(
      "rms_norm_quant_fp8(Tensor(a!) q, Tensor(b!) scales, Tensor(c!)? out, Tensor(d!) x, "
      "Tensor(e!)? residual, Tensor weight, float eps) -> ()");
  m.def(
      "rms_norm_gated(Tensor(a!) out, Tensor x, Tensor z, Tensor weight, int group, float eps) -> ()");
  m.def("act_and_mul(Tensor(a!) out, Tensor x, int kind=0, float limit=0.0) -> ()");
  m.def("silu_mul_fp8_quant(Tensor(a!) out, Tensor(b!) scales, Tensor x, float limit=0.0) -> ()");
  m.def("group_quant_fp8(Tensor(a!) out, Tensor(b!) scales, Tensor x) -> ()");
  m.def(
      "kv_insert(Tensor key, Tensor value, Tensor(a!) k_cache, Tensor(b!) v_cache, "
      "Tensor slot_mapping) -> ()");
  m.def(
      "rope_kv(Tensor(a!) qkv, Tensor positions, Tensor cos_sin, Tensor? q_norm_w, Tensor? "
      "k_norm_w, Tensor(b!)? k_cache, Tensor(c!)? v_cache, Tensor slot_mapping, int num_q_heads, "
      "int num_kv_heads, int rot_dim, bool neox=True, float eps=1e-6, int head_dim=0, "
      "int[]? mrope_section=None, bool mrope_interleaved=False) -> ()");
  m.def(
      "paged_decode(Tensor q, Tensor(a!) out, Tensor k_cache, Tensor v_cache, Tensor "
      "block_tables, Tensor seq_lens, int num_q_heads, int num_kv_heads, int max_seq_len, float "
      "scale, int num_splits=1, Tensor(b!)? ws_o=None, Tensor(c!)? ws_lse=None, "
      "Tensor? sinks=None) -> ()");
  m.def(
      "paged_prefill(Tensor q, Tensor(a!) out, Tensor k_cache, Tensor v_cache, Tensor cu_q, "
      "Tensor seq_lens, Tensor block_tables, Tensor(b!) tile_offsets, int num_q_heads, int "
      "num_kv_heads, float scale, int window=0, Tensor? sinks=None, bool causal=True, "
      "Tensor? tree_mask=None) -> ()");
  m.def(
      "sample(Tensor logits, Tensor? temperature, Tensor? top_k, Tensor? top_p, Tensor? min_p, "
      "Tensor? seeds, Tensor? steps, int vocab_offset, Tensor(a!) out_idx, Tensor(b!)? "
      "out_val=None) -> ()");
  m.def("merge_candidates(Tensor vals, Tensor idx, Tensor(a!) out) -> ()");
  m.def("apply_penalties(Tensor(a!) logits, Tensor entries, Tensor rep, Tensor pres, Tensor freq, "
        "int vocab_offset) -> ()");
  m.def("apply_token_bitmask(Tensor(a!) logits, Tensor bitmask, Tensor rows, int vocab_offset) "
        "-> ()");
  m.def("embedding(Tensor(a!) out, Tensor table, Tensor ids, int vocab_start=0) -> ()");
  m.def("gather_rows(Tensor(a!) out, Tensor x, Tensor idx) -> ()");
  m.def(
      "mla_prep(Tensor(a!) q, Tensor kv, Tensor kv_norm_w, float eps, Tensor positions, "
      "Tensor cos_sin, Tensor(b!) cache, Tensor slot_mapping, int Hq) -> ()");
  m.def(
      "mla_attention(Tensor q_lat, Tensor q_pe, Tensor cache, Tensor block_tables, Tensor cu_q, "
      "Tensor seq_lens, Tensor? indices, Tensor(a!) out, float scale, int splits, "
      "Tensor? ws_o=None, Tensor? ws_lse=None, int dcp_size=1, int dcp_rank=0, "
      "Tensor(b!)? lse_out=None) -> ()");
  m.def(
      "indexer_k_prep(Tensor k, Tensor ln_w, Tensor ln_b, float eps, Tensor positions, "
      "Tensor cos_sin, Tensor(a!) cache, Tensor slot_mapping) -> ()");
  m.def(
      "indexer_scores(Tensor q, Tensor w, Tensor cache, Tensor block_tables, Tensor cu_q, "
      "Tensor seq_lens, Tensor(a!) scores) -> ()");
  m.def("mla_topk(Tensor scores, Tensor cu_q, Tensor seq_lens, Tensor(a!) out) -> ()");
  m.def(
      "gemm_fp8(Tensor A, Tensor sa, Tensor B, Tensor sb, Tensor(a!) C, int splits=0, "
      "Tensor? workspace=None, Tensor? counters=None, Tensor? tile_expert=None, "
      "Tensor? num_tiles=None, int num_experts=0) -> ()");
  m.def(
      "gemm_grouped_bf16(Tensor A, Tensor B, Tensor(a!) C, Tensor tile_expert, Tensor num_tiles, "
      "int num_experts, int mode=0, int bn=0) -> ()");
  m.def("topk_softmax(Tensor logits, Tensor(a!) ids, Tensor(b!) w, bool renorm=True) -> ()");
  m.def(
      "grouped_topk(Tensor logits, Tensor? bias, Tensor(a!) ids, Tensor(b!) w, int n_group, "
      "int topk_group, bool sigmoid, bool renorm, float scale) -> ()");
  m.def(
      "moe_align(Tensor ids, int num_experts, Tensor(a!) sorted_ids, Tensor(b!) tile_expert, "
      "Tensor(c!) offsets, Tensor(d!) pos, Tensor(e!) num_tiles, int expert_offset=0) -> ()");
  m.def("moe_gather(Tensor x, Tensor sorted_ids, Tensor num_tiles, int k, Tensor(a!) out) -> ()");
  m.def("w4_dequant(Tensor(a!) out, Tensor packed, Tensor scales, Tensor? offsets) -> ()");
  m.def("row_fp8_qdq(Tensor(a!) out, Tensor x, bool swiglu, float limit, Tensor? num_tiles) -> ()");
  m.def("moe_gemv(Tensor x, Tensor ids, int E, int expert_offset, Tensor w_gu, Tensor w_down, "
        "Tensor(a!) h, Tensor(b!) y, Tensor(c!) pos) -> ()");
  m.def("moe_combine(Tensor y, Tensor pos, Tensor w, Tensor? shared, Tensor(a!) out, "
      "Tensor? shared_gate=None) -> ()");
  m.def(
      "causal_conv1d(Tensor x, Tensor w, Tensor(a!) state, Tensor cu_q, Tensor seq_lens, "
      "Tensor slots, Tensor(b!) out, Tensor? bias=None) -> ()");
  m.def(
      "mamba2_scan(Tensor xbc, int b_off, int c_off, Tensor dt, Tensor dt_bias, Tensor A_log, "
      "Tensor D, Tensor(a!) state, Tensor cu_q, Tensor seq_lens, Tensor slots, Tensor(b!) y, "
      "int H, int G, int P, int N, float dt_min, float dt_max) -> ()");
  m.def(
      "mamba2_chunked(Tensor xbc, int b_off, int c_off, Tensor dt, Tensor dt_bias, "
      "Tensor A_log, Tensor D, Tensor(a!) state, Tensor cu_q, Tensor seq_lens, Tensor slots, "
      "Tensor(b!) y, int H, int G, int P, int N, float dt_min, float dt_max, "
      "Tensor(c!) chunk_offsets, Tensor(d!) states, Tensor(e!) start_bf16, Tensor(f!) decay, "
      "int num_tokens) -> ()");
  m.def("gated_rmsnorm(Tensor(a!) out, Tensor y, Tensor z, Tensor w, int group, float eps) -> ()");
  m.def(
      "gdn_recurrent(Tensor qkv, Tensor ba, Tensor A_log, Tensor dt_bias, Tensor(a!) state, "
      "Tensor cu_q, Tensor seq_lens, Tensor slots, int Hk, int Hv, Tensor(b!) out, "
      "bool single_token=False) -> ()");
  m.def(
      "gdn_chunked(Tensor qkv, Tensor ba, Tensor A_log, Tensor dt_bias, Tensor(a!) state, "
      "Tensor cu_q, Tensor seq_lens, Tensor slots, int Hk, int Hv, Tensor(b!) out, "
      "Tensor(c!) ws, Tensor(d!) chunk_offsets, Tensor(e!) gam_c) -> ()");
  m.def("sigmoid_gate(Tensor(a!) out, Tensor gate) -> ()");
}

TORCH_LIBRARY_IMPL(b200, CUDA, m) {
  m.impl("gemm_bf16", &gemm_bf16);
  m.impl("rms_norm", &rms_norm);
  m.impl("fused_add_rms_norm", &fused_add_rms_norm);
  m.impl("rms_norm_gated", &rms_norm_gated);
  m.impl("rms_norm_quant_fp8", &rms_norm_quant_fp8);
  m.impl("act_and_mul", &act_and_mul);
  m.impl("silu_mul_fp8_quant", &silu_mul_fp8_quant);
  m.impl("group_quant_fp8", &group_quant_fp8);
  m.impl("rope_kv", &rope_kv);
  m.impl("paged_decode", &paged_decode);
  m.impl("tq_store", &tq_store);
  m.impl("tq_decode", &tq_decode);
  m.impl("tq_dequant", &tq_dequant);
  m.impl("paged_prefill", &paged_prefill);
  m.impl("sample", &sample);
  m.impl("merge_candidates", &merge_candidates);
  m.impl("kv_insert", &kv_insert);
  m.impl("apply_penalties", &apply_penalties);
  m.impl("apply_token_bitmask", &apply_token_bitmask);
  m.impl("embedding", &embedding);
  m.impl("gather_rows", &gather_rows);
  m.impl("gemm_grouped_bf16", &gemm_grouped_bf16);
  m.impl("topk_softmax", &topk_softmax);
  m.impl("grouped_topk", &grouped_topk);
  m.impl("moe_align", &moe_align);
  m.impl("gemm_fp8", &gemm_fp8);
  m.impl("mla_prep", &mla_prep);
  m.impl("mla_attention", &mla_attention);
  m.impl("indexer_k_prep", &indexer_k_prep);
  m.impl("indexer_scores", &indexer_scores);
  m.impl("mla_topk", &mla_topk);
  m.impl("moe_gather", &moe_gather);
  m.impl("w4_dequant", &w4_dequant);
  m.impl("row_fp8_qdq", &row_fp8_qdq);
  m.impl("moe_combine", &moe_combine);
  m.impl("moe_gemv", &moe_gemv);
  m.impl("causal_conv1d", &causal_conv1d);
  m.impl("mamba2_scan", &mamba2_scan);
  m.impl("mamba2_chunked", &mamba2_chunked);
  m.impl("gated_rmsnorm", &gated_rmsnorm);
  m.impl("gdn_recurrent", &gdn_recurrent);
  m.impl("gdn_chunked", &gdn_chunked);
  m.impl("sigmoid_gate", &sigmoid_gate);
}

void register_runtime(pybind11::module_& m);  // csrc/runtime/bindings.cpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "vllm_musa_b200 native extension (sm_100a kernels + host runtime)";
  m.def("gemm_plan", &gemm_plan, "automatic (bn, splits, workspace_floats) for a bf16 GEMM");
  m.def("gemm_set_katoms", [](int64_t k) { b200::gemm::set_katoms((int)k); },
        "64-element K atoms per bf16 GEMM pipeline stage: 0 automatic, 1 / 2 / 4 forced");
  m.def("set_prefill_tc2", [](bool on) { b200::attn::set_prefill_tc2(on); },
        "allow (true) the two-heads-per-CTA tcgen05 prefill kernel for even GQA groups");
  m.def("set_prefill_tc", [](bool on) { b200::attn::set_prefill_tc(on); },
        "select the tcgen05 (true) or mma.sync (false) prefill attention kernel for head_dim 128");
  m.def("gemm_fp8_plan", &gemm_fp8_plan, "automatic (splits, workspace_floats, counters) for fp8");
  m.def("decode_num_splits", &decode_num_splits, "split-KV count for a decode batch");
  m.def("tq_slot_bytes", &tq_slot_bytes, "TurboQuant slot bytes for (head_dim, key_bits, value_bits)");
  m.def("moe_max_rows", [](int64_t n, int64_t E) { return (int64_t)b200::moe::align_max_rows(n, E); },
        "rows of the expert-sorted buffer for n assignments over E experts");
  m.def("error_word", &error_word, "per-device error word of the bounded waits");
  m.def("fused_allreduce", &fused_allreduce, "NVSwitch all-reduce (+ residual + RMSNorm)",
        py::arg("like"), py::arg("bufs"), py::arg("epochs_ptr"), py::arg("rank"),
        py::arg("world"), py::arg("T"), py::arg("H"), py::arg("blocks"), py::arg("parity"),
        py::arg("two_shot"), py::arg("residual"), py::arg("weight"), py::arg("eps"),
        py::arg("rs_rows") = 0, py::arg("end_barrier") = false);
  m.def("cand_row_bytes", &cand_row_bytes, "bytes of one candidate row");
  m.def("shard_candidates", &shard_candidates, "per-shard top-k candidates of each logits row",
        py::arg("logits"), py::arg("temperature"), py::arg("seeds"), py::arg("steps"),
        py::arg("vocab_offset"), py::arg("out"));
  m.def("merge_candidates_local", &merge_candidates_local,
        "merge [world][R] candidate rows held locally and sample (top-k / top-p / min-p)");
  m.def("topk_exchange", &topk_exchange,
        "exchange candidate rows over NVLink, then merge and sample each row");
  m.def("nvls_allreduce", &nvls_allreduce,
        "NVLS (multimem) all-reduce (+ residual + RMSNorm, + optional 1x128 e4m3 output)",
        py::arg("like"), py::arg("ptrs"), py::arg("rank"), py::arg("world"), py::arg("T"),
        py::arg("H"), py::arg("two_shot"), py::arg("residual"), py::arg("weight"),
        py::arg("eps"), py::arg("rows_per_warp") = 0);
  m.def("nvls_flag_bytes", []() { return (int64_t)b200::comm::kNvlsFlagBytes; });
  m.def("ep_dispatch", &ep_dispatch, "expert-parallel dispatch over NVLink (+ count exchange)");
  m.def("exchange_candidates", &exchange_candidates,
        "vocab-parallel sampling: per-row candidates exchanged over NVLink and merged");
  m.def("ep_return", &ep_return, "expert-parallel combine into the sources' staging slots");
  m.def("gemm_bf16_rs", &gemm_bf16_rs,
        "row-parallel GEMM with the reduce-scatter in its epilogue (NVLink stores)",
        py::arg("A"), py::arg("B"), py::arg("recv"), py::arg("rs_rows"), py::arg("rank"),
        py::arg("bn") = 0, py::arg("splits") = 0, py::arg("mt") = 0,
        py::arg("workspace") = py::none(), py::arg("counters") = py::none());
  m.def("ipc_malloc", [](size_t n) { return (int64_t)reinterpret_cast<uintptr_t>(b200::comm::ipc_malloc(n)); });
  m.def("ipc_free", [](int64_t p) { b200::comm::ipc_free(reinterpret_cast<void*>(p)); });
  m.def("ipc_handle", [](int64_t p) { return pybind11::bytes(b200::comm::ipc_handle(reinterpret_cast<void*>(p))); });
  m.def("ipc_open", [](const std::string& h) { return (int64_t)reinterpret_cast<uintptr_t>(b200::comm::ipc_open(h)); });
  m.def("ipc_close", [](int64_t p) { b200::comm::ipc_close(reinterpret_cast<void*>(p)); });
  m.def("tensor_from_ptr",
        [](int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype, int64_t device) {
          // non-owning view of device memory this library manages (IPC buffers)
          return torch::from_blob(reinterpret_cast<void*>(ptr), shape, [](void*) {},
                                  at::TensorOptions().dtype(dtype).device(at::kCUDA, device));
        });
  m.def("comm_flag_bytes", []() { return (int64_t)(b200::comm::kFlagBytes + b200::comm::kEpochBytes); });
  m.def("comm_max_blocks", []() { return (int64_t)b200::comm::kMaxBlocks; });
  m.def("launch_count", []() { return (long long)b200::launch_counter().load(); },
        "kernels launched (or recorded into CUDA graphs) by this library so far");
  m.attr("BUILT_ARCH") = "sm_100a";
  register_runtime(m);
}
