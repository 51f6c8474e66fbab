// Allocation-free split-KV paged decode (declaration and usage notes: decode_noalloc.h).
// The split partials (fp32 O and log-sum-exp per (sequence, head, split)) are written to a
// file-scope device array instead of a caller-provided workspace; the attention kernels are
// the same ones paged_decode launches (paged_attention.cu).
#include <stdint.h>
#include <stdio.h>

#include <exception>
#include <mutex>

#include "../b200_kernels.h"
#include "decode_noalloc.h"

static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[B200_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices];  // device address of the array, per device (set-up once)

// Device address of the scratch array for the current device.  In host code the array's
// name is only a host-side stand-in, so the address must come from cudaGetSymbolAddress,
// queried once per device with that device current.
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return B200_NOALLOC_ERR_SETUP;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_decode_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      fprintf(stderr, "b200_paged_decode_noalloc: cudaGetSymbolAddress failed on device %d: %s\n",
              dev, cudaGetErrorString(e));
      return B200_NOALLOC_ERR_SETUP;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return B200_NOALLOC_OK;
}

}  // namespace

extern "C" int b200_paged_decode_noalloc(const void* q, int64_t ld_q, void* out, int64_t ld_out,
                                         void* k_cache, void* v_cache, int num_blocks,
                                         const int32_t* block_tables, int64_t bt_stride,
                                         const int32_t* seq_lens, int batch, int num_q_heads,
                                         int num_kv_heads, int head_dim, int block_size,
                                         int max_seq_len, int num_splits, float scale,
                                         int* status, cudaStream_t stream) {
  if (!q || !out || !k_cache || !v_cache || !block_tables || !seq_lens || batch < 0 ||
      num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || num_splits < 1 ||
      max_seq_len < 1 || num_blocks < 1)
    return B200_NOALLOC_ERR_ARGS;
  // geometry the decode kernels serve (checked here so that a bad argument is reported as
  // such, before anything is queued on the stream)
  if (num_q_heads % num_kv_heads != 0 || num_q_heads / num_kv_heads > 16)
    return B200_NOALLOC_ERR_ARGS;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return B200_NOALLOC_ERR_ARGS;
  if (block_size < 16 || block_size % 16 != 0 || (block_size > 64 && block_size % 64 != 0))
    return B200_NOALLOC_ERR_ARGS;
  if (ld_q < (int64_t)num_q_heads * head_dim ||
      ld_out < (int64_t)num_q_heads * head_dim || bt_stride < 1)
    return B200_NOALLOC_ERR_ARGS;
  // the caches are read by TMA: 16-byte aligned base addresses
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0)
    return B200_NOALLOC_ERR_ARGS;
  // scratch layout: partial O [batch, Hq, splits, D] fp32, 256-byte aligned LSE after it
  const size_t o_bytes = (size_t)batch * num_q_heads * num_splits * head_dim * sizeof(float);
  const size_t o_pad = (o_bytes + 255) / 256 * 256;
  const size_t lse_bytes = (size_t)batch * num_q_heads * num_splits * sizeof(float);
  if (num_splits > 1 && o_pad + lse_bytes > B200_DECODE_NOALLOC_SCRATCH_BYTES) {
    fprintf(stderr,
            "b200_paged_decode_noalloc: %d sequences x %d heads x %d splits x head_dim %d needs "
            "%zu bytes of split scratch; the static scratch holds %u bytes (use fewer splits or "
            "a smaller batch per call)\n",
            batch, num_q_heads, num_splits, head_dim, o_pad + lse_bytes,
            B200_DECODE_NOALLOC_SCRATCH_BYTES);
    return B200_NOALLOC_ERR_TOO_LARGE;
  }
  void* base = nullptr;
  const int rc = scratch_address(&base);
  if (rc != B200_NOALLOC_OK) return rc;
  if (status != nullptr && cudaMemsetAsync(status, 0, sizeof(int), stream) != cudaSuccess)
    return B200_NOALLOC_ERR_LAUNCH;
  if (batch == 0) return B200_NOALLOC_OK;
  b200::attn::DecodeArgs a{};
  a.q = q;
  a.ld_q = ld_q;
  a.o = out;
  a.ld_o = ld_out;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = bt_stride;
  a.seq_lens = seq_lens;
  a.B = batch;
  a.Hq = num_q_heads;
  a.Hkv = num_kv_heads;
  a.D = head_dim;
  a.block_size = block_size;
  a.max_seq_len = max_seq_len;
  a.num_splits = num_splits;
  a.scale = scale;
  a.ws_o = reinterpret_cast<float*>(base);
  a.ws_lse = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(base) + o_pad);
  a.err = status;
  try {
    b200::attn::run_decode(a, stream);
  } catch (const std::exception& e) {
    fprintf(stderr, "b200_paged_decode_noalloc: %s\n", e.what());
    return B200_NOALLOC_ERR_LAUNCH;
  }
  return B200_NOALLOC_OK;
}
