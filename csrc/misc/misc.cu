// Small data-movement kernels: token embedding lookup (optionally vocab-sharded: ids outside
// [vocab_start, vocab_start + vocab) produce zero rows) and row gather (e.g. selecting the last
// token of every sequence before the LM head).  128-bit vector copies, one CTA row per token.
#include <algorithm>

#include "../b200_kernels.h"
#include "../common/common.cuh"

namespace b200 {
namespace misc {

__global__ void embedding_kernel(uint4* __restrict__ out, const uint4* __restrict__ table,
                                 const int32_t* __restrict__ ids, int H8, int64_t vocab,
                                 int64_t vocab_start) {
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int64_t id = (int64_t)ids[t] - vocab_start;
  const bool ok = id >= 0 && id < vocab;
  for (int c = threadIdx.x; c < H8; c += blockDim.x)
    out[(int64_t)t * H8 + c] = ok ? table[id * H8 + c] : make_uint4(0, 0, 0, 0);
}

__global__ void gather_rows_kernel(uint4* __restrict__ out, const uint8_t* __restrict__ in,
                                   int64_t ld_in_bytes, const int32_t* __restrict__ idx, int W16) {
  const int r = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(in + (int64_t)idx[r] * ld_in_bytes);
  for (int c = threadIdx.x; c < W16; c += blockDim.x) out[(int64_t)r * W16 + c] = src[c];
}

void run_embedding(void* out, const void* table, const int32_t* ids, int T, int H, int64_t vocab,
                   int64_t vocab_start, cudaStream_t s) {
  B200_REQUIRE(H % 8 == 0, "embedding: hidden size must be a multiple of 8");
  if (T == 0) return;
  const int H8 = H / 8;
  embedding_kernel<<<T, std::min(256, std::max(32, H8)), 0, s>>>(
      reinterpret_cast<uint4*>(out), reinterpret_cast<const uint4*>(table), ids, H8, vocab,
      vocab_start);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

void run_gather_rows(void* out, const void* in, int64_t ld_in, const int32_t* idx, int R, int H,
                     int elem_bytes, cudaStream_t s) {
  B200_REQUIRE((H * elem_bytes) % 16 == 0 && (ld_in * elem_bytes) % 16 == 0,
               "gather_rows: rows must be 16-byte multiples");
  if (R == 0) return;
  const int W16 = H * elem_bytes / 16;
  gather_rows_kernel<<<R, std::min(256, std::max(32, W16)), 0, s>>>(
      reinterpret_cast<uint4*>(out), reinterpret_cast<const uint8_t*>(in), ld_in * elem_bytes,
      idx, W16);
  B200_CUDA_OK(cudaGetLastError());
  count_launch();
}

}  // namespace misc
}  // namespace b200
