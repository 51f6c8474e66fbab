// Parameters of the NVSwitch fused all-reduce kernels (custom_ar.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace b200 {
namespace comm {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 128;
// flags region: [4 phases][kMaxBlocks][kMaxRanks] uint32, then the local epoch counters.
constexpr size_t kFlagBytes = 4 * kMaxBlocks * kMaxRanks * sizeof(uint32_t);
constexpr size_t kEpochBytes = kMaxBlocks * sizeof(uint32_t);

struct ArParams {
  int rank, world, T, H, blocks, parity;
  bool two_shot;
  const void* staging[kMaxRanks];  // this call's staging slot of every rank (peer VAs)
  void* out[kMaxRanks];            // this call's output slot of every rank
  uint32_t* flags[kMaxRanks];      // flag region of every rank
  uint32_t* epochs;                // this rank's per-block epoch counters (local)
  void* residual;                  // [T, H] bf16, updated in place (nullptr: plain AR)
  const void* weight;              // RMSNorm weight (nullptr: no norm, plain all-reduce)
  float eps;
  int* err;
  // > 0: the reduce-scatter already happened in the producing GEMM's epilogue (two-shot
  // only): this rank's staging slot holds `world` blocks of rs_rows rows, block p = rank p's
  // partial sums of the rows this rank owns, so the reduction reads local memory only.
  int rs_rows = 0;
};

void run_fused_allreduce(const ArParams& a, cudaStream_t s);
void* ipc_malloc(size_t bytes);
void ipc_free(void* p);
std::string ipc_handle(void* p);
void* ipc_open(const std::string& handle);
void ipc_close(void* p);

}  // namespace comm
}  // namespace b200
