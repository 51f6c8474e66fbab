// Parameters of the NVSwitch fused all-reduce kernels (custom_ar.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace b200 {
namespace comm {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 128;
// flags region: [6 phases][kMaxBlocks][kMaxRanks] uint32 (all-reduce start / end barriers by
// parity, sampling exchange by parity), then the local epoch counters.
constexpr size_t kFlagBytes = 6 * kMaxBlocks * kMaxRanks * sizeof(uint32_t);
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
  // one-shot calls end with a barrier too (callers whose buffer parity does not strictly
  // alternate between consecutive calls)
  bool end_barrier = false;
};

void run_fused_allreduce(const ArParams& a, cudaStream_t s);

// NVLS variant (nvls_ar.cu): the buffers are bound to an NVLink multicast object; `mc_*` are
// multicast addresses of this call's slots, the other pointers this rank's own copies.
struct NvlsParams {
  int rank, world, T, H, blocks;
  bool two_shot;
  const void* mc_staging;  // [T, H] bf16 partial sums of every rank, read with ld_reduce
  void* mc_out;            // two-shot: normalised rows, stored to every rank
  void* out_local;         // one-shot: this rank's output copy
  uint32_t* mc_flags;      // barrier counters [2 phases][kMaxBlocks] (multicast address)
  uint32_t* flags;         // the same counters, this rank's copy
  uint32_t* epochs;        // local per-block call counts [2 phases][kMaxBlocks]
  void* residual;          // [T, H] bf16, updated in place (nullptr: plain all-reduce)
  const void* weight;      // RMSNorm weight (nullptr: no norm)
  float eps;
  // per-token 1x128 e4m3 output instead of the bf16 rows (needs the norm): q [T, H] e4m3 and
  // scales [T, H / 128] fp32; multicast addresses (two-shot) or local copies (one-shot)
  void* mc_q = nullptr;
  void* q_local = nullptr;
  float* mc_s = nullptr;
  float* s_local = nullptr;
  int* err;
};
constexpr size_t kNvlsFlagBytes = 2 * kMaxBlocks * sizeof(uint32_t);
void run_nvls_allreduce(const NvlsParams& a, cudaStream_t s);
int nvls_blocks(int T, int world, bool two_shot, int rows_per_warp = 0);

// Vocab-parallel sampling exchange: every rank's per-row (score, token) candidate is stored into
// every peer's candidate region [src rank][row]; after a per-block epoch barrier each rank picks
// the row maxima (ties -> smaller token id) from local memory.
struct CandParams {
  int rank, world, R, parity;
  float* vals[kMaxRanks];      // this call's candidate score region of every rank [world][R]
  int64_t* ids[kMaxRanks];     // this call's candidate id region of every rank [world][R]
  uint32_t* flags[kMaxRanks];  // flag region of every rank (phases 4 / 5 by parity)
  uint32_t* epochs;            // local per-block epoch counters (own slice)
  const float* my_vals;        // [R] this rank's candidates
  const int64_t* my_ids;
  int64_t* out;                // [R] merged tokens
  int* err;
};
void run_exchange_candidates(const CandParams& a, cudaStream_t s);
void* ipc_malloc(size_t bytes);
void ipc_free(void* p);
std::string ipc_handle(void* p);
void* ipc_open(const std::string& handle);
void ipc_close(void* p);

}  // namespace comm
}  // namespace b200
