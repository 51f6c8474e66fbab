// Allocation-free C entry point for split-KV paged decode attention.
//
// This entry point has no counterpart in the reference (MooreThreads/vllm-musa).  It exists
// for callers that cannot allocate GPU memory while they run attention: hosts that hand this
// library a fixed device-memory budget and forbid it from growing (inference servers with
// their own allocator, embedded / real-time deployments that reserve all memory up front),
// and foreign-language runtimes that link the shared library with no PyTorch allocator to
// draw a workspace from.  Instead of a caller- or torch-allocated workspace, the split-KV
// partial results live in a file-scope device array of B200_DECODE_NOALLOC_SCRATCH_BYTES
// (16 MiB), which every GPU that loads the library keeps until the process exits.
//
// Usage notes:
//  * The first call on a device performs set-up for that device (it looks up the scratch
//    array's device address with cudaGetSymbolAddress and registers the kernel's shared-memory
//    size).  Make that first call before any stream capture.
//  * All calls share the one scratch array, and it keeps the previous call's contents.  Calls
//    whose executions overlap on the GPU (different streams, or different host threads) race
//    on it: serialise them.
//  * Inputs and outputs are caller-owned device memory with the layouts of paged_decode
//    (torch.ops.b200.paged_decode): q [batch, >= Hq*D] bf16 rows (stride ld_q), out
//    [batch, >= Hq*D] bf16 (stride ld_out), caches [num_blocks, Hkv, block_size, D] bf16,
//    block_tables [batch, bt_stride] int32, seq_lens [batch] int32.
//  * `status` (optional, device int) is zeroed on the stream and receives a non-zero code if
//    a bounded wait in the kernel gave up.
//  * No cudaMalloc, cudaFree or other allocating routine is called.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define B200_DECODE_NOALLOC_SCRATCH_BYTES (16u << 20)

#define B200_NOALLOC_OK 0
#define B200_NOALLOC_ERR_TOO_LARGE 1  // split partials would exceed the scratch array
#define B200_NOALLOC_ERR_SETUP 2      // no current device / symbol address lookup failed
#define B200_NOALLOC_ERR_ARGS 3       // null / misaligned pointer or unsupported geometry:
                                      // head_dim not 64, 128 or 256; num_q_heads not a multiple
                                      // of num_kv_heads or a GQA group above 16; block_size not
                                      // 16, 32, 64 or a multiple of 64
#define B200_NOALLOC_ERR_LAUNCH 4     // the kernel launch failed

#ifdef __cplusplus
extern "C" {
#endif

int b200_paged_decode_noalloc(const void* q, int64_t ld_q, void* out, int64_t ld_out,
                              void* k_cache, void* v_cache, int num_blocks,
                              const int32_t* block_tables, int64_t bt_stride,
                              const int32_t* seq_lens, int batch, int num_q_heads,
                              int num_kv_heads, int head_dim, int block_size, int max_seq_len,
                              int num_splits, float scale, int* status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
