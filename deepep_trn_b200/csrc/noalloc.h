// Allocation-free C entry point of the dispatch-layout kernel.
//
// This entry point has no counterpart in the reference library: it exists for
// callers of this library that cannot allocate device memory at the point where
// they need the routing layout. Typical cases are inference engines that plan
// every byte of device memory ahead of time and forbid allocation inside their
// execution callbacks (an allocation there could fail or stall mid-request),
// plugin interfaces whose enqueue step must not call the CUDA allocator, and
// callers outside PyTorch that have no caching allocator at all. The regular
// layout op takes a scratch tensor from the caller; this variant keeps its
// scratch in a fixed-size array compiled into the library instead.
//
// int b200ep_dispatch_layout_noalloc(topk_idx, num_tokens, topk, num_experts, num_ranks,
//                                    num_tokens_per_rank, num_tokens_per_expert,
//                                    is_token_in_rank, stream)
//
//   topk_idx               [num_tokens, topk] int64 device array, -1 = masked entry
//   num_tokens_per_rank    [num_ranks] int32 device output
//   num_tokens_per_expert  [num_experts] int32 device output
//   is_token_in_rank       [num_tokens, num_ranks] bool device output
//   stream                 CUDA stream to launch on (0 = legacy default stream)
//
// Results are identical to the regular layout op. Limits: num_experts <= 4096,
// 1 <= num_ranks <= 32, num_experts divisible by num_ranks. Returns 0 on success,
// B200EP_NOALLOC_TOO_LARGE (-2) when a size is beyond those limits or negative,
// or the CUDA error code of the failing runtime call.
//
// The scratch array (about 16 KB) lives in every GPU that loads the library until
// the process exits. All calls on a device share it and it keeps the state of the
// last call; the kernel returns it to zero before it finishes, so calls that run
// one after another on the GPU are correct, but calls that overlap on the GPU
// (different streams without ordering between them) race on it and must be avoided.
// The first call on each device looks up the array's device address (with that device
// current) and clears the array with an asynchronous memset on the caller's stream, so
// the clearing is ordered before that call's kernel; make that first call before any
// CUDA stream capture.
// No call allocates or frees memory.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define B200EP_NOALLOC_TOO_LARGE (-2)
#define B200EP_NOALLOC_MAX_EXPERTS 4096
#define B200EP_NOALLOC_MAX_RANKS 32

extern "C" __attribute__((visibility("default"))) int b200ep_dispatch_layout_noalloc(
    const int64_t* topk_idx, int num_tokens, int topk, int num_experts, int num_ranks,
    int32_t* num_tokens_per_rank, int32_t* num_tokens_per_expert, bool* is_token_in_rank, cudaStream_t stream);
