// N1: dispatch layout on the device (no host round trip).
//
// topk_idx [T, K] (int64 or int32) -> num_tokens_per_rank [R] int32,
// num_tokens_per_expert [E] int32, is_token_in_rank [T, R] bool.
// Same results as deep_ep_trn/layout.py:15-29 (which runs on the host after a
// topk_idx.cpu() at buffer.py:165).
//
// One thread per token. Per-CTA counts are reduced in shared memory with warp
// ballots (ranks) and shared atomics (experts), then folded into a scratch
// accumulator in global memory. The last CTA to finish copies the scratch
// totals to the outputs and zeroes the scratch, so the whole op is one launch
// and needs no memset. Scratch layout: [R + E] counts, then one arrival counter.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ops.h"

namespace b200ep {

constexpr int kLayoutThreads = 256;
constexpr int kLayoutSmemExperts = 4096;

template <typename IdxT>
__global__ void __launch_bounds__(kLayoutThreads) layout_kernel(const IdxT* __restrict__ topk, int T, int K, int E,
                                                                 int R, int EL, int32_t* __restrict__ ntr,
                                                                 int32_t* __restrict__ nte, bool* __restrict__ itr,
                                                                 int32_t* __restrict__ scratch) {
  __shared__ int32_t s_rank[B200EP_MAX_RANKS];
  __shared__ int32_t s_exp[kLayoutSmemExperts];
  __shared__ bool s_last;
  const bool smem_hist = E <= kLayoutSmemExperts;
  for (int i = threadIdx.x; i < B200EP_MAX_RANKS; i += blockDim.x) s_rank[i] = 0;
  if (smem_hist)
    for (int i = threadIdx.x; i < E; i += blockDim.x) s_exp[i] = 0;
  __syncthreads();

  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t mask = 0;
  if (t < T) {
    for (int k = 0; k < K; ++k) {
      const int64_t e = static_cast<int64_t>(topk[static_cast<int64_t>(t) * K + k]);
      if (e < 0 || e >= E) continue;
      mask |= 1u << static_cast<uint32_t>(e / EL);
      if (smem_hist)
        atomicAdd(&s_exp[e], 1);
      else
        atomicAdd(&scratch[R + e], 1);
    }
    bool* row = itr + static_cast<int64_t>(t) * R;
    for (int r = 0; r < R; ++r) row[r] = (mask >> r) & 1u;
  }
  for (int r = 0; r < R; ++r) {
    const uint32_t b = __ballot_sync(0xffffffffu, (mask >> r) & 1u);
    if (lane_id() == 0 && b) atomicAdd(&s_rank[r], __popc(b));
  }
  __syncthreads();
  for (int r = threadIdx.x; r < R; r += blockDim.x)
    if (s_rank[r]) atomicAdd(&scratch[r], s_rank[r]);
  if (smem_hist)
    for (int e = threadIdx.x; e < E; e += blockDim.x)
      if (s_exp[e]) atomicAdd(&scratch[R + e], s_exp[e]);

  // last CTA publishes and resets the scratch accumulators
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int prev = atomicAdd(&scratch[R + E], 1);
    s_last = (prev == static_cast<int>(gridDim.x) - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int r = threadIdx.x; r < R; r += blockDim.x) {
    ntr[r] = atomicExch(&scratch[r], 0);
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    nte[e] = atomicExch(&scratch[R + e], 0);
  }
  __syncthreads();
  if (threadIdx.x == 0) atomicExch(&scratch[R + E], 0);
}

void layout(const at::Tensor& topk_idx, int64_t num_experts, int64_t num_ranks, at::Tensor ntr, at::Tensor nte,
            at::Tensor itr, at::Tensor scratch) {
  TORCH_CHECK(topk_idx.is_cuda() && topk_idx.dim() == 2 && topk_idx.is_contiguous(), "topk_idx must be [T, K] CUDA");
  TORCH_CHECK(num_ranks >= 1 && num_ranks <= B200EP_MAX_RANKS, "num_ranks must be in [1, 32]");
  TORCH_CHECK(num_experts % num_ranks == 0, "num_experts must be divisible by num_ranks");
  TORCH_CHECK(ntr.scalar_type() == at::kInt && nte.scalar_type() == at::kInt && itr.scalar_type() == at::kBool,
              "output dtypes: int32, int32, bool");
  TORCH_CHECK(scratch.scalar_type() == at::kInt && scratch.numel() >= num_ranks + num_experts + 1,
              "scratch too small");
  const c10::cuda::CUDAGuard guard(topk_idx.device());
  const int T = static_cast<int>(topk_idx.size(0)), K = static_cast<int>(topk_idx.size(1));
  const int E = static_cast<int>(num_experts), R = static_cast<int>(num_ranks);
  const int grid = std::max(1, (T + kLayoutThreads - 1) / kLayoutThreads);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (topk_idx.scalar_type() == at::kLong) {
    layout_kernel<int64_t><<<grid, kLayoutThreads, 0, stream>>>(
        topk_idx.data_ptr<int64_t>(), T, K, E, R, E / R, ntr.data_ptr<int32_t>(), nte.data_ptr<int32_t>(),
        itr.data_ptr<bool>(), scratch.data_ptr<int32_t>());
  } else {
    TORCH_CHECK(topk_idx.scalar_type() == at::kInt, "topk_idx must be int64 or int32");
    layout_kernel<int32_t><<<grid, kLayoutThreads, 0, stream>>>(
        topk_idx.data_ptr<int32_t>(), T, K, E, R, E / R, ntr.data_ptr<int32_t>(), nte.data_ptr<int32_t>(),
        itr.data_ptr<bool>(), scratch.data_ptr<int32_t>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace b200ep

// ============================================================================ allocation-free variant
// The same kernel with its scratch in a file-scope device array (see noalloc.h).
#include <cstdio>
#include <mutex>

#include "noalloc.h"

namespace b200ep {
namespace {

constexpr int kNoAllocScratch = B200EP_NOALLOC_MAX_RANKS + B200EP_NOALLOC_MAX_EXPERTS + 1;

// [R + E] accumulators and one arrival counter; zero at load time and returned to zero
// by the last CTA of every launch.
__device__ __align__(256) int32_t g_layout_scratch[kNoAllocScratch];

constexpr int kMaxDevices = 64;
int32_t* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device, looked up once per device.
// In host code the symbol is only a host-side handle; the kernel needs this address.
// The first call on a device also clears the array with an asynchronous memset on the
// caller's stream, so the clearing is ordered before that call's kernel on the same
// stream (the array is zero at module load as well, and every launch leaves it at zero).
cudaError_t scratch_for_current_device(cudaStream_t stream, int32_t** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_layout_scratch);
    if (err != cudaSuccess) return err;
    err = cudaMemsetAsync(p, 0, sizeof(g_layout_scratch), stream);
    if (err != cudaSuccess) return err;
    g_scratch_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace b200ep

extern "C" int b200ep_dispatch_layout_noalloc(const int64_t* topk_idx, int num_tokens, int topk, int num_experts,
                                              int num_ranks, int32_t* num_tokens_per_rank,
                                              int32_t* num_tokens_per_expert, bool* is_token_in_rank,
                                              cudaStream_t stream) {
  using namespace b200ep;
  if (num_tokens < 0 || topk < 0 || num_experts <= 0 || num_ranks < 1 || num_ranks > B200EP_NOALLOC_MAX_RANKS ||
      num_experts > B200EP_NOALLOC_MAX_EXPERTS || num_experts % num_ranks != 0) {
    std::fprintf(stderr,
                 "b200ep_dispatch_layout_noalloc: sizes outside the compiled limits (num_tokens=%d topk=%d "
                 "num_experts=%d (max %d, divisible by num_ranks) num_ranks=%d (1..%d))\n",
                 num_tokens, topk, num_experts, B200EP_NOALLOC_MAX_EXPERTS, num_ranks, B200EP_NOALLOC_MAX_RANKS);
    return B200EP_NOALLOC_TOO_LARGE;
  }
  int32_t* scratch = nullptr;
  cudaError_t err = scratch_for_current_device(stream, &scratch);
  if (err != cudaSuccess) return static_cast<int>(err);
  const int grid = num_tokens > 0 ? (num_tokens + kLayoutThreads - 1) / kLayoutThreads : 1;
  layout_kernel<int64_t><<<grid, kLayoutThreads, 0, stream>>>(topk_idx, num_tokens, topk, num_experts, num_ranks,
                                                              num_experts / num_ranks, num_tokens_per_rank,
                                                              num_tokens_per_expert, is_token_in_rank, scratch);
  return static_cast<int>(cudaGetLastError());
}
