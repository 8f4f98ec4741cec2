// Device barrier over the EP group and a probe of the bounded-wait error path.
//
// The probe waits on a flag of the local signal pad that no kernel ever writes,
// with a caller-given budget, so the timeout branch (error status written to the
// host-mapped page, kernel returns) runs without any fault or hang.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ops.h"

namespace b200ep {

__global__ void device_barrier_kernel(HeapView hv) {
  LocalState* ls = hv.local();
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(&ls->epoch[kEpBar]) + 1u;
  const int tid = threadIdx.x;
  if (tid < hv.R) {
    fence_sys();
    st_release_sys(&hv.sig(tid)->barrier[hv.rank], e);
    wait_epoch(&hv.sig(hv.rank)->barrier[tid], e, hv.timeout_ns, hv.status, kTimeoutBarrier, 7, hv.rank, tid);
  }
  __syncthreads();
  if (tid == 0) ls->epoch[kEpBar] = e;
}

__global__ void wait_probe_kernel(HeapView hv, uint64_t budget_ns) {
  // pad[] is never written by any kernel, so this wait must run out
  const uint32_t* flag = &hv.sig(hv.rank)->pad[0];
  const uint32_t want = ld_acquire_sys(flag) + 1u;
  wait_epoch(flag, want, budget_ns, hv.status, kTimeoutBarrier, 99, hv.rank, -1);
}

void device_barrier(SymmHeap& heap) {
  const c10::cuda::CUDAGuard guard(heap.device());
  device_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(heap.view());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void wait_probe(SymmHeap& heap, int64_t budget_ns) {
  const c10::cuda::CUDAGuard guard(heap.device());
  wait_probe_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream()>>>(heap.view(), static_cast<uint64_t>(budget_ns));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace b200ep
