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
  if (tid == 0) {
    ls->epoch[kEpBar] = e;
    ls->trace[kTrBarrierExit] = global_ns();
  }
}

__global__ void wait_probe_kernel(HeapView hv, uint64_t budget_ns) {
  // pad[] is never written by any kernel, so this wait must run out
  const uint32_t* flag = &hv.sig(hv.rank)->pad[0];
  const uint32_t want = ld_acquire_sys(flag) + 1u;
  wait_epoch(flag, want, budget_ns, hv.status, kTimeoutBarrier, 99, hv.rank, -1);
}

// Cost of making a CTA's stores visible before a flag: every CTA writes `bytes` into the
// heap of rank `peer` (its own rank for a local measurement), then thread 0 times one
// fence of the given scope (0 = gpu, 1 = sys, 2 = none: st.release.sys alone) plus the
// flag store. out[cta] = nanoseconds of that fence + store.
__global__ void fence_cost_kernel(HeapView hv, int peer, int64_t bytes, int scope, int64_t* out) {
  uint8_t* dst = hv.base[peer] + hv.L.lc_rows[0] + static_cast<int64_t>(blockIdx.x) * bytes;
  const int4 v = make_int4(blockIdx.x, 1, 2, 3);
  for (int64_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) reinterpret_cast<int4*>(dst)[i] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = global_ns();
    if (scope == 0) asm volatile("fence.acq_rel.gpu;" ::: "memory");
    if (scope == 1) asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(&hv.sig(peer)->pad[1], static_cast<uint32_t>(blockIdx.x));
    out[blockIdx.x] = static_cast<int64_t>(global_ns() - t0);
  }
}

void fence_cost(SymmHeap& heap, int64_t peer, int64_t bytes, int64_t scope, at::Tensor out) {
  const c10::cuda::CUDAGuard guard(heap.device());
  HeapView hv = heap.view();
  TORCH_CHECK(peer >= 0 && peer < hv.R && bytes % 16 == 0, "bad peer / size");
  TORCH_CHECK(out.numel() * bytes <= hv.L.lc_rows[1] - hv.L.lc_rows[0], "probe exceeds the scratch region");
  fence_cost_kernel<<<static_cast<int>(out.numel()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      hv, static_cast<int>(peer), bytes, static_cast<int>(scope), out.data_ptr<int64_t>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
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
