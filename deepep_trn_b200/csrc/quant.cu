// N6: standalone per-token, per-128-channel e4m3 quantisation (the same
// device function the dispatch kernels fuse into their send path).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ops.h"

namespace b200ep {

template <typename T16>
__global__ void __launch_bounds__(256) quant_fp8_kernel(const T16* __restrict__ x, uint8_t* __restrict__ q,
                                                        float* __restrict__ scales, int64_t T, int H,
                                                        int round_scale) {
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t GW = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t t = gw; t < T; t += GW)
    warp_quant_row<T16>(q + t * H, scales + t * (H / 128), x + t * H, H, round_scale);
}

void quant_fp8(const at::Tensor& x, at::Tensor q, at::Tensor scales, bool round_scale) {
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.is_contiguous() && q.is_contiguous() && scales.is_contiguous(), "contiguous tensors expected");
  const int H = static_cast<int>(x.size(-1));
  TORCH_CHECK(H % 128 == 0, "hidden must be a multiple of 128");
  const int64_t T = x.numel() / H;
  TORCH_CHECK(q.element_size() == 1 && q.numel() == x.numel(), "q must be a 1-byte tensor shaped like x");
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.numel() == T * (H / 128), "scales must be fp32 [.., H/128]");
  if (T == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((T + 7) / 8, 148 * 16));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kHalf)
    quant_fp8_kernel<__half><<<blocks, 256, 0, stream>>>(reinterpret_cast<const __half*>(x.data_ptr()),
                                                        static_cast<uint8_t*>(q.data_ptr()), scales.data_ptr<float>(),
                                                        T, H, round_scale);
  else
    quant_fp8_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), static_cast<uint8_t*>(q.data_ptr()),
        scales.data_ptr<float>(), T, H, round_scale);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace b200ep
