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

// Inverse of the above: e4m3 [T, H] with fp32 scales [T, H/128] -> bf16 (scale * value,
// rounded once). A thread per 16 channels.
__global__ void __launch_bounds__(256) dequant_fp8_kernel(const uint8_t* __restrict__ q, const float* __restrict__ sc,
                                                          __nv_bfloat16* __restrict__ out, int64_t chunks, int H) {
  const int cpr = H / 16;  // chunks per row
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < chunks; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t t = i / cpr;
    const int j = static_cast<int>(i % cpr);
    const int4 v = reinterpret_cast<const int4*>(q)[i];
    const float f = sc[t * (H / 128) + (j >> 3)];
    const __nv_fp8x2_storage_t* b2 = reinterpret_cast<const __nv_fp8x2_storage_t*>(&v);
    alignas(16) __nv_bfloat162 o[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 x2 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(b2[k], __NV_E4M3)));
      o[k] = __floats2bfloat162_rn(x2.x * f, x2.y * f);
    }
    reinterpret_cast<int4*>(out)[2 * i] = reinterpret_cast<const int4*>(o)[0];
    reinterpret_cast<int4*>(out)[2 * i + 1] = reinterpret_cast<const int4*>(o)[1];
  }
}

void dequant_fp8(const at::Tensor& q, const at::Tensor& scales, at::Tensor out) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.is_contiguous() && scales.is_contiguous() && out.is_contiguous(), "contiguous tensors expected");
  const int H = static_cast<int>(q.size(-1));
  TORCH_CHECK(H % 128 == 0 && q.element_size() == 1, "q must be e4m3 [.., H] with H % 128 == 0");
  const int64_t T = q.numel() / H;
  TORCH_CHECK(scales.scalar_type() == at::kFloat && scales.numel() == T * (H / 128), "scales must be fp32 [.., H/128]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.numel() == q.numel(), "out must be bf16 shaped like q");
  const int64_t chunks = T * (H / 16);
  if (chunks == 0) return;
  const int blocks = static_cast<int>(std::min<int64_t>((chunks + 255) / 256, 148 * 16));
  dequant_fp8_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      static_cast<const uint8_t*>(q.data_ptr()), scales.data_ptr<float>(),
      static_cast<__nv_bfloat16*>(out.data_ptr()), chunks, H);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace b200ep
