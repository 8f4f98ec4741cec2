// MoE-layer kernels around the grouped GEMM (N8 backward, N9, N10):
//
//  router_topk        logits [T, E] fp32 -> top-k ids (ties to the lower id) and softmax over
//                     the chosen k; warp per token.
//  router_topk_bwd    d_logits[t, e_k] = w_k * (dw_k - sum_j w_j dw_j), zero elsewhere.
//  permute_*          received rows [N, H] with local top-k ids [N, K] -> expert-major rows
//                     [rows, H]; each expert's segment starts at a multiple of 128 and keeps
//                     row order (deterministic), padding rows are zeroed. Three launches:
//                     per-block expert counts, one-CTA scan (offsets + block bases), scatter.
//  unpermute          y[n] = sum_k w[n, k] * out[pos[n, k]] in fp32 (one bf16 cast).
//  unpermute_bwd      d_out[pos[n, k]] = w[n, k] * dy[n]; dw[n, k] = <out[pos[n, k]], dy[n]>.
//  permute_bwd        dx[n] = sum_k d_rows[pos[n, k]].
//  swiglu_bwd         from d_h and the saved [gate | up] pre-activation (128-column interleave).
//  transpose          bf16 [B, R, C] -> [B, C, R] through 64x64 shared-memory tiles.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>

#include "ops.h"

namespace b200ep {

// ============================================================================ router
template <int EPT>  // experts per lane (E <= 32 * EPT)
__global__ void __launch_bounds__(256) router_topk_kernel(const float* __restrict__ logits, int T, int E, int K,
                                                          int64_t* __restrict__ idx, float* __restrict__ w) {
  const int lane = lane_id();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  float v[EPT];
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? logits[static_cast<int64_t>(t) * E + e] : -INFINITY;
  }
  float sel[32];
  int sid[32];
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bid = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = i * 32 + lane;
      if (e < E && (v[i] > best || (v[i] == best && e < bid))) {
        best = v[i];
        bid = e;
      }
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bid, m);
      if (ob > best || (ob == best && oi < bid)) {
        best = ob;
        bid = oi;
      }
    }
    if (k < 32) {
      sel[k] = best;
      sid[k] = bid;
    }
    if ((bid & 31) == lane) v[bid >> 5] = -INFINITY;  // remove the winner
  }
  // softmax over the chosen k (values are sorted descending: sel[0] is the max)
  if (lane == 0) {
    float sum = 0.f;
    for (int k = 0; k < K; ++k) sum += __expf(sel[k] - sel[0]);
    for (int k = 0; k < K; ++k) {
      idx[static_cast<int64_t>(t) * K + k] = sid[k];
      w[static_cast<int64_t>(t) * K + k] = __expf(sel[k] - sel[0]) / sum;
    }
  }
}

void router_topk(const at::Tensor& logits, int64_t topk, at::Tensor idx, at::Tensor w) {
  const c10::cuda::CUDAGuard guard(logits.device());
  TORCH_CHECK(logits.is_contiguous() && logits.scalar_type() == at::kFloat, "logits must be contiguous fp32");
  const int T = static_cast<int>(logits.size(0)), E = static_cast<int>(logits.size(1)), K = static_cast<int>(topk);
  TORCH_CHECK(K >= 1 && K <= 32 && K <= E && E <= 1024, "need 1 <= k <= 32, k <= E <= 1024");
  if (T == 0) return;
  const int blocks = (T * 32 + 255) / 256;
  auto s = at::cuda::getCurrentCUDAStream();
  const float* l = logits.data_ptr<float>();
  int64_t* ip = idx.data_ptr<int64_t>();
  float* wp = w.data_ptr<float>();
  if (E <= 64) router_topk_kernel<2><<<blocks, 256, 0, s>>>(l, T, E, K, ip, wp);
  else if (E <= 128) router_topk_kernel<4><<<blocks, 256, 0, s>>>(l, T, E, K, ip, wp);
  else if (E <= 256) router_topk_kernel<8><<<blocks, 256, 0, s>>>(l, T, E, K, ip, wp);
  else router_topk_kernel<32><<<blocks, 256, 0, s>>>(l, T, E, K, ip, wp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

__global__ void router_topk_bwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ w,
                                       const float* __restrict__ dw, float* __restrict__ dlogits, int T, int E, int K) {
  const int t = blockIdx.x;
  float* row = dlogits + static_cast<int64_t>(t) * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) row[e] = 0.f;
  __syncthreads();
  if (threadIdx.x == 0) {
    float dot = 0.f;
    for (int k = 0; k < K; ++k) dot += w[t * K + k] * dw[t * K + k];
    for (int k = 0; k < K; ++k) {
      const int64_t e = idx[t * K + k];
      if (e >= 0 && e < E) row[e] = w[t * K + k] * (dw[t * K + k] - dot);
    }
  }
}

void router_topk_bwd(const at::Tensor& idx, const at::Tensor& w, const at::Tensor& dw, at::Tensor dlogits) {
  const c10::cuda::CUDAGuard guard(w.device());
  const int T = static_cast<int>(w.size(0)), K = static_cast<int>(w.size(1)), E = static_cast<int>(dlogits.size(1));
  if (T == 0) return;
  router_topk_bwd_kernel<<<T, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int64_t>(), w.data_ptr<float>(), dw.data_ptr<float>(), dlogits.data_ptr<float>(), T, E, K);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ permute
constexpr int kPermRows = 32;      // rows per block of the count/scatter passes (one warp)
constexpr int kPermMaxExperts = 1024;

// Per 32-row block: cnt[block][e] = #rows of the block routed to local expert e.
template <typename IdxT>
__global__ void __launch_bounds__(32) permute_count_kernel(const IdxT* __restrict__ ids, int N, int K, int EL,
                                                            int32_t* __restrict__ cnt) {
  const int lane = lane_id();
  const int n = blockIdx.x * kPermRows + lane;
  int32_t e_of[32];
  for (int k = 0; k < 32; ++k) e_of[k] = -1;
  if (n < N)
    for (int k = 0; k < K && k < 32; ++k) {
      const int64_t e = static_cast<int64_t>(ids[static_cast<int64_t>(n) * K + k]);
      e_of[k] = (e >= 0 && e < EL) ? static_cast<int32_t>(e) : -1;
    }
  for (int e = 0; e < EL; ++e) {
    bool has = false;
    for (int k = 0; k < K && k < 32; ++k) has |= e_of[k] == e;
    const uint32_t b = __ballot_sync(0xffffffffu, has);
    if (lane == 0) cnt[static_cast<int64_t>(blockIdx.x) * EL + e] = __popc(b);
  }
}

// One CTA: padded segment offsets [EL + 1] and base[block][e] (first row of the block's rows of e).
__global__ void permute_scan_kernel(int32_t* __restrict__ cnt_base, int nblocks, int EL, int align,
                                    int64_t* __restrict__ offsets, int32_t* __restrict__ counts) {
  __shared__ int64_t s_off[kPermMaxExperts + 1];
  for (int e = threadIdx.x; e < EL; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < nblocks; ++b) run += cnt_base[static_cast<int64_t>(b) * EL + e];
    counts[e] = run;
    s_off[e] = (run + align - 1) / align * align;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int e = 0; e < EL; ++e) {
      const int64_t sz = s_off[e];
      s_off[e] = acc;
      acc += sz;
    }
    s_off[EL] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= EL; e += blockDim.x) offsets[e] = s_off[e];
  for (int e = threadIdx.x; e < EL; e += blockDim.x) {
    int64_t run = s_off[e];
    for (int b = 0; b < nblocks; ++b) {
      const int c = cnt_base[static_cast<int64_t>(b) * EL + e];
      cnt_base[static_cast<int64_t>(b) * EL + e] = static_cast<int32_t>(run);
      run += c;
    }
  }
}

// Per 32-row block (one warp): the rows of expert e keep row order. Top-k ids are
// distinct per row, so "row n has e" is one bit per lane and the lane prefix of the
// ballot is the position within the block.
template <typename IdxT>
__global__ void __launch_bounds__(32) permute_scatter_kernel(const IdxT* __restrict__ ids, int N, int K, int EL,
                                                              const int32_t* __restrict__ base,
                                                              int32_t* __restrict__ pos) {
  const int lane = lane_id();
  const int n = blockIdx.x * kPermRows + lane;
  int32_t e_of[32];
  for (int k = 0; k < 32; ++k) e_of[k] = -1;
  if (n < N)
    for (int k = 0; k < K && k < 32; ++k) {
      const int64_t e = static_cast<int64_t>(ids[static_cast<int64_t>(n) * K + k]);
      e_of[k] = (e >= 0 && e < EL) ? static_cast<int32_t>(e) : -1;
      pos[static_cast<int64_t>(n) * K + k] = -1;
    }
  for (int e = 0; e < EL; ++e) {
    int hit_k = -1;
    for (int k = 0; k < K && k < 32; ++k)
      if (e_of[k] == e) hit_k = k;
    const uint32_t b = __ballot_sync(0xffffffffu, hit_k >= 0);
    if (hit_k >= 0)
      pos[static_cast<int64_t>(n) * K + hit_k] =
          base[static_cast<int64_t>(blockIdx.x) * EL + e] + __popc(b & lanemask_lt());
  }
}

// Copy rows to their expert-major slots and zero the padding rows.
__global__ void __launch_bounds__(256) permute_copy_kernel(const uint8_t* __restrict__ x, int64_t x_stride, int N,
                                                           int K, int64_t row_bytes, const int32_t* __restrict__ pos,
                                                           uint8_t* __restrict__ out, const int64_t* __restrict__ offsets,
                                                           const int32_t* __restrict__ counts, int EL) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int GW = (gridDim.x * blockDim.x) >> 5;
  for (int n = gw; n < N; n += GW) {
    for (int k = 0; k < K; ++k) {
      const int p = pos[static_cast<int64_t>(n) * K + k];
      if (p >= 0) warp_copy(out + static_cast<int64_t>(p) * row_bytes, x + static_cast<int64_t>(n) * x_stride, row_bytes);
    }
  }
  // padding rows of every segment
  for (int e = 0; e < EL; ++e) {
    const int64_t s = offsets[e] + counts[e], t = offsets[e + 1];
    for (int64_t r = s + gw; r < t; r += GW) {
      int4* d = reinterpret_cast<int4*>(out + r * row_bytes);
      for (int64_t i = lane_id(); i < row_bytes / 16; i += 32) d[i] = make_int4(0, 0, 0, 0);
    }
  }
}

// The same copy driven by the bulk-copy engine: one thread per CTA streams the CTA's
// source rows into a ring of shared-memory stages (each row read once) and, as each
// lands, issues one bulk store per destination slot (up to K). The other warps zero
// the CTA's share of the padding rows meanwhile. Waits are bounded; a timed-out wait
// sets *error, lets the loads in flight land and stops.
constexpr int kPermCopyThreads = 128;
constexpr int kPermCopyTok = 64;   // tokens per CTA pass (their pos rows are staged in smem)

__global__ void __launch_bounds__(kPermCopyThreads) permute_copy_bulk_kernel(
    const uint8_t* __restrict__ x, int64_t x_stride, int N, int K, int64_t row_bytes, const int32_t* __restrict__ pos,
    uint8_t* __restrict__ out, const int64_t* __restrict__ offsets, const int32_t* __restrict__ counts, int EL,
    int stage_bytes, int nstages, uint32_t* __restrict__ error, uint64_t timeout_ns) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<int64_t>(nstages) * stage_bytes);
  __shared__ int32_t s_pos[kPermCopyTok * 32];
  const int tid = threadIdx.x;
  const int n0 = static_cast<int>(static_cast<int64_t>(N) * blockIdx.x / gridDim.x);
  const int n1 = static_cast<int>(static_cast<int64_t>(N) * (blockIdx.x + 1) / gridDim.x);
  if (tid == 0) {
    for (int i = 0; i < nstages; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  uint32_t phase_bits = 0;
  bool ok = true;
  for (int c0 = n0; c0 < n1; c0 += kPermCopyTok) {
    const int n = min(kPermCopyTok, n1 - c0);
    __syncthreads();  // the previous pass is done with s_pos
    for (int i = tid; i < n * K; i += kPermCopyThreads) s_pos[i] = pos[static_cast<int64_t>(c0) * K + i];
    __syncthreads();
    if (tid == 0 && ok) {
      auto issue = [&](int q) {
        const int st = q % nstages;
        mbar_arrive_expect_tx(&bars[st], static_cast<uint32_t>(row_bytes));
        bulk_load(smem + static_cast<int64_t>(st) * stage_bytes, x + static_cast<int64_t>(c0 + q) * x_stride,
                  static_cast<uint32_t>(row_bytes), &bars[st]);
      };
      const int pro = min(n, nstages);
      for (int q = 0; q < pro; ++q) issue(q);
      for (int m = 0; m < n; ++m) {
        const int st = m % nstages;
        if (!mbar_wait(&bars[st], (phase_bits >> st) & 1u, timeout_ns)) {
          atomicExch(error, 1u);
          const int last = min(n - 1, m >= 1 ? m - 2 + nstages : pro - 1);
          for (int q = m + 1; q <= last; ++q)
            mbar_wait(&bars[q % nstages], (phase_bits >> (q % nstages)) & 1u, timeout_ns);
          ok = false;
          break;
        }
        phase_bits ^= 1u << st;
        const uint8_t* src = smem + static_cast<int64_t>(st) * stage_bytes;
        for (int k = 0; k < K; ++k) {
          const int p = s_pos[m * K + k];
          if (p >= 0) bulk_store(out + static_cast<int64_t>(p) * row_bytes, src, static_cast<uint32_t>(row_bytes));
        }
        bulk_commit();
        const int q = m - 1 + nstages;
        if (m >= 1 && q < n) {
          bulk_wait_read<1>();  // the stores of token m - 1 have read their stage
          issue(q);
        }
      }
      bulk_wait_read<0>();
    }
  }
  // padding rows of every segment: warps 1.. of all CTAs, plain 16-byte stores
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int kZeroWarps = kPermCopyThreads / 32 - 1;
  if (warp >= 1) {
    const int gw = blockIdx.x * kZeroWarps + (warp - 1), GW = gridDim.x * kZeroWarps;
    for (int e = 0; e < EL; ++e) {
      const int64_t s0 = offsets[e] + counts[e], t = offsets[e + 1];
      for (int64_t r = s0 + gw; r < t; r += GW) {
        int4* d = reinterpret_cast<int4*>(out + r * row_bytes);
        for (int64_t i = lane; i < row_bytes / 16; i += 32) d[i] = make_int4(0, 0, 0, 0);
      }
    }
  }
  if (tid == 0) bulk_wait<0>();  // the row stores are complete before the CTA exits
}

// fp8 input (e4m3 rows with one fp32 scale per 128 channels, as an fp8 dispatch delivers
// them): a warp per token reads the row once and stores it to every destination slot of the
// token, either dequantised to bf16 (DEQUANT) or as e4m3 bytes plus the scales (for the fp8
// GEMM; padding rows get zero bytes and scale 1).
template <bool DEQUANT>
__global__ void __launch_bounds__(256) permute_copy_fp8_kernel(const uint8_t* __restrict__ q, int64_t q_stride,
                                                               const float* __restrict__ sc, int64_t s_stride, int N,
                                                               int K, int H, const int32_t* __restrict__ pos,
                                                               void* __restrict__ out_v, float* __restrict__ out_s,
                                                               const int64_t* __restrict__ offsets,
                                                               const int32_t* __restrict__ counts, int EL) {
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(out_v);
  uint8_t* out_q = static_cast<uint8_t*>(out_v);
  const int nsb = H / 128;
  const int lane = lane_id();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int GW = (gridDim.x * blockDim.x) >> 5;
  const int nch = H / 16;  // 16 fp8 channels per chunk
  for (int n = gw; n < N; n += GW) {
    int p[32];
    int np = 0;
    for (int k = 0; k < K; ++k) {
      const int v = pos[static_cast<int64_t>(n) * K + k];
      if (v >= 0) p[np++] = v;
    }
    if (np == 0) continue;
    const uint8_t* qr = q + static_cast<int64_t>(n) * q_stride;
    const float* sr = sc + static_cast<int64_t>(n) * s_stride;
    if (!DEQUANT) {
      for (int j = lane; j < nch; j += 32) {
        const int4 v = reinterpret_cast<const int4*>(qr)[j];
        for (int i = 0; i < np; ++i) reinterpret_cast<int4*>(out_q + static_cast<int64_t>(p[i]) * H)[j] = v;
      }
      for (int b = lane; b < nsb; b += 32) {
        const float f = sr[b];
        for (int i = 0; i < np; ++i) out_s[static_cast<int64_t>(p[i]) * nsb + b] = f;
      }
      continue;
    }
    for (int j = lane; j < nch; j += 32) {
      const int4 v = reinterpret_cast<const int4*>(qr)[j];
      const float f = sr[j >> 3];  // 8 chunks of 16 per 128-channel block
      const __nv_fp8x2_storage_t* b2 = reinterpret_cast<const __nv_fp8x2_storage_t*>(&v);
      alignas(16) __nv_bfloat162 o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __half2 h = __half2(__nv_cvt_fp8x2_to_halfraw2(b2[i], __NV_E4M3));
        const float2 x2 = __half22float2(h);
        o[i] = __floats2bfloat162_rn(x2.x * f, x2.y * f);
      }
      for (int i = 0; i < np; ++i) {
        int4* d = reinterpret_cast<int4*>(out + static_cast<int64_t>(p[i]) * H) + 2 * j;
        d[0] = reinterpret_cast<const int4*>(o)[0];
        d[1] = reinterpret_cast<const int4*>(o)[1];
      }
    }
  }
  const int64_t row_bytes = DEQUANT ? 2LL * H : H;
  for (int e = 0; e < EL; ++e) {
    const int64_t s0 = offsets[e] + counts[e], t = offsets[e + 1];
    for (int64_t r = s0 + gw; r < t; r += GW) {
      int4* d = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(out_v) + r * row_bytes);
      for (int64_t i = lane; i < row_bytes / 16; i += 32) d[i] = make_int4(0, 0, 0, 0);
      if (!DEQUANT)
        for (int b = lane; b < nsb; b += 32) out_s[r * nsb + b] = 1.f;
    }
  }
}

void permute(const at::Tensor& x, const at::Tensor& ids, int64_t num_local_experts, at::Tensor out, at::Tensor pos,
             at::Tensor offsets, at::Tensor counts, at::Tensor scratch, const OptTensor& error,
             const OptTensor& x_scales, const OptTensor& out_scales) {
  const c10::cuda::CUDAGuard guard(x.device());
  const int N = static_cast<int>(x.size(0)), K = static_cast<int>(ids.size(1)), EL = static_cast<int>(num_local_experts);
  TORCH_CHECK(EL <= kPermMaxExperts, "too many local experts");
  TORCH_CHECK(x.stride(1) == 1 && out.is_contiguous() && ids.is_contiguous(), "layouts");
  const int64_t row_bytes = x.size(1) * x.element_size();
  TORCH_CHECK(row_bytes % 16 == 0, "row bytes must be a multiple of 16");
  const int nblocks = std::max(1, (N + kPermRows - 1) / kPermRows);
  TORCH_CHECK(scratch.numel() >= int64_t(nblocks) * EL, "scratch too small");
  TORCH_CHECK(K <= 32, "top-k above 32 is not supported by permute");
  auto s = at::cuda::getCurrentCUDAStream();
  int32_t* cb = scratch.data_ptr<int32_t>();
  if (ids.scalar_type() == at::kLong) {
    permute_count_kernel<int64_t><<<nblocks, 32, 0, s>>>(ids.data_ptr<int64_t>(), N, K, EL, cb);
  } else {
    permute_count_kernel<int32_t><<<nblocks, 32, 0, s>>>(ids.data_ptr<int32_t>(), N, K, EL, cb);
  }
  permute_scan_kernel<<<1, 1024, 0, s>>>(cb, nblocks, EL, 128, offsets.data_ptr<int64_t>(), counts.data_ptr<int32_t>());
  if (ids.scalar_type() == at::kLong) {
    permute_scatter_kernel<int64_t><<<nblocks, 32, 0, s>>>(ids.data_ptr<int64_t>(), N, K, EL, cb,
                                                           pos.data_ptr<int32_t>());
  } else {
    permute_scatter_kernel<int32_t><<<nblocks, 32, 0, s>>>(ids.data_ptr<int32_t>(), N, K, EL, cb,
                                                           pos.data_ptr<int32_t>());
  }
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  if (x_scales.has_value()) {
    const bool keep = out_scales.has_value();  // e4m3 rows + scales out, else bf16 rows
    TORCH_CHECK(x.element_size() == 1 && out.size(1) == x.size(1) && x.size(1) % 128 == 0 &&
                    x_scales->scalar_type() == at::kFloat && unit_inner(*x_scales) &&
                    x_scales->size(1) * 128 == x.size(1) && x.stride(0) % 16 == 0 &&
                    (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0,
                "fp8 permute: x [N, H] e4m3 (H % 128 == 0, 16-byte aligned rows), scales [N, H/128] fp32");
    TORCH_CHECK(keep ? (out.element_size() == 1 && out_scales->scalar_type() == at::kFloat &&
                        out_scales->is_contiguous() && out_scales->size(0) == out.size(0) &&
                        out_scales->size(1) == x_scales->size(1))
                     : out.scalar_type() == at::kBFloat16,
                "fp8 permute: bf16 rows out, or e4m3 rows + [P, H/128] fp32 scales out");
    auto kern = keep ? permute_copy_fp8_kernel<false> : permute_copy_fp8_kernel<true>;
    kern<<<sms * 4, 256, 0, s>>>(static_cast<const uint8_t*>(x.data_ptr()), x.stride(0), x_scales->data_ptr<float>(),
                                 x_scales->stride(0), N, K, static_cast<int>(x.size(1)), pos.data_ptr<int32_t>(),
                                 out.data_ptr(), keep ? out_scales->data_ptr<float>() : nullptr,
                                 offsets.data_ptr<int64_t>(), counts.data_ptr<int32_t>(), EL);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  const int64_t xs = x.stride(0) * x.element_size();
  const uintptr_t xp = reinterpret_cast<uintptr_t>(x.data_ptr()), op = reinterpret_cast<uintptr_t>(out.data_ptr());
  const bool bulk = error.has_value() && ((xp | op) & 15) == 0 && xs % 16 == 0 && row_bytes <= 65536 &&
                    !std::getenv("B200EP_PERMUTE_WARPCOPY");
  if (bulk) {
    const int stage_bytes = static_cast<int>((row_bytes + 127) / 128 * 128);
    const int nstages = static_cast<int>(std::max<int64_t>(2, std::min<int64_t>(8, (96 * 1024) / stage_bytes)));
    const size_t smem = static_cast<size_t>(nstages) * stage_bytes + nstages * 8;
    static std::atomic<uint64_t> seen{0};
    AT_CUDA_CHECK(set_smem_limit_once(seen, permute_copy_bulk_kernel, 200 * 1024));
    const int grid = std::max(1, std::min(N, sms * 2));
    permute_copy_bulk_kernel<<<grid, kPermCopyThreads, smem, s>>>(
        static_cast<const uint8_t*>(x.data_ptr()), xs, N, K, row_bytes, pos.data_ptr<int32_t>(),
        static_cast<uint8_t*>(out.data_ptr()), offsets.data_ptr<int64_t>(), counts.data_ptr<int32_t>(), EL, stage_bytes,
        nstages, reinterpret_cast<uint32_t*>(error->data_ptr<int32_t>()), 10ull * 1000 * 1000 * 1000);
  } else {
    permute_copy_kernel<<<sms * 4, 256, 0, s>>>(static_cast<const uint8_t*>(x.data_ptr()), xs, N, K, row_bytes,
                                                pos.data_ptr<int32_t>(), static_cast<uint8_t*>(out.data_ptr()),
                                                offsets.data_ptr<int64_t>(), counts.data_ptr<int32_t>(), EL);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ unpermute
// y[n] = sum_k w[n,k] * rows[pos[n,k]]; thread per 8-element chunk, all K loads in flight.
__global__ void __launch_bounds__(256) unpermute_kernel(const __nv_bfloat16* __restrict__ rows, const int32_t* __restrict__ pos,
                                                        const float* __restrict__ w, int N, int K, int H,
                                                        __nv_bfloat16* __restrict__ y) {
  const int nch = H / 8;
  const int64_t total = static_cast<int64_t>(N) * nch;
  for (int64_t it = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; it < total; it += int64_t(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(it / nch), j = static_cast<int>(it % nch);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int4 v[8];
    float wk[8];
    bool ok[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int p = k < K ? pos[static_cast<int64_t>(n) * K + k] : -1;
      ok[k] = p >= 0;
      wk[k] = ok[k] ? w[static_cast<int64_t>(n) * K + k] : 0.f;
      if (ok[k]) v[k] = reinterpret_cast<const int4*>(rows + static_cast<int64_t>(p) * H)[j];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (ok[k]) {
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v[k]);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(h[i]) * wk[k];
      }
    }
    for (int k = 8; k < K; ++k) {
      const int p = pos[static_cast<int64_t>(n) * K + k];
      if (p < 0) continue;
      const float ww = w[static_cast<int64_t>(n) * K + k];
      const int4 r = reinterpret_cast<const int4*>(rows + static_cast<int64_t>(p) * H)[j];
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(h[i]) * ww;
    }
    int4 o;
    __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) oh[i] = __float2bfloat16_rn(acc[i]);
    reinterpret_cast<int4*>(y + static_cast<int64_t>(n) * H)[j] = o;
  }
}

void unpermute(const at::Tensor& rows, const at::Tensor& pos, const at::Tensor& w, at::Tensor y) {
  const c10::cuda::CUDAGuard guard(rows.device());
  const int N = static_cast<int>(pos.size(0)), K = static_cast<int>(pos.size(1)), H = static_cast<int>(rows.size(1));
  TORCH_CHECK(H % 8 == 0 && rows.is_contiguous() && y.is_contiguous() && w.is_contiguous(), "layouts");
  if (N == 0) return;
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  unpermute_kernel<<<sms * 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(rows.data_ptr()), pos.data_ptr<int32_t>(), w.data_ptr<float>(), N, K, H,
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// d_rows[pos[n,k]] = w[n,k] * dy[n] (warp per (n, k)), dw[n,k] = <rows[pos[n,k]], dy[n]>.
__global__ void __launch_bounds__(256) unpermute_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                            const __nv_bfloat16* __restrict__ rows,
                                                            const int32_t* __restrict__ pos, const float* __restrict__ w,
                                                            int N, int K, int H, __nv_bfloat16* __restrict__ drows,
                                                            float* __restrict__ dw, const int64_t* __restrict__ offsets,
                                                            const int32_t* __restrict__ counts, int EL) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int GW = (gridDim.x * blockDim.x) >> 5;
  const int lane = lane_id();
  for (int64_t it = gw; it < static_cast<int64_t>(N) * K; it += GW) {
    const int n = static_cast<int>(it / K), k = static_cast<int>(it % K);
    const int p = pos[it];
    if (p < 0) {
      if (dw && lane == 0) dw[it] = 0.f;
      continue;
    }
    const float ww = w[it];
    float dot = 0.f;
    const int4* dyr = reinterpret_cast<const int4*>(dy + static_cast<int64_t>(n) * H);
    const int4* rr = reinterpret_cast<const int4*>(rows + static_cast<int64_t>(p) * H);
    int4* dr = reinterpret_cast<int4*>(drows + static_cast<int64_t>(p) * H);
    for (int j = lane; j < H / 8; j += 32) {
      const int4 a = dyr[j];
      const int4 b = rr[j];
      const __nv_bfloat16* ah = reinterpret_cast<const __nv_bfloat16*>(&a);
      const __nv_bfloat16* bh = reinterpret_cast<const __nv_bfloat16*>(&b);
      int4 o;
      __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float av = __bfloat162float(ah[i]);
        dot += av * __bfloat162float(bh[i]);
        oh[i] = __float2bfloat16_rn(av * ww);
      }
      dr[j] = o;
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, m);
    if (dw && lane == 0) dw[it] = dot;
  }
  // padding rows feed the weight-gradient GEMMs: they must be zeros, not stale memory
  for (int e = 0; e < EL; ++e) {
    const int64_t s = offsets[e] + counts[e], t = offsets[e + 1];
    for (int64_t r = s + gw; r < t; r += GW) {
      int4* d = reinterpret_cast<int4*>(drows + r * H);
      for (int i = lane; i < H / 8; i += 32) d[i] = make_int4(0, 0, 0, 0);
    }
  }
}

void unpermute_bwd(const at::Tensor& dy, const at::Tensor& rows, const at::Tensor& pos, const at::Tensor& w,
                   at::Tensor drows, const c10::optional<at::Tensor>& dw, const at::Tensor& offsets,
                   const at::Tensor& counts) {
  const c10::cuda::CUDAGuard guard(dy.device());
  const int N = static_cast<int>(pos.size(0)), K = static_cast<int>(pos.size(1)), H = static_cast<int>(dy.size(1));
  TORCH_CHECK(H % 8 == 0 && dy.is_contiguous() && rows.is_contiguous() && drows.is_contiguous(), "layouts");
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  unpermute_bwd_kernel<<<sms * 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(rows.data_ptr()),
      pos.data_ptr<int32_t>(), w.data_ptr<float>(), N, K, H, reinterpret_cast<__nv_bfloat16*>(drows.data_ptr()),
      dw.has_value() ? dw->data_ptr<float>() : nullptr, offsets.data_ptr<int64_t>(), counts.data_ptr<int32_t>(),
      static_cast<int>(counts.numel()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dx[n] = sum_k d_rows[pos[n,k]] (fp32 accumulate).
__global__ void __launch_bounds__(256) permute_bwd_kernel(const __nv_bfloat16* __restrict__ drows,
                                                          const int32_t* __restrict__ pos, int N, int K, int H,
                                                          __nv_bfloat16* __restrict__ dx) {
  const int nch = H / 8;
  const int64_t total = static_cast<int64_t>(N) * nch;
  for (int64_t it = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; it < total; it += int64_t(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(it / nch), j = static_cast<int>(it % nch);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < K; ++k) {
      const int p = pos[static_cast<int64_t>(n) * K + k];
      if (p < 0) continue;
      const int4 r = reinterpret_cast<const int4*>(drows + static_cast<int64_t>(p) * H)[j];
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += __bfloat162float(h[i]);
    }
    int4 o;
    __nv_bfloat16* oh = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) oh[i] = __float2bfloat16_rn(acc[i]);
    reinterpret_cast<int4*>(dx + static_cast<int64_t>(n) * H)[j] = o;
  }
}

void permute_bwd(const at::Tensor& drows, const at::Tensor& pos, at::Tensor dx) {
  const c10::cuda::CUDAGuard guard(drows.device());
  const int N = static_cast<int>(pos.size(0)), K = static_cast<int>(pos.size(1)), H = static_cast<int>(dx.size(1));
  TORCH_CHECK(H % 8 == 0 && drows.is_contiguous() && dx.is_contiguous(), "layouts");
  if (N == 0) return;
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  permute_bwd_kernel<<<sms * 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(drows.data_ptr()), pos.data_ptr<int32_t>(), N, K, H,
      reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ SwiGLU backward
// pre [rows, 2I] interleaved in 128-column blocks (gate block, up block); dh [rows, I].
// d_pre[gate j] = dh * up * silu'(gate), d_pre[up j] = dh * silu(gate).
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh,
                                                         const __nv_bfloat16* __restrict__ pre, int64_t rows, int I,
                                                         __nv_bfloat16* __restrict__ dpre) {
  const int64_t total = rows * (I / 8);
  for (int64_t it = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; it < total; it += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = it / (I / 8);
    const int j = static_cast<int>(it % (I / 8)) * 8;  // column in I space
    const int blk = j / 128, within = j % 128;
    const int64_t gcol = static_cast<int64_t>(blk) * 256 + within, ucol = gcol + 128;
    const int4 dv = *reinterpret_cast<const int4*>(dh + r * I + j);
    const int4 gv = *reinterpret_cast<const int4*>(pre + r * 2 * I + gcol);
    const int4 uv = *reinterpret_cast<const int4*>(pre + r * 2 * I + ucol);
    const __nv_bfloat16* d = reinterpret_cast<const __nv_bfloat16*>(&dv);
    const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&gv);
    const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&uv);
    int4 og, ou;
    __nv_bfloat16* ogh = reinterpret_cast<__nv_bfloat16*>(&og);
    __nv_bfloat16* ouh = reinterpret_cast<__nv_bfloat16*>(&ou);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float gf = __bfloat162float(g[i]), uf = __bfloat162float(u[i]), df = __bfloat162float(d[i]);
      const float sg = 1.f / (1.f + __expf(-gf));
      const float silu = gf * sg;
      ogh[i] = __float2bfloat16_rn(df * uf * sg * (1.f + gf * (1.f - sg)));
      ouh[i] = __float2bfloat16_rn(df * silu);
    }
    *reinterpret_cast<int4*>(dpre + r * 2 * I + gcol) = og;
    *reinterpret_cast<int4*>(dpre + r * 2 * I + ucol) = ou;
  }
}

void swiglu_bwd(const at::Tensor& dh, const at::Tensor& pre, at::Tensor dpre) {
  const c10::cuda::CUDAGuard guard(dh.device());
  const int64_t rows = dh.size(0);
  const int I = static_cast<int>(dh.size(1));
  TORCH_CHECK(I % 128 == 0 && pre.size(1) == 2 * I && dh.is_contiguous() && pre.is_contiguous(), "layouts");
  if (rows == 0) return;
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  swiglu_bwd_kernel<<<sms * 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()),
      rows, I, reinterpret_cast<__nv_bfloat16*>(dpre.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ transpose
// [B, R, C] -> [B, C, R], bf16, 64x64 tiles through padded shared memory.
__global__ void __launch_bounds__(256) transpose_kernel(const uint16_t* __restrict__ in, uint16_t* __restrict__ out,
                                                        int64_t R, int64_t C, int64_t in_ld, int64_t out_ld,
                                                        int64_t in_bs, int64_t out_bs) {
  __shared__ uint16_t tile[64][66];
  const int64_t b = blockIdx.z;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 64, c0 = static_cast<int64_t>(blockIdx.x) * 64;
  const uint16_t* src = in + b * in_bs;
  uint16_t* dst = out + b * out_bs;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
  for (int i = ty; i < 64; i += 8) {
    const int64_t r = r0 + i;
    for (int j = tx; j < 64; j += 32) {
      const int64_t c = c0 + j;
      tile[i][j] = (r < R && c < C) ? src[r * in_ld + c] : 0;
    }
  }
  __syncthreads();
  for (int i = ty; i < 64; i += 8) {
    const int64_t c = c0 + i;
    for (int j = tx; j < 64; j += 32) {
      const int64_t r = r0 + j;
      if (r < R && c < C) dst[c * out_ld + r] = tile[j][i];
    }
  }
}

void transpose(const at::Tensor& in, at::Tensor out) {
  const c10::cuda::CUDAGuard guard(in.device());
  TORCH_CHECK(in.element_size() == 2 && out.element_size() == 2, "16-bit tensors");
  const bool batched = in.dim() == 3;
  const int64_t B = batched ? in.size(0) : 1;
  const int64_t R = in.size(-2), C = in.size(-1);
  TORCH_CHECK(in.stride(-1) == 1 && out.stride(-1) == 1, "unit inner stride");
  dim3 grid(static_cast<unsigned>((C + 63) / 64), static_cast<unsigned>((R + 63) / 64), static_cast<unsigned>(B));
  if (R == 0 || C == 0 || B == 0) return;
  transpose_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      static_cast<const uint16_t*>(in.data_ptr()), static_cast<uint16_t*>(out.data_ptr()), R, C, in.stride(-2),
      out.stride(-2), batched ? in.stride(0) : 0, batched ? out.stride(0) : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace b200ep
