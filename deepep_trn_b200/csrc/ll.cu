// Low-latency dispatch / combine (N4, N5), CUDA-graph capturable, split into a
// send kernel and a receive kernel so ``return_recv_hook`` can defer the wait.
//
// Reference semantics: deep_ep_trn/buffer.py:269-364. The receiver sees
// ``recv_x[EL, R*M, H]`` where each local expert's rows are packed in
// (source rank, source token) order, ``layout_range[e, s] = (start << 32) | count``
// and ``src_info`` holds the source token (-1 past the count). Combine returns one
// row per (token, expert) and the source applies the top-k weights in fp32.
//
// Wire: one row per (token, destination rank), as in the reference, written
// directly into the destination's slot [src][token] of its receive area by
// 16-byte peer stores; fp8 rows are quantised 1x128 in registers on the way out.
// Every (src, token) slot of every destination also gets the token's K global
// expert ids and an epoch flag, so the receiver needs no count exchange: one
// CTA per local expert walks the slots in (src, token) order, waits on each
// flag, and compacts the matching rows into recv_x. No host synchronisation.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ops.h"

namespace b200ep {

constexpr int kLLSendThreads = 256;
constexpr int kLLRecvThreads = 512;

__device__ __forceinline__ uint32_t ldv_u32(const uint32_t* p) { return *reinterpret_cast<const volatile uint32_t*>(p); }

// ============================================================================ dispatch send
struct LLSendArgs {
  HeapView hv;
  const uint8_t* x;   // [T, H] bf16 (or fp16)
  int64_t x_stride;   // bytes
  int x_fp16;
  const void* topk;
  int topk_i32;
  int T, H, K, E;
  int use_fp8, round_scale;
};

template <typename T16>
__global__ void __launch_bounds__(kLLSendThreads) ll_dispatch_send_kernel(LLSendArgs a) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t e = ldv_u32(&ls->epoch[kEpLLD]) + 1u;
  const int slot = e & 1u;
  const int me = hv.rank, R = hv.R, Mll = hv.cfg.Mll;
  const int64_t rs = hv.L.row_stride;
  const int H = a.H, K = a.K, EL = a.E / R;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kLLSendThreads / 32;
  __shared__ int s_last;

  const int T = min(a.T, Mll);
  if (blockIdx.x == 0 && tid < R)
    st_release_sys64(&hv.sig(tid)->ll_hdr[slot][me], (static_cast<uint64_t>(e) << 32) | static_cast<uint32_t>(T));
  if (a.T > Mll && blockIdx.x == 0 && tid == 0) report_error(hv.status, kCapacity, 4, me, -1, Mll, a.T);

  for (int t = blockIdx.x * nwarps + warp; t < T; t += gridDim.x * nwarps) {
    int32_t g = -1;
    if (lane < K) {
      const int64_t i = static_cast<int64_t>(t) * K + lane;
      g = a.topk_i32 ? static_cast<const int32_t*>(a.topk)[i] : static_cast<int32_t>(static_cast<const int64_t*>(a.topk)[i]);
      if (g >= a.E) g = -1;
    }
    const uint32_t dmask = __reduce_or_sync(0xffffffffu, g >= 0 ? (1u << (g / EL)) : 0u);
    const int64_t slot_row = static_cast<int64_t>(me) * Mll + t;
    const T16* src = reinterpret_cast<const T16*>(a.x + static_cast<int64_t>(t) * a.x_stride);
    if (!a.use_fp8) {
      // bf16 rows: each 16-byte chunk is loaded once and stored to every destination
      for (int c = lane * 8; c < H; c += 256) {
        const int4 v = *reinterpret_cast<const int4*>(src + c);
        for (uint32_t m = dmask; m; m &= m - 1) {
          const int p = __ffs(m) - 1;
          *reinterpret_cast<int4*>(hv.base[p] + hv.L.ll_rows[slot] + slot_row * rs + c * 2) = v;
        }
      }
    } else {
      for (int c = 0; c < H; c += 256) {
        const int off = c + lane * 8;
        const bool act = off < H;
        float v[8];
        load8(v, src + off, act);
        const Quant8 qr = quant8_e4m3(v, a.round_scale);
        if (act) {
          const uint2 q = qr.q;
          const float scale = qr.scale;
          for (uint32_t m = dmask; m; m &= m - 1) {
            const int p = __ffs(m) - 1;
            uint8_t* row = hv.base[p] + hv.L.ll_rows[slot] + slot_row * rs;
            *reinterpret_cast<uint2*>(row + off) = q;
            if ((lane & 15) == 0) reinterpret_cast<float*>(row + H)[off / 128] = scale;
          }
        }
      }
    }
    // ids go to every rank (a non-routed rank learns that it is not a destination)
    if (lane < K)
      for (int p = 0; p < R; ++p) hv.at<int32_t>(p, hv.L.ll_ids[slot])[slot_row * K + lane] = g;
    __syncwarp();
    if (lane < R) {
      fence_sys();
      st_release_sys(hv.at<uint32_t>(lane, hv.L.ll_flags[slot]) + slot_row, e);
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&ls->arrive[kEpLLD], 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && tid == 0) {
    ls->arrive[kEpLLD] = 0;
    ls->epoch[kEpLLD] = e;
  }
}

void ll_dispatch_send(SymmHeap& heap, const at::Tensor& x, const at::Tensor& topk_idx, int64_t num_experts,
                      bool use_fp8, bool round_scale, int64_t num_sms) {
  const c10::cuda::CUDAGuard guard(x.device());
  HeapView hv = heap.view();
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.element_size() == 2, "x must be 16-bit [T, H]");
  TORCH_CHECK(topk_idx.is_contiguous() && topk_idx.dim() == 2, "topk_idx must be contiguous [T, K]");
  LLSendArgs a{};
  a.hv = hv;
  a.x = static_cast<const uint8_t*>(x.data_ptr());
  a.x_stride = x.stride(0) * 2;
  a.x_fp16 = x.scalar_type() == at::kHalf;
  a.topk = topk_idx.data_ptr();
  a.topk_i32 = topk_idx.scalar_type() == at::kInt;
  a.T = static_cast<int>(x.size(0));
  a.H = static_cast<int>(x.size(1));
  a.K = static_cast<int>(topk_idx.size(1));
  a.E = static_cast<int>(num_experts);
  a.use_fp8 = use_fp8;
  a.round_scale = round_scale;
  TORCH_CHECK(a.H % 8 == 0 && a.H <= hv.cfg.H, "low-latency hidden must be a multiple of 8 within the buffer");
  TORCH_CHECK(!use_fp8 || a.H % 128 == 0, "fp8 needs hidden % 128 == 0");
  TORCH_CHECK(a.K <= 32 && a.K <= hv.cfg.K && a.E <= hv.cfg.E && a.E % hv.R == 0, "bad top-k / experts");
  TORCH_CHECK((a.x_stride % 16) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0, "x rows must be 16-byte aligned");
  const int warps_needed = std::max(1, (std::min(a.T, hv.cfg.Mll) + 7) / 8);
  int grid = num_sms > 0 ? static_cast<int>(num_sms) : heap.num_sms();
  grid = std::max(1, std::min(grid, warps_needed));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (a.x_fp16)
    ll_dispatch_send_kernel<__half><<<grid, kLLSendThreads, 0, stream>>>(a);
  else
    ll_dispatch_send_kernel<__nv_bfloat16><<<grid, kLLSendThreads, 0, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ dispatch recv
struct LLRecvArgs {
  HeapView hv;
  uint8_t* recv_x;          // [EL, R*Mll, H] (fp8 or 16-bit)
  uint8_t* recv_scales;     // fp32 [EL, R*Mll, H/128] or ue8m0 bytes [EL, R*Mll, H/128]
  int32_t* recv_count;      // [EL]
  int32_t* src_info;        // [EL, R*Mll]
  int64_t* layout_range;    // [EL, R]
  int32_t* pair_meta;       // [EL, R*Mll]: src * K + k
  int32_t* cum_stats;       // [EL] or null
  int64_t* wait_stats;      // [R] or null
  int H, K, E;
  int use_fp8, ue8m0;
};

__global__ void __launch_bounds__(kLLRecvThreads) ll_dispatch_recv_kernel(LLRecvArgs a) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t e = ldv_u32(&ls->epoch[kEpLLD]);
  const int slot = e & 1u;
  const int me = hv.rank, R = hv.R, Mll = hv.cfg.Mll;
  const int64_t rs = hv.L.row_stride;
  const int H = a.H, K = a.K, EL = a.E / R;
  const int le = blockIdx.x;
  const int32_t want = me * EL + le;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kLLRecvThreads / 32;
  const int64_t RM = static_cast<int64_t>(R) * Mll;
  const int64_t PB = a.use_fp8 ? H : 2LL * H;   // payload bytes
  const int nsb = H / 128;                      // scale blocks

  __shared__ int s_T, s_fail;
  __shared__ int s_wcnt[nwarps];
  __shared__ int s_tok[kLLRecvThreads];
  __shared__ int s_dst[kLLRecvThreads];
  int running = 0;
  if (tid == 0) s_fail = 0;
  for (int s = 0; s < R; ++s) {
    if (tid == 0) {
      const uint64_t* hdr = &hv.sig(me)->ll_hdr[slot][s];
      uint64_t v = ld_acquire_sys64(hdr);
      const uint64_t t0 = global_ns();
      uint32_t spins = 0;
      while (!epoch_reached(static_cast<uint32_t>(v >> 32), e)) {
        if ((++spins & 63u) == 0u && (global_ns() - t0 > hv.timeout_ns || has_error(hv.status))) {
          report_error(hv.status, kTimeoutLLHeader, 5, me, s, e, static_cast<uint32_t>(v >> 32));
          s_fail = 1;
          break;
        }
        v = ld_acquire_sys64(hdr);
      }
      s_T = s_fail ? 0 : static_cast<int>(v & 0xffffffffu);
      if (a.wait_stats && le == 0) atomicAdd(reinterpret_cast<unsigned long long*>(&a.wait_stats[s]),
                                             static_cast<unsigned long long>(global_ns() - t0));
    }
    __syncthreads();
    const int Ts = s_T;
    const int start = running;
    for (int tile = 0; tile < Ts; tile += kLLRecvThreads) {
      const int t = tile + tid;
      int hit = -1;
      if (t < Ts && !s_fail) {
        const int64_t slot_row = static_cast<int64_t>(s) * Mll + t;
        if (wait_epoch(hv.at<uint32_t>(me, hv.L.ll_flags[slot]) + slot_row, e, hv.timeout_ns, hv.status,
                       kTimeoutLLRow, 5, me, s)) {
          const int32_t* ids = hv.at<int32_t>(me, hv.L.ll_ids[slot]) + slot_row * K;
          for (int k = 0; k < K; ++k)
            if (hit < 0 && *reinterpret_cast<const volatile int32_t*>(ids + k) == want) hit = k;
        } else {
          s_fail = 1;
        }
      }
      const uint32_t b = __ballot_sync(0xffffffffu, hit >= 0);
      if (lane == 0) s_wcnt[warp] = __popc(b);
      __syncthreads();
      if (tid == 0) {
        int run = 0;
        for (int w = 0; w < nwarps; ++w) {
          const int c = s_wcnt[w];
          s_wcnt[w] = run;
          run += c;
        }
        s_T = run;  // reuse as the tile total
      }
      __syncthreads();
      const int tile_total = s_T;
      if (hit >= 0) {
        const int q = s_wcnt[warp] + __popc(b & lanemask_lt());
        const int p = running + q;
        s_tok[q] = t;
        s_dst[q] = p;
        a.src_info[le * RM + p] = t;
        a.pair_meta[le * RM + p] = s * K + hit;
      }
      __syncthreads();
      fence_sys();
      for (int q = warp; q < tile_total; q += nwarps) {
        const int t2 = s_tok[q], p = s_dst[q];
        const uint8_t* row = hv.at<uint8_t>(me, hv.L.ll_rows[slot]) + (static_cast<int64_t>(s) * Mll + t2) * rs;
        const int64_t o = le * RM + p;
        warp_copy(a.recv_x + o * PB, row, PB);
        if (a.use_fp8) {
          const float* sc = reinterpret_cast<const float*>(row + H);
          if (a.ue8m0) {
            for (int i = lane; i < nsb; i += 32)
              a.recv_scales[o * nsb + i] = static_cast<uint8_t>((__float_as_uint(sc[i]) >> 23) & 0xFFu);
          } else {
            warp_copy(a.recv_scales + o * nsb * 4, sc, nsb * 4LL);
          }
        }
      }
      running += tile_total;
      __syncthreads();
      if (tid == 0) s_T = Ts;
      __syncthreads();
    }
    if (tid == 0) a.layout_range[le * R + s] = (static_cast<int64_t>(start) << 32) | static_cast<int64_t>(running - start);
    __syncthreads();
  }
  for (int64_t p = running + tid; p < RM; p += kLLRecvThreads) a.src_info[le * RM + p] = -1;
  if (tid == 0) {
    a.recv_count[le] = running;
    if (a.cum_stats) atomicAdd(&a.cum_stats[le], running);
  }
}

void ll_dispatch_recv(SymmHeap& heap, at::Tensor recv_x, const OptTensor& recv_scales, at::Tensor recv_count,
                      at::Tensor src_info, at::Tensor layout_range, at::Tensor pair_meta, int64_t num_experts,
                      bool use_fp8, bool ue8m0, const OptTensor& cum_stats, const OptTensor& wait_stats) {
  const c10::cuda::CUDAGuard guard(recv_x.device());
  HeapView hv = heap.view();
  LLRecvArgs a{};
  a.hv = hv;
  a.recv_x = static_cast<uint8_t*>(recv_x.data_ptr());
  a.H = static_cast<int>(recv_x.size(2));
  a.K = hv.cfg.K;
  a.E = static_cast<int>(num_experts);
  a.use_fp8 = use_fp8;
  a.ue8m0 = ue8m0;
  const int EL = a.E / hv.R;
  TORCH_CHECK(recv_x.size(0) == EL && recv_x.size(1) == int64_t(hv.R) * hv.cfg.Mll, "recv_x shape");
  if (use_fp8) {
    TORCH_CHECK(recv_scales.has_value(), "fp8 needs recv_scales");
    a.recv_scales = static_cast<uint8_t*>(recv_scales->data_ptr());
  }
  a.recv_count = recv_count.data_ptr<int32_t>();
  a.src_info = src_info.data_ptr<int32_t>();
  a.layout_range = layout_range.data_ptr<int64_t>();
  a.pair_meta = pair_meta.data_ptr<int32_t>();
  if (cum_stats.has_value()) a.cum_stats = cum_stats->data_ptr<int32_t>();
  if (wait_stats.has_value()) a.wait_stats = wait_stats->data_ptr<int64_t>();
  ll_dispatch_recv_kernel<<<EL, kLLRecvThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ combine send
struct LCSendArgs {
  HeapView hv;
  const uint8_t* x;     // [EL, R*Mll, H] 16-bit
  int64_t x_row_stride; // bytes between rows
  int64_t x_exp_stride; // bytes between experts
  const int32_t* recv_count;
  const int32_t* src_info;
  const int32_t* pair_meta;
  int H, K, EL, cta_per_expert;
};

__global__ void __launch_bounds__(kLLSendThreads) ll_combine_send_kernel(LCSendArgs a) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t e = ldv_u32(&ls->epoch[kEpLLC]) + 1u;
  const int slot = e & 1u;
  const int R = hv.R, Mll = hv.cfg.Mll, H = a.H, K = a.K;
  const int64_t RM = static_cast<int64_t>(R) * Mll;
  const int64_t RB = 2LL * H;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kLLSendThreads / 32;
  __shared__ int s_last;
  const int le = blockIdx.x / a.cta_per_expert, sub = blockIdx.x % a.cta_per_expert;
  const int count = static_cast<int>(a.recv_count[le] < RM ? a.recv_count[le] : RM);
  for (int p = sub * nwarps + warp; p < count; p += a.cta_per_expert * nwarps) {
    const int t = a.src_info[le * RM + p];
    const int sk = a.pair_meta[le * RM + p];
    const int s = sk / K, k = sk % K;
    if (t < 0 || t >= Mll || s < 0 || s >= R) continue;
    uint8_t* dst = hv.base[s] + hv.L.lc_rows[slot] + (static_cast<int64_t>(t) * K + k) * RB;
    warp_copy(dst, a.x + le * a.x_exp_stride + p * a.x_row_stride, RB);
    __syncwarp();
    if (lane == 0) {
      fence_sys();
      st_release_sys(hv.at<uint32_t>(s, hv.L.lc_flags[slot]) + static_cast<int64_t>(t) * K + k, e);
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&ls->arrive[kEpLLC], 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && tid == 0) {
    ls->arrive[kEpLLC] = 0;
    ls->epoch[kEpLLC] = e;
  }
}

void ll_combine_send(SymmHeap& heap, const at::Tensor& x, const at::Tensor& recv_count, const at::Tensor& src_info,
                     const at::Tensor& pair_meta, int64_t num_experts, int64_t num_sms) {
  const c10::cuda::CUDAGuard guard(x.device());
  HeapView hv = heap.view();
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && x.element_size() == 2, "x must be 16-bit [EL, R*M, H]");
  LCSendArgs a{};
  a.hv = hv;
  a.x = static_cast<const uint8_t*>(x.data_ptr());
  a.x_row_stride = x.stride(1) * 2;
  a.x_exp_stride = x.stride(0) * 2;
  a.recv_count = recv_count.data_ptr<int32_t>();
  a.src_info = src_info.data_ptr<int32_t>();
  a.pair_meta = pair_meta.data_ptr<int32_t>();
  a.H = static_cast<int>(x.size(2));
  a.K = hv.cfg.K;
  a.EL = static_cast<int>(num_experts / hv.R);
  TORCH_CHECK(x.size(0) == a.EL && x.size(1) == int64_t(hv.R) * hv.cfg.Mll, "x shape must be [EL, R*M, H]");
  TORCH_CHECK(a.H % 8 == 0 && a.x_row_stride % 16 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0,
              "x rows must be 16-byte aligned");
  const int sms = num_sms > 0 ? static_cast<int>(num_sms) : heap.num_sms();
  a.cta_per_expert = std::max(1, (2 * sms) / std::max(1, a.EL));
  ll_combine_send_kernel<<<a.EL * a.cta_per_expert, kLLSendThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ combine recv
struct LCRecvArgs {
  HeapView hv;
  const void* topk;
  int topk_i32;
  const float* w;
  uint8_t* out;     // [T, H] bf16
  int T, H, K, E;
};

template <typename T16>
__global__ void __launch_bounds__(kLLSendThreads) ll_combine_recv_kernel(LCRecvArgs a) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t e = ldv_u32(&ls->epoch[kEpLLC]);
  const int slot = e & 1u;
  const int me = hv.rank, H = a.H, K = a.K;
  const int64_t RB = 2LL * H;
  const int lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kLLSendThreads / 32;
  __shared__ float s_w[nwarps][32];
  const uint8_t* rows = hv.at<uint8_t>(me, hv.L.lc_rows[slot]);
  for (int t = blockIdx.x * nwarps + warp; t < a.T; t += gridDim.x * nwarps) {
    float wk = 0.f;
    bool valid = false;
    if (lane < K) {
      const int64_t i = static_cast<int64_t>(t) * K + lane;
      const int64_t g = a.topk_i32 ? static_cast<const int32_t*>(a.topk)[i] : static_cast<const int64_t*>(a.topk)[i];
      valid = g >= 0 && g < a.E;
      wk = valid ? a.w[i] : 0.f;
      if (valid && !wait_epoch(hv.at<uint32_t>(me, hv.L.lc_flags[slot]) + i, e, hv.timeout_ns, hv.status,
                               kTimeoutLLCombine, 6, me, -1))
        valid = false;
    }
    s_w[warp][lane] = valid ? wk : 0.f;
    const uint32_t vmask = __ballot_sync(0xffffffffu, valid);
    __syncwarp();
    fence_sys();
    T16* out = reinterpret_cast<T16*>(a.out) + static_cast<int64_t>(t) * H;
    for (int c = lane * 8; c < H; c += 256) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (uint32_t m = vmask; m; m &= m - 1) {
        const int k = __ffs(m) - 1;
        const float wv = s_w[warp][k];
        const int4 raw = *reinterpret_cast<const int4*>(rows + (static_cast<int64_t>(t) * K + k) * RB + c * 2);
        const T16* h = reinterpret_cast<const T16*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += static_cast<float>(h[i]) * wv;
      }
      int4 o;
      T16* oh = reinterpret_cast<T16*>(&o);
#pragma unroll
      for (int i = 0; i < 8; ++i) oh[i] = static_cast<T16>(acc[i]);
      *reinterpret_cast<int4*>(out + c) = o;
    }
    __syncwarp();
  }
}

void ll_combine_recv(SymmHeap& heap, const at::Tensor& topk_idx, const at::Tensor& topk_w, at::Tensor out,
                     int64_t num_sms) {
  const c10::cuda::CUDAGuard guard(out.device());
  HeapView hv = heap.view();
  TORCH_CHECK(out.is_contiguous() && out.element_size() == 2, "out must be contiguous 16-bit [T, H]");
  TORCH_CHECK(topk_idx.is_contiguous() && topk_w.is_contiguous() && topk_w.scalar_type() == at::kFloat,
              "topk_idx / topk_weights must be contiguous (weights fp32)");
  LCRecvArgs a{};
  a.hv = hv;
  a.topk = topk_idx.data_ptr();
  a.topk_i32 = topk_idx.scalar_type() == at::kInt;
  a.w = topk_w.data_ptr<float>();
  a.out = static_cast<uint8_t*>(out.data_ptr());
  a.T = static_cast<int>(out.size(0));
  a.H = static_cast<int>(out.size(1));
  a.K = static_cast<int>(topk_idx.size(1));
  a.E = hv.cfg.E;
  TORCH_CHECK(a.H % 8 == 0 && a.T <= hv.cfg.Mll && a.K <= hv.cfg.K, "combine shape exceeds the buffer");
  constexpr int nwarps = kLLSendThreads / 32;
  int grid = std::max(1, (a.T + nwarps - 1) / nwarps);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (out.scalar_type() == at::kHalf)
    ll_combine_recv_kernel<__half><<<grid, kLLSendThreads, 0, stream>>>(a);
  else
    ll_combine_recv_kernel<__nv_bfloat16><<<grid, kLLSendThreads, 0, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  (void)num_sms;
}

}  // namespace b200ep
