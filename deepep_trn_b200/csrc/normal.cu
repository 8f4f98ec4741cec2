// Normal-mode dispatch and combine over NVLink peer memory (N2, N3, N6 fused).
//
// Reference semantics: deep_ep_trn/buffer.py:169-266. Received rows are ordered
// by (source rank, source token); combine sums each token's returned rows in
// fp32 and casts once. The reference packs rows on the host and runs one
// fixed-slot all-to-all-v per op; here:
//
//  dispatch = nd_prepare (every rank stages its tokens in its own symmetric heap,
//             optionally quantising to fp8 1x128 on the way, builds its per-destination
//             token lists with a block scan, exchanges counts through peer flags and
//             publishes the receive size in host-mapped memory)
//           + nd_pull   (each receiver pulls exactly its rows from the peers'
//             staging with TMA bulk loads into shared memory and bulk stores into
//             recv_x: no pack/unpack pass and no slot padding).
//  combine  = nc_combine (one cooperative kernel: push each row back into its source's
//             return block with 16-byte peer stores, signal, then every source
//             reduces its tokens' rows in fp32, adds the optional bias, casts).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>

#include "ops.h"

namespace b200ep {

constexpr int kPrepThreads = 512;
constexpr int kPrepMaxExperts = 8192;
constexpr int kScanBytes = 16384;  // is_token_in_rank bytes staged per scan chunk
constexpr int kPullThreads = 256;
constexpr int kPullChunk = 256;
constexpr int kCombThreads = 512;

__device__ __forceinline__ int32_t ld_volatile_i32(const int32_t* p) {
  return *reinterpret_cast<const volatile int32_t*>(p);
}
__device__ __forceinline__ float ld_volatile_f32(const float* p) {
  return *reinterpret_cast<const volatile float*>(p);
}
__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// ============================================================================ prepare
struct NdPrepArgs {
  HeapView hv;
  const uint8_t* x;
  int64_t x_stride;      // bytes between rows of x
  const float* xs;       // pre-quantised scales [T, H/128] (mode 1)
  int64_t xs_stride;     // elements
  int mode;              // 0: 16-bit payload, 1: fp8 payload + scales given, 2: quantise 16-bit -> fp8
  int x_fp16;
  int round_scale;
  const void* topk;       // [T, K] or null (cached dispatch)
  int topk_i32;
  const float* topk_w;
  const int32_t* nte;     // caller's num_tokens_per_expert [E]
  int has_nte;            // explicit: an empty topk tensor may have a null pointer
  const bool* in_rank;
  int32_t* token_pos;    // [T, R]
  int64_t* recv_off;     // [R + 1] copy for the handle
  int T, H, K, E;
  uint64_t ticket;
  int local_direct;      // the receiver reads its own rows from x directly: stage only rows peers need
};

__global__ void __launch_bounds__(kPrepThreads) nd_prepare_kernel(NdPrepArgs a) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t e = ld_volatile_u32(&ls->epoch[kEpND]) + 1u;
  const int slot = e & 1u;
  const int me = hv.rank, R = hv.R, M = hv.cfg.M;
  const int64_t rs = hv.L.row_stride;
  const int T = a.T, H = a.H, K = a.K;
  uint8_t* stage_x = hv.at<uint8_t>(me, hv.L.nd_x[slot]);
  int32_t* stage_topk = hv.at<int32_t>(me, hv.L.nd_topk[slot]);
  float* stage_w = hv.at<float>(me, hv.L.nd_w[slot]);
  int32_t* stage_lists = hv.at<int32_t>(me, hv.L.nd_lists[slot]);

  __shared__ int32_t s_cnt[B200EP_MAX_RANKS][kPrepThreads / 32];
  __shared__ int32_t s_base[B200EP_MAX_RANKS];
  __shared__ int s_last, s_fail;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kPrepThreads / 32;

  if (T > M) {
    if (blockIdx.x == 0 && tid == 0) report_error(hv.status, kCapacity, 1, me, -1, M, T);
  }
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrPrepStart] = global_ns();

  // ---------------------------------------------------------------- CTA 0: per-destination scan
  // Each thread owns a contiguous chunk of tokens; one block-wide exclusive scan per
  // destination gives every (token, destination) its row in that destination's list,
  // in token order.
  if (blockIdx.x == 0) {
    const int Tc = min(T, M);
    __shared__ __align__(16) uint8_t s_mask[kScanBytes];
    if (tid < R) s_base[tid] = 0;
    const int TC = kScanBytes / R;  // tokens per chunk staged in shared memory
    for (int cs = 0; cs < Tc; cs += TC) {
      const int n = min(TC, Tc - cs);
      const int nbytes = n * R;
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.in_rank) + static_cast<int64_t>(cs) * R;
      if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        for (int i = tid; i < nbytes / 16; i += kPrepThreads)
          reinterpret_cast<int4*>(s_mask)[i] = reinterpret_cast<const int4*>(src)[i];
        for (int i = (nbytes / 16) * 16 + tid; i < nbytes; i += kPrepThreads) s_mask[i] = src[i];
      } else {
        for (int i = tid; i < nbytes; i += kPrepThreads) s_mask[i] = src[i];
      }
      __syncthreads();
      const int tpt = (n + kPrepThreads - 1) / kPrepThreads;
      const int c0 = min(n, tid * tpt), c1 = min(n, c0 + tpt);
      int cnt[B200EP_MAX_RANKS];
#pragma unroll
      for (int r = 0; r < B200EP_MAX_RANKS; ++r) cnt[r] = 0;
      for (int t = c0; t < c1; ++t) {
#pragma unroll
        for (int r = 0; r < B200EP_MAX_RANKS; ++r)
          if (r < R && s_mask[t * R + r]) ++cnt[r];
      }
      int incl[B200EP_MAX_RANKS];
#pragma unroll
      for (int r = 0; r < B200EP_MAX_RANKS; ++r) {
        if (r >= R) continue;
        int v = cnt[r];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, v, d);
          if (lane >= d) v += u;
        }
        incl[r] = v;
        if (lane == 31) s_cnt[r][warp] = v;
      }
      __syncthreads();
      if (tid < R) {
        int run = s_base[tid];
        for (int w = 0; w < nwarps; ++w) {
          const int c = s_cnt[tid][w];
          s_cnt[tid][w] = run;
          run += c;
        }
        s_base[tid] = run;  // rows for destination tid so far
      }
      __syncthreads();
      int off[B200EP_MAX_RANKS];
#pragma unroll
      for (int r = 0; r < B200EP_MAX_RANKS; ++r)
        if (r < R) off[r] = s_cnt[r][warp] + incl[r] - cnt[r];
      for (int t = c0; t < c1; ++t) {
        int32_t* pos_row = a.token_pos + static_cast<int64_t>(cs + t) * R;
#pragma unroll
        for (int r = 0; r < B200EP_MAX_RANKS; ++r) {
          if (r >= R) continue;
          if (s_mask[t * R + r]) {
            pos_row[r] = off[r];
            stage_lists[static_cast<int64_t>(r) * M + off[r]] = cs + t;
            ++off[r];
          } else {
            pos_row[r] = -1;
          }
        }
      }
      __syncthreads();
    }
    int32_t* stage_counts = hv.at<int32_t>(me, hv.L.nd_counts[slot]);
    int32_t* stage_nte = hv.at<int32_t>(me, hv.L.nd_nte[slot]);
    if (tid < R) stage_counts[tid] = s_base[tid];
    if (a.has_nte)
      for (int i = tid; i < a.E; i += kPrepThreads) stage_nte[i] = a.nte[i];
    if (tid == 0) ls->trace[kTrPrepScanDone] = global_ns();
  }

  // ---------------------------------------------------------------- copiers: stage rows + top-k
  if (gridDim.x == 1 || blockIdx.x > 0) {
    const int cta = gridDim.x == 1 ? 0 : blockIdx.x - 1;
    const int ncta = gridDim.x == 1 ? 1 : gridDim.x - 1;
    const int gw = cta * nwarps + warp, GW = ncta * nwarps;
    const int Tc = min(T, M);
    for (int t = gw; t < Tc; t += GW) {
      uint8_t* dst = stage_x + static_cast<int64_t>(t) * rs;
      const uint8_t* src = a.x + static_cast<int64_t>(t) * a.x_stride;
      bool stage = true;
      if (a.local_direct) {
        const bool peer = lane < R && lane != me && a.in_rank[static_cast<int64_t>(t) * R + lane];
        stage = __any_sync(0xffffffffu, peer);
      }
      if (!stage) {
        // only this rank receives the token: the pull reads it from x
      } else if (a.mode == 0) {
        warp_copy(dst, src, 2LL * H);
      } else if (a.mode == 1) {
        warp_copy(dst, src, H);
        warp_copy(dst + H, a.xs + static_cast<int64_t>(t) * a.xs_stride, (H / 128) * 4);
      } else if (a.x_fp16) {
        warp_quant_row<__half>(dst, reinterpret_cast<float*>(dst + H), reinterpret_cast<const __half*>(src), H, a.round_scale);
      } else {
        warp_quant_row<__nv_bfloat16>(dst, reinterpret_cast<float*>(dst + H), reinterpret_cast<const __nv_bfloat16*>(src), H, a.round_scale);
      }
      if (lane < K) {
        const int64_t i = static_cast<int64_t>(t) * K + lane;
        int32_t g = -1;
        if (a.topk) g = a.topk_i32 ? static_cast<const int32_t*>(a.topk)[i]
                                   : static_cast<int32_t>(static_cast<const int64_t*>(a.topk)[i]);
        stage_topk[i] = g;
        stage_w[i] = a.topk_w ? a.topk_w[i] : 0.f;
      }
    }
  }

  // ---------------------------------------------------------------- grid completion
  // staging is local memory that peers read after the last CTA's system-scope release,
  // so a GPU-scope fence before the arrival is enough here
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&ls->arrive[kEpND], 1u);
    s_last = (prev == gridDim.x - 1);
    s_fail = 0;
  }
  __syncthreads();
  if (!s_last) return;

  // ---------------------------------------------------------------- last CTA: notify
  if (tid == 0) ls->trace[kTrPrepCopiesDone] = global_ns();
  if (tid < R) {
    fence_sys();  // acquire side of the arrival counter, then release to the peer
    st_release_sys(&hv.sig(tid)->nd_ready[slot][me], e);
  }
  if (tid < R) {
    if (!wait_epoch(&hv.sig(me)->nd_ready[slot][tid], e, hv.timeout_ns, hv.status, kTimeoutReady, 1, me, tid))
      atomicExch(&s_fail, 1);
  }
  __syncthreads();
  if (tid == 0) ls->trace[kTrPrepPeersReady] = global_ns();
  __shared__ int32_t s_rc[B200EP_MAX_RANKS];
  if (tid < R) {
    int32_t c = s_fail ? 0 : ld_volatile_i32(hv.at<int32_t>(tid, hv.L.nd_counts[slot]) + me);
    if (c < 0 || c > M) {
      report_error(hv.status, kCapacity, 1, me, tid, M, static_cast<uint32_t>(c));
      c = 0;
    }
    s_rc[tid] = c;
  }
  __syncthreads();
  HostPage* host = hv.host;
  if (tid == 0) {
    int64_t off = 0;
    for (int s = 0; s < R; ++s) {
      ls->nd_recv_off[slot][s] = off;
      if (a.recv_off) a.recv_off[s] = off;
      host->notify.recv_counts[s] = s_rc[s];
      off += s_rc[s];
    }
    ls->nd_recv_off[slot][R] = off;
    ls->nd_num_recv[slot] = off;
    if (a.recv_off) a.recv_off[R] = off;
    host->notify.num_recv = off;
  }
  const int EL = a.E / R;
  if (a.has_nte) {
    for (int le = tid; le < EL && le < 1024; le += kPrepThreads) {
      int32_t sum = 0;
      if (!s_fail)
        for (int s = 0; s < R; ++s) sum += ld_volatile_i32(hv.at<int32_t>(s, hv.L.nd_nte[slot]) + me * EL + le);
      host->notify.per_expert[le] = sum;
    }
  }
  __syncthreads();
  if (tid == 0) {
    ls->epoch[kEpND] = e;
    ls->arrive[kEpND] = 0;
    __threadfence_system();
    st_release_sys64(const_cast<uint64_t*>(&host->notify.ticket), a.ticket);
    ls->trace[kTrPrepNotified] = global_ns();
  }
}

void nd_prepare(SymmHeap& heap, const at::Tensor& x, const OptTensor& x_scales, int64_t mode, bool round_scale,
                const OptTensor& topk_idx, const OptTensor& topk_w, const OptTensor& nte, const at::Tensor& in_rank,
                at::Tensor token_pos, at::Tensor recv_off, int64_t num_experts, int64_t ticket, int64_t num_sms) {
  const c10::cuda::CUDAGuard guard(x.device());
  HeapView hv = heap.view();
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [T, H] with unit inner stride");
  TORCH_CHECK(in_rank.is_contiguous() && in_rank.scalar_type() == at::kBool && in_rank.size(1) == hv.R,
              "is_token_in_rank must be a contiguous [T, R] bool tensor");
  TORCH_CHECK(token_pos.is_contiguous() && token_pos.scalar_type() == at::kInt, "token_pos must be int32");
  TORCH_CHECK(recv_off.numel() == hv.R + 1 && recv_off.scalar_type() == at::kLong, "recv_off must be [R+1] int64");
  TORCH_CHECK(num_experts <= kPrepMaxExperts && num_experts <= hv.cfg.E, "num_experts exceeds the buffer");
  NdPrepArgs a{};
  a.hv = hv;
  a.T = static_cast<int>(x.size(0));
  a.H = static_cast<int>(x.size(1));
  TORCH_CHECK(a.H <= hv.cfg.H, "hidden exceeds the buffer's hidden size");
  a.x = static_cast<const uint8_t*>(x.data_ptr());
  a.x_stride = x.stride(0) * x.element_size();
  a.mode = static_cast<int>(mode);
  if (mode == 0) {
    TORCH_CHECK(x.element_size() == 2, "16-bit payload expected");
  } else {
    TORCH_CHECK(a.H % 128 == 0, "fp8 dispatch needs hidden % 128 == 0");
  }
  if (mode == 1) {
    TORCH_CHECK(x.element_size() == 1 && x_scales.has_value(), "fp8 input needs (x_fp8, scales)");
    TORCH_CHECK(x_scales->scalar_type() == at::kFloat && unit_inner(*x_scales), "scales must be fp32");
    a.xs = x_scales->data_ptr<float>();
    a.xs_stride = x_scales->stride(0);
  }
  if (mode == 2) {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kHalf, "quantise needs bf16/fp16 x");
    TORCH_CHECK(x.is_contiguous(), "quantise needs contiguous x");
  }
  a.x_fp16 = x.scalar_type() == at::kHalf;
  a.round_scale = round_scale;
  a.K = topk_idx.has_value() ? static_cast<int>(topk_idx->size(1)) : hv.cfg.K;
  TORCH_CHECK(a.K <= 32 && a.K <= hv.cfg.K, "top-k exceeds the buffer");
  if (topk_idx.has_value()) {
    TORCH_CHECK(topk_idx->is_contiguous(), "topk_idx must be contiguous");
    a.topk = topk_idx->data_ptr();
    a.topk_i32 = topk_idx->scalar_type() == at::kInt;
  }
  if (topk_w.has_value()) {
    TORCH_CHECK(topk_w->is_contiguous() && topk_w->scalar_type() == at::kFloat, "topk_weights must be fp32");
    a.topk_w = topk_w->data_ptr<float>();
  }
  if (nte.has_value()) {
    TORCH_CHECK(nte->is_contiguous() && nte->scalar_type() == at::kInt && nte->numel() == num_experts,
                "num_tokens_per_expert must be a contiguous [E] int32 tensor");
    a.nte = nte->data_ptr<int32_t>();
    a.has_nte = 1;
  }
  a.in_rank = in_rank.data_ptr<bool>();
  a.token_pos = token_pos.data_ptr<int32_t>();
  a.recv_off = recv_off.data_ptr<int64_t>();
  a.E = static_cast<int>(num_experts);
  a.ticket = static_cast<uint64_t>(ticket);
  a.local_direct = mode != 2 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (a.x_stride & 15) == 0 &&
                   (mode == 0 || ((reinterpret_cast<uintptr_t>(a.xs) & 15) == 0 && (a.xs_stride * 4) % 16 == 0));
  int grid = num_sms > 0 ? static_cast<int>(num_sms) : heap.num_sms();
  grid = std::max(1, std::min(grid, std::max(1, a.T / 2 + 1)));
  nd_prepare_kernel<<<grid, kPrepThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ pull
struct NdPullArgs {
  HeapView hv;
  uint8_t* recv_x;
  float* recv_scales;
  void* recv_topk;
  int recv_topk_i32;
  float* recv_w;
  void* recv_src;
  int recv_src_i32;
  int64_t capacity;
  int mode, H, K, E;
  int use_tma, nstages;
  int stage_bytes;
  const uint8_t* local_x;      // rows from this rank come straight from x (null: use staging)
  int64_t local_x_stride;      // bytes
  const uint8_t* local_scales; // fp8 tuple input: scales rows
  int64_t local_scales_stride; // bytes
};

__global__ void __launch_bounds__(kPullThreads) nd_pull_kernel(NdPullArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t e = ld_volatile_u32(&ls->epoch[kEpND]);
  const int slot = e & 1u;
  const int me = hv.rank, R = hv.R, M = hv.cfg.M;
  const int64_t rs = hv.L.row_stride;
  const int H = a.H, K = a.K, EL = a.E / R, lo = me * EL;
  const int64_t MD = a.mode == 0 ? 2LL * H : H;            // payload bytes per row
  const int64_t SB = a.mode == 0 ? 0 : (H / 128) * 4LL;    // scale bytes per row
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kPullThreads / 32;

  __shared__ int64_t s_off[B200EP_MAX_RANKS + 1];
  __shared__ int32_t s_src[kPullChunk];
  __shared__ int32_t s_tok[kPullChunk];
  if (tid <= R) s_off[tid] = ls->nd_recv_off[slot][tid];
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrPullStart] = global_ns();
  __syncthreads();
  int64_t N = s_off[R];
  if (N > a.capacity) {
    if (blockIdx.x == 0 && tid == 0)
      report_error(hv.status, kCapacity, 2, me, -1, static_cast<uint32_t>(a.capacity), static_cast<uint32_t>(N));
    N = a.capacity;
  }
  const int64_t i0 = N * blockIdx.x / gridDim.x, i1 = N * (blockIdx.x + 1) / gridDim.x;

  uint8_t* stages = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<int64_t>(a.nstages) * a.stage_bytes);
  uint32_t phase_bits = 0;
  bool tma_ok = true;
  if (a.use_tma && tid == 0) {
    for (int s = 0; s < a.nstages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    fence_proxy_async_global();  // peer data acquired by the prepare kernel is read through the async proxy
  }
  __syncthreads();

  for (int64_t chunk = i0; chunk < i1; chunk += kPullChunk) {
    const int n = static_cast<int>(i1 - chunk < kPullChunk ? i1 - chunk : kPullChunk);
    for (int q = tid; q < n; q += kPullThreads) {
      const int64_t i = chunk + q;
      int s = 0;
      while (s + 1 < R && s_off[s + 1] <= i) ++s;
      const int64_t j = i - s_off[s];
      s_src[q] = s;
      s_tok[q] = ld_volatile_i32(hv.at<int32_t>(s, hv.L.nd_lists[slot]) + static_cast<int64_t>(me) * M + j);
    }
    __syncthreads();

    if (a.use_tma) {
      if (tid == 0 && tma_ok) {
        auto src_of = [&](int q) -> const uint8_t* {
          if (a.local_x && s_src[q] == me) return a.local_x + static_cast<int64_t>(s_tok[q]) * a.local_x_stride;
          return hv.base[s_src[q]] + hv.L.nd_x[slot] + static_cast<int64_t>(s_tok[q]) * rs;
        };
        auto issue = [&](int q) {
          const int st = q % a.nstages;
          mbar_arrive_expect_tx(&bars[st], static_cast<uint32_t>(MD));
          bulk_load(stages + static_cast<int64_t>(st) * a.stage_bytes, src_of(q), static_cast<uint32_t>(MD), &bars[st]);
        };
        const int pro = min(n, a.nstages);
        for (int q = 0; q < pro; ++q) issue(q);
        for (int m = 0; m < n; ++m) {
          const int st = m % a.nstages;
          if (!mbar_wait(&bars[st], (phase_bits >> st) & 1u, hv.timeout_ns)) {
            report_error(hv.status, kTimeoutReady, 2, me, s_src[m], 0, 0, 1);
            tma_ok = false;
            // let the loads still in flight (at most one per stage) land before the CTA exits
            const int last = min(n - 1, m >= 1 ? m - 2 + a.nstages : pro - 1);
            for (int q = m + 1; q <= last; ++q)
              mbar_wait(&bars[q % a.nstages], (phase_bits >> (q % a.nstages)) & 1u, hv.timeout_ns);
            break;
          }
          phase_bits ^= 1u << st;
          bulk_store(a.recv_x + (chunk + m) * MD, stages + static_cast<int64_t>(st) * a.stage_bytes,
                     static_cast<uint32_t>(MD));
          bulk_commit();
          const int q = m - 1 + a.nstages;
          if (m >= 1 && q < n) {
            bulk_wait_read<1>();
            issue(q);
          }
        }
        bulk_wait_read<0>();
      }
    } else {
      for (int q = warp; q < n; q += nwarps) {
        const uint8_t* src = (a.local_x && s_src[q] == me)
                                 ? a.local_x + static_cast<int64_t>(s_tok[q]) * a.local_x_stride
                                 : hv.base[s_src[q]] + hv.L.nd_x[slot] + static_cast<int64_t>(s_tok[q]) * rs;
        warp_copy(a.recv_x + (chunk + q) * MD, src, MD);
      }
    }
    // metadata (and fp8 scales): warps 1.. when warp 0 drives TMA, every warp otherwise
    const int w0 = a.use_tma ? 1 : 0, nw = a.use_tma ? nwarps - 1 : nwarps;
    for (int q = warp - w0; q >= 0 && q < n; q += nw) {
      const int64_t i = chunk + q;
      const int s = s_src[q], t = s_tok[q];
      if (lane == 0) {
        if (a.recv_src_i32)
          static_cast<int32_t*>(a.recv_src)[i] = t;
        else
          static_cast<int64_t*>(a.recv_src)[i] = t;
      }
      if (a.recv_topk && lane < K) {
        const int64_t ki = static_cast<int64_t>(t) * K + lane;
        const int32_t g = ld_volatile_i32(hv.at<int32_t>(s, hv.L.nd_topk[slot]) + ki);
        const bool local = g >= lo && g < lo + EL;
        const int64_t o = i * K + lane;
        if (a.recv_topk_i32)
          static_cast<int32_t*>(a.recv_topk)[o] = local ? g - lo : -1;
        else
          static_cast<int64_t*>(a.recv_topk)[o] = local ? g - lo : -1;
        if (a.recv_w) a.recv_w[o] = local ? ld_volatile_f32(hv.at<float>(s, hv.L.nd_w[slot]) + ki) : 0.f;
      }
      if (SB) {
        const uint8_t* src = (a.local_x && s == me)
                                 ? a.local_scales + static_cast<int64_t>(t) * a.local_scales_stride
                                 : hv.base[s] + hv.L.nd_x[slot] + static_cast<int64_t>(t) * rs + H;
        warp_copy(reinterpret_cast<uint8_t*>(a.recv_scales) + i * SB, src, SB);
      }
    }
    __syncthreads();
  }
  if (a.use_tma && tid == 0) bulk_wait<0>();
  // last CTA stamps the end of the pull
  __syncthreads();
  if (tid == 0 && atomicAdd(&ls->arrive2[kEpND], 1u) == gridDim.x - 1) {
    ls->arrive2[kEpND] = 0;
    ls->trace[kTrPullEnd] = global_ns();
  }
}

void nd_pull(SymmHeap& heap, at::Tensor recv_x, const OptTensor& recv_scales, const OptTensor& recv_topk,
             const OptTensor& recv_w, at::Tensor recv_src, int64_t mode, int64_t num_experts, int64_t num_sms,
             bool use_tma, const OptTensor& local_x, const OptTensor& local_scales) {
  const c10::cuda::CUDAGuard guard(recv_x.device());
  HeapView hv = heap.view();
  NdPullArgs a{};
  a.hv = hv;
  TORCH_CHECK(recv_x.is_contiguous(), "recv_x must be contiguous");
  a.recv_x = static_cast<uint8_t*>(recv_x.data_ptr());
  a.capacity = recv_x.size(0);
  a.H = static_cast<int>(recv_x.size(1));
  a.mode = static_cast<int>(mode);
  a.E = static_cast<int>(num_experts);
  a.K = hv.cfg.K;
  if (mode != 0) {
    TORCH_CHECK(recv_scales.has_value() && recv_scales->is_contiguous(), "fp8 dispatch needs recv_scales");
    a.recv_scales = recv_scales->data_ptr<float>();
  }
  if (recv_topk.has_value()) {
    a.recv_topk = recv_topk->data_ptr();
    a.recv_topk_i32 = recv_topk->scalar_type() == at::kInt;
    a.K = static_cast<int>(recv_topk->size(1));
  }
  if (recv_w.has_value()) a.recv_w = recv_w->data_ptr<float>();
  a.recv_src = recv_src.data_ptr();
  a.recv_src_i32 = recv_src.scalar_type() == at::kInt;
  // same rule as nd_prepare's local_direct: rows for this rank were not staged in that case
  if (local_x.has_value() && mode != 2) {
    const uintptr_t xp = reinterpret_cast<uintptr_t>(local_x->data_ptr());
    const int64_t xs = local_x->stride(0) * local_x->element_size();
    bool ok = (xp & 15) == 0 && (xs & 15) == 0;
    if (mode == 1) {
      TORCH_CHECK(local_scales.has_value(), "fp8 input needs its scales");
      const uintptr_t sp = reinterpret_cast<uintptr_t>(local_scales->data_ptr());
      ok = ok && (sp & 15) == 0 && (local_scales->stride(0) * 4) % 16 == 0;
      a.local_scales = static_cast<const uint8_t*>(local_scales->data_ptr());
      a.local_scales_stride = local_scales->stride(0) * 4;
    }
    if (ok) {
      a.local_x = static_cast<const uint8_t*>(local_x->data_ptr());
      a.local_x_stride = xs;
    }
  }
  const int64_t MD = mode == 0 ? 2LL * a.H : a.H;
  const bool aligned = (reinterpret_cast<uintptr_t>(a.recv_x) & 15) == 0 && (MD % 16) == 0 && MD < (1 << 20);
  a.use_tma = use_tma && aligned;
  size_t smem = 0;
  if (a.use_tma) {
    a.stage_bytes = static_cast<int>(align_up(MD, 128));
    const int64_t budget = 160 * 1024;
    a.nstages = static_cast<int>(std::max<int64_t>(2, std::min<int64_t>(16, budget / a.stage_bytes)));
    smem = static_cast<size_t>(a.nstages) * a.stage_bytes + a.nstages * sizeof(uint64_t);
    TORCH_CHECK(smem <= 200 * 1024, "row too large for the TMA pipeline");
    static std::atomic<uint64_t> seen{0};
    AT_CUDA_CHECK(set_smem_limit_once(seen, nd_pull_kernel, 220 * 1024));
  }
  const int grid = num_sms > 0 ? static_cast<int>(num_sms) : heap.num_sms();
  nd_pull_kernel<<<grid, kPullThreads, smem, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ combine
struct NcArgs {
  HeapView hv;
  const uint8_t* x;
  int64_t x_stride;     // bytes
  const float* w;       // [N, K]
  int64_t w_stride;
  const int64_t* recv_off;
  const int32_t* token_pos;
  uint8_t* out;
  float* out_w;
  const uint8_t* bias0;
  const uint8_t* bias1;
  int T, H, K;
  int use_tma;            // rows of x are contiguous and 16-byte aligned: push with bulk copies
  int chunk_bytes;        // bytes per bulk copy (multiple of 16)
  int nstages;
};

template <typename T16>
__device__ __forceinline__ void acc8(float (&acc)[8], const int4& raw) {
  const T16* h = reinterpret_cast<const T16*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] += static_cast<float>(h[i]);
}

template <typename T16>
__global__ void __launch_bounds__(kCombThreads) nc_combine_kernel(NcArgs a) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t e = ld_volatile_u32(&ls->epoch[kEpNC]) + 1u;
  const int slot = e & 1u;
  const int me = hv.rank, R = hv.R, M = hv.cfg.M;
  const int H = a.H, K = a.K;
  const int64_t RB = 2LL * H;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kCombThreads / 32;
  const int gw = blockIdx.x * nwarps + warp, GW = gridDim.x * nwarps;

  __shared__ int64_t s_off[B200EP_MAX_RANKS + 1];
  __shared__ int s_last, s_fail;
  if (tid <= R) s_off[tid] = a.recv_off[tid];
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrCombStart] = global_ns();
  __syncthreads();
  const int64_t N = s_off[R];

  // ---------------------------------------------------------------- push rows home
  // Rows from source s occupy x[off[s], off[s+1]) and land contiguously in s's return
  // block [me][0, count), so each peer's share is one contiguous byte range.
  if (a.use_tma) {
    extern __shared__ __align__(1024) uint8_t smem_push[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem_push + static_cast<int64_t>(a.nstages) * a.chunk_bytes);
    // chunks of every peer's byte range, in rank order (own rows excluded); a peer's last
    // chunk may be short, and no chunk spans two peers
    int64_t nchunks = 0;
    for (int s = 0; s < R; ++s)
      if (s != me) nchunks += ((s_off[s + 1] - s_off[s]) * RB + a.chunk_bytes - 1) / a.chunk_bytes;
    const int64_t c0 = nchunks * blockIdx.x / gridDim.x, c1 = nchunks * (blockIdx.x + 1) / gridDim.x;
    if (tid == 0 && c1 > c0) {
      for (int st = 0; st < a.nstages; ++st) mbar_init(&bars[st], 1);
      fence_mbar_init();
      auto locate = [&](int64_t c, const uint8_t*& src, uint8_t*& dst, uint32_t& bytes) {
        for (int s = 0; s < R; ++s) {
          if (s == me) continue;
          const int64_t len = (s_off[s + 1] - s_off[s]) * RB;
          const int64_t nc = (len + a.chunk_bytes - 1) / a.chunk_bytes;
          if (c < nc) {
            const int64_t byte = c * a.chunk_bytes;
            src = a.x + s_off[s] * RB + byte;
            dst = hv.at<uint8_t>(s, hv.L.nc_rows[slot]) + static_cast<int64_t>(me) * M * RB + byte;
            bytes = static_cast<uint32_t>(len - byte < a.chunk_bytes ? len - byte : a.chunk_bytes);
            return;
          }
          c -= nc;
        }
        bytes = 0;
      };
      uint32_t phase_bits = 0;
      const int64_t n = c1 - c0;
      auto issue = [&](int64_t q) {
        const int st = static_cast<int>(q % a.nstages);
        const uint8_t* src;
        uint8_t* dst;
        uint32_t bytes;
        locate(c0 + q, src, dst, bytes);
        mbar_arrive_expect_tx(&bars[st], bytes);
        if (bytes) bulk_load(smem_push + static_cast<int64_t>(st) * a.chunk_bytes, src, bytes, &bars[st]);
      };
      const int64_t pro = n < a.nstages ? n : a.nstages;
      for (int64_t q = 0; q < pro; ++q) issue(q);
      for (int64_t m = 0; m < n; ++m) {
        const int st = static_cast<int>(m % a.nstages);
        if (!mbar_wait(&bars[st], (phase_bits >> st) & 1u, hv.timeout_ns)) {
          report_error(hv.status, kTimeoutCombine, 3, me, -1, 0, 0, 1);
          break;
        }
        phase_bits ^= 1u << st;
        const uint8_t* src;
        uint8_t* dst;
        uint32_t bytes;
        locate(c0 + m, src, dst, bytes);
        if (bytes) bulk_store(dst, smem_push + static_cast<int64_t>(st) * a.chunk_bytes, bytes);
        bulk_commit();
        const int64_t q = m - 1 + a.nstages;
        if (m >= 1 && q < n) {
          bulk_wait_read<1>();
          issue(q);
        }
      }
      bulk_wait<0>();              // this CTA's peer writes are complete
      fence_proxy_async_global();  // order them before the generic-proxy arrival below
    }
    // weights: small, plain stores
    if (a.w) {
      for (int64_t i = blockIdx.x * kCombThreads + tid; i < N * K; i += static_cast<int64_t>(gridDim.x) * kCombThreads) {
        const int64_t row = i / K, k = i % K;
        int s = 0;
        while (s + 1 < R && s_off[s + 1] <= row) ++s;
        if (s == me) continue;
        const int64_t j = row - s_off[s];
        hv.at<float>(s, hv.L.nc_w[slot])[(static_cast<int64_t>(me) * M + j) * K + k] = a.w[row * a.w_stride + k];
      }
    }
  } else {
    for (int64_t i = gw; i < N; i += GW) {
      int s = 0;
      while (s + 1 < R && s_off[s + 1] <= i) ++s;
      const int64_t j = i - s_off[s];
      if (j >= M || s == me) continue;  // own rows are read from x in place by the reduce
      const int64_t slot_row = static_cast<int64_t>(me) * M + j;
      warp_copy(hv.at<uint8_t>(s, hv.L.nc_rows[slot]) + slot_row * RB, a.x + i * a.x_stride, RB);
      if (a.w && lane < K) hv.at<float>(s, hv.L.nc_w[slot])[slot_row * K + lane] = a.w[i * a.w_stride + lane];
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(&ls->arrive[kEpNC], 1u);
    s_last = (prev == gridDim.x - 1);
    s_fail = 0;
  }
  __syncthreads();
  if (s_last) {
    if (tid < R) {
      fence_sys();
      st_release_sys(&hv.sig(tid)->nc_ready[slot][me], e);
    }
    if (tid == 0) {
      ls->arrive[kEpNC] = 0;
      ls->epoch[kEpNC] = e;
      ls->trace[kTrCombPushDone] = global_ns();
    }
  }

  // ---------------------------------------------------------------- reduce at the source
  if (tid < R) {
    if (!wait_epoch(&hv.sig(me)->nc_ready[slot][tid], e, hv.timeout_ns, hv.status, kTimeoutCombine, 3, me, tid))
      atomicExch(&s_fail, 1);
  }
  __syncthreads();  // every thread reads rows whose flags threads < R acquired
  if (s_fail) return;
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrCombPeersReady] = global_ns();
  const uint8_t* rows = hv.at<uint8_t>(me, hv.L.nc_rows[slot]);
  const float* wrows = hv.at<float>(me, hv.L.nc_w[slot]);
  const bool vec = (H % 8) == 0;
  __shared__ int32_t s_pos[nwarps][B200EP_MAX_RANKS];
  for (int t = gw; t < a.T; t += GW) {
    // every lane learns the token's row position in each rank's return block
    if (lane < R) s_pos[warp][lane] = a.token_pos[static_cast<int64_t>(t) * R + lane];
    __syncwarp();
    const int32_t* pos = s_pos[warp];
    T16* out = reinterpret_cast<T16*>(a.out) + static_cast<int64_t>(t) * H;
    const T16* b0 = a.bias0 ? reinterpret_cast<const T16*>(a.bias0) + static_cast<int64_t>(t) * H : nullptr;
    const T16* b1 = a.bias1 ? reinterpret_cast<const T16*>(a.bias1) + static_cast<int64_t>(t) * H : nullptr;
    if (vec) {
      // rows of this token present in the return blocks
      const uint8_t* rp[B200EP_MAX_RANKS];
      int nr = 0;
      for (int r = 0; r < R; ++r) {
        if (pos[r] < 0) continue;
        rp[nr++] = r == me ? a.x + (s_off[me] + pos[r]) * a.x_stride
                           : rows + (static_cast<int64_t>(r) * M + pos[r]) * RB;
      }
      // eight 256-element chunks per pass: up to 8 x nr independent 16-byte loads per lane
      constexpr int U = 8;
      for (int c0 = lane * 8; c0 < H; c0 += 256 * U) {
        float acc[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[u][i] = 0.f;
        for (int r = 0; r < nr; ++r) {
          int4 v[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + u * 256 < H) v[u] = *reinterpret_cast<const int4*>(rp[r] + (c0 + u * 256) * 2);
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + u * 256 < H) acc8<T16>(acc[u], v[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + u * 256;
          if (c >= H) continue;
          if (b0) acc8<T16>(acc[u], *reinterpret_cast<const int4*>(b0 + c));
          if (b1) acc8<T16>(acc[u], *reinterpret_cast<const int4*>(b1 + c));
          int4 o;
          T16* oh = reinterpret_cast<T16*>(&o);
#pragma unroll
          for (int i = 0; i < 8; ++i) oh[i] = static_cast<T16>(acc[u][i]);
          *reinterpret_cast<int4*>(out + c) = o;
        }
      }
    } else {
      for (int c = lane; c < H; c += 32) {
        float acc = 0.f;
        for (int r = 0; r < R; ++r) {
          const int p = pos[r];
          if (p < 0) continue;
          const uint8_t* row = r == me ? a.x + (s_off[me] + p) * a.x_stride
                                       : rows + (static_cast<int64_t>(r) * M + p) * RB;
          acc += static_cast<float>(reinterpret_cast<const T16*>(row)[c]);
        }
        if (b0) acc += static_cast<float>(b0[c]);
        if (b1) acc += static_cast<float>(b1[c]);
        out[c] = static_cast<T16>(acc);
      }
    }
    if (a.out_w && lane < K) {
      float s = 0.f;
      for (int r = 0; r < R; ++r) {
        const int p = pos[r];
        if (p < 0) continue;
        s += r == me ? a.w[(s_off[me] + p) * a.w_stride + lane] : wrows[(static_cast<int64_t>(r) * M + p) * K + lane];
      }
      a.out_w[static_cast<int64_t>(t) * K + lane] = s;
    }
    __syncwarp();
  }
  __syncthreads();
  if (tid == 0 && atomicAdd(&ls->arrive2[kEpNC], 1u) == gridDim.x - 1) {
    ls->arrive2[kEpNC] = 0;
    ls->trace[kTrCombEnd] = global_ns();
  }
}


// ============================================================================ combine (pull form)
// Each expert rank stages the rows its peers need in its own heap (a local copy) and
// publishes its receive offsets; every source then streams its tokens' rows in with
// TMA bulk loads (the faster NVLink direction on this fabric) through a shared-memory
// ring and reduces them in fp32 as they arrive, adds the optional bias and casts once.
struct NcPullArgs {
  HeapView hv;
  const uint8_t* x;
  int64_t x_stride;     // bytes
  const float* w;
  int64_t w_stride;
  const int64_t* recv_off;
  const int32_t* token_pos;
  uint8_t* out;
  float* out_w;
  const uint8_t* bias0;
  const uint8_t* bias1;
  int T, H, K;
  int nstages, stage_bytes;
};

constexpr int kPullTok = 32;        // tokens per batch (their row lists are built together)
constexpr int kPullConsumers = kCombThreads / 32 - 1;   // warp 0 drives the loads, the rest reduce

// Row stream of the pull combine. Warp 0's lane 0 issues one bulk load per row into a ring
// of shared-memory stages (full barrier: transaction bytes; empty barrier: one arrival
// per consumer warp); warps 1.. each own fixed 16-byte chunks of the row, accumulate
// in fp32 and store a token's output after its last row, without CTA-wide barriers
// between rows.
template <typename T16>
__global__ void __launch_bounds__(kCombThreads) nc_pull_kernel(NcPullArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_ring[];
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t e = ld_volatile_u32(&ls->epoch[kEpNC]) + 1u;
  const int slot = e & 1u;
  const int me = hv.rank, R = hv.R;
  const int H = a.H, K = a.K;
  const int64_t RB = 2LL * H;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kCombThreads / 32;
  const int gw = blockIdx.x * nwarps + warp, GW = gridDim.x * nwarps;
  const int ns = a.nstages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_ring + static_cast<int64_t>(ns) * a.stage_bytes);
  uint64_t* empty = full + ns;

  __shared__ int64_t s_off[B200EP_MAX_RANKS + 1];
  __shared__ int64_t s_roff[B200EP_MAX_RANKS];
  __shared__ int s_last;
  __shared__ volatile int s_fail;
  __shared__ const uint8_t* s_rows[kPullTok * B200EP_MAX_RANKS];  // the batch's rows, token-major
  __shared__ int16_t s_rtok[kPullTok * B200EP_MAX_RANKS];         // token of the row if it is its last, else -1
  __shared__ int s_cnt[kPullTok];
  __shared__ int s_n[kPullTok + 1];
  if (tid <= R) s_off[tid] = a.recv_off[tid];
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrCombStart] = global_ns();
  __syncthreads();
  const int64_t N = s_off[R];

  // ---------------------------------------------------------------- stage rows for the peers
  uint8_t* send = hv.at<uint8_t>(me, hv.L.nc_send[slot]);
  float* send_w = hv.at<float>(me, hv.L.nc_send_w[slot]);
  for (int64_t i = gw; i < N; i += GW) {
    if (i >= s_off[me] && i < s_off[me + 1]) continue;  // own rows are read in place
    warp_copy(send + i * RB, a.x + i * a.x_stride, RB);
    if (a.w && lane < K) send_w[i * K + lane] = a.w[i * a.w_stride + lane];
  }
  if (blockIdx.x == 0 && tid <= R) hv.at<int64_t>(me, hv.L.nc_send_off[slot])[tid] = s_off[tid];
  __syncthreads();
  if (tid == 0) {
    __threadfence();  // local data; peers read it after the last CTA's system-scope release
    s_last = atomicAdd(&ls->arrive[kEpNC], 1u) == gridDim.x - 1;
    s_fail = 0;
  }
  __syncthreads();
  if (s_last) {
    if (tid < R) {
      fence_sys();
      st_release_sys(&hv.sig(tid)->nc_ready[slot][me], e);
    }
    if (tid == 0) {
      ls->arrive[kEpNC] = 0;
      ls->epoch[kEpNC] = e;
      ls->trace[kTrCombPushDone] = global_ns();
    }
  }
  // ---------------------------------------------------------------- wait for every expert rank
  if (tid < R) {
    if (!wait_epoch(&hv.sig(me)->nc_ready[slot][tid], e, hv.timeout_ns, hv.status, kTimeoutCombine, 3, me, tid))
      s_fail = 1;
    else
      s_roff[tid] = tid == me ? s_off[me] : *reinterpret_cast<const volatile int64_t*>(
                                                 hv.at<int64_t>(tid, hv.L.nc_send_off[slot]) + me);
  }
  __syncthreads();
  if (s_fail) return;
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrCombPeersReady] = global_ns();
  if (tid == 0) {
    for (int st = 0; st < ns; ++st) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kPullConsumers);
    }
    fence_mbar_init();
    fence_proxy_async_global();
  }
  __syncthreads();

  // ---------------------------------------------------------------- row stream + reduce
  const int nch = H / 8;                           // 16-byte chunks per row
  const int t0 = static_cast<int>(static_cast<int64_t>(a.T) * blockIdx.x / gridDim.x);
  const int t1 = static_cast<int>(static_cast<int64_t>(a.T) * (blockIdx.x + 1) / gridDim.x);
  uint32_t g = 0;  // rows streamed so far by this CTA (drives stage and parity)
  for (int tb = t0; tb < t1 && !s_fail; tb += kPullTok) {
    const int nt = min(kPullTok, t1 - tb);
    // per token: its rows (one per rank it visited) and its combined weights
    int pv[kPullTok / nwarps];
#pragma unroll
    for (int u = 0; u < kPullTok / nwarps; ++u) {
      const int i = warp + u * nwarps;
      pv[u] = -1;
      if (i >= nt) continue;
      const int t = tb + i;
      const int p = lane < R ? a.token_pos[static_cast<int64_t>(t) * R + lane] : -1;
      pv[u] = p;
      const uint32_t bt = __ballot_sync(0xffffffffu, p >= 0);  // every lane takes part
      if (lane == 0) s_cnt[i] = __popc(bt);
      if (a.out_w) {
        float acc_w = 0.f;
        for (int r = 0; r < R; ++r) {
          const int pr = __shfl_sync(0xffffffffu, p, r);
          if (pr < 0 || lane >= K) continue;
          acc_w += r == me ? a.w[(s_off[me] + pr) * a.w_stride + lane]
                           : *reinterpret_cast<const volatile float*>(
                                 hv.at<float>(r, hv.L.nc_send_w[slot]) + (s_roff[r] + pr) * K + lane);
        }
        if (lane < K) a.out_w[static_cast<int64_t>(t) * K + lane] = acc_w;
      }
    }
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the row counts
      const int c = lane < nt ? s_cnt[lane] : 0;
      int v = c;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += o;
      }
      s_n[lane] = v - c;
      if (lane == 31) s_n[kPullTok] = v;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kPullTok / nwarps; ++u) {
      const int i = warp + u * nwarps;
      if (i >= nt) continue;
      const int p = pv[u];
      const uint32_t b = __ballot_sync(0xffffffffu, p >= 0);
      if (p >= 0) {
        const int q = __popc(b & lanemask_lt());
        const int k = s_n[i] + q;
        s_rows[k] = lane == me ? a.x + (s_off[me] + p) * a.x_stride
                               : hv.base[lane] + hv.L.nc_send[slot] + (s_roff[lane] + p) * RB;
        s_rtok[k] = static_cast<int16_t>(q == __popc(b) - 1 ? i : -1);
      }
    }
    __syncthreads();
    const int nrows = s_n[kPullTok];

    if (warp == 0) {
      // ------------------------------------------------------------ producer
      if (lane == 0) {
        int k = 0;
        for (; k < nrows; ++k) {
          const uint32_t gk = g + k;
          const int st = static_cast<int>(gk % ns);
          if (gk >= static_cast<uint32_t>(ns) &&
              !mbar_wait(&empty[st], ((gk / ns) + 1u) & 1u, hv.timeout_ns)) {
            s_fail = 1;
            break;
          }
          if (s_fail) break;
          mbar_arrive_expect_tx(&full[st], static_cast<uint32_t>(RB));
          bulk_load(smem_ring + static_cast<int64_t>(st) * a.stage_bytes, s_rows[k], static_cast<uint32_t>(RB),
                    &full[st]);
        }
        if (s_fail) {
          // let the loads still in flight land before the CTA's shared memory is released
          for (int kk = max(0, k - ns); kk < k; ++kk) {
            const uint32_t gk = g + kk;
            mbar_wait(&full[gk % ns], (gk / ns) & 1u, hv.timeout_ns);
          }
        }
      }
    } else {
      // ------------------------------------------------------------ consumers
      const int ct = tid - 32;                   // 0 .. 32 * kPullConsumers - 1
      constexpr int CT = 32 * kPullConsumers;
      float acc[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[u][q] = 0.f;
      for (int k = 0; k < nrows; ++k) {
        const uint32_t gk = g + k;
        const int st = static_cast<int>(gk % ns);
        if (!mbar_wait(&full[st], (gk / ns) & 1u, hv.timeout_ns)) {
          s_fail = 1;
          break;
        }
        if (s_fail) break;
        const uint8_t* row = smem_ring + static_cast<int64_t>(st) * a.stage_bytes;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = ct + u * CT;
          if (j < nch) acc8<T16>(acc[u], *reinterpret_cast<const int4*>(row + j * 16));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_local(&empty[st]);
        const int i = s_rtok[k];
        if (i >= 0) {
          // last row of token i: bias, cast, store, reset
          const int64_t t = tb + i;
          T16* out = reinterpret_cast<T16*>(a.out) + t * H;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = ct + u * CT;
            if (j >= nch) continue;
            if (a.bias0) acc8<T16>(acc[u], reinterpret_cast<const int4*>(a.bias0 + t * RB)[j]);
            if (a.bias1) acc8<T16>(acc[u], reinterpret_cast<const int4*>(a.bias1 + t * RB)[j]);
            int4 o;
            T16* oh = reinterpret_cast<T16*>(&o);
#pragma unroll
            for (int q = 0; q < 8; ++q) oh[q] = static_cast<T16>(acc[u][q]);
            reinterpret_cast<int4*>(out)[j] = o;
#pragma unroll
            for (int q = 0; q < 8; ++q) acc[u][q] = 0.f;
          }
        }
      }
      // tokens routed nowhere (all top-k masked) still get bias (or zeros)
      for (int i = warp - 1; i < nt; i += kPullConsumers) {
        if (s_cnt[i] != 0) continue;
        const int64_t t = tb + i;
        T16* out = reinterpret_cast<T16*>(a.out) + t * H;
        for (int j = lane; j < nch; j += 32) {
          float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if (a.bias0) acc8<T16>(z, reinterpret_cast<const int4*>(a.bias0 + t * RB)[j]);
          if (a.bias1) acc8<T16>(z, reinterpret_cast<const int4*>(a.bias1 + t * RB)[j]);
          int4 o;
          T16* oh = reinterpret_cast<T16*>(&o);
#pragma unroll
          for (int q = 0; q < 8; ++q) oh[q] = static_cast<T16>(z[q]);
          reinterpret_cast<int4*>(out)[j] = o;
        }
      }
    }
    g += static_cast<uint32_t>(nrows);
    __syncthreads();  // the batch's lists are free again
  }
  if (s_fail) {
    if (tid == 0) report_error(hv.status, kTimeoutCombine, 3, me, -1, 0, 0, 2);
    return;
  }
  __syncthreads();
  if (tid == 0 && atomicAdd(&ls->arrive2[kEpNC], 1u) == gridDim.x - 1) {
    ls->arrive2[kEpNC] = 0;
    ls->trace[kTrCombEnd] = global_ns();
  }
}

void nc_combine(SymmHeap& heap, const at::Tensor& x, const OptTensor& w, const at::Tensor& recv_off,
                const at::Tensor& token_pos, at::Tensor out, const OptTensor& out_w, const OptTensor& bias0,
                const OptTensor& bias1, int64_t num_sms) {
  const c10::cuda::CUDAGuard guard(x.device());
  HeapView hv = heap.view();
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.element_size() == 2, "combine x must be 16-bit [N, H]");
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == x.scalar_type(), "out must match x");
  TORCH_CHECK(recv_off.scalar_type() == at::kLong && recv_off.numel() == hv.R + 1, "recv_off must be [R+1] int64");
  TORCH_CHECK(token_pos.is_contiguous() && token_pos.scalar_type() == at::kInt, "token_pos must be int32");
  NcArgs a{};
  a.hv = hv;
  a.x = static_cast<const uint8_t*>(x.data_ptr());
  a.x_stride = x.stride(0) * 2;
  a.H = static_cast<int>(x.size(1));
  TORCH_CHECK(a.H <= hv.cfg.H, "hidden exceeds the buffer's hidden size");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(a.x) & 15) == 0 || a.H % 8 != 0, "x must be 16-byte aligned");
  a.K = 0;
  if (w.has_value()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && unit_inner(*w), "topk_weights must be fp32");
    a.w = w->data_ptr<float>();
    a.w_stride = w->stride(0);
    a.K = static_cast<int>(w->size(1));
    TORCH_CHECK(a.K <= hv.cfg.K, "top-k exceeds the buffer");
  }
  a.recv_off = recv_off.data_ptr<int64_t>();
  a.token_pos = token_pos.data_ptr<int32_t>();
  a.out = static_cast<uint8_t*>(out.data_ptr());
  a.T = static_cast<int>(out.size(0));
  if (out_w.has_value()) a.out_w = out_w->data_ptr<float>();
  if (bias0.has_value()) {
    TORCH_CHECK(bias0->is_contiguous() && bias0->scalar_type() == x.scalar_type(), "bias dtype/layout");
    a.bias0 = static_cast<const uint8_t*>(bias0->data_ptr());
  }
  if (bias1.has_value()) {
    TORCH_CHECK(bias1->is_contiguous() && bias1->scalar_type() == x.scalar_type(), "bias dtype/layout");
    a.bias1 = static_cast<const uint8_t*>(bias1->data_ptr());
  }
  int grid = num_sms > 0 ? static_cast<int>(num_sms) : heap.num_sms();
  void* kfn = x.scalar_type() == at::kHalf ? reinterpret_cast<void*>(nc_combine_kernel<__half>)
                                           : reinterpret_cast<void*>(nc_combine_kernel<__nv_bfloat16>);
  const uintptr_t xp = reinterpret_cast<uintptr_t>(a.x);
  const bool aligned = (xp & 15) == 0 && (a.x_stride % 16) == 0 && (a.H % 8) == 0 && a.H <= 4 * 8 * 32 * kPullConsumers;
  if (aligned && !getenv("B200EP_COMBINE_PUSH")) {
    NcPullArgs p{};
    p.hv = a.hv;
    p.x = a.x;
    p.x_stride = a.x_stride;
    p.w = a.w;
    p.w_stride = a.w_stride;
    p.recv_off = a.recv_off;
    p.token_pos = a.token_pos;
    p.out = a.out;
    p.out_w = a.out_w;
    p.bias0 = a.bias0;
    p.bias1 = a.bias1;
    p.T = a.T;
    p.H = a.H;
    p.K = a.K;
    p.stage_bytes = static_cast<int>(align_up(2LL * a.H, 128));
    p.nstages = static_cast<int>(std::max<int64_t>(2, std::min<int64_t>(12, (176 * 1024) / p.stage_bytes)));
    const size_t psmem = static_cast<size_t>(p.nstages) * p.stage_bytes + p.nstages * 16;
    void* pfn = x.scalar_type() == at::kHalf ? reinterpret_cast<void*>(nc_pull_kernel<__half>)
                                             : reinterpret_cast<void*>(nc_pull_kernel<__nv_bfloat16>);
    static std::atomic<uint64_t> pseen[2];
    AT_CUDA_CHECK(set_smem_limit_once(pseen[x.scalar_type() == at::kHalf ? 1 : 0], pfn, 200 * 1024));
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pfn, kCombThreads, psmem);
    const int g = std::max(1, std::min(grid, per_sm * heap.num_sms()));
    void* pargs[] = {&p};
    // cooperative: every CTA waits for the other ranks after staging, so all CTAs must be resident
    AT_CUDA_CHECK(cudaLaunchCooperativeKernel(pfn, dim3(g), dim3(kCombThreads), pargs, psmem,
                                              at::cuda::getCurrentCUDAStream()));
    return;
  }
  a.use_tma = (xp & 15) == 0 && a.x_stride == 2LL * a.H && (a.x_stride % 16) == 0 && !getenv("B200EP_NO_TMA");
  a.chunk_bytes = 16384;
  a.nstages = 8;
  if (const char* v = getenv("B200EP_PUSH_CHUNK")) a.chunk_bytes = std::max(1024, atoi(v)) / 16 * 16;
  if (const char* v = getenv("B200EP_PUSH_STAGES")) a.nstages = std::max(2, std::min(16, atoi(v)));
  while (static_cast<int64_t>(a.nstages) * a.chunk_bytes > 150 * 1024 && a.nstages > 2) --a.nstages;
  const size_t smem = a.use_tma ? static_cast<size_t>(a.nstages) * a.chunk_bytes + a.nstages * 8 : 0;
  static std::atomic<uint64_t> seen[2];
  AT_CUDA_CHECK(set_smem_limit_once(seen[x.scalar_type() == at::kHalf ? 1 : 0], kfn, 160 * 1024));
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kCombThreads, smem);
  grid = std::max(1, std::min(grid, per_sm * heap.num_sms()));
  void* args[] = {&a};
  // cooperative: every CTA waits for the peers after its own pushes, so all CTAs must be resident
  AT_CUDA_CHECK(cudaLaunchCooperativeKernel(kfn, dim3(grid), dim3(kCombThreads), args, smem,
                                            at::cuda::getCurrentCUDAStream()));
}

}  // namespace b200ep
