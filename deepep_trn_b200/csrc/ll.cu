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
// expert ids, so the receiver needs no count exchange: one CTA per local expert
// walks all slots in (src, token) order and compacts the matching rows into
// recv_x. No host synchronisation.
//
// Completion signalling is batched: each sending CTA adds the number of slots
// (dispatch) or rows (combine) it wrote to a per-(parity, source) counter in the
// destination's signal pad with one system-scope fence and one red.release.sys
// per destination. Counters are cumulative; the receiver keeps what it has
// already consumed in its local state, so nothing is ever reset. A system-scope
// fence per row would also order against host-mapped memory and costs far more.
//
// Parallelism: CTAs own contiguous token blocks on the send side (16-byte chunks
// spread over their threads), a CTA per token on the combine receive side with all
// K slot loads of a chunk issued together.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ops.h"

namespace b200ep {

constexpr int kLLThreads = 256;
constexpr int kLLRecvThreads = 512;

__device__ __forceinline__ uint32_t ldv_u32(const uint32_t* p) { return *reinterpret_cast<const volatile uint32_t*>(p); }

// Last CTA of the grid publishes the new epoch of `which` and resets the arrival counter.
__device__ __forceinline__ void finish_epoch(LocalState* ls, int which, uint32_t e, int trace_point) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&ls->arrive[which], 1u);
    s_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    ls->arrive[which] = 0;
    ls->epoch[which] = e;
    ls->trace[trace_point] = global_ns();
  }
}

// ============================================================================ dispatch send
struct LLSendArgs {
  HeapView hv;
  const uint8_t* x;   // [T, H] bf16 (or fp16)
  int64_t x_stride;   // bytes
  const void* topk;
  int topk_i32;
  int T, H, K, E;
  int use_fp8, round_scale;
};

// grid: CTAs own contiguous blocks of tokens
// One sending CTA's share (tokens [T*b/G, T*(b+1)/G)) for epoch e; any multiple of 32 threads.
template <typename T16>
__device__ void ll_dispatch_send_body(const LLSendArgs& a, uint32_t e) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const int nthr = blockDim.x;
  const int slot = e & 1u;
  const int me = hv.rank, R = hv.R, Mll = hv.cfg.Mll;
  const int64_t rs = hv.L.row_stride;
  const int H = a.H, K = a.K, EL = a.E / R;
  const int tid = threadIdx.x;
  const int T = min(a.T, Mll);
  __shared__ int32_t s_ids[32];
  __shared__ uint32_t s_mask;

  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLLSendStart] = global_ns();
  if (blockIdx.x == 0 && tid < R)
    st_release_sys64(&hv.sig(tid)->ll_hdr[slot][me], (static_cast<uint64_t>(e) << 32) | static_cast<uint32_t>(T));
  if (a.T > Mll && blockIdx.x == 0 && tid == 0) report_error(hv.status, kCapacity, 4, me, -1, Mll, a.T);

  const int t0 = static_cast<int>(static_cast<int64_t>(T) * blockIdx.x / gridDim.x);
  const int t1 = static_cast<int>(static_cast<int64_t>(T) * (blockIdx.x + 1) / gridDim.x);
  for (int t = t0; t < t1; ++t) {
    if (tid < 32) {
      int32_t g = -1;
      if (tid < K) {
        const int64_t i = static_cast<int64_t>(t) * K + tid;
        g = a.topk_i32 ? static_cast<const int32_t*>(a.topk)[i]
                       : static_cast<int32_t>(static_cast<const int64_t*>(a.topk)[i]);
        if (g >= a.E) g = -1;
      }
      s_ids[tid] = g;
      const uint32_t m = __reduce_or_sync(0xffffffffu, g >= 0 ? (1u << (g / EL)) : 0u);
      if (tid == 0) s_mask = m;
    }
    __syncthreads();
    const uint32_t dmask = s_mask;
    const int64_t slot_row = static_cast<int64_t>(me) * Mll + t;
    const T16* src = reinterpret_cast<const T16*>(a.x + static_cast<int64_t>(t) * a.x_stride);
    const int nchunk = H / 8;  // 16-byte chunks of the 16-bit row
    if (!a.use_fp8) {
      for (int j0 = tid; j0 < nchunk; j0 += 4 * nthr) {
        int4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = j0 + u * nthr;
          if (j < nchunk) v[u] = reinterpret_cast<const int4*>(src)[j];
        }
        for (uint32_t m = dmask; m; m &= m - 1) {
          const int p = __ffs(m) - 1;
          int4* dst = reinterpret_cast<int4*>(hv.base[p] + hv.L.ll_rows[slot] + slot_row * rs);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = j0 + u * nthr;
            if (j < nchunk) dst[j] = v[u];
          }
        }
      }
    } else {
      // a half-warp quantises one 128-element block; every thread runs the same number of
      // iterations so the shuffles inside quant8_e4m3 always see full warps
      const int iters = (nchunk + nthr - 1) / nthr;
      for (int it0 = 0; it0 < iters; it0 += 4) {
        float vv[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = (it0 + u) * nthr + tid;
          load8(vv[u], src + static_cast<int64_t>(j) * 8, it0 + u < iters && j < nchunk);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
        if (it0 + u >= iters) break;
        const int j = (it0 + u) * nthr + tid;
        const bool act = j < nchunk;
        const Quant8 qr = quant8_e4m3(vv[u], a.round_scale);
        if (act) {
          for (uint32_t m = dmask; m; m &= m - 1) {
            const int p = __ffs(m) - 1;
            uint8_t* row = hv.base[p] + hv.L.ll_rows[slot] + slot_row * rs;
            *reinterpret_cast<uint2*>(row + j * 8) = qr.q;
            if ((tid & 15) == 0) reinterpret_cast<float*>(row + H)[j / 16] = qr.scale;
          }
        }
        }
      }
    }
    // ids go to every rank (a non-routed rank learns that it is not a destination)
    for (int i = tid; i < R * K; i += nthr) {
      const int p = i / K, k = i % K;
      hv.at<int32_t>(p, hv.L.ll_ids[slot])[slot_row * K + k] = s_ids[k];
    }
    __syncthreads();
  }
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLLSendStored] = global_ns();
  if (tid < R && t1 > t0) {
    signal_add(&hv.sig(tid)->ll_cnt[slot][me], static_cast<uint32_t>(t1 - t0), tid == me);
  }
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLLSendReleased] = global_ns();
}

template <typename T16>
__global__ void __launch_bounds__(kLLThreads) ll_dispatch_send_kernel(LLSendArgs a) {
  LocalState* ls = a.hv.local();
  const uint32_t e = ldv_u32(&ls->epoch[kEpLLD]) + 1u;
  ll_dispatch_send_body<T16>(a, e);
  finish_epoch(ls, kEpLLD, e, kTrLLSendEnd);
}

static LLSendArgs ll_send_args(SymmHeap& heap, const at::Tensor& x, const at::Tensor& topk_idx,
                               int64_t num_experts, bool use_fp8, bool round_scale) {
  HeapView hv = heap.view();
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.element_size() == 2, "x must be 16-bit [T, H]");
  TORCH_CHECK(topk_idx.is_contiguous() && topk_idx.dim() == 2, "topk_idx must be contiguous [T, K]");
  LLSendArgs a{};
  a.hv = hv;
  a.x = static_cast<const uint8_t*>(x.data_ptr());
  a.x_stride = x.stride(0) * 2;
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
  TORCH_CHECK(a.T == 0 || ((a.x_stride % 16) == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0),
              "x rows must be 16-byte aligned");
  return a;
}

void ll_dispatch_send(SymmHeap& heap, const at::Tensor& x, const at::Tensor& topk_idx, int64_t num_experts,
                      bool use_fp8, bool round_scale, int64_t num_sms) {
  const c10::cuda::CUDAGuard guard(x.device());
  const LLSendArgs a = ll_send_args(heap, x, topk_idx, num_experts, use_fp8, round_scale);
  const int sms = num_sms > 0 ? static_cast<int>(num_sms) : heap.num_sms();
  const int grid = std::max(1, std::min(std::min(a.T, a.hv.cfg.Mll), 2 * sms));
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x.scalar_type() == at::kHalf)
    ll_dispatch_send_kernel<__half><<<grid, kLLThreads, 0, stream>>>(a);
  else
    ll_dispatch_send_kernel<__nv_bfloat16><<<grid, kLLThreads, 0, stream>>>(a);
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
  int split;                // CTAs per local expert
};

// grid: `split` CTAs per local expert. Every CTA of an expert walks the (src, token) slots of
// all sources flattened in (src, token) order, 512 slots per tile, up to the end of its
// share of the slots: the ids of the earlier slots give it the position of its first row
// (no communication between the CTAs), and it copies the rows of its own slots. The last
// CTA of the expert, which has walked every slot, writes the counts and layout_range.
// Receive side for epoch e; blockDim.x == kLLRecvThreads, gridDim.x == EL * split.
__device__ void ll_dispatch_recv_body(const LLRecvArgs& a, uint32_t e) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const int slot = e & 1u;
  const int me = hv.rank, R = hv.R, Mll = hv.cfg.Mll;
  const int64_t rs = hv.L.row_stride;
  const int H = a.H, K = a.K, EL = a.E / R;
  const int le = blockIdx.x / a.split, part = blockIdx.x % a.split;
  const bool last_part = part == a.split - 1;
  const int32_t want = me * EL + le;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kLLRecvThreads / 32;
  const int64_t RM = static_cast<int64_t>(R) * Mll;
  const int64_t PB = a.use_fp8 ? H : 2LL * H;   // payload bytes
  const int nsb = H / 128;                      // scale blocks

  __shared__ int s_T[B200EP_MAX_RANKS];
  __shared__ int s_toff[B200EP_MAX_RANKS + 1];   // prefix of T over sources
  __shared__ int s_bcnt[B200EP_MAX_RANKS];       // rows of this expert per source
  __shared__ int s_fail, s_tile_total;
  __shared__ int s_wcnt[nwarps];
  __shared__ int s_tok[kLLRecvThreads];
  __shared__ int s_src[kLLRecvThreads];
  __shared__ int s_dst[kLLRecvThreads];
  if (tid == 0) s_fail = 0;
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLLRecvStart] = global_ns();
  __syncthreads();
  // headers: one thread per source
  if (tid < R) {
    const uint64_t* hdr = &hv.sig(me)->ll_hdr[slot][tid];
    const uint64_t t0 = global_ns();
    uint64_t v = ld_relaxed_sys64(hdr);
    uint32_t spins = 0;
    while (!epoch_reached(static_cast<uint32_t>(v >> 32), e)) {
      if ((++spins & 31u) == 0u && (global_ns() - t0 > hv.timeout_ns || has_error(hv.status))) {
        report_error(hv.status, kTimeoutLLHeader, 5, me, tid, e, static_cast<uint32_t>(v >> 32));
        s_fail = 1;
        break;
      }
      __nanosleep(32);
      v = ld_relaxed_sys64(hdr);
    }
    if (!s_fail) v = ld_acquire_sys64(hdr);
    s_T[tid] = epoch_reached(static_cast<uint32_t>(v >> 32), e) ? static_cast<int>(v & 0xffffffffu) : 0;
    s_bcnt[tid] = 0;
    // every slot of source tid has landed once its counter passes what was consumed before
    if (!s_fail && s_T[tid] > 0) {
      const uint32_t target = ls->ll_expect[slot][tid] + static_cast<uint32_t>(s_T[tid]);
      if (!wait_epoch(&hv.sig(me)->ll_cnt[slot][tid], target, hv.timeout_ns, hv.status, kTimeoutLLRow, 5, me, tid))
        s_fail = 1;
    }
    if (a.wait_stats && blockIdx.x == 0)
      atomicAdd(reinterpret_cast<unsigned long long*>(&a.wait_stats[tid]),
                static_cast<unsigned long long>(global_ns() - t0));
  }
  __syncthreads();
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLLRecvReady] = global_ns();
  if (tid == 0) {
    int run = 0;
    for (int s = 0; s < R; ++s) {
      s_toff[s] = run;
      run += min(s_T[s], Mll);
    }
    s_toff[R] = run;
  }
  __syncthreads();
  const int total = s_toff[R];
  const int lo_slot = static_cast<int>(static_cast<int64_t>(total) * part / a.split);
  const int hi_slot = static_cast<int>(static_cast<int64_t>(total) * (part + 1) / a.split);
  __shared__ int s_own[kLLRecvThreads];
  int running = 0;
  for (int tile = 0; tile < hi_slot; tile += kLLRecvThreads) {
    const int i = tile + tid;
    int hit = -1, s = 0, t = 0;
    if (i < hi_slot && !s_fail) {
      while (s + 1 < R && s_toff[s + 1] <= i) ++s;
      t = i - s_toff[s];
      const int64_t slot_row = static_cast<int64_t>(s) * Mll + t;
      const int32_t* ids = hv.at<int32_t>(me, hv.L.ll_ids[slot]) + slot_row * K;
      if ((K & 3) == 0) {
        // the counter acquire above ordered these loads; vector loads keep the chain short
        for (int k0 = 0; k0 < K && hit < 0; k0 += 4) {
          const int4 v = *reinterpret_cast<const int4*>(ids + k0);
          if (v.x == want) hit = k0;
          else if (v.y == want) hit = k0 + 1;
          else if (v.z == want) hit = k0 + 2;
          else if (v.w == want) hit = k0 + 3;
        }
      } else {
        for (int k = 0; k < K; ++k)
          if (hit < 0 && ids[k] == want) hit = k;
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
      s_tile_total = run;
    }
    __syncthreads();
    const int tile_total = s_tile_total;
    if (hit >= 0) {
      const int q = s_wcnt[warp] + __popc(b & lanemask_lt());
      const int p = running + q;
      const bool own = i >= lo_slot;
      s_tok[q] = t;
      s_src[q] = s;
      s_dst[q] = p;
      s_own[q] = own;
      if (own) {
        a.src_info[le * RM + p] = t;
        a.pair_meta[le * RM + p] = s * K + hit;
      }
      atomicAdd(&s_bcnt[s], 1);
    }
    __syncthreads();  // rows acquired by other threads are ordered by the barrier
    for (int q = warp; q < tile_total; q += nwarps) {
      if (!s_own[q]) continue;
      const int t2 = s_tok[q], s2 = s_src[q], p = s_dst[q];
      const uint8_t* row = hv.at<uint8_t>(me, hv.L.ll_rows[slot]) + (static_cast<int64_t>(s2) * Mll + t2) * rs;
      const int64_t o = le * RM + p;
      warp_copy<8>(a.recv_x + o * PB, row, PB);
      if (a.use_fp8) {
        const float* sc = reinterpret_cast<const float*>(row + H);
        if (a.ue8m0) {
          for (int j = lane; j < nsb; j += 32)
            a.recv_scales[o * nsb + j] = static_cast<uint8_t>((__float_as_uint(sc[j]) >> 23) & 0xFFu);
        } else {
          warp_copy(a.recv_scales + o * nsb * 4, sc, nsb * 4LL);
        }
      }
    }
    running += tile_total;
    __syncthreads();
  }
  if (last_part) {
    if (tid < R) {
      int start = 0;
      for (int s = 0; s < tid; ++s) start += s_bcnt[s];
      a.layout_range[le * R + tid] = (static_cast<int64_t>(start) << 32) | static_cast<int64_t>(s_bcnt[tid]);
    }
    for (int64_t p = running + tid; p < RM; p += kLLRecvThreads) a.src_info[le * RM + p] = -1;
    if (tid == 0) {
      a.recv_count[le] = running;
      if (a.cum_stats) atomicAdd(&a.cum_stats[le], running);
    }
  }
  // the last expert CTA records the slots consumed from each source
  __shared__ int s_last;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&ls->arrive[kArLLRecv], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    if (tid < R) ls->ll_expect[slot][tid] += static_cast<uint32_t>(s_T[tid]);
    if (tid == 0) {
      ls->arrive[kArLLRecv] = 0;
      ls->trace[kTrLLRecvEnd] = global_ns();
    }
  }
}

// two CTAs per SM (<= 64 registers): at EP1 the 256 local experts then fit in one wave
__global__ void __launch_bounds__(kLLRecvThreads, 2) ll_dispatch_recv_kernel(LLRecvArgs a) {
  ll_dispatch_recv_body(a, ldv_u32(&a.hv.local()->epoch[kEpLLD]));
}


static LLRecvArgs ll_recv_args(SymmHeap& heap, at::Tensor recv_x, const OptTensor& recv_scales,
                               at::Tensor recv_count, at::Tensor src_info, at::Tensor layout_range,
                               at::Tensor pair_meta, int64_t num_experts, bool use_fp8, bool ue8m0,
                               const OptTensor& cum_stats, const OptTensor& wait_stats) {
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
  // spread the copies over about 128 CTAs when there are few local experts
  a.split = EL >= 128 ? 1 : std::max(1, std::min(8, 128 / EL));
  return a;
}

void ll_dispatch_recv(SymmHeap& heap, at::Tensor recv_x, const OptTensor& recv_scales, at::Tensor recv_count,
                      at::Tensor src_info, at::Tensor layout_range, at::Tensor pair_meta, int64_t num_experts,
                      bool use_fp8, bool ue8m0, const OptTensor& cum_stats, const OptTensor& wait_stats) {
  const c10::cuda::CUDAGuard guard(recv_x.device());
  const LLRecvArgs a = ll_recv_args(heap, recv_x, recv_scales, recv_count, src_info, layout_range, pair_meta,
                                    num_experts, use_fp8, ue8m0, cum_stats, wait_stats);
  ll_dispatch_recv_kernel<<<(a.E / a.hv.R) * a.split, kLLRecvThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ============================================================================ combine send
struct LCSendArgs {
  HeapView hv;
  const uint8_t* x;     // [EL, >= R*Mll rows, H] 16-bit
  int64_t x_row_stride; // bytes between rows
  int64_t x_exp_stride; // bytes between experts
  const int32_t* recv_count;
  const int32_t* src_info;
  const int32_t* pair_meta;
  int H, K, EL;
};

// persistent grid over (expert, row) items: each warp copies rows home, then the CTA flags
// what it sent to each rank; blockDim.x == kLLThreads
__device__ void ll_combine_send_body(const LCSendArgs& a, uint32_t e) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const int slot = e & 1u;
  const int R = hv.R, Mll = hv.cfg.Mll, H = a.H, K = a.K;
  const int64_t RM = static_cast<int64_t>(R) * Mll;
  const int64_t RB = 2LL * H;
  __shared__ uint32_t s_n[B200EP_MAX_RANKS];
  __shared__ int s_cnt[1025];   // prefix of the per-expert row counts
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  constexpr int nwarps = kLLThreads / 32;
  if (tid < R) s_n[tid] = 0;
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLCSendStart] = global_ns();
  // exclusive prefix of the per-expert row counts: loads in parallel, warp scans, one pass over
  // the warp totals (a serial loop of dependent loads costs a memory latency per expert)
  __shared__ int s_wsum[nwarps];
  __shared__ int s_carry;
  if (tid == 0) s_carry = 0;
  __syncthreads();
  for (int base = 0; base < a.EL; base += kLLThreads) {
    const int le = base + tid;
    const int c = le < a.EL ? min(a.recv_count[le], static_cast<int>(RM)) : 0;
    int v = c;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, d);
      if (lane >= d) v += u;
    }
    if (lane == 31) s_wsum[warp] = v;
    __syncthreads();
    if (tid == 0) {
      int run = s_carry;
      for (int w = 0; w < nwarps; ++w) {
        const int x = s_wsum[w];
        s_wsum[w] = run;
        run += x;
      }
      s_carry = run;
    }
    __syncthreads();
    if (le < a.EL) s_cnt[le] = s_wsum[warp] + v - c;
    __syncthreads();
  }
  if (tid == 0) s_cnt[a.EL] = s_carry;
  __syncthreads();
  const int total = s_cnt[a.EL];
  // valid rows only, one warp per row
  for (int i = blockIdx.x * nwarps + warp; i < total; i += gridDim.x * nwarps) {
    int lo = 0, hi = a.EL - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_cnt[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int le = lo, p = i - s_cnt[le];
    const int t = a.src_info[le * RM + p];
    const int sk = a.pair_meta[le * RM + p];
    const int s = sk / K, k = sk % K;
    if (t < 0 || t >= Mll || s < 0 || s >= R) continue;
    uint8_t* dst = hv.base[s] + hv.L.lc_rows[slot] + (static_cast<int64_t>(t) * K + k) * RB;
    warp_copy<16>(dst, a.x + le * a.x_exp_stride + p * a.x_row_stride, RB);
    if (lane == 0) atomicAdd(&s_n[s], 1u);
  }
  __syncthreads();
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLCSendStored] = global_ns();
  if (tid < R && s_n[tid] > 0) {
    signal_add(&hv.sig(tid)->lc_cnt[slot][hv.rank], s_n[tid], tid == hv.rank);
  }
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLCSendReleased] = global_ns();
}

__global__ void __launch_bounds__(kLLThreads) ll_combine_send_kernel(LCSendArgs a) {
  LocalState* ls = a.hv.local();
  const uint32_t e = ldv_u32(&ls->epoch[kEpLLC]) + 1u;
  ll_combine_send_body(a, e);
  finish_epoch(ls, kEpLLC, e, kTrLCSendEnd);
}

static LCSendArgs lc_send_args(SymmHeap& heap, const at::Tensor& x, const at::Tensor& recv_count,
                               const at::Tensor& src_info, const at::Tensor& pair_meta, int64_t num_experts) {
  HeapView hv = heap.view();
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && x.element_size() == 2, "x must be 16-bit [EL, rows, H]");
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
  TORCH_CHECK(x.size(0) == a.EL && a.EL <= 1024, "x must have one slab per local expert (at most 1024)");
  TORCH_CHECK(a.H % 8 == 0 && a.x_row_stride % 16 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0,
              "x rows must be 16-byte aligned");
  return a;
}

void ll_combine_send(SymmHeap& heap, const at::Tensor& x, const at::Tensor& recv_count, const at::Tensor& src_info,
                     const at::Tensor& pair_meta, int64_t num_experts, int64_t num_sms) {
  const c10::cuda::CUDAGuard guard(x.device());
  const LCSendArgs a = lc_send_args(heap, x, recv_count, src_info, pair_meta, num_experts);
  const int sms = num_sms > 0 ? static_cast<int>(num_sms) : heap.num_sms();
  ll_combine_send_kernel<<<sms, kLLThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
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

// tokens t = blockIdx.x, blockIdx.x + gridDim.x, ...; every thread issues the K slot loads of
// a 16-byte chunk together; blockDim.x == kLLThreads
template <typename T16>
__device__ void ll_combine_recv_body(const LCRecvArgs& a, uint32_t e) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const int slot = e & 1u;
  const int me = hv.rank, H = a.H, K = a.K;
  const int64_t RB = 2LL * H;
  const int tid = threadIdx.x;
  __shared__ float s_w[32];
  __shared__ uint32_t s_valid;
  __shared__ uint32_t s_exp[B200EP_MAX_RANKS];
  __shared__ int s_fail;
  const int R = hv.R, EL = a.E / R;
  const uint8_t* rows = hv.at<uint8_t>(me, hv.L.lc_rows[slot]);
  // rows expected from every rank = this rank's valid (token, k) entries owned by it
  if (tid < R) s_exp[tid] = 0;
  if (tid == 0) s_fail = 0;
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLCRecvStart] = global_ns();
  __syncthreads();
  for (int64_t i = tid; i < static_cast<int64_t>(a.T) * K; i += kLLThreads) {
    const int64_t g = a.topk_i32 ? static_cast<const int32_t*>(a.topk)[i] : static_cast<const int64_t*>(a.topk)[i];
    if (g >= 0 && g < a.E) atomicAdd(&s_exp[g / EL], 1u);
  }
  __syncthreads();
  if (tid < R && s_exp[tid] > 0) {
    const uint32_t target = ls->lc_expect[slot][tid] + s_exp[tid];
    if (!wait_epoch(&hv.sig(me)->lc_cnt[slot][tid], target, hv.timeout_ns, hv.status, kTimeoutLLCombine, 6, me, tid))
      s_fail = 1;
  }
  __syncthreads();  // rows acquired by threads < R are read by every thread after this
  if (blockIdx.x == 0 && tid == 0) ls->trace[kTrLCRecvReady] = global_ns();
  for (int t = blockIdx.x; t < a.T && !s_fail; t += gridDim.x) {
    if (tid < 32) {
      bool valid = false;
      float wk = 0.f;
      if (tid < K) {
        const int64_t i = static_cast<int64_t>(t) * K + tid;
        const int64_t g = a.topk_i32 ? static_cast<const int32_t*>(a.topk)[i] : static_cast<const int64_t*>(a.topk)[i];
        valid = g >= 0 && g < a.E;
        wk = valid ? a.w[i] : 0.f;
      }
      s_w[tid] = wk;
      const uint32_t vm = __ballot_sync(0xffffffffu, valid);
      if (tid == 0) s_valid = vm;
    }
    __syncthreads();
    const uint32_t vmask = s_valid;
    const uint8_t* trow = rows + static_cast<int64_t>(t) * K * RB;
    T16* out = reinterpret_cast<T16*>(a.out) + static_cast<int64_t>(t) * H;
    const int nchunk = H / 8;
    for (int j = tid; j < nchunk; j += kLLThreads) {
      int4 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k < K && ((vmask >> k) & 1u)) v[k] = reinterpret_cast<const int4*>(trow + k * RB)[j];
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k < K && ((vmask >> k) & 1u)) {
          const float wv = s_w[k];
          const T16* h = reinterpret_cast<const T16*>(&v[k]);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += static_cast<float>(h[i]) * wv;
        }
      }
      for (int k = 8; k < K; ++k) {  // top-k above 8: remaining slots one at a time
        if ((vmask >> k) & 1u) {
          const int4 r = reinterpret_cast<const int4*>(trow + k * RB)[j];
          const float wv = s_w[k];
          const T16* h = reinterpret_cast<const T16*>(&r);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[i] += static_cast<float>(h[i]) * wv;
        }
      }
      int4 o;
      T16* oh = reinterpret_cast<T16*>(&o);
#pragma unroll
      for (int i = 0; i < 8; ++i) oh[i] = static_cast<T16>(acc[i]);
      reinterpret_cast<int4*>(out)[j] = o;
    }
    __syncthreads();
  }
  // the last CTA records the rows consumed from each rank
  __shared__ int s_last;
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(&ls->arrive[kArLCRecv], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last) {
    if (tid < R) ls->lc_expect[slot][tid] += s_exp[tid];
    if (tid == 0) {
      ls->arrive[kArLCRecv] = 0;
      ls->trace[kTrLCRecvEnd] = global_ns();
    }
  }
}

template <typename T16>
__global__ void __launch_bounds__(kLLThreads) ll_combine_recv_kernel(LCRecvArgs a) {
  ll_combine_recv_body<T16>(a, ldv_u32(&a.hv.local()->epoch[kEpLLC]));
}


static LCRecvArgs lc_recv_args(SymmHeap& heap, const at::Tensor& topk_idx, const at::Tensor& topk_w,
                               at::Tensor out) {
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
  TORCH_CHECK(a.H % 8 == 0 && a.T <= hv.cfg.Mll && a.K <= hv.cfg.K && a.K <= 32, "combine shape exceeds the buffer");
  return a;
}

void ll_combine_recv(SymmHeap& heap, const at::Tensor& topk_idx, const at::Tensor& topk_w, at::Tensor out,
                     int64_t num_sms) {
  const c10::cuda::CUDAGuard guard(out.device());
  const LCRecvArgs a = lc_recv_args(heap, topk_idx, topk_w, out);
  if (a.T == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (out.scalar_type() == at::kHalf)
    ll_combine_recv_kernel<__half><<<a.T, kLLThreads, 0, stream>>>(a);
  else
    ll_combine_recv_kernel<__nv_bfloat16><<<a.T, kLLThreads, 0, stream>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  (void)num_sms;
}

}  // namespace b200ep
