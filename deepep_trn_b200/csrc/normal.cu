// Normal-mode dispatch and combine over NVLink peer memory (N2, N3, N6 fused).
//
// Reference semantics: deep_ep_trn/buffer.py:169-266. Received rows are ordered by
// (source rank, source token); combine sums each token's returned rows in fp32 and
// casts once. The reference packs rows on the host, runs one fixed-slot all-to-all-v
// per op and unpacks (transport/nki_a2av.py:47-75, buffer.py:143-156); here each op
// is one cooperative kernel in which sending and receiving overlap row by row.
//
// Dispatch (nd_kernel), CTA b of G owns source tokens [T*b/G, T*(b+1)/G):
//   1. scan: the CTA counts its range's rows per destination; after a grid barrier (held
//      by CTA 0 until every peer has entered this dispatch, so the ranks push together)
//      every CTA knows where its range starts in each destination's block, writes the
//      token -> row map (token_pos) and sends each destination (first row, rows) of its
//      range; CTA 0 sends this rank's row totals and per-expert counts. These control
//      words are self-tagged and sent with relaxed stores before any row (second grid
//      barrier).
//   2. push (every warp): each token row goes straight from x to every other rank that
//      owns one of its experts, 16-byte stores into that rank's inbox over NVLink
//      (fp8 e4m3 + 1x128 scales quantised in registers on the way when asked), with
//      the token's top-k ids, weights and index appended; then one thread per destination
//      publishes that the CTA's range has landed (a system-scope release).
//   3. receive (every warp): as soon as every source's total is in, CTA 0 publishes the
//      receive size to the host; every CTA then copies, for each source s, the rows
//      that s's CTA b pushed (once its progress word is in) from the inbox to recv_x
//      at recv_off[s] + row, with the metadata. Rows a rank keeps come from x directly.
// Combine (nc_kernel), same grid and the same ranges: expert rank r's CTA b pushes the
// rows of every source s's range b back into s's combine inbox (weights appended) and publishes;
// then source s's CTA b reduces the tokens of range b in fp32 as their rows are in (own
// rows read from x in place), adds the optional bias and casts once. The CTAs of a GPU
// are not in step, so some push while others already receive.
//
// Ordering: payload stores, a block barrier, then a system-scope fence and release store
// of the progress word by one thread per destination; receivers poll the word with
// system-scope relaxed loads and acquire it before reading rows. Dispatch and combine have
// separate inboxes, progress words and sequence numbers: a rank writes into a peer's inbox
// of one kind for op q only after that peer reported that it finished reading that inbox
// for op q - 1 (inbox_free / cinbox_free), which every rank sends at the end of its kernel.
// Every wait is bounded by the buffer's timeout and reports into the host-mapped status page.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cstdlib>

#include "ops.h"

namespace b200ep {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
// Each CTA first pushes (every warp), then publishes one progress word per destination,
// then receives or reduces (every warp). Splitting the roles in time rather than across the
// warps of an SM was measured to matter: while receiving warps of the same SM were active,
// the system-scope release that follows a CTA's NVLink stores took 0.7-2.2 ms to complete
// (B200, EP2); with the SM doing nothing else it completes as soon as the stores have landed,
// and CTAs still overlap with one another (some push while others receive).
__device__ __forceinline__ int32_t ldv_i32(const int32_t* p) { return *reinterpret_cast<const volatile int32_t*>(p); }
__device__ __forceinline__ uint32_t ldv_u32(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

// Destination bits of token row `p` (R bytes of is_token_in_rank).
__device__ __forceinline__ uint32_t row_mask(const bool* p, int R) {
  uint32_t m = 0;
  const uint8_t* b = reinterpret_cast<const uint8_t*>(p);
  for (int r = 0; r < R; ++r) m |= (b[r] != 0 ? 1u : 0u) << r;
  return m;
}

// Bounded spin on a 64-bit (q << 32) | value word until its tag is q; returns the value
// (or -1 after recording a timeout). The word is written by another GPU, so it is polled
// with system-scope relaxed loads (a GPU-scope load need not observe a peer GPU's store: the
// peer's thread is outside the .gpu scope), backing off between polls, and acquired once at
// system scope when the tag matches. Callers keep the pollers few (one thread per peer and
// CTA): thousands of threads polling a few L2 lines were measured to slow the NVLink writes
// arriving at the GPU.
__device__ __forceinline__ int64_t wait_tagged(const uint64_t* p, uint32_t q, const HeapView& hv, uint32_t code,
                                               uint32_t op, int peer) {
  uint64_t v = ld_relaxed_sys64(p);
  if (static_cast<uint32_t>(v >> 32) != q) {
    const uint64_t t0 = global_ns();
    uint32_t spins = 0;
    while (true) {
      __nanosleep(128);
      v = ld_relaxed_sys64(p);
      if (static_cast<uint32_t>(v >> 32) == q) break;
      if ((++spins & 15u) == 0u && (global_ns() - t0 > hv.timeout_ns || has_error(hv.status))) {
        report_error(hv.status, code, op, hv.rank, peer, q, static_cast<uint32_t>(v >> 32));
        return -1;
      }
    }
  }
  v = ld_acquire_sys64(p);
  return static_cast<int64_t>(v & 0xffffffffu);
}

// Bounded wait until a tagged progress word reports at least `want` rows for op q (one
// thread polls; same system-scope polling and final acquire as wait_tagged). Returns the rows seen.
__device__ __forceinline__ int64_t wait_progress(const uint64_t* p, uint32_t q, int64_t want, const HeapView& hv,
                                                 uint32_t op, int peer) {
  auto ok = [&](uint64_t x) {
    return static_cast<uint32_t>(x >> 32) == q && static_cast<int64_t>(x & 0xffffffffu) >= want;
  };
  uint64_t v = ld_relaxed_sys64(p);
  if (!ok(v)) {
    const uint64_t t0 = global_ns();
    uint32_t spins = 0;
    while (true) {
      __nanosleep(128);
      v = ld_relaxed_sys64(p);
      if (ok(v)) break;
      if ((++spins & 15u) == 0u && (global_ns() - t0 > hv.timeout_ns || has_error(hv.status))) {
        report_error(hv.status, kTimeoutReady, op, hv.rank, peer, static_cast<uint32_t>(want),
                     static_cast<uint32_t>(v & 0xffffffffu));
        return -1;
      }
    }
  }
  v = ld_acquire_sys64(p);
  return static_cast<int64_t>(v & 0xffffffffu);
}

// Bounded spin until the bits `mask` of a self-tagged control word equal `tag`; the word's
// other bits are its value, so no acquire follows (nothing else is read on its account).
// Same polling as wait_tagged. Returns false after recording a timeout.
__device__ __forceinline__ bool wait_word(const uint64_t* p, uint64_t mask, uint64_t tag, const HeapView& hv,
                                          uint32_t op, int peer, uint64_t* out) {
  uint64_t v = ld_relaxed_sys64(p);
  if ((v & mask) != tag) {
    const uint64_t t0 = global_ns();
    uint32_t spins = 0;
    while (true) {
      __nanosleep(128);
      v = ld_relaxed_sys64(p);
      if ((v & mask) == tag) break;
      if ((++spins & 15u) == 0u && (global_ns() - t0 > hv.timeout_ns || has_error(hv.status))) {
        report_error(hv.status, kTimeoutReady, op, hv.rank, peer, static_cast<uint32_t>(tag >> 32),
                     static_cast<uint32_t>(v >> 32));
        return false;
      }
    }
  }
  *out = v;
  return true;
}

// Barrier over the CTAs of a cooperative launch (all resident); bounded. Every CTA must
// call it the same number of times, errors included.
__device__ bool grid_barrier(LocalState* ls, const HeapView& hv, uint32_t op) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    s_ok = 1;
    const uint32_t gen = ldv_u32(&ls->gbar_gen);
    __threadfence();
    if (atomicAdd(&ls->gbar_count, 1u) == gridDim.x - 1) {
      ls->gbar_count = 0;
      __threadfence();
      atomicExch(&ls->gbar_gen, gen + 1u);
    } else {
      const uint64_t t0 = global_ns();
      while (ldv_u32(&ls->gbar_gen) == gen) {
        __nanosleep(32);
        if (global_ns() - t0 > hv.timeout_ns) {
          report_error(hv.status, kTimeoutBarrier, op, hv.rank, -1, gen + 1u, gen);
          s_ok = 0;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
  return s_ok != 0;
}

// Last CTA to arrive ends the op: publishes the sequence number of its kind (kEpInbox for
// dispatch, kEpCInbox for combine) locally and tells every peer that this rank's inbox of that
// kind may be written for the next op.
__device__ void finish_op(LocalState* ls, const HeapView& hv, int which, uint32_t q, int trace_point) {
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(&ls->arrive[which], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  if (threadIdx.x == 0) {
    ls->arrive[which] = 0;
    ls->epoch[which] = q;
    ls->trace[trace_point] = global_ns();
  }
  if (threadIdx.x < hv.R) {
    Signals* sp = hv.sig(threadIdx.x);
    st_release_sys(which == kEpInbox ? &sp->inbox_free[hv.rank] : &sp->cinbox_free[hv.rank], q);
  }
}

// Wait (threads < R) until every peer finished reading its inbox of kind `which` for op q - 1.
__device__ void wait_inboxes_free(const HeapView& hv, int which, uint32_t q, int* s_fail) {
  if (threadIdx.x < hv.R && threadIdx.x != hv.rank) {
    Signals* sp = hv.sig(hv.rank);
    const uint32_t* f = which == kEpInbox ? &sp->inbox_free[threadIdx.x] : &sp->cinbox_free[threadIdx.x];
    if (!wait_epoch(f, q - 1u, hv.timeout_ns, hv.status, kTimeoutReady, which == kEpInbox ? 10 : 11, hv.rank,
                    threadIdx.x))
      atomicExch(s_fail, 1);
  }
}

template <typename T16>
__device__ __forceinline__ void acc8(float (&acc)[8], const int4& raw) {
  const T16* h = reinterpret_cast<const T16*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] += static_cast<float>(h[i]);
}

}  // namespace

// ============================================================================ dispatch
struct NdArgs {
  HeapView hv;
  const uint8_t* x;
  int64_t x_stride;       // bytes between rows of x
  const float* xs;        // mode 1: scales [T, H/128]
  int64_t xs_stride;      // elements
  int mode;               // 0: 16-bit payload, 1: fp8 payload + scales given, 2: quantise 16-bit -> fp8
  int x_fp16, round_scale;
  const void* topk;       // [T, K] or null (cached dispatch)
  int topk_i32;
  const float* topk_w;    // [T, K] or null
  const int32_t* nte;     // [E] tokens per expert of this rank, or null
  const bool* in_rank;    // [T, R]
  int32_t* token_pos;     // out [T, R]: row of token t in rank r's block for this source, -1 if not sent
  int32_t* send_start;    // out [G, R]: first row of CTA b's range in each destination's block
  int32_t* recv_info;     // out [R, kMaxGrid, 2]: (first row, rows) of each (source, CTA) range here
  int64_t* recv_off;      // out [R + 1]: first received row of each source
  uint8_t* recv_x;
  float* recv_scales;
  void* recv_topk;
  int recv_topk_i32;
  float* recv_w;
  void* recv_src;
  int recv_src_i32;
  int64_t capacity;       // rows of the receive outputs
  int T, H, K, E;
  uint64_t ticket;
  int pad_rows;           // fill the metadata of rows [N, capacity) (sync-free sizing)
};

// Push warp `pw` writes token t to every destination of `dmask`: payload, scales, ids,
// weights, token index. Rows for destination p go to p's inbox block `me`, row pos[p].
template <typename T16>
__device__ void push_token(const NdArgs& a, int t, uint32_t dmask, const int32_t* pos) {
  const HeapView& hv = a.hv;
  const int lane = lane_id(), me = hv.rank, M = hv.cfg.M, H = a.H, K = a.K;
  const int64_t IS = hv.L.inbox_stride;
  const int P = a.mode == 0 ? 2 * H : H;
  const int S = a.mode == 0 ? 0 : (H / 128) * 4;
  auto row_of = [&](int p) -> uint8_t* {
    return hv.base[p] + hv.L.inbox + (static_cast<int64_t>(me) * M + pos[p]) * IS;
  };
  const uint8_t* src = a.x + static_cast<int64_t>(t) * a.x_stride;
  if (a.mode == 0 || a.mode == 1) {
    // 16-byte chunks, eight loads in flight per lane, each stored to every destination
    const int64_t n = P >> 4;
    const int4* s = reinterpret_cast<const int4*>(src);
    int64_t i = lane;
    for (; i + 224 < n; i += 256) {
      int4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = s[i + 32 * u];
      for (uint32_t m = dmask; m; m &= m - 1) {
        int4* d = reinterpret_cast<int4*>(row_of(__ffs(m) - 1));
#pragma unroll
        for (int u = 0; u < 8; ++u) d[i + 32 * u] = v[u];
      }
    }
    for (; i < n; i += 32) {
      const int4 v = s[i];
      for (uint32_t m = dmask; m; m &= m - 1) reinterpret_cast<int4*>(row_of(__ffs(m) - 1))[i] = v;
    }
    if (a.mode == 1) {
      const float* sc = a.xs + static_cast<int64_t>(t) * a.xs_stride;
      for (int j = lane; j < H / 128; j += 32) {
        const float v = sc[j];
        for (uint32_t m = dmask; m; m &= m - 1) reinterpret_cast<float*>(row_of(__ffs(m) - 1) + P)[j] = v;
      }
    }
  } else {
    // quantise 1x128 blocks in registers: four 256-element chunks per pass, each lane 8 values
    const T16* xv = reinterpret_cast<const T16*>(src);
    for (int c0 = 0; c0 < H; c0 += 1024) {
      float v[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int off = c0 + u * 256 + lane * 8;
        load8(v[u], xv + off, off < H);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int off = c0 + u * 256 + lane * 8;
        const Quant8 r = quant8_e4m3(v[u], a.round_scale);
        if (off < H) {
          for (uint32_t m = dmask; m; m &= m - 1) {
            uint8_t* row = row_of(__ffs(m) - 1);
            *reinterpret_cast<uint2*>(row + off) = r.q;
            if ((lane & 15) == 0) reinterpret_cast<float*>(row + P)[off / 128] = r.scale;
          }
        }
      }
    }
  }
  // metadata: ids and weights (lanes < K), token index (lane 31)
  if (lane < K || lane == 31) {
    int32_t id = -1;
    float w = 0.f;
    if (lane < K) {
      const int64_t i = static_cast<int64_t>(t) * K + lane;
      if (a.topk) id = a.topk_i32 ? static_cast<const int32_t*>(a.topk)[i]
                                  : static_cast<int32_t>(static_cast<const int64_t*>(a.topk)[i]);
      if (a.topk_w) w = a.topk_w[i];
    }
    for (uint32_t m = dmask; m; m &= m - 1) {
      uint8_t* meta = row_of(__ffs(m) - 1) + P + S;
      if (lane < K) {
        reinterpret_cast<int32_t*>(meta)[lane] = id;
        reinterpret_cast<float*>(meta + 4 * K)[lane] = w;
      } else {
        *reinterpret_cast<int32_t*>(meta + 8 * K) = t;
      }
    }
  }
}

// Receive warp: write row `i` of the outputs from source s's token t (payload at `payload`,
// scales at `scales` if fp8; ids / weights from `ids` / `wts`, or from the caller's arrays).
__device__ __forceinline__ void emit_meta(const NdArgs& a, int64_t i, int t, const int32_t* ids, const float* wts) {
  const int lane = lane_id(), K = a.K, R = a.hv.R;
  const int EL = a.E / R, lo = a.hv.rank * EL;
  if (lane == 0) {
    if (a.recv_src_i32)
      static_cast<int32_t*>(a.recv_src)[i] = t;
    else
      static_cast<int64_t*>(a.recv_src)[i] = t;
  }
  if (a.recv_topk && lane < K) {
    const int32_t g = ids[lane];
    const bool local = g >= lo && g < lo + EL;
    const int64_t o = i * K + lane;
    if (a.recv_topk_i32)
      static_cast<int32_t*>(a.recv_topk)[o] = local ? g - lo : -1;
    else
      static_cast<int64_t*>(a.recv_topk)[o] = local ? g - lo : -1;
    if (a.recv_w) a.recv_w[o] = local && wts ? wts[lane] : 0.f;
  }
}

template <typename T16>
__global__ void __launch_bounds__(kThreads, 1) nd_kernel(NdArgs a) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t q = ldv_u32(&ls->epoch[kEpInbox]) + 1u;
  const int me = hv.rank, R = hv.R, M = hv.cfg.M, H = a.H, K = a.K;
  const int G = gridDim.x, b = blockIdx.x;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  const int T = min(a.T, M);
  const int t0 = static_cast<int>(static_cast<int64_t>(T) * b / G);
  const int t1 = static_cast<int>(static_cast<int64_t>(T) * (b + 1) / G);
  const int64_t IS = hv.L.inbox_stride;
  const int P = a.mode == 0 ? 2 * H : H;
  const int S = a.mode == 0 ? 0 : (H / 128) * 4;

  __shared__ int s_fail;
  __shared__ int32_t s_cnt[B200EP_MAX_RANKS];     // rows of my range per destination
  __shared__ int32_t s_start[B200EP_MAX_RANKS];   // first row of my range in each destination's block
  __shared__ int32_t s_tot[B200EP_MAX_RANKS];     // this rank's rows per destination
  __shared__ int32_t s_run[B200EP_MAX_RANKS];
  __shared__ int32_t s_wcnt[kWarps][B200EP_MAX_RANKS];
  __shared__ int64_t s_roff[B200EP_MAX_RANKS + 1];
  __shared__ int32_t s_rcount[B200EP_MAX_RANKS];  // rows each source sends this rank
  __shared__ int32_t s_pos[kWarps][B200EP_MAX_RANKS];

  if (tid == 0) s_fail = 0;
  if (tid < R) s_cnt[tid] = 0;
  if (a.T > M && b == 0 && tid == 0) report_error(hv.status, kCapacity, 1, me, -1, M, a.T);
  if (b == 0 && tid == 0) {
    ls->trace[kTrNdStart] = global_ns();
    ls->trace[kTrNdWaitNs] = 0;
  }
  // CTA 0 tells every peer that this rank entered dispatch q (relaxed: a timing signal only)
  if (b == 0 && tid < R && tid != me) st_relaxed_sys(&hv.sig(tid)->nd_start[me], q);
  __syncthreads();
  wait_inboxes_free(hv, kEpInbox, q, &s_fail);
  if (b == 0) {  // block-uniform
    __syncthreads();
    if (tid == 0) ls->trace[kTrNdFreeIn] = global_ns();
  }

  // ---------------------------------------------------------------- scan
  for (int tt = t0; tt < t1; tt += kThreads) {
    const int t = tt + tid;
    const uint32_t m = t < t1 ? row_mask(a.in_rank + static_cast<int64_t>(t) * R, R) : 0u;
    for (int r = 0; r < R; ++r) {
      const uint32_t bb = __ballot_sync(0xffffffffu, (m >> r) & 1u);
      if (lane == 0 && bb) atomicAdd(&s_cnt[r], __popc(bb));
    }
  }
  __syncthreads();
  int32_t* rcnt = hv.at<int32_t>(me, hv.L.nd_rcnt);
  if (tid < R) rcnt[b * R + tid] = s_cnt[tid];
  // The ranks start pushing together: CTA 0 holds the grid barrier below until every peer has
  // entered this dispatch. Without it a rank that finished its previous combine early pushed
  // alone, then waited for the late rank's rows, and the lead swapped ranks from op to op
  // (B200, EP2: ~110 us of skew, 0.51 ms per step against 0.31 ms with the ranks in phase).
  if (b == 0 && tid < R && tid != me &&
      !wait_epoch(&hv.sig(me)->nd_start[tid], q, hv.timeout_ns, hv.status, kTimeoutReady, 12, me, tid))
    s_fail = 1;
  if (!grid_barrier(ls, hv, 1) && tid == 0) s_fail = 1;
  if (b == 0 && tid == 0) ls->trace[kTrNdBarrier] = global_ns();
  for (int r = warp; r < R; r += kWarps) {
    int before = 0, all = 0;
    for (int c = lane; c < G; c += 32) {
      const int v = ldv_i32(rcnt + c * R + r);
      all += v;
      if (c < b) before += v;
    }
    before = warp_sum(before);
    all = warp_sum(all);
    if (lane == 0) {
      s_start[r] = before;
      s_run[r] = before;
      s_tot[r] = all;
    }
  }
  __syncthreads();
  for (int tt = t0; tt < t1; tt += kThreads) {
    const int t = tt + tid;
    const uint32_t m = t < t1 ? row_mask(a.in_rank + static_cast<int64_t>(t) * R, R) : 0u;
    int pre[B200EP_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < B200EP_MAX_RANKS; ++r) {
      if (r < R) {
        const uint32_t bb = __ballot_sync(0xffffffffu, (m >> r) & 1u);
        pre[r] = __popc(bb & lanemask_lt());
        if (lane == 0) s_wcnt[warp][r] = __popc(bb);
      }
    }
    __syncthreads();
    if (tid < R) {
      int run = s_run[tid];
      for (int w = 0; w < kWarps; ++w) {
        const int c = s_wcnt[w][tid];
        s_wcnt[w][tid] = run;
        run += c;
      }
      s_run[tid] = run;
    }
    __syncthreads();
    if (t < t1) {
      int32_t* pos = a.token_pos + static_cast<int64_t>(t) * R;
#pragma unroll
      for (int r = 0; r < B200EP_MAX_RANKS; ++r)
        if (r < R) pos[r] = ((m >> r) & 1u) ? s_wcnt[warp][r] + pre[r] : -1;
    }
    __syncthreads();
  }
  if (tid < R) a.send_start[b * R + tid] = s_start[tid];
  if (tid == 0) {  // this rank's own range b in its own block (used by combine's pair mode)
    a.recv_info[(static_cast<int64_t>(me) * kMaxGrid + b) * 2] = s_start[me];
    a.recv_info[(static_cast<int64_t>(me) * kMaxGrid + b) * 2 + 1] = s_cnt[me];
  }
  __syncthreads();  // s_fail from the inbox waits
  const bool fail0 = s_fail != 0;
  if (!fail0) {
    // Control words are self-tagged 64-bit values written with relaxed stores: a word is valid
    // once its tag is this op's, so no fence orders them and none waits for earlier remote
    // stores to be acknowledged. (A release behind remote stores completes only after their
    // acks, which queue behind the peer's own row traffic in the other direction: totals sent
    // that way reached a busy peer ~120 us late at EP2.) To destination p:
    //   info[me][b]  (q & 0xffff) << 48 | first row of my range b in p's block << 24 | its rows
    //   nd_cnt[me]   q << 32 | (my CTAs - 1) << 24 | my rows for p          (CTA 0)
    //   nd_nte[me][le]  q << 32 | my tokens for p's local expert le         (CTA 0)
    if (tid < R) {
      st_relaxed_sys64(hv.at<uint64_t>(tid, hv.L.info) + static_cast<int64_t>(me) * kMaxGrid + b,
                       (static_cast<uint64_t>(q & 0xffffu) << 48) |
                           (static_cast<uint64_t>(s_start[tid]) << 24) | static_cast<uint64_t>(s_cnt[tid]));
      if (b == 0)
        st_relaxed_sys64(&hv.sig(tid)->nd_cnt[me], (static_cast<uint64_t>(q) << 32) |
                                                       (static_cast<uint64_t>(G - 1) << 24) |
                                                       static_cast<uint64_t>(s_tot[tid]));
    }
    if (b == 0) {
      if (a.nte) {
        const int EL = a.E / R;
        for (int i = tid; i < a.E; i += kThreads) {
          const int p = i / EL;
          st_relaxed_sys64(hv.at<uint64_t>(p, hv.L.nd_nte) + me * EL + (i - p * EL),
                           (static_cast<uint64_t>(q) << 32) | static_cast<uint32_t>(a.nte[i]));
        }
      }
      if (tid == 0) ls->trace[kTrNdScanned] = global_ns();
    }
  }
  // Every CTA's control words leave before any CTA pushes rows, so they do not queue behind
  // row traffic: a receiver cannot place any row before it has every source's total. The
  // barrier is taken on every path (errors included).
  if (!grid_barrier(ls, hv, 2) && tid == 0) s_fail = 1;
  __syncthreads();
  const bool fail1 = s_fail != 0;

  // ---------------------------------------------------------------- push (every warp)
  if (!fail1) {
    for (int t = t0 + warp; t < t1; t += kWarps) {
      uint32_t m = 0;
      if (lane < R) {
        const int32_t p = a.token_pos[static_cast<int64_t>(t) * R + lane];
        s_pos[warp][lane] = p;
        m = (p >= 0 && lane != me) ? 1u : 0u;
      }
      const uint32_t dmask = __ballot_sync(0xffffffffu, m);
      __syncwarp();
      if (dmask) push_token<T16>(a, t, dmask, s_pos[warp]);
      __syncwarp();
    }
  }
  __syncthreads();
  if (b == 0 && tid == 0) ls->trace[kTrNdPushed] = global_ns();
  // one release per destination covers every row of this CTA's range (an empty range too)
  if (!fail1 && tid < R && tid != me) {
    fence_sys();
    st_release_sys64(hv.at<uint64_t>(tid, hv.L.prog) + static_cast<int64_t>(me) * kMaxGrid + b,
                     (static_cast<uint64_t>(q) << 32) | static_cast<uint32_t>(s_cnt[tid]));
  }
  if (b == 0 && tid == 0) ls->trace[kTrNdPublished] = global_ns();

  // ---------------------------------------------------------------- receive (every warp)
  __shared__ int s_rfail;
  if (tid == 0) s_rfail = fail1 ? 1 : 0;
  __syncthreads();
  __shared__ int32_t s_istart[B200EP_MAX_RANKS], s_icnt[B200EP_MAX_RANKS];  // source s's range b here
  if (!fail1) {
    uint64_t v = 0;
    if (tid < R) {
      // source tid's rows for this rank, and its grid size
      if (!wait_word(&hv.sig(me)->nd_cnt[tid], 0xffffffff00000000ull, static_cast<uint64_t>(q) << 32, hv, 1, tid,
                     &v)) {
        s_rfail = 1;
        s_rcount[tid] = 0;
      } else {
        const int g = static_cast<int>((v >> 24) & 0xffu) + 1;
        s_rcount[tid] = static_cast<int32_t>(v & 0xffffffu);
        if (g != G) {
          report_error(hv.status, kBadInput, 1, me, tid, G, static_cast<uint32_t>(g));
          s_rfail = 1;
        }
      }
    } else if (tid >= 32 && tid < 32 + R) {
      // source s's range b: first row in block s and rows (another warp polls these)
      const int s = tid - 32;
      if (s == me) {
        s_istart[s] = s_start[me];
        s_icnt[s] = s_cnt[me];
      } else if (wait_word(hv.at<uint64_t>(me, hv.L.info) + static_cast<int64_t>(s) * kMaxGrid + b,
                           0xffff000000000000ull, static_cast<uint64_t>(q & 0xffffu) << 48, hv, 1, s, &v)) {
        s_istart[s] = static_cast<int32_t>((v >> 24) & 0xffffffu);
        s_icnt[s] = static_cast<int32_t>(v & 0xffffffu);
        if (s_istart[s] + s_icnt[s] > M) {  // a range must lie inside the source's block
          report_error(hv.status, kBadInput, 1, me, s, M, static_cast<uint32_t>(s_istart[s] + s_icnt[s]));
          s_icnt[s] = 0;
          s_rfail = 1;
        }
      } else {
        s_istart[s] = 0;
        s_icnt[s] = 0;
        s_rfail = 1;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    int64_t off = 0;
    for (int s = 0; s < R; ++s) {
      s_roff[s] = off;
      off += s_rfail ? 0 : s_rcount[s];
    }
    s_roff[R] = off;
    if (off > a.capacity) {
      report_error(hv.status, kCapacity, 2, me, -1, static_cast<uint32_t>(a.capacity), static_cast<uint32_t>(off));
      s_rfail = 1;
    }
  }
  __syncthreads();
  const bool rfail = s_rfail != 0;
  const int64_t N = rfail ? 0 : s_roff[R];
  if (b == 0) {
    // handle offsets and the host notify page
    if (tid <= R) a.recv_off[tid] = rfail ? 0 : s_roff[tid];
    HostPage* host = hv.host;
    if (tid < R) host->notify.recv_counts[tid] = rfail ? 0 : s_rcount[tid];
    const int EL = a.E / R;
    for (int le = tid; le < EL && le < 1024; le += kThreads) {
      int32_t sum = 0;
      if (!rfail && a.nte)
        for (int s = 0; s < R; ++s) {
          uint64_t v = 0;
          if (wait_word(hv.at<uint64_t>(me, hv.L.nd_nte) + s * EL + le, 0xffffffff00000000ull,
                        static_cast<uint64_t>(q) << 32, hv, 1, s, &v))
            sum += static_cast<int32_t>(v & 0xffffffffu);
        }
      host->notify.per_expert[le] = sum;
    }
    if (tid == 0) {
      ls->trace[kTrNdCounts] = global_ns();
      host->notify.num_recv = N;
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence_system();
      st_release_sys64(const_cast<uint64_t*>(&host->notify.ticket), a.ticket);
      ls->trace[kTrNdNotified] = global_ns();
    }
  }
  if (!rfail) {
    // rows this rank keeps: straight from x (or quantised from it) into their final place
    const int64_t base = s_roff[me];
    for (int t = t0 + warp; t < t1; t += kWarps) {
      const int32_t p = a.token_pos[static_cast<int64_t>(t) * R + me];
      if (p < 0) continue;
      const int64_t i = base + p;
      const uint8_t* src = a.x + static_cast<int64_t>(t) * a.x_stride;
      if (a.mode == 0) {
        warp_copy(a.recv_x + i * P, src, P);
      } else if (a.mode == 1) {
        warp_copy(a.recv_x + i * P, src, P);
        warp_copy(a.recv_scales + i * (H / 128), a.xs + static_cast<int64_t>(t) * a.xs_stride, S);
      } else {
        warp_quant_row<T16>(a.recv_x + i * P, a.recv_scales + i * (H / 128), reinterpret_cast<const T16*>(src), H,
                            a.round_scale);
      }
      // metadata from the caller's arrays
      if (lane == 0) {
        if (a.recv_src_i32)
          static_cast<int32_t*>(a.recv_src)[i] = t;
        else
          static_cast<int64_t*>(a.recv_src)[i] = t;
      }
      if (a.recv_topk && lane < K) {
        const int EL = a.E / R, lo = me * EL;
        const int64_t k = static_cast<int64_t>(t) * K + lane;
        const int32_t g = a.topk_i32 ? static_cast<const int32_t*>(a.topk)[k]
                                     : static_cast<int32_t>(static_cast<const int64_t*>(a.topk)[k]);
        const bool local = g >= lo && g < lo + EL;
        const int64_t o = i * K + lane;
        if (a.recv_topk_i32)
          static_cast<int32_t*>(a.recv_topk)[o] = local ? g - lo : -1;
        else
          static_cast<int64_t*>(a.recv_topk)[o] = local ? g - lo : -1;
        if (a.recv_w) a.recv_w[o] = local && a.topk_w ? a.topk_w[k] : 0.f;
      }
    }
    uint64_t waited = 0;  // ns this warp spent waiting for progress words (CTA 0 reports it)
    // rows pushed by other ranks: for each source (rotated), the rows of its CTA b's range
    for (int k = 1; k < R; ++k) {
      const int s = (me + R - k) % R;
      const int64_t start = s_istart[s], cnt = s_icnt[s];
      if (tid == 0) {
        const uint64_t tw = global_ns();
        // the whole range lands before its one progress word
        if (cnt > 0 && wait_progress(hv.at<uint64_t>(me, hv.L.prog) + static_cast<int64_t>(s) * kMaxGrid + b, q,
                                     cnt, hv, 1, s) < 0)
          s_rfail = 1;
        waited += global_ns() - tw;
      }
      __syncthreads();  // every thread reads rows that thread 0 acquired
      if (s_rfail) break;
      if (tid == 0) {
        a.recv_info[(static_cast<int64_t>(s) * kMaxGrid + b) * 2] = static_cast<int32_t>(start);
        a.recv_info[(static_cast<int64_t>(s) * kMaxGrid + b) * 2 + 1] = static_cast<int32_t>(cnt);
      }
      const uint8_t* blk = hv.at<uint8_t>(me, hv.L.inbox) + static_cast<int64_t>(s) * M * IS;
      for (int64_t u = warp; u < cnt; u += kWarps) {
        const int64_t j = start + u;
        const uint8_t* row = blk + j * IS;
        const int64_t i = s_roff[s] + j;
        warp_copy(a.recv_x + i * P, row, P);
        if (S) warp_copy(a.recv_scales + i * (H / 128), row + P, S);
        const int32_t* ids = reinterpret_cast<const int32_t*>(row + P + S);
        const float* wts = reinterpret_cast<const float*>(row + P + S + 4 * K);
        const int t = *reinterpret_cast<const int32_t*>(row + P + S + 8 * K);
        emit_meta(a, i, t, ids, wts);
      }
      __syncthreads();
    }
    if (tid == 0 && s_rfail) report_error(hv.status, kTimeoutReady, 1, me, -1, 0, 0, 3);
    if (b == 0 && tid == 0) ls->trace[kTrNdWaitNs] = waited;
  }
  // sync-free sizing: the rows past N carry no expert (-1), weight 0 and source -1
  if (a.pad_rows) {
    for (int64_t i = N + static_cast<int64_t>(b) * kThreads + tid; i < a.capacity;
         i += static_cast<int64_t>(G) * kThreads) {
      if (a.recv_src_i32)
        static_cast<int32_t*>(a.recv_src)[i] = -1;
      else
        static_cast<int64_t*>(a.recv_src)[i] = -1;
      if (a.recv_topk)
        for (int k = 0; k < K; ++k) {
          if (a.recv_topk_i32)
            static_cast<int32_t*>(a.recv_topk)[i * K + k] = -1;
          else
            static_cast<int64_t*>(a.recv_topk)[i * K + k] = -1;
          if (a.recv_w) a.recv_w[i * K + k] = 0.f;
        }
    }
  }
  if (b == 0 && tid == 0) ls->trace[kTrNdRecvd] = global_ns();
  __syncthreads();
  finish_op(ls, hv, kEpInbox, q, kTrNdEnd);
}

void nd_dispatch(SymmHeap& heap, const at::Tensor& x, const OptTensor& x_scales, int64_t mode, bool round_scale,
                 const OptTensor& topk_idx, const OptTensor& topk_w, const OptTensor& nte, const at::Tensor& in_rank,
                 at::Tensor token_pos, at::Tensor send_start, at::Tensor recv_info, at::Tensor recv_off,
                 at::Tensor recv_x, const OptTensor& recv_scales, const OptTensor& recv_topk,
                 const OptTensor& recv_w, at::Tensor recv_src, int64_t num_experts, int64_t ticket, int64_t grid,
                 bool pad_rows) {
  const c10::cuda::CUDAGuard guard(x.device());
  HeapView hv = heap.view();
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [T, H] with unit inner stride");
  TORCH_CHECK(in_rank.is_contiguous() && in_rank.scalar_type() == at::kBool && in_rank.size(1) == hv.R,
              "is_token_in_rank must be a contiguous [T, R] bool tensor");
  TORCH_CHECK(token_pos.is_contiguous() && token_pos.scalar_type() == at::kInt, "token_pos must be int32");
  TORCH_CHECK(recv_off.numel() == hv.R + 1 && recv_off.scalar_type() == at::kLong, "recv_off must be [R+1] int64");
  TORCH_CHECK(num_experts <= hv.cfg.E && num_experts % hv.R == 0, "num_experts exceeds the buffer");
  TORCH_CHECK(hv.cfg.M < (1 << 24), "at most 2^24 - 1 tokens per rank (24-bit row fields of the control words)");
  NdArgs a{};
  a.hv = hv;
  a.T = static_cast<int>(x.size(0));
  a.H = static_cast<int>(x.size(1));
  TORCH_CHECK(a.H <= hv.cfg.H && a.H % 8 == 0, "hidden must be a multiple of 8 within the buffer's hidden size");
  a.x = static_cast<const uint8_t*>(x.data_ptr());
  a.x_stride = x.stride(0) * x.element_size();
  TORCH_CHECK(a.T == 0 || ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && a.x_stride % 16 == 0),
              "x rows must be 16-byte aligned");
  a.mode = static_cast<int>(mode);
  if (mode == 0) TORCH_CHECK(x.element_size() == 2, "16-bit payload expected");
  if (mode != 0) TORCH_CHECK(a.H % 128 == 0, "fp8 dispatch needs hidden % 128 == 0");
  if (mode == 1) {
    TORCH_CHECK(x.element_size() == 1 && x_scales.has_value(), "fp8 input needs (x_fp8, scales)");
    TORCH_CHECK(x_scales->scalar_type() == at::kFloat && unit_inner(*x_scales), "scales must be fp32");
    a.xs = x_scales->data_ptr<float>();
    a.xs_stride = x_scales->stride(0);
  }
  if (mode == 2)
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kHalf, "quantise needs bf16/fp16 x");
  a.x_fp16 = x.scalar_type() == at::kHalf;
  a.round_scale = round_scale;
  a.K = topk_idx.has_value() ? static_cast<int>(topk_idx->size(1)) : hv.cfg.K;
  TORCH_CHECK(a.K <= 30 && a.K <= hv.cfg.K, "top-k exceeds the buffer (at most 30)");
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
  }
  a.in_rank = in_rank.data_ptr<bool>();
  a.token_pos = token_pos.data_ptr<int32_t>();
  a.E = static_cast<int>(num_experts);
  a.ticket = static_cast<uint64_t>(ticket);
  const int G = grid > 0 ? static_cast<int>(std::min<int64_t>(grid, kMaxGrid)) : heap.num_sms();
  TORCH_CHECK(G >= 1 && G <= kMaxGrid, "grid out of range");
  TORCH_CHECK(send_start.is_contiguous() && send_start.numel() >= static_cast<int64_t>(G) * hv.R &&
                  send_start.scalar_type() == at::kInt, "send_start must hold [grid, R] int32");
  TORCH_CHECK(recv_info.is_contiguous() && recv_info.numel() >= static_cast<int64_t>(hv.R) * kMaxGrid * 2 &&
                  recv_info.scalar_type() == at::kInt, "recv_info must hold [R, 256, 2] int32");
  a.send_start = send_start.data_ptr<int32_t>();
  a.recv_info = recv_info.data_ptr<int32_t>();
  a.recv_off = recv_off.data_ptr<int64_t>();
  TORCH_CHECK(recv_x.is_contiguous() && recv_x.size(1) == a.H, "recv_x must be contiguous [cap, H]");
  a.recv_x = static_cast<uint8_t*>(recv_x.data_ptr());
  a.capacity = recv_x.size(0);
  if (mode != 0) {
    TORCH_CHECK(recv_scales.has_value() && recv_scales->is_contiguous(), "fp8 dispatch needs recv_scales");
    a.recv_scales = recv_scales->data_ptr<float>();
  }
  if (recv_topk.has_value()) {
    a.recv_topk = recv_topk->data_ptr();
    a.recv_topk_i32 = recv_topk->scalar_type() == at::kInt;
    TORCH_CHECK(recv_topk->size(1) == a.K, "recv_topk width must equal top-k");
  }
  if (recv_w.has_value()) a.recv_w = recv_w->data_ptr<float>();
  a.recv_src = recv_src.data_ptr();
  a.recv_src_i32 = recv_src.scalar_type() == at::kInt;
  a.pad_rows = pad_rows ? 1 : 0;
  void* fn = a.x_fp16 ? reinterpret_cast<void*>(nd_kernel<__half>) : reinterpret_cast<void*>(nd_kernel<__nv_bfloat16>);
  void* args[] = {&a};
  // cooperative: CTAs wait for one another (grid barrier) and for peers' CTAs, so all must be resident
  AT_CUDA_CHECK(cudaLaunchCooperativeKernel(fn, dim3(G), dim3(kThreads), args, 0, at::cuda::getCurrentCUDAStream()));
}

// ============================================================================ combine
struct NcArgs {
  HeapView hv;
  const uint8_t* x;         // [N, H] rows received by this rank's dispatch (expert outputs)
  int64_t x_stride;         // bytes
  const float* w;           // [N, K] (may be null when N == 0)
  int64_t w_stride;
  int has_w;                // the op carries top-k weights (every rank passes them)
  const int64_t* recv_off;  // [R + 1]
  const int32_t* recv_info; // [R, kMaxGrid, 2]
  const int32_t* token_pos; // [T, R]
  const int32_t* send_start;// [G, R]
  uint8_t* out;
  float* out_w;
  const uint8_t* bias0;
  const uint8_t* bias1;
  int T, H, K;
  // pair mode: row i of x is sum_k pair_w[i, k] * pairs[pair_pos[i, k]] (fp32, one cast), formed
  // by the pushing warps from the expert outputs in permuted order (an unpermute fused in)
  const uint8_t* pairs;     // [P, H] 16-bit, or null
  const int32_t* pair_pos;  // [N, PK], -1 = no pair
  const float* pair_w;      // [N, PK]
  int PK;
};

// Pair mode: one warp forms row i = sum_k w[i, k] * pairs[pos[i, k]] in fp32 (k ascending) and
// stores its 16-bit cast at dst.
template <typename T16>
__device__ void push_pair_row(const NcArgs& a, int64_t i, uint8_t* dst) {
  const int lane = lane_id(), PK = a.PK, nch = a.H / 8;
  const int32_t mp = lane < PK ? a.pair_pos[i * PK + lane] : -1;
  const float mw = lane < PK ? a.pair_w[i * PK + lane] : 0.f;
  constexpr int U = 4;
  // the loop bounds are warp-uniform (every lane takes part in the shuffles)
  for (int base = 0; base < nch; base += 32 * U) {
    const int c0 = base + lane;
    float acc[U][8];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[u][e] = 0.f;
    for (int k = 0; k < PK; ++k) {
      const int32_t p = __shfl_sync(0xffffffffu, mp, k);
      const float wk = __shfl_sync(0xffffffffu, mw, k);
      if (p < 0) continue;
      const int4* src = reinterpret_cast<const int4*>(a.pairs + static_cast<int64_t>(p) * a.H * 2);
      int4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (c0 + 32 * u < nch) v[u] = src[c0 + 32 * u];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (c0 + 32 * u >= nch) continue;
        const T16* h = reinterpret_cast<const T16*>(&v[u]);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[u][e] += static_cast<float>(h[e]) * wk;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = c0 + 32 * u;
      if (c >= nch) continue;
      int4 o;
      T16* oh = reinterpret_cast<T16*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) oh[e] = static_cast<T16>(acc[u][e]);
      reinterpret_cast<int4*>(dst)[c] = o;
    }
  }
}

template <typename T16>
__global__ void __launch_bounds__(kThreads, 1) nc_kernel(NcArgs a) {
  const HeapView& hv = a.hv;
  LocalState* ls = hv.local();
  const uint32_t q = ldv_u32(&ls->epoch[kEpCInbox]) + 1u;
  const int me = hv.rank, R = hv.R, M = hv.cfg.M, H = a.H, K = a.K;
  const int G = gridDim.x, b = blockIdx.x;
  const int tid = threadIdx.x, lane = lane_id(), warp = warp_id();
  const int64_t IS = hv.L.cinbox_stride;
  const int64_t RB = 2LL * H;

  __shared__ int s_fail;
  __shared__ int64_t s_off[B200EP_MAX_RANKS + 1];
  __shared__ int32_t s_start[B200EP_MAX_RANKS], s_cnt[B200EP_MAX_RANKS];
  if (tid == 0) s_fail = 0;
  if (tid <= R) s_off[tid] = a.recv_off[tid];
  if (tid < R) {
    s_start[tid] = a.recv_info[(static_cast<int64_t>(tid) * kMaxGrid + b) * 2];
    // own rows are read from x in place; in pair mode they are formed and written locally too
    s_cnt[tid] = (tid == me && !a.pairs) ? 0 : a.recv_info[(static_cast<int64_t>(tid) * kMaxGrid + b) * 2 + 1];
  }
  if (b == 0 && tid == 0) {
    ls->trace[kTrNcStart] = global_ns();
    ls->trace[kTrNcWaitNs] = 0;
  }
  __syncthreads();
  wait_inboxes_free(hv, kEpCInbox, q, &s_fail);
  __syncthreads();
  const bool fail0 = s_fail != 0;

  // ---------------------------------------------------------------- push rows home (every warp)
  if (!fail0) {
    // rows of every source's range, the sources rotated per CTA so the CTAs of a rank spread
    // their stores over all peers at once
    for (int it = warp;; it += kWarps) {
      int s = -1, u = 0, rem = it;
      for (int k = 1; k <= R; ++k) {
        const int ss = (me + b + k) % R;   // (own rows have no count unless in pair mode)
        if (rem < s_cnt[ss]) {
          s = ss;
          u = rem;
          break;
        }
        rem -= s_cnt[ss];
      }
      if (s < 0) break;
      const int64_t j = s_start[s] + u;
      const int64_t i = s_off[s] + j;
      uint8_t* dst = hv.base[s] + hv.L.cinbox + (static_cast<int64_t>(me) * M + j) * IS;
      if (a.pairs)
        push_pair_row<T16>(a, i, dst);
      else
        warp_copy(dst, a.x + i * a.x_stride, RB);
      if (a.has_w && lane < K) reinterpret_cast<float*>(dst + RB)[lane] = a.w[i * a.w_stride + lane];
    }
  }
  __syncthreads();
  if (b == 0 && tid == 0) ls->trace[kTrNcPushed] = global_ns();
  // one release per source covers every row of its range (an empty range too)
  if (!fail0 && tid < R && (tid != me || a.pairs)) {
    uint64_t* pw = hv.at<uint64_t>(tid, hv.L.cprog) + static_cast<int64_t>(me) * kMaxGrid + b;
    const uint64_t word = (static_cast<uint64_t>(q) << 32) | static_cast<uint32_t>(s_cnt[tid]);
    if (tid == me) {  // pair mode's own rows: writer and readers on this GPU
      fence_gpu();
      st_release_gpu64(pw, word);
    } else {
      fence_sys();
      st_release_sys64(pw, word);
    }
  }
  if (b == 0 && tid == 0) ls->trace[kTrNcPublished] = global_ns();
  // ---------------------------------------------------------------- wait for this range's rows
  // One thread per rank polls that rank's progress word for range b (one word per range, so its
  // tag alone says the range has landed). Keeping the pollers few matters: a few thousand
  // threads polling the same few lines of L2 slowed the NVLink writes arriving at this GPU
  // to a trickle (B200, EP2).
  __shared__ int s_wfail;
  if (tid == 0) s_wfail = fail0 ? 1 : 0;
  __syncthreads();
  uint64_t waited = 0;
  if (!fail0 && tid < R && (tid != me || a.pairs)) {
    const uint64_t tw = global_ns();
    if (wait_tagged(hv.at<uint64_t>(me, hv.L.cprog) + static_cast<int64_t>(tid) * kMaxGrid + b, q, hv,
                    kTimeoutCombine, 3, tid) < 0)
      s_wfail = 1;
    waited = global_ns() - tw;
  }
  __syncthreads();  // every thread reads rows that the pollers acquired
  if (b == 0 && tid < R) atomicMax(reinterpret_cast<unsigned long long*>(&ls->trace[kTrNcWaitNs]),
                                   static_cast<unsigned long long>(waited));
  {
    // ------------------------------------------------------------ reduce my tokens (every warp)
    const int rw = warp;
    const int t0 = static_cast<int>(static_cast<int64_t>(a.T) * b / G);
    const int t1 = static_cast<int>(static_cast<int64_t>(a.T) * (b + 1) / G);
    __shared__ const uint8_t* s_rows[kWarps][B200EP_MAX_RANKS];
    __shared__ const float* s_wrows[kWarps][B200EP_MAX_RANKS];
    const uint8_t* inbox = hv.at<uint8_t>(me, hv.L.cinbox);
    const int nch = H / 8;
    const bool wfail = s_wfail != 0;
    for (int t = t0 + rw; t < t1 && !wfail; t += kWarps) {
      // this token's rows: one per rank that received it
      int32_t pos = lane < R ? a.token_pos[static_cast<int64_t>(t) * R + lane] : -1;
      const uint8_t* rp = nullptr;
      const float* wp = nullptr;
      if (pos >= 0) {
        if (lane == me && !a.pairs) {
          const int64_t i = s_off[me] + pos;
          rp = a.x + i * a.x_stride;
          wp = a.has_w ? a.w + i * a.w_stride : nullptr;
        } else {
          rp = inbox + (static_cast<int64_t>(lane) * M + pos) * IS;
          wp = a.has_w ? reinterpret_cast<const float*>(rp + RB) : nullptr;
        }
      }
      const uint32_t have = __ballot_sync(0xffffffffu, pos >= 0);
      const int nr = __popc(have);
      if (pos >= 0) {
        const int k = __popc(have & lanemask_lt());
        s_rows[rw][k] = rp;
        s_wrows[rw][k] = wp;
      }
      __syncwarp();
      T16* out = reinterpret_cast<T16*>(a.out) + static_cast<int64_t>(t) * H;
      const T16* b0 = a.bias0 ? reinterpret_cast<const T16*>(a.bias0) + static_cast<int64_t>(t) * H : nullptr;
      const T16* b1 = a.bias1 ? reinterpret_cast<const T16*>(a.bias1) + static_cast<int64_t>(t) * H : nullptr;
      constexpr int U = 4;
      for (int c0 = lane; c0 < nch; c0 += 32 * U) {
        float acc[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[u][e] = 0.f;
        int r = 0;
        for (; r + 1 < nr; r += 2) {
          const uint8_t* p0 = s_rows[rw][r];
          const uint8_t* p1 = s_rows[rw][r + 1];
          int4 v0[U], v1[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int c = c0 + 32 * u;
            if (c < nch) {
              v0[u] = reinterpret_cast<const int4*>(p0)[c];
              v1[u] = reinterpret_cast<const int4*>(p1)[c];
            }
          }
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + 32 * u < nch) {
              acc8<T16>(acc[u], v0[u]);
              acc8<T16>(acc[u], v1[u]);
            }
        }
        if (r < nr) {
          const uint8_t* p0 = s_rows[rw][r];
          int4 v0[U];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + 32 * u < nch) v0[u] = reinterpret_cast<const int4*>(p0)[c0 + 32 * u];
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (c0 + 32 * u < nch) acc8<T16>(acc[u], v0[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + 32 * u;
          if (c >= nch) continue;
          if (b0) acc8<T16>(acc[u], reinterpret_cast<const int4*>(b0)[c]);
          if (b1) acc8<T16>(acc[u], reinterpret_cast<const int4*>(b1)[c]);
          int4 o;
          T16* oh = reinterpret_cast<T16*>(&o);
#pragma unroll
          for (int e = 0; e < 8; ++e) oh[e] = static_cast<T16>(acc[u][e]);
          reinterpret_cast<int4*>(out)[c] = o;
        }
      }
      if (a.out_w && lane < K) {
        float sw = 0.f;
        for (int r = 0; r < nr; ++r) {
          const float* wr = s_wrows[rw][r];
          if (wr) sw += wr[lane];
        }
        a.out_w[static_cast<int64_t>(t) * K + lane] = sw;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  if (b == 0 && tid == 0) ls->trace[kTrNcReduced] = global_ns();
  finish_op(ls, hv, kEpCInbox, q, kTrNcEnd);
}

void nc_combine(SymmHeap& heap, const at::Tensor& x, const OptTensor& w, const at::Tensor& recv_off,
                const at::Tensor& recv_info, const at::Tensor& token_pos, const at::Tensor& send_start, at::Tensor out,
                const OptTensor& out_w, const OptTensor& bias0, const OptTensor& bias1, int64_t grid,
                const OptTensor& pair_pos, const OptTensor& pair_w) {
  const c10::cuda::CUDAGuard guard(out.device());
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
  TORCH_CHECK(a.H <= hv.cfg.H && a.H % 8 == 0, "hidden must be a multiple of 8 within the buffer's hidden size");
  TORCH_CHECK(x.size(0) == 0 || ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && a.x_stride % 16 == 0),
              "combine x rows must be 16-byte aligned");
  a.K = 0;
  if (w.has_value()) {
    TORCH_CHECK(w->scalar_type() == at::kFloat && unit_inner(*w), "topk_weights must be fp32");
    a.w = w->data_ptr<float>();
    a.w_stride = w->stride(0);
    a.has_w = 1;
    a.K = static_cast<int>(w->size(1));
    TORCH_CHECK(a.K <= hv.cfg.K && a.K <= 32, "top-k exceeds the buffer");
  }
  a.recv_off = recv_off.data_ptr<int64_t>();
  a.recv_info = recv_info.data_ptr<int32_t>();
  a.token_pos = token_pos.data_ptr<int32_t>();
  a.send_start = send_start.data_ptr<int32_t>();
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
  if (pair_pos.has_value()) {
    // x holds the expert outputs in permuted order; rows are formed from it by pair_pos / pair_w
    TORCH_CHECK(pair_w.has_value() && pair_pos->is_contiguous() && pair_pos->scalar_type() == at::kInt &&
                    pair_w->is_contiguous() && pair_w->scalar_type() == at::kFloat &&
                    pair_w->sizes() == pair_pos->sizes() && pair_pos->size(1) <= 32,
                "pair mode needs contiguous pair_pos [N, K] int32 and pair_w [N, K] fp32 (K <= 32)");
    TORCH_CHECK(x.is_contiguous(), "pair mode needs contiguous expert outputs");
    a.pairs = a.x;
    a.pair_pos = pair_pos->data_ptr<int32_t>();
    a.pair_w = pair_w->data_ptr<float>();
    a.PK = static_cast<int>(pair_pos->size(1));
  }
  const int G = static_cast<int>(grid);
  TORCH_CHECK(G >= 1 && G <= kMaxGrid && send_start.numel() >= static_cast<int64_t>(G) * hv.R,
              "combine must run on the grid of its dispatch");
  void* fn = x.scalar_type() == at::kHalf ? reinterpret_cast<void*>(nc_kernel<__half>)
                                          : reinterpret_cast<void*>(nc_kernel<__nv_bfloat16>);
  void* args[] = {&a};
  AT_CUDA_CHECK(cudaLaunchCooperativeKernel(fn, dim3(G), dim3(kThreads), args, 0, at::cuda::getCurrentCUDAStream()));
}

}  // namespace b200ep
