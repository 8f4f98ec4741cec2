// Raw NVLink transfer engines, measured in isolation (no routing, no flags).
//
// Every rank moves `bytes_per_peer` bytes to or from every other rank of the EP group at
// the same time (the all-to-all pattern of dispatch and combine), with one of the engines
// the data paths can use:
//
//   0  pull, TMA   : one thread per CTA drives a ring of cp.async.bulk loads from the peer
//                    into shared memory and bulk stores into local memory
//   1  pull, LSU   : warps load 16-byte vectors from the peer, store them locally
//   2  push, TMA   : bulk loads of local memory, bulk stores into the peer
//   3  push, LSU   : warps load locally, store 16-byte vectors into the peer
//   4  pull, TMA, no local store (NVLink read rate alone)
//   5  pull, TMA, one ring per warp (lane 0 of every warp drives its own stages)
//
// Chunks alternate between peers so every link carries traffic at once. The source of a
// pull is the peer's region [me][off], its destination this rank's region [p][off]; a push
// mirrors that. The regions are the two halves of the normal-mode inbox of the heap.
// Reference counterpart: the raw transport curve of bench/bench_transport.py (an NKI
// all-to-all-v there).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "ops.h"

namespace b200ep {

namespace {

struct BwArgs {
  HeapView hv;
  int mode;
  int64_t bpp;      // bytes per peer
  int chunk;        // bytes per transfer (multiple of 16)
  int nstages;      // ring stages per driving thread
  int64_t src_off, dst_off;
};

__device__ __forceinline__ void bw_addr(const BwArgs& a, int64_t q, const uint8_t*& src, uint8_t*& dst) {
  const HeapView& hv = a.hv;
  const int me = hv.rank, R = hv.R;
  const int np = R > 1 ? R - 1 : 1;
  const int p = R > 1 ? (me + 1 + static_cast<int>(q % np)) % R : me;
  const int64_t off = (q / np) * a.chunk;
  const bool push = a.mode == 2 || a.mode == 3;
  if (!push) {
    src = hv.base[p] + a.src_off + static_cast<int64_t>(me) * a.bpp + off;
    dst = hv.base[me] + a.dst_off + static_cast<int64_t>(p) * a.bpp + off;
  } else {
    src = hv.base[me] + a.src_off + static_cast<int64_t>(p) * a.bpp + off;
    dst = hv.base[p] + a.dst_off + static_cast<int64_t>(me) * a.bpp + off;
  }
}

// One driving thread: chunks q = q0, q0 + qs, ... (< nq) through `ns` stages of `ring`.
__device__ void bw_tma_ring(const BwArgs& a, int64_t q0, int64_t qs, int64_t nq, uint8_t* ring, uint64_t* bars,
                            int ns, bool store) {
  if (q0 >= nq) return;
  const int64_t n = (nq - q0 + qs - 1) / qs;
  const uint32_t bytes = static_cast<uint32_t>(a.chunk);
  auto issue = [&](int64_t i) {
    const int st = static_cast<int>(i % ns);
    const uint8_t* src;
    uint8_t* dst;
    bw_addr(a, q0 + i * qs, src, dst);
    mbar_arrive_expect_tx(&bars[st], bytes);
    bulk_load(ring + static_cast<int64_t>(st) * a.chunk, src, bytes, &bars[st]);
  };
  uint32_t phase = 0;
  const int64_t pro = n < ns ? n : ns;
  for (int64_t i = 0; i < pro; ++i) issue(i);
  int64_t m = 0;
  for (; m < n; ++m) {
    const int st = static_cast<int>(m % ns);
    if (!mbar_wait(&bars[st], (phase >> st) & 1u, a.hv.timeout_ns)) {
      report_error(a.hv.status, kTimeoutReady, 90, a.hv.rank, -1, 0, 0, 1);
      break;
    }
    phase ^= 1u << st;
    if (store) {
      const uint8_t* src;
      uint8_t* dst;
      bw_addr(a, q0 + m * qs, src, dst);
      bulk_store(dst, ring + static_cast<int64_t>(st) * a.chunk, bytes);
      bulk_commit();
      const int64_t i = m - 1 + ns;
      if (m >= 1 && i < n) {
        bulk_wait_read<1>();
        issue(i);
      }
    } else if (m + ns < n) {
      issue(m + ns);
    }
  }
  if (m < n) {
    // a wait ran out: let the loads still in flight land before shared memory is released
    for (int64_t i = m + 1; i < n && i < m + ns; ++i) {
      const int st = static_cast<int>(i % ns);
      mbar_wait(&bars[st], (phase >> st) & 1u, a.hv.timeout_ns);
    }
  }
  if (store) bulk_wait<0>();
}

__global__ void __launch_bounds__(512) nvl_bw_kernel(BwArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int R = a.hv.R;
  const int np = R > 1 ? R - 1 : 1;
  const int64_t nq = (a.bpp / a.chunk) * np;
  const int tid = threadIdx.x, warp = warp_id(), lane = lane_id();
  const int nwarps = blockDim.x / 32;
  if (a.mode == 1 || a.mode == 3) {
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * nwarps + warp, GW = static_cast<int64_t>(gridDim.x) * nwarps;
    for (int64_t q = gw; q < nq; q += GW) {
      const uint8_t* src;
      uint8_t* dst;
      bw_addr(a, q, src, dst);
      warp_copy(dst, src, a.chunk);
    }
    return;
  }
  const bool per_warp = a.mode == 5;
  const int ns = a.nstages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<int64_t>(per_warp ? nwarps : 1) * ns * a.chunk);
  if (tid == 0) {
    for (int i = 0; i < (per_warp ? nwarps : 1) * ns; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (!per_warp) {
    if (tid == 0) bw_tma_ring(a, blockIdx.x, gridDim.x, nq, smem, bars, ns, a.mode != 4);
  } else if (lane == 0) {
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * nwarps + warp, GW = static_cast<int64_t>(gridDim.x) * nwarps;
    bw_tma_ring(a, gw, GW, nq, smem + static_cast<int64_t>(warp) * ns * a.chunk, bars + warp * ns, ns, true);
  }
}

}  // namespace

void nvl_bw(SymmHeap& heap, int64_t mode, int64_t bytes_per_peer, int64_t chunk, int64_t nstages, int64_t grid,
            int64_t threads) {
  const c10::cuda::CUDAGuard guard(heap.device());
  HeapView hv = heap.view();
  TORCH_CHECK(mode >= 0 && mode <= 5, "mode must be 0..5");
  TORCH_CHECK(chunk >= 16 && chunk % 16 == 0 && chunk <= (1 << 20), "chunk must be a multiple of 16 bytes");
  TORCH_CHECK(bytes_per_peer % chunk == 0, "bytes_per_peer must be a multiple of chunk");
  TORCH_CHECK(threads >= 32 && threads <= 512 && threads % 32 == 0, "threads must be 32..512, a multiple of 32");
  const int64_t region = (static_cast<int64_t>(hv.R) * hv.cfg.M * hv.L.inbox_stride) / 2 / 256 * 256;
  TORCH_CHECK(static_cast<int64_t>(hv.R) * bytes_per_peer <= region, "bytes_per_peer exceeds the staging region");
  BwArgs a{};
  a.hv = hv;
  a.mode = static_cast<int>(mode);
  a.bpp = bytes_per_peer;
  a.chunk = static_cast<int>(chunk);
  a.nstages = static_cast<int>(std::max<int64_t>(1, nstages));
  a.src_off = hv.L.inbox;
  a.dst_off = hv.L.inbox + region;
  size_t smem = 0;
  if (mode != 1 && mode != 3) {
    const int rings = mode == 5 ? static_cast<int>(threads / 32) : 1;
    smem = static_cast<size_t>(rings) * a.nstages * a.chunk + static_cast<size_t>(rings) * a.nstages * 8;
    TORCH_CHECK(smem <= 220 * 1024, "ring does not fit in shared memory");
    static std::atomic<uint64_t> seen{0};
    AT_CUDA_CHECK(set_smem_limit_once(seen, nvl_bw_kernel, 227 * 1024));
  }
  const int g = grid > 0 ? static_cast<int>(grid) : heap.num_sms();
  nvl_bw_kernel<<<g, static_cast<int>(threads), smem, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace b200ep
