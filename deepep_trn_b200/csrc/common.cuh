// Device primitives shared by every kernel of the library (sm_100a only).
//
// * scoped memory operations for cross-GPU signalling over NVLink
//   (ld.acquire.sys / st.release.sys / red.release.sys),
// * bounded waits on %globaltimer that record an error in a host-mapped status
//   page and return instead of trapping or hanging,
// * TMA bulk copies (cp.async.bulk, no tensor map; every CTA fetches its own data)
//   completed through shared-memory mbarriers or bulk async-groups.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <atomic>

// Sets a kernel's dynamic shared-memory limit once per device. The attribute belongs to the
// device's context, so a process that drives several GPUs must set it on each of them;
// `seen` keeps one bit per device (setting it twice, from two threads, is harmless).
template <typename Fn>
inline cudaError_t set_smem_limit_once(std::atomic<uint64_t>& seen, Fn fn, int bytes) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
  if (bit != 0 && (seen.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  err = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (err == cudaSuccess) seen.fetch_or(bit, std::memory_order_release);
  return err;
}

#ifndef B200EP_MAX_RANKS
#define B200EP_MAX_RANKS 32
#endif

namespace b200ep {

// ----------------------------------------------------------------------------- status page
// One page of host-mapped memory per Buffer. Kernels write the first error they
// see; the host reads it after a synchronisation point and raises.
enum ErrorCode : uint32_t {
  kOk = 0,
  kTimeoutReady = 1,      // a peer never signalled its staged data
  kTimeoutCombine = 2,    // a peer never delivered combine rows
  kTimeoutLLHeader = 3,   // low-latency: a source never wrote its header
  kTimeoutLLRow = 4,      // low-latency: a row flag never arrived
  kTimeoutLLCombine = 5,  // low-latency combine: a (token, k) slot never arrived
  kCapacity = 6,          // a count exceeded the buffer capacity
  kTimeoutBarrier = 7,
  kBadInput = 8,
};

struct Status {
  uint32_t code;
  uint32_t op;
  int32_t rank;
  int32_t peer;
  uint32_t expected;
  uint32_t seen;
  uint32_t aux;
  uint32_t pad;
};

// Host notify area for normal-mode dispatch (written by the prepare kernel).
struct NotifyPage {
  volatile uint64_t ticket;         // last field written; equals the host's ticket when valid
  int64_t num_recv;                 // rows this rank will receive
  int32_t recv_counts[B200EP_MAX_RANKS];
  int32_t per_expert[1024];         // received (row, local expert) pairs per local expert
};

struct HostPage {
  Status status;
  uint8_t pad0[64 - sizeof(Status)];
  NotifyPage notify;
};

#if defined(__CUDACC__)
__device__ __forceinline__ void report_error(Status* st, uint32_t code, uint32_t op, int rank, int peer,
                                             uint32_t expected, uint32_t seen, uint32_t aux = 0) {
  if (st == nullptr) return;
  if (atomicCAS(&st->code, 0u, code) == 0u) {
    st->op = op;
    st->rank = rank;
    st->peer = peer;
    st->expected = expected;
    st->seen = seen;
    st->aux = aux;
    __threadfence_system();
  }
}

__device__ __forceinline__ bool has_error(const Status* st) {
  return st != nullptr && *reinterpret_cast<const volatile uint32_t*>(&st->code) != 0u;
}

// ----------------------------------------------------------------------------- scoped ops
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_acquire_sys64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_relaxed_sys64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
// For a flag whose writer and readers are on the same GPU (a rank signalling itself) GPU scope
// suffices; a system-scope fence took ~6 us on B200 even with only local stores outstanding.
__device__ __forceinline__ void fence_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void red_add_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Release of a flag at rank `dst`: GPU scope when the flag and its readers are on this GPU.
__device__ __forceinline__ void signal_add(uint32_t* p, uint32_t v, bool local) {
  if (local) {
    fence_gpu();
    red_add_release_gpu(p, v);
  } else {
    fence_sys();
    red_add_release_sys(p, v);
  }
}
// Orders generic-proxy accesses of this thread with its later async-proxy (TMA) ones.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Epochs grow by one per call and wrap at 2^32; compare by signed difference.
__device__ __forceinline__ bool epoch_reached(uint32_t seen, uint32_t want) {
  return static_cast<int32_t>(seen - want) >= 0;
}

// Spin until *flag reaches `want` or the budget runs out. Returns false on timeout
// (after recording it); callers then skip their work and return. Flags are written by other
// GPUs, so they are polled with system-scope relaxed loads (a GPU-scope load need not observe
// a peer's store: with GPU-scope polling a low-latency round took 247 us instead of 63 us at
// EP2 on B200), with a short back-off between polls, and acquired once at system scope.
__device__ __forceinline__ bool wait_epoch(const uint32_t* flag, uint32_t want, uint64_t budget_ns, Status* st,
                                           uint32_t code, uint32_t op, int rank, int peer,
                                           uint64_t* waited_ns = nullptr) {
  uint32_t v = ld_relaxed_sys(flag);
  if (!epoch_reached(v, want)) {
    const uint64_t t0 = global_ns();
    uint32_t spins = 0;
    while (true) {
      __nanosleep(32);
      v = ld_relaxed_sys(flag);
      if (epoch_reached(v, want)) break;
      if ((++spins & 31u) == 0u) {
        const uint64_t dt = global_ns() - t0;
        if (dt > budget_ns || has_error(st)) {
          report_error(st, code, op, rank, peer, want, v);
          return false;
        }
      }
    }
    if (waited_ns) *waited_ns += global_ns() - t0;
  }
  (void)ld_acquire_sys(flag);
  return true;
}

// ----------------------------------------------------------------------------- warp helpers
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Copy n bytes with one warp, using the widest access both pointers allow.
// The 16-byte path keeps U loads per lane in flight (U * 512 bytes per warp; U = 16 covers a
// 7168-wide bf16 row in two round trips, for latency-bound copies of few rows).
template <int U = 8>
__device__ __forceinline__ void warp_copy(void* __restrict__ dst, const void* __restrict__ src, int64_t n) {
  const int lane = lane_id();
  const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src);
  if ((a & 15) == 0 && (n & 15) == 0) {
    const int64_t m = n >> 4;
    int4* d = reinterpret_cast<int4*>(dst);
    const int4* s = reinterpret_cast<const int4*>(src);
    int64_t i = lane;
    for (; i + 32 * (U - 1) < m; i += 32 * U) {
      int4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = s[i + 32 * u];
#pragma unroll
      for (int u = 0; u < U; ++u) d[i + 32 * u] = v[u];
    }
    for (; i < m; i += 32) d[i] = s[i];
  } else if ((a & 3) == 0 && (n & 3) == 0) {
    const int64_t m = n >> 2;
    for (int64_t i = lane; i < m; i += 32)
      reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
  } else {
    for (int64_t i = lane; i < n; i += 32)
      reinterpret_cast<uint8_t*>(dst)[i] = reinterpret_cast<const uint8_t*>(src)[i];
  }
}

// Copy n bytes (multiple of 16, both ends 16-byte aligned) with a whole CTA,
// four 16-byte loads per thread in flight.
__device__ __forceinline__ void cta_copy16(void* __restrict__ dst, const void* __restrict__ src, int64_t n) {
  const int64_t m = n >> 4;
  int4* d = reinterpret_cast<int4*>(dst);
  const int4* s = reinterpret_cast<const int4*>(src);
  const int nt = blockDim.x;
  int64_t i = threadIdx.x;
  for (; i + 3 * nt < m; i += 4 * nt) {
    int4 v0 = s[i], v1 = s[i + nt], v2 = s[i + 2 * nt], v3 = s[i + 3 * nt];
    d[i] = v0; d[i + nt] = v1; d[i + 2 * nt] = v2; d[i + 3 * nt] = v3;
  }
  for (; i < m; i += nt) d[i] = s[i];
}

// ----------------------------------------------------------------------------- mbarrier + TMA bulk
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded mbarrier wait; false if the transaction never completed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t budget_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > budget_ns) return false;
  }
  return true;
}
// plain arrival (count 1) on a CTA-local mbarrier
__device__ __forceinline__ void mbar_arrive_local(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// global (local or peer) -> shared, completion counted on `bar`.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// shared -> global (local or peer), tracked by the bulk async-group of this thread.
__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ----------------------------------------------------------------------------- fp8
// e4m3 with round-to-nearest-even and saturation to +-448 (cvt.rn.satfinite).
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float a, float b) {
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3));
}

// Smallest power of two >= s for a positive normal float, by exponent arithmetic.
__device__ __forceinline__ float pow2_ceil(float s) {
  uint32_t b = __float_as_uint(s);
  uint32_t e = (b >> 23) & 0xFFu;
  if (b & 0x7FFFFFu) e += 1u;
  return __uint_as_float(e << 23);
}

// One lane's share of a 1x128 block quantisation: 8 contiguous values, the
// other 15 lanes of the same half-warp hold the rest of the block. Every lane of
// the warp must call this (it shuffles); inactive lanes pass zeros.
// scale = max(amax, 1e-4) / 448 (or its power-of-two ceiling); q = rn_satfinite(v * (448 / amax)).
struct Quant8 {
  uint2 q;
  float scale;
};
__device__ __forceinline__ Quant8 quant8_e4m3(const float (&v)[8], bool round_scale) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int m = 8; m >= 1; m >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, m));
  amax = fmaxf(amax, 1e-4f);
  float scale, inv;
  if (round_scale) {
    scale = pow2_ceil(__fdiv_rn(amax, 448.f));
    inv = __fdiv_rn(1.f, scale);
  } else {
    scale = __fdiv_rn(amax, 448.f);
    inv = __fdiv_rn(448.f, amax);
  }
  Quant8 r;
  r.q.x = uint32_t(f32x2_to_e4m3x2(v[0] * inv, v[1] * inv)) | (uint32_t(f32x2_to_e4m3x2(v[2] * inv, v[3] * inv)) << 16);
  r.q.y = uint32_t(f32x2_to_e4m3x2(v[4] * inv, v[5] * inv)) | (uint32_t(f32x2_to_e4m3x2(v[6] * inv, v[7] * inv)) << 16);
  r.scale = scale;
  return r;
}

// Load 8 contiguous 16-bit values as fp32 (zeros when !act).
template <typename T16>
__device__ __forceinline__ void load8(float (&v)[8], const T16* p, bool act) {
  if (act) {
    const int4 raw = *reinterpret_cast<const int4*>(p);
    const T16* h = reinterpret_cast<const T16*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = static_cast<float>(h[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
  }
}

// Quantise one row of bf16/fp16 into [H fp8 | H/128 fp32 scales] with one warp (H % 128 == 0).
// Four 256-element chunks are loaded before any is quantised (four loads in flight per lane).
template <typename T16>
__device__ __forceinline__ void warp_quant_row(uint8_t* __restrict__ dst, float* __restrict__ scales,
                                               const T16* __restrict__ src, int H, bool round_scale) {
  const int lane = lane_id();
  for (int c0 = 0; c0 < H; c0 += 1024) {
    float v[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int off = c0 + u * 256 + lane * 8;
      load8(v[u], src + off, off < H);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int off = c0 + u * 256 + lane * 8;
      const Quant8 r = quant8_e4m3(v[u], round_scale);
      if (off < H) {
        *reinterpret_cast<uint2*>(dst + off) = r.q;
        if ((lane & 15) == 0) scales[off / 128] = r.scale;
      }
    }
  }
}

#endif  // __CUDACC__

}  // namespace b200ep
