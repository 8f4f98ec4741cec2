// Symmetric heap layout: one cudaMalloc'd region per rank, mapped into every
// peer of the EP group through CUDA IPC. All ranks compute the same offsets
// from the same HeapConfig, so a region of rank p is reached as base[p] + off.
//
// Every staging region is double-buffered on the parity of its op's epoch,
// which removes the "peer finished reading" round trip: a rank only overwrites
// slot e&1 at epoch e after it has seen every peer's epoch e-1 signal, and a
// peer only sends that signal after its epoch e-2 reads were complete (stream
// order on the peer). The argument holds for each op family separately.
#pragma once

#include <cstdint>
#include <cstddef>
#include "common.cuh"

namespace b200ep {

// Device trace points: the last op of each kind stamps %globaltimer at fixed phases.
enum TracePoint : int {
  kTrPrepStart = 0, kTrPrepScanDone, kTrPrepCopiesDone, kTrPrepPeersReady, kTrPrepNotified,
  kTrPullStart = 8, kTrPullEnd,
  kTrCombStart = 16, kTrCombPushDone, kTrCombPeersReady, kTrCombEnd,  // push done = rows staged (pull form)
  kTrLLSendStart = 24, kTrLLSendEnd, kTrLLRecvStart, kTrLLRecvReady, kTrLLRecvEnd,
  kTrLCSendStart = 32, kTrLCSendEnd, kTrLCRecvStart, kTrLCRecvReady, kTrLCRecvEnd,
  kTracePoints = 40,
};

enum EpochId : int {
  kEpND = 0,    // normal dispatch (prepare kernel advances it)
  kEpNC = 1,    // normal combine
  kEpLLD = 2,   // low-latency dispatch (send kernel advances it)
  kEpLLC = 3,   // low-latency combine (send kernel advances it)
  kEpBar = 4,   // device barrier
  kArLLRecv = 5,  // arrival counter of the low-latency dispatch receive kernel
  kArLCRecv = 6,  // arrival counter of the low-latency combine receive kernel
  kNumEpochs = 8,
};

// Written by peers (remote stores), polled locally.
struct Signals {
  uint32_t nd_ready[2][B200EP_MAX_RANKS];   // source s staged its dispatch data for epoch e
  uint32_t nc_ready[2][B200EP_MAX_RANKS];   // rank r delivered all its combine rows for epoch e
  uint64_t ll_hdr[2][B200EP_MAX_RANKS];     // (epoch << 32) | num_tokens of source s
  uint32_t ll_cnt[2][B200EP_MAX_RANKS];     // cumulative token slots source s has written (per parity)
  uint32_t lc_cnt[2][B200EP_MAX_RANKS];     // cumulative combine rows rank r has written home
  uint32_t barrier[B200EP_MAX_RANKS];
  uint32_t pad[B200EP_MAX_RANKS];
};

// Only touched by the owning rank.
struct LocalState {
  uint32_t epoch[kNumEpochs];
  uint32_t arrive[kNumEpochs];   // grid-completion counters (reset by the last CTA)
  int64_t nd_recv_off[2][B200EP_MAX_RANKS + 1];   // exclusive prefix of rows per source
  int64_t nd_num_recv[2];
  uint32_t ll_expect[2][B200EP_MAX_RANKS];        // ll_cnt values already consumed
  uint32_t lc_expect[2][B200EP_MAX_RANKS];        // lc_cnt values already consumed
  uint32_t arrive2[kNumEpochs];                   // second arrival counters (phase ends)
  uint64_t trace[kTracePoints];                   // %globaltimer stamps of the last op of each kind
};

struct HeapConfig {
  int32_t R;     // EP ranks
  int32_t M;     // normal-mode max tokens per rank
  int32_t Mll;   // low-latency max tokens per rank
  int32_t H;     // hidden size (elements)
  int32_t K;     // top-k
  int32_t E;     // experts
};

struct HeapLayout {
  int64_t sig, local;
  int64_t row_stride;      // bytes per staged row: align16(2H); fp8 rows use [H payload | H/32 scales]
  // normal dispatch staging (x2)
  int64_t nd_x[2], nd_topk[2], nd_w[2], nd_lists[2], nd_counts[2], nd_nte[2];
  // normal combine receive (x2): [R][M] rows of 2H bytes, [R][M][K] weights (push form)
  int64_t nc_rows[2], nc_w[2];
  // normal combine send (x2, pull form): [R*M] rows of 2H bytes, [R*M][K] weights, [R+1] offsets
  int64_t nc_send[2], nc_send_w[2], nc_send_off[2];
  // low-latency dispatch receive (x2): [R][Mll] rows, [R][Mll][K] ids
  int64_t ll_rows[2], ll_ids[2];
  // low-latency combine receive (x2): [Mll][K] rows of 2H bytes
  int64_t lc_rows[2];
  int64_t total;
};

__host__ __device__ inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Every region is followed by a 256-byte guard zone that the host fills with kCanaryByte at
// construction and checks on request (SymmHeap::check_canaries): a kernel that writes past
// the end of a region, on any rank, changes it.
constexpr int64_t kGuardBytes = 256;
constexpr int kCanaryByte = 0xA5;

inline HeapLayout make_layout(const HeapConfig& c, int64_t* guards = nullptr, int* nguards = nullptr) {
  HeapLayout L{};
  int64_t off = 0;
  int ng = 0;
  auto take = [&](int64_t bytes) {
    int64_t o = off;
    off = align_up(off + bytes, 256);
    if (guards != nullptr) guards[ng] = off;
    ++ng;
    off += kGuardBytes;
    return o;
  };
  L.sig = take(sizeof(Signals));
  L.local = take(sizeof(LocalState));
  L.row_stride = align_up(2LL * c.H, 16);
  for (int b = 0; b < 2; ++b) {
    L.nd_x[b] = take(int64_t(c.M) * L.row_stride);
    L.nd_topk[b] = take(int64_t(c.M) * c.K * 4);
    L.nd_w[b] = take(int64_t(c.M) * c.K * 4);
    L.nd_lists[b] = take(int64_t(c.R) * c.M * 4);
    L.nd_counts[b] = take(int64_t(c.R) * 4);
    L.nd_nte[b] = take(int64_t(c.E) * 4);
  }
  for (int b = 0; b < 2; ++b) {
    L.nc_rows[b] = take(int64_t(c.R) * c.M * 2LL * c.H);
    L.nc_w[b] = take(int64_t(c.R) * c.M * c.K * 4);
  }
  for (int b = 0; b < 2; ++b) {
    L.nc_send[b] = take(int64_t(c.R) * c.M * 2LL * c.H);
    L.nc_send_w[b] = take(int64_t(c.R) * c.M * c.K * 4);
    L.nc_send_off[b] = take(int64_t(c.R + 1) * 8);
  }
  for (int b = 0; b < 2; ++b) {
    L.ll_rows[b] = take(int64_t(c.R) * c.Mll * L.row_stride);
    L.ll_ids[b] = take(int64_t(c.R) * c.Mll * c.K * 4);
  }
  for (int b = 0; b < 2; ++b) L.lc_rows[b] = take(int64_t(c.Mll) * c.K * 2LL * c.H);
  L.total = off;
  if (nguards != nullptr) *nguards = ng;
  return L;
}
constexpr int kMaxGuards = 64;

// What a kernel needs to reach every peer's heap. Passed by value.
struct HeapView {
  uint8_t* base[B200EP_MAX_RANKS];
  int32_t rank;
  int32_t R;
  HeapConfig cfg;
  HeapLayout L;
  Status* status;        // host-mapped
  HostPage* host;        // host-mapped (device pointer)
  uint64_t timeout_ns;

  __device__ __forceinline__ Signals* sig(int p) const { return reinterpret_cast<Signals*>(base[p] + L.sig); }
  __device__ __forceinline__ LocalState* local() const {
    return reinterpret_cast<LocalState*>(base[rank] + L.local);
  }
  template <typename T>
  __device__ __forceinline__ T* at(int p, int64_t off) const {
    return reinterpret_cast<T*>(base[p] + off);
  }
};

}  // namespace b200ep
