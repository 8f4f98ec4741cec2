// Symmetric heap layout: one cudaMalloc'd region per rank, mapped into every
// peer of the EP group through CUDA IPC. All ranks compute the same offsets
// from the same HeapConfig, so a region of rank p is reached as base[p] + off.
//
// Normal mode has two inboxes per rank, each R blocks of M rows: block s of the dispatch
// inbox holds the rows source s pushed to this rank, block s of the combine inbox the rows
// expert rank s sent back. Each kind of op has its own sequence number: a source writes into
// a peer's inbox of one kind (and its progress / info words) for op q only after that peer
// reported that it finished reading that inbox for op q - 1. With separate inboxes a rank's
// combine does not wait for the peers to finish reading their dispatch rows (and the next
// dispatch not for the peers' combines), so the ranks are not held in lockstep between ops;
// nothing is double-buffered and nothing is ever reset. Low-latency mode keeps two parities
// of its own receive areas (its own protocol, no host sync).
#pragma once

#include <cstdint>
#include <cstddef>
#include "common.cuh"

namespace b200ep {

// Device trace points: the last op of each kind stamps %globaltimer at fixed phases.
enum TracePoint : int {
  // normal dispatch: kernel start, scan done (counts published), peers' counts in, host
  // notified, CTA 0's pushes done, CTA 0's receives done, kernel end, CTA 0's last progress
  // word released
  kTrNdStart = 0, kTrNdScanned, kTrNdCounts, kTrNdNotified, kTrNdPushed, kTrNdRecvd, kTrNdEnd, kTrNdPublished,
  kTrNdWaitNs = 8,  // not a stamp: mean ns a receiving warp of CTA 0 waited for progress words
  kTrNdFreeIn = 9,  // CTA 0: every peer's dispatch inbox is free (the scan follows)
  kTrNdBarrier,     // CTA 0: past the grid barrier of the scan
  kTrBarrierExit = 15,  // the device barrier's exit (every rank's within a flag latency): aligns
                        // the ranks' clocks in a trace
  // normal combine: kernel start, CTA 0's pushes done, CTA 0's reduction done, kernel end,
  // CTA 0's last progress word released
  kTrNcStart = 16, kTrNcPushed, kTrNcReduced, kTrNcEnd, kTrNcPublished,
  kTrNcWaitNs = 21,  // not a stamp: mean ns a reducing warp of CTA 0 waited for progress words
  // low-latency send kernels also stamp when CTA 0 has issued its row stores and when its
  // releases (the fence that waits for those stores to land) are done
  kTrLLSendStart = 24, kTrLLSendEnd, kTrLLRecvStart, kTrLLRecvReady, kTrLLRecvEnd, kTrLLSendStored,
  kTrLLSendReleased,
  kTrLCSendStart = 32, kTrLCSendEnd, kTrLCRecvStart, kTrLCRecvReady, kTrLCRecvEnd, kTrLCSendStored,
  kTrLCSendReleased,
  kTracePoints = 40,
};

enum EpochId : int {
  kEpInbox = 0,   // normal-mode dispatch sequence (dispatch inbox)
  kEpCInbox = 1,  // normal-mode combine sequence (combine inbox)
  kEpLLD = 2,     // low-latency dispatch (send kernel advances it)
  kEpLLC = 3,     // low-latency combine (send kernel advances it)
  kEpBar = 4,     // device barrier
  kArLLRecv = 5,  // arrival counter of the low-latency dispatch receive kernel
  kArLCRecv = 6,  // arrival counter of the low-latency combine receive kernel
  kNumEpochs = 8,
};

// Largest CTA count of a normal-mode kernel (one CTA per SM on B200: 148).
constexpr int kMaxGrid = 256;

// Written by peers (remote stores), polled locally.
struct Signals {
  uint64_t nd_cnt[B200EP_MAX_RANKS];    // (q << 32) | (source s's CTAs - 1) << 24 | rows s sends this rank
  uint32_t nd_start[B200EP_MAX_RANKS];     // peer p started dispatch q (a timing signal: orders nothing)
  uint32_t inbox_free[B200EP_MAX_RANKS];   // peer p finished reading its dispatch inbox for dispatch q
  uint32_t cinbox_free[B200EP_MAX_RANKS];  // peer p finished reading its combine inbox for combine q
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
  uint32_t ll_expect[2][B200EP_MAX_RANKS];        // ll_cnt values already consumed
  uint32_t lc_expect[2][B200EP_MAX_RANKS];        // lc_cnt values already consumed
  uint32_t arrive2[kNumEpochs];                   // second arrival counters (phase ends)
  uint32_t gbar_count;                            // grid barrier of the normal-mode kernels
  uint32_t gbar_gen;
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
  int64_t row_stride;      // bytes per low-latency row: 2H rounded up to 128; fp8 rows use [H payload | H/32 scales]
  int64_t inbox_stride;    // bytes per dispatch inbox row: payload, scales, top-k ids and weights, source token
  int64_t inbox;           // dispatch inbox: [R][M] rows of inbox_stride bytes
  int64_t cinbox_stride;   // bytes per combine inbox row: 16-bit payload, top-k weights
  int64_t cinbox;          // combine inbox: [R][M] rows of cinbox_stride bytes
  int64_t nd_nte;          // [R][E/R] uint64: (q << 32) | tokens each source sends to each local expert
  int64_t nd_rcnt;         // [kMaxGrid][R] int32: rows of each CTA's token range per destination
  int64_t info;            // [R][kMaxGrid] uint64: (q & 0xffff) << 48 | first row << 24 | rows of (source, CTA)
  int64_t prog;            // [R][kMaxGrid] uint64: (q << 32) | rows dispatch (source, CTA) has pushed here
  int64_t cprog;           // [R][kMaxGrid] uint64: (q << 32) | rows combine (expert rank, CTA) has pushed here
  // low-latency dispatch receive (x2): [R][Mll] rows, [R][Mll][K] ids
  int64_t ll_rows[2], ll_ids[2];
  // low-latency combine receive (x2): [Mll][K] rows of 2H bytes
  int64_t lc_rows[2];
  int64_t total;
};

__host__ __device__ inline int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Dispatch inbox row: [payload: 2H (16-bit) or H (fp8) | fp8 scales: H/32 | ids: 4K | weights: 4K |
// token: 4]; combine inbox row: [payload: 2H | weights: 4K]. Rows start on 128-byte lines, so a
// warp's 512-byte run of 16-byte stores covers whole lines (a run that starts mid-line leaves
// partly written 32-byte sectors at both ends, each one a masked write over NVLink).
__host__ __device__ inline int64_t inbox_row_bytes(int64_t H, int64_t K) { return align_up(2 * H + 8 * K + 4, 128); }
__host__ __device__ inline int64_t cinbox_row_bytes(int64_t H, int64_t K) { return align_up(2 * H + 4 * K, 128); }

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
  L.row_stride = align_up(2LL * c.H, 128);
  L.inbox_stride = inbox_row_bytes(c.H, c.K);
  L.inbox = take(int64_t(c.R) * c.M * L.inbox_stride);
  L.cinbox_stride = cinbox_row_bytes(c.H, c.K);
  L.cinbox = take(int64_t(c.R) * c.M * L.cinbox_stride);
  L.nd_nte = take(int64_t(c.E) * 8);
  L.nd_rcnt = take(int64_t(kMaxGrid) * c.R * 4);
  L.info = take(int64_t(c.R) * kMaxGrid * 8);
  L.prog = take(int64_t(c.R) * kMaxGrid * 8);
  L.cprog = take(int64_t(c.R) * kMaxGrid * 8);
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
