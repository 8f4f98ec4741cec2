// Host-side declarations of the runtime and every kernel launcher exported to Python.
#pragma once

#include <atomic>
#include <chrono>
#include <cstdint>
#include <string>
#include <tuple>
#include <vector>

#include <ATen/ATen.h>
#include <c10/util/Optional.h>

#include "heap.cuh"

namespace b200ep {

class SymmHeap {
 public:
  SymmHeap(int rank, int world, int M, int Mll, int H, int K, int E, int device, double timeout_s);
  ~SymmHeap();
  SymmHeap(const SymmHeap&) = delete;
  SymmHeap& operator=(const SymmHeap&) = delete;

  std::string ipc_handle() const;
  void open(const std::vector<std::string>& handles);
  void close();
  HeapView view() const;
  std::vector<int64_t> status() const;
  void clear_status();
  std::vector<int64_t> trace() const;
  std::vector<int64_t> wait_notify(uint64_t ticket, int num_local_experts, double timeout_s) const;
  // Offsets (bytes into this rank's heap) of the guard zones whose canary bytes changed.
  std::vector<int64_t> check_canaries() const;
  // Zero the grid-barrier and arrival counters of this rank's local state (after a device
  // error left a kernel part-way; epochs and sequence numbers are kept).
  void reset_counters();

  int rank() const { return rank_; }
  int world() const { return world_; }
  int device() const { return device_; }
  int num_sms() const { return num_sms_; }
  int64_t total_bytes() const { return layout_.total; }
  const HeapConfig& config() const { return cfg_; }
  bool is_open() const { return local_ != nullptr; }

 private:
  int rank_, world_, device_, num_sms_ = 0;
  HeapConfig cfg_{};
  HeapLayout layout_{};
  int64_t guards_[kMaxGuards] = {};
  int nguards_ = 0;
  uint64_t timeout_ns_ = 0;
  void* local_ = nullptr;
  std::vector<void*> peers_;
  HostPage* host_ = nullptr;
  HostPage* host_dev_ = nullptr;
  bool opened_ = false;
};

using OptTensor = c10::optional<at::Tensor>;

// Unit stride in the last dimension, or a last dimension of one element (whose stride torch
// leaves arbitrary, e.g. the scales of a 128-wide fp8 row or top-1 routing weights).
inline bool unit_inner(const at::Tensor& t) { return t.size(-1) <= 1 || t.stride(-1) == 1; }

// layout.cu
void layout(const at::Tensor& topk_idx, int64_t num_experts, int64_t num_ranks, at::Tensor ntr, at::Tensor nte,
            at::Tensor itr, at::Tensor scratch);

// normal.cu
void nd_dispatch(SymmHeap& heap, const at::Tensor& x, const OptTensor& x_scales, int64_t mode, bool round_scale,
                 const OptTensor& topk_idx, const OptTensor& topk_w, const OptTensor& nte, const at::Tensor& in_rank,
                 at::Tensor token_pos, at::Tensor send_start, at::Tensor recv_info, at::Tensor recv_off,
                 at::Tensor recv_x, const OptTensor& recv_scales, const OptTensor& recv_topk,
                 const OptTensor& recv_w, at::Tensor recv_src, int64_t num_experts, int64_t ticket, int64_t grid,
                 bool pad_rows);
void nc_combine(SymmHeap& heap, const at::Tensor& x, const OptTensor& w, const at::Tensor& recv_off,
                const at::Tensor& recv_info, const at::Tensor& token_pos, const at::Tensor& send_start, at::Tensor out,
                const OptTensor& out_w, const OptTensor& bias0, const OptTensor& bias1, int64_t grid,
                const OptTensor& pair_pos, const OptTensor& pair_w);

// host_ops.cpp: the normal-mode ops as one native call each (outputs, launch, notify wait)
std::tuple<at::Tensor, at::Tensor, at::Tensor> layout_op(const at::Tensor& topk_idx, int64_t num_experts,
                                                         int64_t num_ranks, at::Tensor scratch);
std::tuple<at::Tensor, OptTensor, OptTensor, OptTensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
           int64_t, std::vector<int64_t>>
dispatch_op(SymmHeap& heap, const at::Tensor& x, const OptTensor& x_scales, int64_t mode, bool round_scale,
            const OptTensor& topk_idx, const OptTensor& topk_w, const OptTensor& nte, const at::Tensor& in_rank,
            int64_t num_experts, int64_t grid, int64_t cap, bool pad_rows, bool wait, int64_t ticket,
            double timeout_s);
std::tuple<at::Tensor, OptTensor> combine_op(SymmHeap& heap, const at::Tensor& x, const OptTensor& w,
                                             const at::Tensor& recv_off, const at::Tensor& recv_info,
                                             const at::Tensor& token_pos, const at::Tensor& send_start,
                                             const OptTensor& bias0, const OptTensor& bias1, int64_t grid,
                                             const OptTensor& pair_pos, const OptTensor& pair_w);

// ll.cu
void ll_dispatch_send(SymmHeap& heap, const at::Tensor& x, const at::Tensor& topk_idx, int64_t num_experts,
                      bool use_fp8, bool round_scale, int64_t num_sms);
void ll_dispatch_recv(SymmHeap& heap, at::Tensor recv_x, const OptTensor& recv_scales, at::Tensor recv_count,
                      at::Tensor src_info, at::Tensor layout_range, at::Tensor pair_meta, int64_t num_experts,
                      bool use_fp8, bool ue8m0, const OptTensor& cum_stats, const OptTensor& wait_stats);
void ll_combine_send(SymmHeap& heap, const at::Tensor& x, const at::Tensor& recv_count, const at::Tensor& src_info,
                     const at::Tensor& pair_meta, int64_t num_experts, int64_t num_sms);
void ll_combine_recv(SymmHeap& heap, const at::Tensor& topk_idx, const at::Tensor& topk_w, at::Tensor out,
                     int64_t num_sms);

// diag.cu
void device_barrier(SymmHeap& heap);
void wait_probe(SymmHeap& heap, int64_t budget_ns);
void fence_cost(SymmHeap& heap, int64_t peer, int64_t bytes, int64_t scope, at::Tensor out);

// nvlbench.cu
void nvl_bw(SymmHeap& heap, int64_t mode, int64_t bytes_per_peer, int64_t chunk, int64_t nstages, int64_t grid,
            int64_t threads);

// gemm.cu
void grouped_gemm_m(const at::Tensor& A, const at::Tensor& B, const at::Tensor& offsets, const OptTensor& C,
                    const OptTensor& Hout, int64_t epilogue, at::Tensor error, int64_t num_sms, double timeout_s,
                    bool b_kn, const OptTensor& residual);
at::Tensor sf_tiles(const at::Tensor& sc, int64_t groups, int64_t rows_per_group);
void grouped_gemm_fp8_m(const at::Tensor& A, const at::Tensor& sa, const at::Tensor& B, const at::Tensor& sb,
                        const at::Tensor& offsets, const OptTensor& C, const OptTensor& Hout, int64_t epilogue,
                        at::Tensor error, int64_t num_sms, double timeout_s);
void grouped_gemm_k(const at::Tensor& A, const at::Tensor& B, const at::Tensor& offsets, at::Tensor C,
                    at::Tensor error, int64_t num_sms, double timeout_s, bool tok_major);

// moe.cu
void router_topk(const at::Tensor& logits, int64_t topk, at::Tensor idx, at::Tensor w);
void router_topk_bwd(const at::Tensor& idx, const at::Tensor& w, const at::Tensor& dw, at::Tensor dlogits);
void permute(const at::Tensor& x, const at::Tensor& ids, int64_t num_local_experts, at::Tensor out, at::Tensor pos,
             at::Tensor offsets, at::Tensor counts, at::Tensor scratch, const OptTensor& error,
             const OptTensor& x_scales, const OptTensor& out_scales);
void unpermute(const at::Tensor& rows, const at::Tensor& pos, const at::Tensor& w, at::Tensor y);
void unpermute_bwd(const at::Tensor& dy, const at::Tensor& rows, const at::Tensor& pos, const at::Tensor& w,
                   at::Tensor drows, const OptTensor& dw, const at::Tensor& offsets, const at::Tensor& counts);
void permute_bwd(const at::Tensor& drows, const at::Tensor& pos, at::Tensor dx);
void swiglu_bwd(const at::Tensor& dh, const at::Tensor& pre, at::Tensor dpre);
void transpose(const at::Tensor& in, at::Tensor out);

// quant.cu
void quant_fp8(const at::Tensor& x, at::Tensor q, at::Tensor scales, bool round_scale);
void dequant_fp8(const at::Tensor& q, const at::Tensor& scales, at::Tensor out);

}  // namespace b200ep
