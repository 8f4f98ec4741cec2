// Host side of the normal-mode ops as single native calls.
//
// A dispatch needs a dozen output tensors (receive rows, scales, top-k ids and weights,
// sources, the handle's maps), a launch, the wait for the receive size on the notify page
// and the slicing of the outputs to that size. Done from Python, that is a dozen tensor
// constructions at several microseconds each on the critical path between the layout, the
// dispatch and the combine launches; at one or two GPUs, where a kernel runs for tens of
// microseconds, the GPU then waits for the host. Here each op is one crossing into C++:
// outputs come from the caching allocator (at::empty), the kernel is queued, and for a
// dispatch the host waits on the notify page while the kernel is still moving rows.
// Reference counterpart: the host-side packing of deep_ep_trn/buffer.py:143-156 and
// 169-266 (there the host builds and unpacks the rows itself).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>

#include <tuple>
#include <vector>

#include "ops.h"

namespace b200ep {

std::tuple<at::Tensor, at::Tensor, at::Tensor> layout_op(const at::Tensor& topk_idx, int64_t num_experts,
                                                         int64_t num_ranks, at::Tensor scratch) {
  const c10::cuda::CUDAGuard guard(topk_idx.device());
  auto i32 = topk_idx.options().dtype(at::kInt);
  at::Tensor ntr = at::empty({num_ranks}, i32);
  at::Tensor nte = at::empty({num_experts}, i32);
  at::Tensor itr = at::empty({topk_idx.size(0), num_ranks}, topk_idx.options().dtype(at::kBool));
  layout(topk_idx.is_contiguous() ? topk_idx : topk_idx.contiguous(), num_experts, num_ranks, ntr, nte, itr,
         scratch);
  return {ntr, nte, itr};
}

// Returns (recv_x, recv_scales, recv_topk, recv_w, recv_src, token_pos, send_start, recv_info,
// recv_off, num_recv, notify) where notify = [rows from each source..., rows per local
// expert...] when `wait` (the outputs are then cut to num_recv rows), else empty and the
// outputs keep `cap` rows.
std::tuple<at::Tensor, OptTensor, OptTensor, OptTensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
           int64_t, std::vector<int64_t>>
dispatch_op(SymmHeap& heap, const at::Tensor& x, const OptTensor& x_scales, int64_t mode, bool round_scale,
            const OptTensor& topk_idx, const OptTensor& topk_w, const OptTensor& nte, const at::Tensor& in_rank,
            int64_t num_experts, int64_t grid, int64_t cap, bool pad_rows, bool wait, int64_t ticket,
            double timeout_s) {
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), H = x.size(1), R = heap.world();
  auto opt = x.options();
  at::Tensor token_pos = at::empty({T, R}, opt.dtype(at::kInt));
  at::Tensor send_start = at::empty({grid, R}, opt.dtype(at::kInt));
  at::Tensor recv_info = at::empty({R, kMaxGrid, 2}, opt.dtype(at::kInt));
  at::Tensor recv_off = at::empty({R + 1}, opt.dtype(at::kLong));
  at::Tensor recv_x;
  OptTensor recv_s, recv_topk, recv_w;
  if (mode == 0) {
    recv_x = at::empty({cap, H}, opt);
  } else {
    recv_x = at::empty({cap, H}, opt.dtype(at::kFloat8_e4m3fn));
    recv_s = at::empty({cap, H / 128}, opt.dtype(at::kFloat));
  }
  if (topk_idx.has_value()) {
    recv_topk = at::empty({cap, topk_idx->size(1)}, topk_idx->options());
    if (topk_w.has_value()) recv_w = at::empty({cap, topk_idx->size(1)}, opt.dtype(at::kFloat));
  }
  at::Tensor recv_src = at::empty({cap}, opt.dtype(at::kLong));
  nd_dispatch(heap, mode == 1 ? x.view(at::kByte) : x, x_scales, mode, round_scale, topk_idx, topk_w, nte, in_rank,
              token_pos, send_start, recv_info, recv_off, recv_x, recv_s, recv_topk, recv_w, recv_src, num_experts,
              ticket, grid, pad_rows);
  int64_t n = cap;
  std::vector<int64_t> notify;
  if (wait) {
    std::vector<int64_t> info = heap.wait_notify(static_cast<uint64_t>(ticket), static_cast<int>(num_experts / R),
                                                 timeout_s);
    n = info[0];
    notify.assign(info.begin() + 1, info.end());
    recv_x = recv_x.narrow(0, 0, n);
    recv_src = recv_src.narrow(0, 0, n);
    if (recv_s) recv_s = recv_s->narrow(0, 0, n);
    if (recv_topk) recv_topk = recv_topk->narrow(0, 0, n);
    if (recv_w) recv_w = recv_w->narrow(0, 0, n);
  }
  return {recv_x, recv_s, recv_topk, recv_w, recv_src, token_pos, send_start, recv_info, recv_off, n, notify};
}

// Returns (out [T, H], out_w [T, K] or None).
std::tuple<at::Tensor, OptTensor> combine_op(SymmHeap& heap, const at::Tensor& x, const OptTensor& w,
                                             const at::Tensor& recv_off, const at::Tensor& recv_info,
                                             const at::Tensor& token_pos, const at::Tensor& send_start,
                                             const OptTensor& bias0, const OptTensor& bias1, int64_t grid,
                                             const OptTensor& pair_pos, const OptTensor& pair_w) {
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty({token_pos.size(0), x.size(1)}, x.options());
  OptTensor out_w;
  if (w.has_value()) out_w = at::empty({token_pos.size(0), w->size(1)}, x.options().dtype(at::kFloat));
  nc_combine(heap, x, w, recv_off, recv_info, token_pos, send_start, out, out_w, bias0, bias1, grid, pair_pos,
             pair_w);
  return {out, out_w};
}

}  // namespace b200ep
