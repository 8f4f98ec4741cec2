// Host runtime: the symmetric heap (one cudaMalloc per rank, exported and
// imported with CUDA IPC handles) and the host-mapped status/notify page.
//
// Reference counterpart: the reference allocates nothing at Buffer init and
// stages every exchange through the Neuron collective runtime
// (deep_ep_trn/buffer.py:95-119, transport/nki_a2av.py:47-75). Here the
// buffers are allocated once and every later op is a kernel that reads and
// writes peer memory directly.
#include "ops.h"

#include <cstring>
#include <stdexcept>
#include <string>

namespace b200ep {

#define B200EP_CUDA_CHECK(expr)                                                                   \
  do {                                                                                            \
    cudaError_t _e = (expr);                                                                      \
    if (_e != cudaSuccess)                                                                        \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(_e) + " at " +   \
                               __FILE__ + ":" + std::to_string(__LINE__) + " (" #expr ")");       \
  } while (0)

SymmHeap::SymmHeap(int rank, int world, int M, int Mll, int H, int K, int E, int device, double timeout_s)
    : rank_(rank), world_(world), device_(device) {
  if (world < 1 || world > B200EP_MAX_RANKS) throw std::invalid_argument("EP group size must be in [1, 32]");
  if (rank < 0 || rank >= world) throw std::invalid_argument("rank out of range");
  cfg_ = HeapConfig{world, M, Mll, H, K, E};
  layout_ = make_layout(cfg_, guards_, &nguards_);
  if (nguards_ > kMaxGuards) throw std::logic_error("heap layout has more regions than guard slots");
  timeout_ns_ = static_cast<uint64_t>(timeout_s * 1e9);
  B200EP_CUDA_CHECK(cudaSetDevice(device));
  B200EP_CUDA_CHECK(cudaMalloc(&local_, static_cast<size_t>(layout_.total)));
  B200EP_CUDA_CHECK(cudaMemset(local_, 0, static_cast<size_t>(layout_.total)));
  for (int i = 0; i < nguards_; ++i)
    B200EP_CUDA_CHECK(cudaMemset(static_cast<uint8_t*>(local_) + guards_[i], kCanaryByte, kGuardBytes));
  B200EP_CUDA_CHECK(cudaHostAlloc(&host_, sizeof(HostPage), cudaHostAllocMapped));
  std::memset(host_, 0, sizeof(HostPage));
  B200EP_CUDA_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&host_dev_), host_, 0));
  B200EP_CUDA_CHECK(cudaDeviceSynchronize());
  peers_.assign(world, nullptr);
  peers_[rank] = local_;
  int sms = 0;
  B200EP_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  num_sms_ = sms;
}

SymmHeap::~SymmHeap() {
  try {
    close();
  } catch (...) {
  }
}

std::string SymmHeap::ipc_handle() const {
  cudaIpcMemHandle_t h;
  B200EP_CUDA_CHECK(cudaSetDevice(device_));
  B200EP_CUDA_CHECK(cudaIpcGetMemHandle(&h, local_));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void SymmHeap::open(const std::vector<std::string>& handles) {
  if (static_cast<int>(handles.size()) != world_) throw std::invalid_argument("need one IPC handle per rank");
  B200EP_CUDA_CHECK(cudaSetDevice(device_));
  for (int p = 0; p < world_; ++p) {
    if (p == rank_) continue;
    if (handles[p].size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("bad IPC handle size");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[p].data(), sizeof(h));
    void* ptr = nullptr;
    B200EP_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
    peers_[p] = ptr;
  }
  opened_ = true;
}

void SymmHeap::close() {
  if (local_ == nullptr) return;
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  for (int p = 0; p < world_; ++p) {
    if (p != rank_ && peers_[p] != nullptr) cudaIpcCloseMemHandle(peers_[p]);
    peers_[p] = nullptr;
  }
  cudaFree(local_);
  local_ = nullptr;
  if (host_ != nullptr) cudaFreeHost(host_);
  host_ = nullptr;
  host_dev_ = nullptr;
}

HeapView SymmHeap::view() const {
  if (local_ == nullptr) throw std::runtime_error("symmetric heap is closed");
  HeapView v{};
  for (int p = 0; p < world_; ++p) v.base[p] = static_cast<uint8_t*>(peers_[p]);
  v.rank = rank_;
  v.R = world_;
  v.cfg = cfg_;
  v.L = layout_;
  v.status = &host_dev_->status;
  v.host = host_dev_;
  v.timeout_ns = timeout_ns_;
  return v;
}

std::vector<int64_t> SymmHeap::status() const {
  const volatile Status* s = &host_->status;
  return {s->code, s->op, s->rank, s->peer, s->expected, s->seen, s->aux};
}

void SymmHeap::clear_status() { std::memset(&host_->status, 0, sizeof(Status)); }

// Copy of the device trace stamps (synchronises the device).
std::vector<int64_t> SymmHeap::trace() const {
  std::vector<uint64_t> t(kTracePoints, 0);
  B200EP_CUDA_CHECK(cudaSetDevice(device_));
  B200EP_CUDA_CHECK(cudaDeviceSynchronize());
  B200EP_CUDA_CHECK(cudaMemcpy(t.data(), static_cast<uint8_t*>(local_) + layout_.local + offsetof(LocalState, trace),
                               sizeof(uint64_t) * kTracePoints, cudaMemcpyDeviceToHost));
  return std::vector<int64_t>(t.begin(), t.end());
}

// Spin on the host-mapped notify page until the prepare kernel published `ticket`.
// Returns {num_recv, recv_counts[R]..., per_expert[EL]...}; throws on timeout or
// on a device-side error.
std::vector<int64_t> SymmHeap::wait_notify(uint64_t ticket, int num_local_experts, double timeout_s) const {
  const volatile NotifyPage* n = &host_->notify;
  const volatile Status* s = &host_->status;
  auto t0 = std::chrono::steady_clock::now();
  uint64_t spins = 0;
  while (n->ticket != ticket) {
    if (s->code != 0) throw std::runtime_error("device error while waiting for dispatch notify (code " +
                                               std::to_string(s->code) + ")");
    if ((++spins & 1023u) == 0u) {
      double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      if (dt > timeout_s) throw std::runtime_error("timeout waiting for dispatch notify");
    }
  }
  std::atomic_thread_fence(std::memory_order_acquire);
  // the kernel publishes the ticket even after a failed wait (with a zero size): report it
  if (s->code != 0) throw std::runtime_error("device error during dispatch (code " + std::to_string(s->code) + ")");
  std::vector<int64_t> out;
  out.reserve(1 + world_ + num_local_experts);
  out.push_back(static_cast<int64_t>(n->num_recv));
  for (int r = 0; r < world_; ++r) out.push_back(static_cast<int64_t>(n->recv_counts[r]));
  for (int e = 0; e < num_local_experts && e < 1024; ++e) out.push_back(static_cast<int64_t>(n->per_expert[e]));
  return out;
}

void SymmHeap::reset_counters() {
  if (local_ == nullptr) return;
  B200EP_CUDA_CHECK(cudaSetDevice(device_));
  B200EP_CUDA_CHECK(cudaDeviceSynchronize());
  uint8_t* ls = static_cast<uint8_t*>(local_) + layout_.local;
  B200EP_CUDA_CHECK(cudaMemset(ls + offsetof(LocalState, arrive), 0, sizeof(LocalState::arrive)));
  B200EP_CUDA_CHECK(cudaMemset(ls + offsetof(LocalState, arrive2), 0, sizeof(LocalState::arrive2)));
  B200EP_CUDA_CHECK(cudaMemset(ls + offsetof(LocalState, gbar_count), 0, sizeof(uint32_t)));
  B200EP_CUDA_CHECK(cudaDeviceSynchronize());
}

std::vector<int64_t> SymmHeap::check_canaries() const {
  std::vector<int64_t> bad;
  if (local_ == nullptr) return bad;
  B200EP_CUDA_CHECK(cudaSetDevice(device_));
  std::vector<uint8_t> zone(static_cast<size_t>(kGuardBytes));
  for (int i = 0; i < nguards_; ++i) {
    B200EP_CUDA_CHECK(cudaMemcpy(zone.data(), static_cast<const uint8_t*>(local_) + guards_[i],
                                 static_cast<size_t>(kGuardBytes), cudaMemcpyDeviceToHost));
    for (uint8_t b : zone)
      if (b != static_cast<uint8_t>(kCanaryByte)) {
        bad.push_back(guards_[i]);
        break;
      }
  }
  return bad;
}

}  // namespace b200ep
