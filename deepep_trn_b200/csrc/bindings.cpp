// Python bindings of the runtime and kernel launchers (module deepep_trn_b200._C).
#include <torch/extension.h>

#include "ops.h"

namespace py = pybind11;
using namespace b200ep;

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels and NVLink symmetric-heap runtime of deepep_trn_b200";
  py::class_<SymmHeap>(m, "SymmHeap")
      .def(py::init<int, int, int, int, int, int, int, int, double>(), py::arg("rank"), py::arg("world"),
           py::arg("max_tokens"), py::arg("max_ll_tokens"), py::arg("hidden"), py::arg("topk"),
           py::arg("num_experts"), py::arg("device"), py::arg("timeout_s"))
      .def("ipc_handle", [](const SymmHeap& h) { return py::bytes(h.ipc_handle()); })
      .def("open", [](SymmHeap& h, const std::vector<py::bytes>& hs) {
        std::vector<std::string> v;
        for (auto& b : hs) v.emplace_back(std::string(b));
        h.open(v);
      })
      .def("close", &SymmHeap::close)
      .def("status", &SymmHeap::status)
      .def("clear_status", &SymmHeap::clear_status)
      .def("trace", &SymmHeap::trace)
      .def("check_canaries", &SymmHeap::check_canaries)
      .def("reset_counters", &SymmHeap::reset_counters)
      .def("wait_notify", &SymmHeap::wait_notify, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("rank", &SymmHeap::rank)
      .def_property_readonly("world", &SymmHeap::world)
      .def_property_readonly("num_sms", &SymmHeap::num_sms)
      .def_property_readonly("total_bytes", &SymmHeap::total_bytes)
      .def_property_readonly("is_open", &SymmHeap::is_open)
      .def_property_readonly("config", [](const SymmHeap& h) {
        const auto& c = h.config();
        return py::make_tuple(c.R, c.M, c.Mll, c.H, c.K, c.E);
      });
  m.def("heap_bytes", [](int R, int M, int Mll, int H, int K, int E) {
    return make_layout(HeapConfig{R, M, Mll, H, K, E}).total;
  });
  // The symmetric-heap layout for a configuration: region offsets, guard-zone offsets, total.
  m.def("heap_layout", [](int R, int M, int Mll, int H, int K, int E) {
    int64_t guards[kMaxGuards] = {};
    int ng = 0;
    const HeapLayout L = make_layout(HeapConfig{R, M, Mll, H, K, E}, guards, &ng);
    py::dict d;
    d["sig"] = L.sig;
    d["local"] = L.local;
    d["row_stride"] = L.row_stride;
    auto pair = [](const int64_t (&v)[2]) { return py::make_tuple(v[0], v[1]); };
    d["inbox_stride"] = L.inbox_stride;
    d["inbox"] = L.inbox;
    d["cinbox_stride"] = L.cinbox_stride;
    d["cinbox"] = L.cinbox;
    d["nd_nte"] = L.nd_nte;
    d["nd_rcnt"] = L.nd_rcnt;
    d["info"] = L.info;
    d["prog"] = L.prog;
    d["cprog"] = L.cprog;
    d["max_grid"] = kMaxGrid;
    d["ll_rows"] = pair(L.ll_rows);
    d["ll_ids"] = pair(L.ll_ids);
    d["lc_rows"] = pair(L.lc_rows);
    d["guards"] = std::vector<int64_t>(guards, guards + ng);
    d["guard_bytes"] = kGuardBytes;
    d["signals_bytes"] = static_cast<int64_t>(sizeof(Signals));
    d["local_state_bytes"] = static_cast<int64_t>(sizeof(LocalState));
    d["total"] = L.total;
    return d;
  });
  m.def("layout", &layout);
  m.def("layout_op", &layout_op);
  m.def("dispatch_op", &dispatch_op);
  m.def("combine_op", &combine_op);
  m.def("nd_dispatch", &nd_dispatch);
  m.def("nc_combine", &nc_combine);
  m.def("ll_dispatch_send", &ll_dispatch_send);
  m.def("ll_dispatch_recv", &ll_dispatch_recv);
  m.def("ll_combine_send", &ll_combine_send);
  m.def("ll_combine_recv", &ll_combine_recv);
  m.def("quant_fp8", &quant_fp8);
  m.def("dequant_fp8", &dequant_fp8);
  m.def("device_barrier", &device_barrier);
  m.def("grouped_gemm_m", &grouped_gemm_m);
  m.def("router_topk", &router_topk);
  m.def("router_topk_bwd", &router_topk_bwd);
  m.def("permute", &permute);
  m.def("unpermute", &unpermute);
  m.def("unpermute_bwd", &unpermute_bwd);
  m.def("permute_bwd", &permute_bwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("transpose", &transpose);
  m.def("grouped_gemm_k", &grouped_gemm_k);
  m.def("grouped_gemm_fp8_m", &grouped_gemm_fp8_m);
  m.def("sf_tiles", &sf_tiles);
  m.def("wait_probe", &wait_probe);
  m.def("fence_cost", &fence_cost);
  m.def("nvl_bw", &nvl_bw, "raw NVLink engine bandwidth probe (all-to-all pattern)");
}
