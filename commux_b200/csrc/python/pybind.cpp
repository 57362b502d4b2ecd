// commux_b200._C: factory + introspection for torch.distributed registration
// (creator signature of reference: python/csrc/commux_pybind.cpp:19-31; the
// timeout is honoured here instead of dropped).

#include <pybind11/chrono.h>
#include <pybind11/stl.h>

#include "clocks.hpp"
#include <torch/csrc/utils/pybind.h>

#include <chrono>
#include <torch/csrc/distributed/c10d/Backend.hpp>
#include <torch/csrc/distributed/c10d/Store.hpp>
#include <utility>

#include "../engine/engine.hpp"
#include "commux/io.hpp"
#include "commux/process_group_ucx.hpp"

namespace py = pybind11;

namespace {

commux::ProcessGroupUCX* as_commux(const c10::intrusive_ptr<c10d::Backend>& b) {
  auto* pg = dynamic_cast<commux::ProcessGroupUCX*>(b.get());
  TORCH_CHECK(pg != nullptr, "not a commux backend (got ", b->getBackendName(), ")");
  return pg;
}

}  // namespace

PYBIND11_MODULE(_C, m) {
  m.doc() = "commux: tag-matching c10d backend (shared memory + NVLink, sm_100a kernels)";
  m.def(
      "create_backend",
      [](c10::intrusive_ptr<c10d::Store> store, int rank, int size, std::chrono::milliseconds timeout) {
        py::gil_scoped_release nogil;
        return c10::static_intrusive_pointer_cast<c10d::Backend>(
            c10::make_intrusive<commux::ProcessGroupUCX>(std::move(store), rank, size, timeout));
      },
      py::arg("store"), py::arg("rank"), py::arg("size"),
      py::arg("timeout") = std::chrono::milliseconds(0));

  m.def(
      "make_ucp_tag",
      [](int sender, std::uint32_t tag, std::uint32_t sub, bool coll) {
        return commux::make_ucp_tag(sender, tag, sub, coll);
      },
      py::arg("sender_rank"), py::arg("user_tag"), py::arg("sub_index") = 0,
      py::arg("collective") = false);
  m.attr("TAG_MASK_ANY_SOURCE") = py::int_(commux::kTagMaskAnySource);

  m.def("is_commux", [](const c10::intrusive_ptr<c10d::Backend>& b) {
    return dynamic_cast<commux::ProcessGroupUCX*>(b.get()) != nullptr;
  });
  m.def("stats", [](const c10::intrusive_ptr<c10d::Backend>& b) {
    py::dict d;
    for (auto& kv : as_commux(b)->stats()) d[py::str(kv.first)] = kv.second;
    return d;
  });
  m.def("reset_stats", [](const c10::intrusive_ptr<c10d::Backend>& b) { as_commux(b)->reset_stats(); });
  py::class_<commux::clocks::Sampler>(m, "ClockSampler")
      .def(py::init<const std::string&, int>(), py::arg("gpu"), py::arg("interval_us") = 1000)
      .def("start", &commux::clocks::Sampler::start)
      .def("stop",
           [](commux::clocks::Sampler& s) {
             py::list out;
             for (auto& x : s.stop())
               out.append(py::make_tuple(x.t_us, x.sm_mhz, x.sm_max_mhz, x.reasons, x.power_mw));
             return out;
           },
           "Stop and return [(t_us, sm_mhz, sm_max_mhz, reasons, power_mw), ...].")
      .def_property_readonly("error", &commux::clocks::Sampler::error);
  m.def("transports", [](const c10::intrusive_ptr<c10d::Backend>& b) {
    auto& e = as_commux(b)->engine();
    py::list kinds;
    for (int p = 0; p < e.size(); ++p) kinds.append(p == e.rank() ? "self" : e.remote(p) ? "tcp" : "shm");
    return kinds;
  }, "Transport used for each peer rank: 'self', 'shm' (same host) or 'tcp'.");
  py::class_<commux::DevicePlan, std::shared_ptr<commux::DevicePlan>>(m, "P2PPlan")
      .def("start", &commux::DevicePlan::start, py::call_guard<py::gil_scoped_release>(),
           "Enqueue one exchange of the plan's buffers on the current CUDA stream.")
      .def("set_max_ctas", &commux::DevicePlan::set_max_ctas, py::arg("ctas"),
           py::call_guard<py::gil_scoped_release>(),
           "Cap the CTAs of the plan's launches (0: default), e.g. to leave SMs to a kernel that runs "
           "beside the exchange.")
      .def("info", [](commux::DevicePlan& p) {
        py::dict d;
        for (auto& kv : p.info()) d[py::str(kv.first)] = kv.second;
        return d;
      });
  m.def(
      "p2p_plan",
      [](const c10::intrusive_ptr<c10d::Backend>& b, std::vector<at::Tensor> recv_tensors,
         std::vector<int> recv_peers, std::vector<int> recv_tags, std::vector<at::Tensor> send_tensors,
         std::vector<int> send_peers, std::vector<int> send_tags) {
        py::gil_scoped_release nogil;
        return as_commux(b)->p2p_plan(recv_tensors, recv_peers, recv_tags, send_tensors, send_peers,
                                      send_tags);
      },
      py::arg("backend"), py::arg("recv_tensors"), py::arg("recv_peers"), py::arg("recv_tags"),
      py::arg("send_tensors"), py::arg("send_peers"), py::arg("send_tags"));
  m.def(
      "_release_all", [] { commux::Engine::release_all(); }, py::call_guard<py::gil_scoped_release>(),
      "Release every backend's CUDA state (atexit hook; the CUDA context is still alive then).");
  m.def(
      "batch_p2p",
      [](const c10::intrusive_ptr<c10d::Backend>& b, std::vector<at::Tensor> recv_tensors,
         std::vector<int> recv_peers, std::vector<int> recv_tags, std::vector<at::Tensor> send_tensors,
         std::vector<int> send_peers, std::vector<int> send_tags) {
        py::gil_scoped_release nogil;
        return as_commux(b)->batch_p2p(recv_tensors, recv_peers, recv_tags, send_tensors, send_peers,
                                       send_tags);
      },
      py::arg("backend"), py::arg("recv_tensors"), py::arg("recv_peers"), py::arg("recv_tags"),
      py::arg("send_tensors"), py::arg("send_peers"), py::arg("send_tags"));

  py::class_<commux::IOContext, std::shared_ptr<commux::IOContext>>(m, "IOContext")
      .def(py::init([](c10::intrusive_ptr<c10d::Store> store, int rank, int size) {
             py::gil_scoped_release nogil;
             return std::make_shared<commux::IOContext>(std::move(store), rank, size);
           }),
           py::arg("store"), py::arg("rank"), py::arg("size"))
      .def_property_readonly("rank", &commux::IOContext::rank)
      .def_property_readonly("size", &commux::IOContext::size)
      .def("barrier", &commux::IOContext::barrier, py::call_guard<py::gil_scoped_release>())
      .def("broadcast_bytes",
           [](commux::IOContext& io, py::bytes data, int root) {
             std::string s = data;
             std::vector<std::uint8_t> v(s.begin(), s.end());
             {
               py::gil_scoped_release nogil;
               io.broadcast_bytes(v, root);
             }
             return py::bytes(reinterpret_cast<const char*>(v.data()), v.size());
           })
      .def("gather_bytes",
           [](commux::IOContext& io, py::bytes data, int root) {
             std::string s = data;
             std::vector<std::uint8_t> v(s.begin(), s.end()), out;
             {
               py::gil_scoped_release nogil;
               out = io.gather_bytes(v, root);
             }
             return py::bytes(reinterpret_cast<const char*>(out.data()), out.size());
           })
      .def("send_bytes",
           [](commux::IOContext& io, py::bytes data, int dst, int tag) {
             std::string s = data;
             py::gil_scoped_release nogil;
             io.send_bytes(s.data(), s.size(), dst, tag);
           })
      .def("recv_bytes",
           [](commux::IOContext& io, std::size_t n, int src, int tag) {
             std::string s(n, '\0');
             {
               py::gil_scoped_release nogil;
               io.recv_bytes(s.data(), n, src, tag);
             }
             return py::bytes(s);
           })
      .def("open_file", &commux::IOContext::open_file, py::call_guard<py::gil_scoped_release>())
      .def("close_file", &commux::IOContext::close_file, py::call_guard<py::gil_scoped_release>())
      .def("write_at",
           [](commux::IOContext& io, int fd, py::bytes data, std::int64_t offset) {
             std::string s = data;
             py::gil_scoped_release nogil;
             io.write_at(fd, s.data(), s.size(), offset);
           })
      .def("sync_file", &commux::IOContext::sync_file, py::call_guard<py::gil_scoped_release>());
  m.def(
      "make_tcp_io_context",
      [](const std::string& host, int port, int rank, int size) {
        py::gil_scoped_release nogil;
        return commux::make_tcp_io_context(host, port, rank, size);
      },
      py::arg("host"), py::arg("port"), py::arg("rank"), py::arg("size"));
}
