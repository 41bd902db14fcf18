// pybind_module.cpp -- Python access to the C++ front end (tests and
// bench.py drive the same Tensor / operations / tape code a C++ user links).
//
// Numpy arrays become constant tensors (device copy cached across
// evaluations, like weights) or materialized tensors (uploaded on every
// evaluation, like a batch of inputs). The arrays behind constant tensors
// are kept alive until clear().
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>
#include <sstream>

#include "Node.hpp"
#include "TapeExecutor.hpp"
#include "operations.hpp"
#include "tt_cuda.h"

namespace py = pybind11;

namespace {
std::vector<py::object>& keepalive() {
    static auto* v = new std::vector<py::object>();
    return *v;
}

std::vector<uint32_t> shape_of(const py::array& a) {
    std::vector<uint32_t> s;
    for (py::ssize_t i = 0; i < a.ndim(); ++i) s.push_back((uint32_t)a.shape(i));
    if (s.empty()) s.push_back(1);
    return s;
}

Tensor from_numpy(py::array_t<float, py::array::c_style | py::array::forcecast> a, bool constant) {
    auto shape = shape_of(a);
    if (shape.size() > 4) throw std::runtime_error("tt_lazy tensors have rank <= 4");
    if (constant) {
        keepalive().push_back(a);
        return Tensor(const_cast<float*>(a.data()), shape);
    }
    Tensor t(shape);
    std::memcpy(t.data_ptr(), a.data(), t.total_elements() * sizeof(float));
    return t;
}

py::array_t<float> to_numpy(Tensor& t) {
    const float* d = t.data_ptr();
    std::vector<py::ssize_t> shape(t.shape(), t.shape() + t.rank());
    py::array_t<float> out(shape);
    std::memcpy(out.mutable_data(), d, t.total_elements() * sizeof(float));
    return out;
}

tt_lazy::TapeEvaluationManager& manager() {
    return static_cast<tt_lazy::TapeEvaluationManager&>(tt_lazy::get_evaluation_manager());
}
}  // namespace

PYBIND11_MODULE(_tt_lazy, m) {
    m.doc() = "tt_lazy front end on the B200 (sm_100a) backend";

    py::class_<Tensor>(m, "Tensor")
        .def_property_readonly("shape", [](const Tensor& t) { return t.shape_vector(); })
        .def_property_readonly("rank", &Tensor::rank)
        .def_property_readonly("is_lazy", &Tensor::is_lazy)
        .def_property_readonly("is_evaluated", &Tensor::is_evaluated)
        .def_property_readonly("is_constant", &Tensor::is_constant)
        .def_property_readonly("producer_node", &Tensor::producer_node)
        .def_property_readonly("output_index", &Tensor::output_index)
        .def("total_elements", &Tensor::total_elements)
        .def("eval", &Tensor::eval)
        .def("numpy", &to_numpy)
        .def("to_vector", &Tensor::to_vector)
        .def("to_string", &Tensor::to_string)
        .def("__repr__", [](const Tensor& t) {
            std::ostringstream o;
            o << "Tensor(shape=[";
            for (int i = 0; i < t.rank(); ++i) o << (i ? ", " : "") << t.size(i);
            o << "], " << (t.is_lazy() ? "lazy" : t.is_constant() ? "constant" : "materialized") << ")";
            return o.str();
        });

    m.def("constant", [](py::array a) { return from_numpy(a, true); }, "constant tensor over a numpy array");
    m.def(
        "streamed",
        [](py::array a) {
            Tensor t = from_numpy(a, true);
            t.set_streamed(true);
            return t;
        },
        "input over a numpy array, re-uploaded on every evaluation");
    m.def("all_reduce_sum", &all_reduce_sum);
    m.def("comm_unique_id", []() {
        auto id = tt_lazy::comm_unique_id();
        return py::bytes(reinterpret_cast<const char*>(id.data()), id.size());
    });
    m.def("comm_init", [](int nranks, int rank, py::bytes id, int timeout_ms) {
        std::string s = id;
        tt_lazy::comm_init(nranks, rank, std::vector<uint8_t>(s.begin(), s.end()), timeout_ms);
    });
    m.def("comm_destroy", &tt_lazy::comm_destroy);

    py::class_<tt_lazy::CompiledTape>(m, "Plan")
        .def(py::init<const std::vector<Tensor>&, int>(), py::arg("outputs"), py::arg("pipeline_chunks") = 1)
        .def("run", &tt_lazy::CompiledTape::run, py::call_guard<py::gil_scoped_release>())
        .def("capture", &tt_lazy::CompiledTape::capture, py::call_guard<py::gil_scoped_release>())
        .def_property_readonly("captured", &tt_lazy::CompiledTape::captured)
        .def("numpy",
             [](const tt_lazy::CompiledTape& p, size_t i) {
                 Tensor t = *p.result(i);
                 return to_numpy(t);
             })
        .def("device_ptr", [](const tt_lazy::CompiledTape& p, size_t i) { return (uintptr_t)p.result(i)->device().ptr(); })
        .def_property_readonly("kernels_last_run", &tt_lazy::CompiledTape::kernels_last_run)
        .def("__len__", &tt_lazy::CompiledTape::size);
    m.def("materialized", [](py::array a) { return from_numpy(a, false); }, "materialized tensor (copy)");

    m.def("relu", &relu);
    m.def("sigmoid", &sigmoid);
    m.def("add", &add);
    m.def("multiply", &multiply);
    m.def("matmul", &matmul, py::arg("a"), py::arg("b"), py::arg("transpose_a") = false,
          py::arg("transpose_b") = false);
    m.def("transpose", &transpose);
    m.def("split", &split, py::arg("input"), py::arg("split_size"), py::arg("dim") = 0);
    m.def("reduce_sum", &reduce_sum, py::arg("input"), py::arg("dims") = std::vector<int32_t>{},
          py::arg("keepdim") = false);
    m.def("reduce_mean", &reduce_mean, py::arg("input"), py::arg("dims") = std::vector<int32_t>{},
          py::arg("keepdim") = false);
    m.def("fused_mlp", &fused_mlp, py::arg("input"), py::arg("weights"), py::arg("bias"),
          py::arg("has_relu") = true);

    m.def(
        "evaluate",
        [](std::vector<Tensor*> ts) {
            tt_lazy::evaluate(ts);
        },
        "materialise several tensors with one tape");

    m.def("clear", []() {
        Context::instance().clear();
        tt_lazy::get_evaluation_manager().clear_cache();
        keepalive().clear();
    });
    m.def("clear_cache", []() { tt_lazy::get_evaluation_manager().clear_cache(); });
    m.def("graph_size", []() { return Context::instance().size(); });
    m.def("set_optimization", [](bool on) { manager().generator().set_optimization_enabled(on); });

    m.def("tape", [](std::vector<Tensor> outs) {
        auto tape = manager().generator().generate_tape(outs);
        py::list ops;
        for (const auto& op : tape->operations()) {
            py::dict d;
            d["node"] = op->node_id;
            const Node* n = Context::instance().get_node(op->node_id);
            std::string name = n ? std::string(n->op_name()) : std::string("?");
            if (op->plan) name = std::string(op->plan->has_matmul ? "FusedGemm" : "FusedChain") + "[" +
                                 op->plan->describe() + "]";
            d["op"] = name;
            d["fused_nodes"] = op->plan ? (int)op->plan->members.size() + (op->plan->has_matmul ? 1 : 0) : 1;
            d["inputs"] = op->input_nodes;
            d["outputs"] = op->output_nodes;
            ops.append(d);
        }
        return ops;
    });

    m.def("stats", []() {
        auto s = tt_lazy::get_evaluation_manager().get_stats();
        auto ms = tt_lazy::MemoryManager::instance().stats();
        py::dict d;
        d["cache_hits"] = s.cache_hits;
        d["cache_misses"] = s.cache_misses;
        d["operations_executed"] = s.operations_executed;
        d["memory_allocated"] = s.memory_allocated;
        d["fused_operations"] = s.fused_operations;
        d["kernels_launched"] = s.kernels_launched;
        d["device_bytes_live"] = ms.bytes_live;
        d["device_bytes_peak"] = ms.bytes_peak;
        d["device_bytes_cached"] = ms.bytes_cached;
        d["device_allocations"] = ms.allocations;
        d["device_reuses"] = ms.reuses;
        return d;
    });
    m.def("reset_peak", []() { tt_lazy::MemoryManager::instance().reset_peak(); });
    m.def("set_canaries", [](bool on) { tt_lazy::MemoryManager::instance().set_canaries(on); },
          "guard bands after every device buffer, checked after each tape operation (debug)");
    m.def("check_canaries", []() { return tt_lazy::MemoryManager::instance().check_canaries("on request"); });
    m.def("canary_offset", [](uintptr_t ptr) {
        return tt_lazy::MemoryManager::instance().canary_offset(reinterpret_cast<const float*>(ptr));
    });
    m.def("set_profiling", &tt_lazy::set_profiling,
          "time every tape operation with CUDA events (and mark it with an NVTX range)");
    m.def("profile", []() {
        py::list out;
        for (const auto& p : tt_lazy::last_profile()) {
            py::dict d;
            d["op"] = p.op;
            d["ms"] = p.ms;
            out.append(d);
        }
        return out;
    });
    m.def(
        "set_gemm_path",
        [](const std::string& p) {
            if (p != "auto" && p != "ffma" && p != "tf32" && p != "tf32x3")
                throw std::invalid_argument("gemm path must be auto, ffma, tf32 or tf32x3");
            tt_lazy::set_gemm_path(p == "ffma"     ? TTC_GEMM_FFMA
                                   : p == "tf32"   ? TTC_GEMM_TF32
                                   : p == "tf32x3" ? TTC_GEMM_TF32X3
                                                   : TTC_GEMM_AUTO);
        },
        "matmul path: auto (TF32 where the tensor-core kernel takes the shape), ffma, tf32, or tf32x3 "
        "(fp32-accurate 3-pass TF32)");
    m.def("synchronize", []() {
        if (tt_lazy::backend_ready() && ttc_synchronize() != TTC_OK) throw std::runtime_error(ttc_last_error());
    });
    m.def("backend_init", &tt_lazy::backend_init);
    m.def("stream", []() { return (uintptr_t)ttc_get_stream(); });
}
