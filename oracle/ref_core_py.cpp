// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// pybind11 re-binding of the reference's `kansai._core` extension module.
// The reference binds its C++ core with nanobind (python/bindings.cpp:17),
// which is not installed in this image and cannot be installed offline.
// pybind11 is installed, so this file exposes the same names and argument
// meanings (python/bindings.cpp:20-135, :207-208) over the reference's own,
// unmodified C++ sources (core/src/*.cpp, backend/cpu/src/*.cpp), which the
// oracle Makefile compiles where they lie in the reference tree.
//
// With this module importable as `kansai._core`, the reference's own Python
// (python/kansai/quantize.py, nn.py, distributed.py, optim.py) runs unmodified
// and is the ground truth the golden fixtures under tests/golden/ come from.
// Compute methods release the GIL, as python/bindings.cpp:63-122 does.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "kansai/Fused.hpp"
#include "kansai/GradOps.hpp"
#include "kansai/Tensor.hpp"

namespace py = pybind11;
using namespace kan;

PYBIND11_MODULE(_core, m) {
    m.doc() = "reference kansai._core re-bound with pybind11 (oracle only)";
    using rel = py::call_guard<py::gil_scoped_release>;

    py::class_<Tensor>(m, "Tensor")
        .def("__repr__", [](const Tensor& t) {
            std::string s = "Tensor(shape=[";
            for (size_t i = 0; i < t.shape().size(); ++i) {
                if (i) s += ", ";
                s += std::to_string(t.shape()[i]);
            }
            return s + "])";
        })
        .def_property_readonly("shape", [](const Tensor& t) { return t.shape(); })
        .def_property_readonly("requires_grad", &Tensor::requires_grad)
        .def_property_readonly("grad", [](const Tensor& t) -> std::optional<Tensor> { return t.grad(); })
        .def("_set_requires_grad", &Tensor::set_requires_grad, py::arg("requires_grad"))
        .def("numel", &Tensor::numel)
        .def("tolist", &Tensor::to_vector)
        .def("backward",
             [](Tensor& t, std::optional<Tensor> g) {
                 if (g.has_value()) t.backward(*g);
                 else t.backward();
             },
             py::arg("grad_output") = py::none())
        .def("zero_grad", &Tensor::zero_grad)
        .def("add_", &Tensor::add_, py::arg("other"), py::arg("alpha") = 1.0f, rel())
        .def("detach", &Tensor::detach, rel())
        .def("add", &Tensor::add, py::arg("other"), rel())
        .def("sub", &Tensor::sub, py::arg("other"), rel())
        .def("mul", &Tensor::mul, py::arg("other"), rel())
        .def("gt", &Tensor::gt, py::arg("other"), rel())
        .def("lt", &Tensor::lt, py::arg("other"), rel())
        .def("eq", &Tensor::eq, py::arg("other"), rel())
        .def("matmul", &Tensor::matmul, py::arg("other"), rel())
        .def("relu", &Tensor::relu, rel())
        .def("sum", static_cast<Tensor (Tensor::*)() const>(&Tensor::sum), rel())
        .def("sum", static_cast<Tensor (Tensor::*)(int64_t, bool) const>(&Tensor::sum),
             py::arg("dim"), py::arg("keepdim") = false, rel())
        .def("mean", static_cast<Tensor (Tensor::*)() const>(&Tensor::mean), rel())
        .def("mean", static_cast<Tensor (Tensor::*)(int64_t, bool) const>(&Tensor::mean),
             py::arg("dim"), py::arg("keepdim") = false, rel())
        .def("max", &Tensor::max, py::arg("dim"), py::arg("keepdim") = false, rel())
        .def("reshape", &Tensor::reshape, py::arg("shape"), rel())
        .def("transpose", &Tensor::transpose, py::arg("dim0"), py::arg("dim1"), rel())
        .def("slice", &Tensor::slice, py::arg("dim"), py::arg("start"), py::arg("stop"), rel())
        .def("sqrt", &Tensor::sqrt, rel())
        .def("reciprocal", &Tensor::reciprocal, rel())
        .def("div", &Tensor::div, py::arg("other"), rel())
        .def("exp", &Tensor::exp, rel())
        .def("log", &Tensor::log, rel())
        .def("tanh", &Tensor::tanh, rel())
        .def("sigmoid", &Tensor::sigmoid, rel())
        .def("gelu", &Tensor::gelu, rel())
        .def("leaky_relu", &Tensor::leaky_relu, py::arg("negative_slope") = 0.01f, rel())
        .def("softmax", &Tensor::softmax, py::arg("dim"), rel())
        .def("cross_entropy", &Tensor::cross_entropy, py::arg("targets"), rel())
        .def("index_select", &Tensor::index_select, py::arg("dim"), py::arg("indices"), rel())
        .def("__add__", &Tensor::add)
        .def("__sub__", &Tensor::sub)
        .def("__mul__", &Tensor::mul)
        .def("__matmul__", &Tensor::matmul)
        .def("__truediv__", &Tensor::div);

    m.def("zeros", &Tensor::zeros, py::arg("shape"), py::arg("requires_grad") = false);
    m.def("ones", &Tensor::ones, py::arg("shape"), py::arg("requires_grad") = false);
    m.def("randn", &Tensor::randn, py::arg("shape"), py::arg("std") = 1.0f,
          py::arg("requires_grad") = false, py::arg("seed") = 0);
    m.def("from_flat", &Tensor::from_flat, py::arg("data"), py::arg("shape"),
          py::arg("requires_grad") = false);
    m.def("cat", &Tensor::cat, py::arg("tensors"), py::arg("dim"), rel());
    m.def("fused_bias_relu", &fused_bias_relu, py::arg("x"), py::arg("bias"), rel());
    m.def("relu_backward", &relu_backward, py::arg("input"), py::arg("grad_output"), rel());
    m.def("sum_axis0", &sum_axis0, py::arg("grad_output"), rel());
    m.def("matmul_nt", &matmul_nt, py::arg("a"), py::arg("b"), rel());
    m.def("matmul_tn", &matmul_tn, py::arg("a"), py::arg("b"), rel());
    m.def("set_grad_enabled", &set_grad_enabled, py::arg("enabled"));
    m.def("grad_enabled", &grad_enabled);
    // The reference reports Metal only on macOS builds (python/bindings.cpp:249-271);
    // a Linux build has no Metal backend.
    m.def("metal_available", []() { return false; });
}
