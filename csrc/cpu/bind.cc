// Python bindings of the CPU backend and the safetensors reader (module mod_b200._cpu).
#include <torch/extension.h>
#include <omp.h>
#include "cpu_ops.h"
#include "safetensors.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mod_b200 C++/OpenMP CPU backend and safetensors mmap reader";
  m.def("linear", &mbcpu::linear);
  m.def("linear_w8", &mbcpu::linear_w8);
  m.def("rmsnorm", &mbcpu::rmsnorm);
  m.def("rope_qknorm", &mbcpu::rope_qknorm);
  m.def("attn_paged", &mbcpu::attn_paged);
  m.def("swiglu", &mbcpu::swiglu);
  m.def("gelu_tanh", &mbcpu::gelu_tanh);
  m.def("embed", &mbcpu::embed);
  m.def("argmax", &mbcpu::argmax);
  m.def("moe_route", &mbcpu::moe_route);
  m.def("moe_experts", &mbcpu::moe_experts);
  m.def("deltanet_recurrence", &mbcpu::deltanet_recurrence);
  m.def("conv1d_causal", &mbcpu::conv1d_causal);
  m.def("resize_bilinear", &mbcpu::resize_bilinear);
  m.def("set_num_threads", [](int n) { omp_set_num_threads(n); });
  m.def("get_max_threads", []() { return omp_get_max_threads(); });
  mbio::bind(m);
}
