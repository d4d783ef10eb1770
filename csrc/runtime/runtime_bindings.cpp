// runtime_bindings.cpp - pybind11 registration of the native ring runtime.
#include <torch/extension.h>

void register_runtime(pybind11::module_& m) { (void)m; }
