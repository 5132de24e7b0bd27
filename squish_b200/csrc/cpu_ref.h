// cpu_ref.h — registration hook of the C++ CPU reference kernels.
#pragma once
#include <pybind11/pybind11.h>

namespace sqcpu {
void register_cpu(pybind11::module& m);
}
