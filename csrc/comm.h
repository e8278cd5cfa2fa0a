// Symmetric peer memory for the fused compute+collective kernels (one process per GPU, NVLink/NVSwitch).
#pragma once
#include <torch/extension.h>

namespace hrm {
void register_comm_bindings(pybind11::module& m);
}
