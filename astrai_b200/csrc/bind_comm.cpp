// Python bindings for the comm kernels (filled in as the kernels land).
#include <torch/extension.h>

void register_comm(pybind11::module& m) { (void)m; }
