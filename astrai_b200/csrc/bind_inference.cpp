// Python bindings for the inference kernels (filled in as the kernels land).
#include <torch/extension.h>

void register_inference(pybind11::module& m) { (void)m; }
