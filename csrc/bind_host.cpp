// Python bindings of the host-side C++ runtime (module mtorus._C).
#include <torch/extension.h>

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mtorus host runtime";
  m.attr("__version__") = "0.1.0";
}
