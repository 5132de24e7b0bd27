// host_module.cpp — the host C++ libraries alone (CPU codecs, entropy codecs, serving helpers,
// JSON / JSON-schema matchers) as their own Python module, for sanitizer builds: compiled
// with AddressSanitizer and UndefinedBehaviorSanitizer by squish_b200/sanitize/__init__.py and
// driven with randomized and malformed inputs by tests/test_sanitize_cpu.py. The production
// extension (_C) registers the same functions next to the CUDA kernels.
#include <torch/extension.h>

namespace sqcpu {
void register_cpu(pybind11::module& m);  // cpu_ref.cpp (+ entropy.cpp)
}
namespace sqhost {
void register_host(pybind11::module& m);  // host_utils.cpp
}
namespace sqgram {
void register_grammar(pybind11::module& m);  // grammar.cpp
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "squish_b200 host C++ libraries (sanitizer build)";
  sqcpu::register_cpu(m);
  sqhost::register_host(m);
  sqgram::register_grammar(m);
}
