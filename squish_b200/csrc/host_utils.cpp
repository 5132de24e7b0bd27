// host_utils.cpp — host-side helpers of the serving loop, in C++ so they cost microseconds per
// call on the engine thread.
//
// detect_token_loop: repetition-loop detection over a request's generated token ids. The
// reference scans the trailing characters of the decoded text for a period p whose last
// p * reps characters match the characters one period earlier at >= 95%
// (squish/serving/loop_guard.py:44-75); here the same test runs on token ids, which needs no
// detokenization and treats every language alike. Short units need `short_reps` repetitions,
// units of at least `block_period` tokens (whole sentences) only `block_reps`.
#include <torch/extension.h>

#include <cstdint>
#include <vector>

namespace sqhost {

bool detect_token_loop(const std::vector<int64_t>& t, int64_t min_period, int64_t max_period, int64_t short_reps,
                       int64_t block_period, int64_t block_reps, double match_ratio) {
  const int64_t n = (int64_t)t.size();
  for (int64_t period = std::max<int64_t>(1, min_period); period <= max_period; ++period) {
    const int64_t reps = period >= block_period ? block_reps : short_reps;
    const int64_t span = period * reps;
    if (span > n) continue;  // block-sized periods need fewer repetitions: keep scanning
    const int64_t base = n - span;
    const int64_t cmp = span - period;  // positions compared against one period earlier
    const int64_t allowed = cmp - (int64_t)((double)cmp * match_ratio);
    int64_t mism = 0;
    bool loop = true;
    for (int64_t i = base + period; i < n; ++i) {
      if (t[i] != t[i - period] && ++mism > allowed) {
        loop = false;
        break;
      }
    }
    if (loop) return true;
  }
  return false;
}

void register_host(pybind11::module& m) {
  auto h = m.def_submodule("host", "host-side serving helpers");
  h.def("detect_token_loop", &detect_token_loop, pybind11::arg("tokens"), pybind11::arg("min_period") = 2,
        pybind11::arg("max_period") = 96, pybind11::arg("short_reps") = 4, pybind11::arg("block_period") = 32,
        pybind11::arg("block_reps") = 2, pybind11::arg("match_ratio") = 0.95);
}

}  // namespace sqhost
