// host_utils.cpp — host-side helpers of the serving loop, in C++ so they cost microseconds per
// call on the engine thread.
//
// detect_token_loop: repetition-loop detection over a request's generated token ids. The
// reference scans the trailing characters of the decoded text for a period p whose last
// p * reps characters match the characters one period earlier at >= 95%
// (squish/serving/loop_guard.py:44-75); here the same test runs on token ids, which needs no
// detokenization and treats every language alike. Short units need `short_reps` repetitions,
// units of at least `block_period` tokens (whole sentences) only `block_reps`.
//
// NGramIndex: the prompt-lookup drafter's index (reference: the n-gram index of
// squish/speculative/prompt_lookup.py:96-182 and the ouroboros n-gram build,
// squish_quant_rs/src/lib.rs:4539). It owns a copy of the request's token stream, maps every
// n-gram (n_min <= n <= n_max) by a 64-bit hash to the positions where it ends, and answers
// "continuations of the current suffix": up to `want` distinct next-k-token runs after earlier
// occurrences of the longest matching suffix, most recent first. Hash hits are verified
// token by token, so collisions cannot produce a wrong draft.
#include <torch/extension.h>

#include <algorithm>
#include <cstdint>
#include <unordered_map>
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

class NGramIndex {
 public:
  NGramIndex(int64_t n_min, int64_t n_max) : n_min_((int)n_min), n_max_((int)n_max), maps_(n_max + 1) {
    TORCH_CHECK(n_min >= 1 && n_max >= n_min && n_max <= 64, "n-gram range must satisfy 1 <= n_min <= n_max <= 64");
  }

  int64_t size() const { return (int64_t)t_.size(); }

  void extend(const std::vector<int64_t>& toks) {
    for (int64_t v : toks) {
      t_.push_back((int32_t)v);
      const int end = (int)t_.size() - 1;
      uint64_t h = kSeed;
      for (int n = 1; n <= n_max_ && n <= end + 1; ++n) {  // grams ending at `end`, growing leftwards
        h = mix(h, (uint64_t)(uint32_t)t_[end + 1 - n]);
        if (n >= n_min_) maps_[n][h].push_back(end);
      }
    }
  }

  std::vector<std::vector<int64_t>> continuations(int64_t k, int64_t want) const {
    std::vector<std::vector<int64_t>> out;
    const int L = (int)t_.size();
    // hashes of the current suffix for every n, built the same way as in extend()
    std::vector<uint64_t> hs(n_max_ + 1, 0);
    uint64_t h = kSeed;
    for (int n = 1; n <= n_max_ && n <= L; ++n) {
      h = mix(h, (uint64_t)(uint32_t)t_[L - n]);
      hs[n] = h;
    }
    for (int n = n_max_; n >= n_min_; --n) {
      if (L < n + 1) continue;
      auto it = maps_[n].find(hs[n]);
      if (it == maps_[n].end()) continue;
      const std::vector<int32_t>& ends = it->second;
      for (auto e = ends.rbegin(); e != ends.rend(); ++e) {
        const int end = *e;
        if (end >= L - 1) continue;  // the suffix itself
        bool same = true;            // verify the gram (hash collisions)
        for (int j = 0; j < n && same; ++j) same = t_[end - j] == t_[L - 1 - j];
        if (!same) continue;
        const int c0 = end + 1, c1 = std::min<int>(L, end + 1 + (int)k);
        if (c1 <= c0) continue;
        std::vector<int64_t> cont(t_.begin() + c0, t_.begin() + c1);
        bool dup = false;
        for (const auto& o : out) dup = dup || o == cont;
        if (dup) continue;
        out.push_back(std::move(cont));
        if ((int64_t)out.size() >= want) return out;
      }
      if (!out.empty()) return out;
    }
    return out;
  }

 private:
  static constexpr uint64_t kSeed = 0x51ED270B27A3F1C5ull;
  static uint64_t mix(uint64_t h, uint64_t v) {  // SplitMix64 finaliser of (h ^ v * odd)
    uint64_t z = h ^ (v * 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  int n_min_, n_max_;
  std::vector<int32_t> t_;
  std::vector<std::unordered_map<uint64_t, std::vector<int32_t>>> maps_;
};

void register_host(pybind11::module& m) {
  auto h = m.def_submodule("host", "host-side serving helpers");
  h.def("detect_token_loop", &detect_token_loop, pybind11::arg("tokens"), pybind11::arg("min_period") = 2,
        pybind11::arg("max_period") = 96, pybind11::arg("short_reps") = 4, pybind11::arg("block_period") = 32,
        pybind11::arg("block_reps") = 2, pybind11::arg("match_ratio") = 0.95);
  pybind11::class_<NGramIndex>(h, "NGramIndex")
      .def(pybind11::init<int64_t, int64_t>())
      .def("extend", &NGramIndex::extend)
      .def("continuations", &NGramIndex::continuations)
      .def("__len__", &NGramIndex::size);
}

}  // namespace sqhost
