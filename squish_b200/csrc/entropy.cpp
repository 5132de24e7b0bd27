// entropy.cpp — host byte codecs for load-time weight decompression: rANS and prefix-code
// (Huffman) coding over a 256-symbol alphabet.
//
// Counterparts of the reference's rans_encode / rans_decode / huffman_encode /
// huffman_decode (squish_quant_rs/src/lib.rs:1637-1830), with the same Python-facing
// signatures (symbols + 256-entry tables in, bytes out). The streams are this library's own:
//
//  * rANS (Duda, "Asymmetric numeral systems", 2013; byte-wise renormalisation): the caller's
//    frequencies are rescaled deterministically to a total of 2^16 (every present symbol keeps
//    a non-zero share), the 32-bit state lives in [2^23, 2^31), symbols are coded in reverse
//    so the decoder reads forward; the stream starts with the final state, big-endian.
//  * Prefix codes: code words are packed most-significant bit first; decoding uses a direct
//    lookup table when the longest code has <= 16 bits and a binary trie otherwise.
//  * huffman_build: code lengths from a standard Huffman merge over the byte histogram (lengths
//    capped at 24 by flattening the histogram), canonical code words from the lengths.
#include <torch/extension.h>

#include <algorithm>
#include <cstring>
#include <array>
#include <cstdint>
#include <queue>
#include <stdexcept>
#include <vector>

namespace sqcpu {
namespace {

constexpr int kScaleBits = 16;
constexpr uint32_t kTotal = 1u << kScaleBits;
constexpr uint32_t kLow = 1u << 23;  // state lower bound

using Table = std::array<uint32_t, 256>;

const uint8_t* u8_data(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.device().is_cpu() && t.scalar_type() == torch::kUInt8 && t.is_contiguous(), name,
              " must be a contiguous uint8 CPU tensor");
  return t.data_ptr<uint8_t>();
}

Table read_table(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.device().is_cpu() && t.numel() == 256, name, " must have 256 entries");
  auto v = t.to(torch::kInt64).contiguous();
  Table out{};
  const int64_t* p = v.data_ptr<int64_t>();
  for (int i = 0; i < 256; ++i) {
    TORCH_CHECK(p[i] >= 0 && p[i] <= 0xFFFFFFFFLL, name, " entries must fit in uint32");
    out[i] = (uint32_t)p[i];
  }
  return out;
}

// Rescale frequencies to sum exactly to 2^16, keeping every non-zero symbol >= 1.
Table normalise(const Table& f) {
  uint64_t total = 0;
  for (uint32_t v : f) total += v;
  TORCH_CHECK(total > 0, "sum of freqs must be > 0");
  Table q{};
  int64_t sum = 0;
  for (int s = 0; s < 256; ++s) {
    if (f[s] == 0) continue;
    q[s] = std::max<uint32_t>(1, (uint32_t)(((uint64_t)f[s] * kTotal) / total));
    sum += q[s];
  }
  // absorb the rounding difference in the largest shares
  auto largest = [&]() {
    int best = 0;
    for (int s = 1; s < 256; ++s)
      if (q[s] > q[best]) best = s;
    return best;
  };
  while (sum > (int64_t)kTotal) {  // at most 256 symbols of >= 1: always reducible
    const int s = largest();
    const int64_t dec = std::min<int64_t>(sum - (int64_t)kTotal, (int64_t)q[s] - 1);
    q[s] -= (uint32_t)dec;
    sum -= dec;
  }
  if (sum < (int64_t)kTotal) q[largest()] += (uint32_t)((int64_t)kTotal - sum);
  return q;
}

Table cumulative(const Table& q) {
  Table c{};
  uint32_t acc = 0;
  for (int s = 0; s < 256; ++s) {
    c[s] = acc;
    acc += q[s];
  }
  return c;
}

torch::Tensor to_tensor(const std::vector<uint8_t>& v) {
  auto t = torch::empty({(int64_t)v.size()}, torch::kUInt8);
  if (!v.empty()) std::memcpy(t.data_ptr<uint8_t>(), v.data(), v.size());
  return t;
}

torch::Tensor rans_encode(torch::Tensor symbols, torch::Tensor freqs) {
  const uint8_t* sym = u8_data(symbols, "symbols");
  const int64_t n = symbols.numel();
  const Table q = normalise(read_table(freqs, "freqs"));
  const Table c = cumulative(q);
  for (int64_t i = 0; i < n; ++i)
    if (q[sym[i]] == 0) throw std::invalid_argument("symbol " + std::to_string((int)sym[i]) + " has zero frequency");
  std::vector<uint8_t> out;
  out.reserve((size_t)n + 8);
  uint32_t x = kLow;
  for (int64_t i = n - 1; i >= 0; --i) {
    const uint32_t f = q[sym[i]];
    const uint32_t x_max = ((kLow >> kScaleBits) << 8) * f;
    while (x >= x_max) {
      out.push_back((uint8_t)(x & 0xFF));
      x >>= 8;
    }
    x = ((x / f) << kScaleBits) + (x % f) + c[sym[i]];
  }
  for (int b = 0; b < 4; ++b) out.push_back((uint8_t)(x >> (8 * b)));  // reversed below: big-endian
  std::reverse(out.begin(), out.end());
  return to_tensor(out);
}

torch::Tensor rans_decode(torch::Tensor data, torch::Tensor freqs, int64_t n_symbols) {
  const uint8_t* d = u8_data(data, "data");
  const int64_t len = data.numel();
  TORCH_CHECK(len >= 4, "data too short");
  TORCH_CHECK(n_symbols >= 0, "n_symbols must be >= 0");
  const Table q = normalise(read_table(freqs, "freqs"));
  const Table c = cumulative(q);
  std::vector<uint8_t> slot_sym(kTotal);
  for (int s = 0; s < 256; ++s)
    for (uint32_t k = c[s]; k < c[s] + q[s]; ++k) slot_sym[k] = (uint8_t)s;
  int64_t pos = 0;
  uint32_t x = 0;
  for (int b = 0; b < 4; ++b) x = (x << 8) | d[pos++];
  auto out = torch::empty({n_symbols}, torch::kUInt8);
  uint8_t* o = out.data_ptr<uint8_t>();
  for (int64_t i = 0; i < n_symbols; ++i) {
    const uint32_t slot = x & (kTotal - 1);
    const uint8_t s = slot_sym[slot];
    o[i] = s;
    x = q[s] * (x >> kScaleBits) + slot - c[s];
    while (x < kLow) {
      TORCH_CHECK(pos < len, "rANS stream ended early");
      x = (x << 8) | d[pos++];
    }
  }
  return out;
}

void check_code(const Table& words, const Table& lens) {
  for (int s = 0; s < 256; ++s) {
    TORCH_CHECK(lens[s] <= 32, "code lengths must be <= 32");
    if (lens[s] > 0 && lens[s] < 32) TORCH_CHECK(words[s] < (1u << lens[s]), "code word wider than its length");
  }
}

torch::Tensor huffman_encode(torch::Tensor symbols, torch::Tensor code_words, torch::Tensor code_lens) {
  const uint8_t* sym = u8_data(symbols, "symbols");
  const int64_t n = symbols.numel();
  const Table w = read_table(code_words, "code_words"), l = read_table(code_lens, "code_lens");
  check_code(w, l);
  std::vector<uint8_t> out;
  out.reserve((size_t)n / 2 + 8);
  uint64_t acc = 0;
  int bits = 0;
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t len = l[sym[i]];
    if (len == 0) throw std::invalid_argument("symbol " + std::to_string((int)sym[i]) + " has no code");
    acc = (acc << len) | w[sym[i]];
    bits += (int)len;
    while (bits >= 8) {
      bits -= 8;
      out.push_back((uint8_t)(acc >> bits));
    }
    acc &= (bits > 0) ? ((1ull << bits) - 1) : 0ull;
  }
  if (bits > 0) out.push_back((uint8_t)(acc << (8 - bits)));
  return to_tensor(out);
}

torch::Tensor huffman_decode(torch::Tensor data, torch::Tensor code_words, torch::Tensor code_lens,
                             int64_t n_symbols) {
  const uint8_t* d = u8_data(data, "data");
  const int64_t len = data.numel();
  const Table w = read_table(code_words, "code_words"), l = read_table(code_lens, "code_lens");
  check_code(w, l);
  uint32_t maxlen = 0;
  for (int s = 0; s < 256; ++s) maxlen = std::max(maxlen, l[s]);
  TORCH_CHECK(maxlen > 0, "empty code");
  auto out = torch::empty({n_symbols}, torch::kUInt8);
  uint8_t* o = out.data_ptr<uint8_t>();
  int64_t bitpos = 0;
  const int64_t total_bits = len * 8;
  auto peek = [&](int nbits) -> uint32_t {  // next nbits (MSB first), zero past the end
    uint32_t v = 0;
    for (int k = 0; k < nbits; ++k) {
      const int64_t b = bitpos + k;
      const uint32_t bit = b < total_bits ? (d[b >> 3] >> (7 - (b & 7))) & 1u : 0u;
      v = (v << 1) | bit;
    }
    return v;
  };
  if (maxlen <= 16) {
    // direct table: every maxlen-bit window -> (symbol, length)
    std::vector<uint16_t> sym_of(1u << maxlen, 0xFFFF);
    std::vector<uint8_t> len_of(1u << maxlen, 0);
    for (int s = 0; s < 256; ++s) {
      if (l[s] == 0) continue;
      const uint32_t span = 1u << (maxlen - l[s]);
      const uint32_t base = w[s] << (maxlen - l[s]);
      for (uint32_t k = 0; k < span; ++k) {
        TORCH_CHECK(sym_of[base + k] == 0xFFFF, "code is not prefix-free");
        sym_of[base + k] = (uint16_t)s;
        len_of[base + k] = (uint8_t)l[s];
      }
    }
    for (int64_t i = 0; i < n_symbols; ++i) {
      const uint32_t win = peek((int)maxlen);
      TORCH_CHECK(sym_of[win] != 0xFFFF, "invalid code in stream");
      o[i] = (uint8_t)sym_of[win];
      bitpos += len_of[win];
      TORCH_CHECK(bitpos <= total_bits, "prefix-code stream ended early");
    }
    return out;
  }
  // binary trie for long codes: node -> children, leaves carry symbol + 1
  std::vector<std::array<int32_t, 2>> kids(1, {0, 0});
  std::vector<int32_t> leaf(1, 0);
  for (int s = 0; s < 256; ++s) {
    if (l[s] == 0) continue;
    int32_t node = 0;
    for (int k = (int)l[s] - 1; k >= 0; --k) {
      TORCH_CHECK(leaf[node] == 0, "code is not prefix-free");
      const int bit = (w[s] >> k) & 1;
      if (kids[node][bit] == 0) {
        kids[node][bit] = (int32_t)kids.size();
        kids.push_back({0, 0});
        leaf.push_back(0);
      }
      node = kids[node][bit];
    }
    TORCH_CHECK(leaf[node] == 0 && kids[node][0] == 0 && kids[node][1] == 0, "code is not prefix-free");
    leaf[node] = s + 1;
  }
  for (int64_t i = 0; i < n_symbols; ++i) {
    int32_t node = 0;
    while (leaf[node] == 0) {
      TORCH_CHECK(bitpos < total_bits, "prefix-code stream ended early");
      const int bit = (d[bitpos >> 3] >> (7 - (bitpos & 7))) & 1;
      ++bitpos;
      node = kids[node][bit];
      TORCH_CHECK(node != 0, "invalid code in stream");
    }
    o[i] = (uint8_t)(leaf[node] - 1);
  }
  return out;
}

// Huffman code over a 256-bin histogram: returns (code_words uint32[256], code_lens uint8[256]).
std::vector<torch::Tensor> huffman_build(torch::Tensor freqs) {
  Table f = read_table(freqs, "freqs");
  int present = 0;
  for (uint32_t v : f) present += v > 0;
  TORCH_CHECK(present > 0, "sum of freqs must be > 0");
  Table lens{};
  for (int attempt = 0;; ++attempt) {
    lens.fill(0);
    if (present == 1) {
      for (int s = 0; s < 256; ++s)
        if (f[s]) lens[s] = 1;
    } else {
      // (weight, node) min-heap; nodes 0..255 are leaves
      using Item = std::pair<uint64_t, int>;
      std::priority_queue<Item, std::vector<Item>, std::greater<Item>> heap;
      std::vector<int> parent(512, -1);
      int next = 256;
      for (int s = 0; s < 256; ++s)
        if (f[s]) heap.push({f[s], s});
      while (heap.size() > 1) {
        const Item a = heap.top();
        heap.pop();
        const Item b = heap.top();
        heap.pop();
        parent[a.second] = next;
        parent[b.second] = next;
        heap.push({a.first + b.first, next++});
      }
      for (int s = 0; s < 256; ++s) {
        if (!f[s]) continue;
        uint32_t depth = 0;
        for (int n = s; parent[n] >= 0; n = parent[n]) ++depth;
        lens[s] = depth;
      }
    }
    uint32_t maxlen = 0;
    for (uint32_t v : lens) maxlen = std::max(maxlen, v);
    if (maxlen <= 24) break;
    TORCH_CHECK(attempt < 64, "could not bound code lengths");
    for (auto& v : f)  // flatten the histogram and rebuild
      if (v) v = (v >> 1) + 1;
  }
  // canonical code words: by (length, symbol)
  Table words{};
  uint32_t code = 0, prev_len = 0;
  std::vector<int> order;
  for (int s = 0; s < 256; ++s)
    if (lens[s]) order.push_back(s);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return lens[a] < lens[b]; });
  for (size_t i = 0; i < order.size(); ++i) {
    const int s = order[i];
    if (i > 0) code = (code + 1) << (lens[s] - prev_len);
    words[s] = code;
    prev_len = lens[s];
  }
  auto tw = torch::empty({256}, torch::kInt64), tl = torch::empty({256}, torch::kUInt8);
  for (int s = 0; s < 256; ++s) {
    tw.data_ptr<int64_t>()[s] = words[s];
    tl.data_ptr<uint8_t>()[s] = (uint8_t)lens[s];
  }
  return {tw, tl};
}

}  // namespace

void register_entropy(pybind11::module& c) {
  c.def("rans_encode", &rans_encode, "rANS-encode uint8 symbols under a 256-entry frequency table");
  c.def("rans_decode", &rans_decode, "decode n_symbols from a rans_encode stream");
  c.def("huffman_encode", &huffman_encode, "pack prefix-code words (MSB first)");
  c.def("huffman_decode", &huffman_decode, "decode n_symbols from huffman_encode output");
  c.def("huffman_build", &huffman_build, "Huffman code (canonical words, lengths <= 24) for a histogram");
}

}  // namespace sqcpu
