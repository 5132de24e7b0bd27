// kv_research.cpp — host C++ kernels of the KV-cache budget / scoring research policies
// (float32, CPU): layer budgets, per-head attention statistics over an observation window,
// low-rank key spectra and projections, cluster scores and LSH-sampled attention.
//
// The reference ships these as Rust functions of squish_quant_rs with no Python caller:
// CAKE attention entropy (src/lib.rs:3585), GreenKV window scores (3981), SVDq head spectra
// (4210), ShadowKV low-rank key fit / projection (4283, 4368), ClusterKV cluster sums (4427),
// PyramidKV layer budgets (4662), MagicPIG attention (5307). On the serving path this
// package scores KV pages on the device (kv_score.cu: attention mass per page, accumulated
// with an optional decay for heavy-hitter eviction); these functions are the offline / analysis
// counterparts. Each states its math below; MagicPIG here is the published SimHash sampling
// estimator (the reference kernel computes exact attention).
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <tuple>
#include <vector>

namespace sqcpu {

namespace {

torch::Tensor f32(const torch::Tensor& t) { return t.to(torch::kCPU, torch::kFloat32).contiguous(); }

// softmax of s[0..n) in place (max-subtracted)
void softmax_inplace(std::vector<float>& s) {
  float m = -INFINITY;
  for (float v : s) m = std::max(m, v);
  double z = 0;
  for (float& v : s) {
    v = std::exp(v - m);
    z += v;
  }
  for (float& v : s) v = (float)(v / z);
}

uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// standard normal from two uniforms of a counter hash (Box-Muller)
float gauss(uint64_t seed, uint64_t i) {
  const uint64_t a = mix64(seed * 0x9E3779B97F4A7C15ull + 2 * i + 1), b = mix64(seed ^ (2 * i + 2) * 0xD1B54A32D192ED03ull);
  const double u1 = ((a >> 11) + 0.5) * (1.0 / 9007199254740992.0), u2 = ((b >> 11) + 0.5) * (1.0 / 9007199254740992.0);
  return (float)(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
}

}  // namespace

// CAKE: mean normalised attention entropy per head over the observation-window queries,
// entropy(p) / ln(T) with p = softmax(q . k / (sqrt(D) temperature)) over the T keys.
// q_obs [W, H, D], k [T, H, D] -> [H].
torch::Tensor cake_entropy(torch::Tensor q_obs, torch::Tensor k, double temperature) {
  auto q = f32(q_obs), kk = f32(k);
  TORCH_CHECK(q.dim() == 3 && kk.dim() == 3 && q.size(1) == kk.size(1) && q.size(2) == kk.size(2),
              "q_obs [W, H, D], k [T, H, D]");
  const int64_t W = q.size(0), H = q.size(1), D = q.size(2), T = kk.size(0);
  auto out = torch::zeros({H}, torch::kFloat32);
  if (T < 2 || W == 0) return out;
  float* op = out.data_ptr<float>();
  const float scale = (float)(1.0 / (std::sqrt((double)D) * temperature));
  const float* qp = q.data_ptr<float>();
  const float* kp = kk.data_ptr<float>();
  std::vector<float> s(T);
  for (int64_t h = 0; h < H; ++h) {
    double acc = 0;
    for (int64_t w = 0; w < W; ++w) {
      const float* qr = qp + (w * H + h) * D;
      for (int64_t t = 0; t < T; ++t) {
        const float* kr = kp + (t * H + h) * D;
        float d = 0.f;
        for (int64_t j = 0; j < D; ++j) d += qr[j] * kr[j];
        s[t] = d * scale;
      }
      softmax_inplace(s);
      double e = 0;
      for (float p : s)
        if (p > 0.f) e -= (double)p * std::log((double)p);
      acc += e / std::log((double)T);
    }
    op[h] = (float)(acc / (double)W);
  }
  return out;
}

// GreenKV / SnapKV-style token scores: per head, the mean over the observation-window queries
// of their softmax attention (scale 1 / sqrt(D)) on every key. q_obs [H, W, D], k [H, T, D]
// -> [H, T].
torch::Tensor green_kv_score(torch::Tensor q_obs, torch::Tensor k) {
  auto q = f32(q_obs), kk = f32(k);
  TORCH_CHECK(q.dim() == 3 && kk.dim() == 3 && q.size(0) == kk.size(0) && q.size(2) == kk.size(2),
              "q_obs [H, W, D], k [H, T, D]");
  const int64_t H = q.size(0), W = q.size(1), D = q.size(2), T = kk.size(1);
  auto out = torch::zeros({H, T}, torch::kFloat32);
  float* op = out.data_ptr<float>();
  const float scale = (float)(1.0 / std::sqrt((double)D));
  std::vector<float> s(T);
  for (int64_t h = 0; h < H; ++h)
    for (int64_t w = 0; w < W; ++w) {
      const float* qr = q.data_ptr<float>() + (h * W + w) * D;
      for (int64_t t = 0; t < T; ++t) {
        const float* kr = kk.data_ptr<float>() + (h * T + t) * D;
        float d = 0.f;
        for (int64_t j = 0; j < D; ++j) d += qr[j] * kr[j];
        s[t] = d * scale;
      }
      if (T) softmax_inplace(s);
      for (int64_t t = 0; t < T; ++t) op[h * T + t] += s[t] / (float)W;
    }
  return out;
}

// SVDq: singular values of every (layer, head) key matrix [T, D]. keys [L, H, T, D] ->
// [L, H, min(T, D)] descending.
torch::Tensor svd_head_spectrum(torch::Tensor keys) {
  auto k = f32(keys);
  TORCH_CHECK(k.dim() == 4, "keys [L, H, T, D]");
  return torch::linalg_svdvals(k);
}

// ShadowKV: per head the top-`rank` right singular vectors of the key matrix [T, D] (the
// low-rank key basis) -> [H, rank, D]; project: keys [H, N, D] x V[h]^T -> [H, N, rank].
torch::Tensor shadow_kv_fit(torch::Tensor keys, int64_t rank) {
  auto k = f32(keys);
  TORCH_CHECK(k.dim() == 3 && rank >= 1 && rank <= std::min(k.size(1), k.size(2)), "keys [H, T, D], 1 <= rank <= min(T, D)");
  auto svd = torch::linalg_svd(k, /*full_matrices=*/false);
  auto vh = std::get<2>(svd);  // [H, min(T, D), D]
  return vh.narrow(1, 0, rank).contiguous();
}

torch::Tensor shadow_kv_project(torch::Tensor keys, torch::Tensor basis) {
  auto k = f32(keys), v = f32(basis);
  TORCH_CHECK(k.dim() == 3 && v.dim() == 3 && k.size(0) == v.size(0) && k.size(2) == v.size(2),
              "keys [H, N, D], basis [H, rank, D]");
  return torch::bmm(k, v.transpose(1, 2)).contiguous();
}

// ClusterKV: total attention weight of the tokens assigned to each cluster.
torch::Tensor cluster_kv_score(torch::Tensor assignments, torch::Tensor attn, int64_t n_clusters) {
  auto a = assignments.to(torch::kCPU, torch::kInt64).contiguous().view({-1});
  auto w = f32(attn).view({-1});
  TORCH_CHECK(a.numel() == w.numel() && n_clusters >= 1, "one cluster id per weight");
  auto out = torch::zeros({n_clusters}, torch::kFloat32);
  float* op = out.data_ptr<float>();
  const int64_t* ap = a.data_ptr<int64_t>();
  const float* wp = w.data_ptr<float>();
  for (int64_t i = 0; i < a.numel(); ++i) {
    TORCH_CHECK(ap[i] >= 0 && ap[i] < n_clusters, "cluster id out of range");
    op[ap[i]] += wp[i];
  }
  return out;
}

// PyramidKV: per-layer KV budgets decaying linearly with depth,
// budget[l] = max(min_budget, round(base (1 - alpha l / (L - 1)))).
torch::Tensor pyramid_kv_budget(int64_t base, double alpha, int64_t n_layers, int64_t min_budget) {
  TORCH_CHECK(n_layers >= 1 && alpha >= 0.0 && alpha <= 1.0, "n_layers >= 1, alpha in [0, 1]");
  auto out = torch::empty({n_layers}, torch::kInt32);
  int32_t* op = out.data_ptr<int32_t>();
  for (int64_t l = 0; l < n_layers; ++l) {
    const double f = n_layers > 1 ? 1.0 - alpha * (double)l / (double)(n_layers - 1) : 1.0;
    op[l] = (int32_t)std::max<int64_t>(min_budget, (int64_t)std::llround((double)base * f));
  }
  return out;
}

// MagicPIG-style attention estimate (Chen et al. 2024): SimHash with `tables` tables of `bits`
// random hyperplanes each; a key is sampled for a query when it shares the query's bucket in at
// least one table; the softmax numerator of each sampled key is divided by its sampling
// probability p = 1 - (1 - (1 - theta / pi)^bits)^tables (theta: the query-key angle), the
// self-normalised estimate sum_i w_i v_i / sum_i w_i. A query with no sampled key falls back
// to exact attention. q [H, Tq, D], k / v [H, S, D] -> ([H, Tq, D], sampled fraction [H, Tq]).
std::tuple<torch::Tensor, torch::Tensor> magic_pig_attention(torch::Tensor q, torch::Tensor k, torch::Tensor v,
                                                             int64_t tables, int64_t bits, int64_t seed) {
  auto Q = f32(q), K = f32(k), V = f32(v);
  TORCH_CHECK(Q.dim() == 3 && K.dim() == 3 && V.dim() == 3 && Q.size(0) == K.size(0) && K.sizes() == V.sizes() &&
                  Q.size(2) == K.size(2),
              "q [H, Tq, D], k / v [H, S, D]");
  TORCH_CHECK(tables >= 1 && bits >= 1 && bits <= 30, "tables >= 1, 1 <= bits <= 30");
  const int64_t H = Q.size(0), Tq = Q.size(1), D = Q.size(2), S = K.size(1);
  auto out = torch::zeros({H, Tq, D}, torch::kFloat32);
  auto frac = torch::zeros({H, Tq}, torch::kFloat32);
  float* fp = frac.data_ptr<float>();
  // hyperplanes [tables * bits, D]
  std::vector<float> planes(tables * bits * D);
  for (size_t i = 0; i < planes.size(); ++i) planes[i] = gauss((uint64_t)seed, i);
  auto code = [&](const float* x, int64_t t) {
    uint32_t c = 0;
    for (int64_t b = 0; b < bits; ++b) {
      const float* pl = planes.data() + (t * bits + b) * D;
      float d = 0.f;
      for (int64_t j = 0; j < D; ++j) d += pl[j] * x[j];
      c |= (d >= 0.f ? 1u : 0u) << b;
    }
    return c;
  };
  const float scale = (float)(1.0 / std::sqrt((double)D));
  const double pi = 3.141592653589793;
  std::vector<uint32_t> kc(S * tables);
  for (int64_t h = 0; h < H; ++h) {
    const float* kh = K.data_ptr<float>() + h * S * D;
    const float* vh = V.data_ptr<float>() + h * S * D;
    std::vector<double> kn(S);
    for (int64_t s = 0; s < S; ++s) {
      double n = 0;
      for (int64_t j = 0; j < D; ++j) n += (double)kh[s * D + j] * kh[s * D + j];
      kn[s] = std::sqrt(n);
      for (int64_t t = 0; t < tables; ++t) kc[s * tables + t] = code(kh + s * D, t);
    }
    for (int64_t i = 0; i < Tq; ++i) {
      const float* qr = Q.data_ptr<float>() + (h * Tq + i) * D;
      std::vector<uint32_t> qc(tables);
      double qn = 0;
      for (int64_t j = 0; j < D; ++j) qn += (double)qr[j] * qr[j];
      qn = std::sqrt(qn);
      for (int64_t t = 0; t < tables; ++t) qc[t] = code(qr, t);
      std::vector<int64_t> idx;
      std::vector<double> logit, corr;
      for (int64_t s = 0; s < S; ++s) {
        bool hit = false;
        for (int64_t t = 0; t < tables && !hit; ++t) hit = kc[s * tables + t] == qc[t];
        if (!hit) continue;
        double d = 0;
        for (int64_t j = 0; j < D; ++j) d += (double)qr[j] * kh[s * D + j];
        const double cosv = (qn > 0 && kn[s] > 0) ? std::max(-1.0, std::min(1.0, d / (qn * kn[s]))) : 1.0;
        const double p1 = 1.0 - std::acos(cosv) / pi;  // one hyperplane agrees
        const double p = 1.0 - std::pow(1.0 - std::pow(p1, (double)bits), (double)tables);
        idx.push_back(s);
        logit.push_back(d * scale);
        corr.push_back(std::max(p, 1e-12));
      }
      float* o = out.data_ptr<float>() + (h * Tq + i) * D;
      fp[h * Tq + i] = S ? (float)idx.size() / (float)S : 0.f;
      if (idx.empty()) {  // no collision: exact attention
        std::vector<float> s(S);
        for (int64_t r = 0; r < S; ++r) {
          float d = 0.f;
          for (int64_t j = 0; j < D; ++j) d += qr[j] * kh[r * D + j];
          s[r] = d * scale;
        }
        if (S) softmax_inplace(s);
        for (int64_t r = 0; r < S; ++r)
          for (int64_t j = 0; j < D; ++j) o[j] += s[r] * vh[r * D + j];
        continue;
      }
      double m = -INFINITY;
      for (double l : logit) m = std::max(m, l);
      double z = 0;
      std::vector<double> w(idx.size());
      for (size_t r = 0; r < idx.size(); ++r) {
        w[r] = std::exp(logit[r] - m) / corr[r];
        z += w[r];
      }
      for (size_t r = 0; r < idx.size(); ++r)
        for (int64_t j = 0; j < D; ++j) o[j] += (float)(w[r] / z) * vh[idx[r] * D + j];
    }
  }
  return {out, frac};
}

void register_kv_research(pybind11::module& c) {
  c.def("cake_entropy", &cake_entropy, pybind11::arg("q_obs"), pybind11::arg("k"), pybind11::arg("temperature") = 1.0);
  c.def("green_kv_score", &green_kv_score);
  c.def("svd_head_spectrum", &svd_head_spectrum);
  c.def("shadow_kv_fit", &shadow_kv_fit);
  c.def("shadow_kv_project", &shadow_kv_project);
  c.def("cluster_kv_score", &cluster_kv_score);
  c.def("pyramid_kv_budget", &pyramid_kv_budget, pybind11::arg("base"), pybind11::arg("alpha"),
        pybind11::arg("n_layers"), pybind11::arg("min_budget") = 1);
  c.def("magic_pig_attention", &magic_pig_attention, pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"),
        pybind11::arg("tables") = 8, pybind11::arg("bits") = 6, pybind11::arg("seed") = 0);
}

}  // namespace sqcpu
