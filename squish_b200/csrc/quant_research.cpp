// quant_research.cpp — host C++ kernels for the convert-time quantization research methods and
// the small numeric helpers of the speculative / adaptive predictors (CPU, float32, OpenMP-free:
// these run once per checkpoint or on a handful of values per step).
//
// The reference ships these as Rust functions of squish_quant_rs (no Python caller besides its
// tests): any4 Lloyd calibration (src/lib.rs:4470), QuaRot group quantization (2870-2932),
// AdaRound steps (3421), FLUTE LUT encode / decode (3764-3827), QMoE block codebooks (4696),
// BitDistiller group quantization and refinement (4969, 5039), GGUF-style blocks with
// super-block scales (5137), PQ cache sub-codebooks (5223), the
// ReDrafter GRU step and batched cosine similarity (1977-2013), logistic / SGD predictor steps
// (2765-2786). Each function here states its math; where this file departs from a reference
// kernel (unsigned codes at 8 bits, the published AdaRound regulariser, nearest-level
// assignment by binary search) the comment says so.
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <numeric>
#include <tuple>
#include <vector>

namespace sqcpu {

namespace {

torch::Tensor f32c(const torch::Tensor& t) { return t.to(torch::kCPU, torch::kFloat32).contiguous(); }

uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// index of the nearest of the ascending levels lv[0..k) (ties go to the lower level)
inline int nearest_sorted(const float* lv, int k, float v) {
  int lo = 0, hi = k - 1;
  while (lo < hi) {  // first level >= v
    const int mid = (lo + hi) >> 1;
    if (lv[mid] < v) lo = mid + 1;
    else hi = mid;
  }
  if (lo > 0 && std::fabs(v - lv[lo - 1]) <= std::fabs(lv[lo] - v)) return lo - 1;
  return lo;
}

inline float sigmoidf(float x) { return 1.f / (1.f + std::exp(-x)); }

}  // namespace

// ---------------------------------------------------------------------------------- any4
// Lloyd iterations of 1-D k-means: assign every value to its nearest centroid, move each
// centroid to the mean of its values; an empty centroid restarts at a value drawn with a
// seeded splitmix64. Centroids are kept sorted (nearest-level search by bisection).
torch::Tensor any4_lloyd(torch::Tensor values, torch::Tensor init, int64_t n_iter, int64_t seed) {
  auto v = f32c(values).view({-1});
  auto c = f32c(init).view({-1}).clone();
  const int64_t n = v.numel(), k = c.numel();
  TORCH_CHECK(k >= 1 && k <= 65536, "1..65536 centroids");
  float* cp = c.data_ptr<float>();
  std::sort(cp, cp + k);
  if (n == 0) return c;
  const float* vp = v.data_ptr<float>();
  std::vector<double> sum(k);
  std::vector<int64_t> cnt(k);
  uint64_t rng = (uint64_t)seed * 0x2545F4914F6CDD1Dull + 1;
  for (int64_t it = 0; it < n_iter; ++it) {
    std::fill(sum.begin(), sum.end(), 0.0);
    std::fill(cnt.begin(), cnt.end(), 0);
    for (int64_t i = 0; i < n; ++i) {
      const int a = nearest_sorted(cp, (int)k, vp[i]);
      sum[a] += vp[i];
      ++cnt[a];
    }
    bool moved = false;
    for (int64_t j = 0; j < k; ++j) {
      const float nv = cnt[j] ? (float)(sum[j] / (double)cnt[j]) : vp[splitmix64(rng) % (uint64_t)n];
      moved |= nv != cp[j];
      cp[j] = nv;
    }
    std::sort(cp, cp + k);
    if (!moved) break;
  }
  return c;
}

// any4 weights: each group of `group` columns of a row is divided by its absolute maximum; one
// 16-level table per tensor is learned by Lloyd over the normalised values (started at the
// NormalFloat-4 levels); codes are the nearest level. Returns (codes uint8 [R, C], absmax float
// [R, C / group], levels float [16] ascending).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> any4_quantize(torch::Tensor w, int64_t group, int64_t n_iter,
                                                                      int64_t seed) {
  auto x = f32c(w);
  TORCH_CHECK(x.dim() == 2 && group > 0 && x.size(1) % group == 0, "w: [R, C], C a multiple of group");
  const int64_t R = x.size(0), C = x.size(1), G = C / group;
  auto scales = torch::empty({R, G}, torch::kFloat32);
  auto norm = torch::empty({R, C}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  float* sp = scales.data_ptr<float>();
  float* np_ = norm.data_ptr<float>();
  for (int64_t r = 0; r < R; ++r)
    for (int64_t g = 0; g < G; ++g) {
      float m = 0.f;
      for (int64_t j = 0; j < group; ++j) m = std::max(m, std::fabs(xp[r * C + g * group + j]));
      sp[r * G + g] = m > 0.f ? m : 1.f;  // (an all-zero group keeps scale 1, as the NF4 codec)
      const float inv = m > 0.f ? 1.f / m : 0.f;
      for (int64_t j = 0; j < group; ++j) np_[r * C + g * group + j] = xp[r * C + g * group + j] * inv;
    }
  static const float kNf4[16] = {-1.0f, -0.6961928f, -0.52507305f, -0.3949175f, -0.28444138f, -0.18477343f,
                                 -0.09105003f, 0.0f, 0.0795803f, 0.1609302f, 0.2461123f, 0.33791524f,
                                 0.44070983f, 0.562617f, 0.72295684f, 1.0f};
  auto levels = any4_lloyd(norm, torch::from_blob((void*)kNf4, {16}, torch::kFloat32).clone(), n_iter, seed);
  const float* lv = levels.data_ptr<float>();
  auto codes = torch::empty({R, C}, torch::kUInt8);
  uint8_t* cp = codes.data_ptr<uint8_t>();
  for (int64_t i = 0; i < R * C; ++i) cp[i] = (uint8_t)nearest_sorted(lv, 16, np_[i]);
  return {codes, scales, levels};
}

// ---------------------------------------------------------------------------------- QuaRot
// Column-group quantization of an (already rotated) weight: one (scale, zero) per group of
// `group` columns over all rows. Symmetric: scale = absmax / q_max, codes in [-q_max, q_max];
// asymmetric: scale = (max - min) / (2 q_max), zero = -min / scale, codes in [0, 2 q_max].
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> quarot_group_quant(torch::Tensor w, int64_t group,
                                                                           double q_max, bool symmetric) {
  auto x = f32c(w);
  TORCH_CHECK(x.dim() == 2 && group > 0 && q_max > 0, "w: [R, C], group > 0, q_max > 0");
  const int64_t R = x.size(0), C = x.size(1), G = (C + group - 1) / group;
  auto codes = torch::empty({R, C}, torch::kInt32);
  auto scales = torch::ones({G}, torch::kFloat32), zeros = torch::zeros({G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  int32_t* cp = codes.data_ptr<int32_t>();
  float *sp = scales.data_ptr<float>(), *zp = zeros.data_ptr<float>();
  const float qm = (float)q_max;
  for (int64_t g = 0; g < G; ++g) {
    const int64_t c0 = g * group, c1 = std::min(C, c0 + group);
    float mn = INFINITY, mx = -INFINITY, am = 0.f;
    for (int64_t r = 0; r < R; ++r)
      for (int64_t c = c0; c < c1; ++c) {
        const float v = xp[r * C + c];
        mn = std::min(mn, v);
        mx = std::max(mx, v);
        am = std::max(am, std::fabs(v));
      }
    if (symmetric) {
      const float s = am < 1e-9f ? 1.f : am / qm;
      sp[g] = s;
      for (int64_t r = 0; r < R; ++r)
        for (int64_t c = c0; c < c1; ++c)
          cp[r * C + c] = (int32_t)std::min(qm, std::max(-qm, std::nearbyint(xp[r * C + c] / s)));
    } else {
      const float s = std::max(mx - mn, 1e-9f) / (2.f * qm), z = -mn / s;
      sp[g] = s;
      zp[g] = z;
      for (int64_t r = 0; r < R; ++r)
        for (int64_t c = c0; c < c1; ++c)
          cp[r * C + c] = (int32_t)std::min(2.f * qm, std::max(0.f, std::nearbyint(xp[r * C + c] / s + z)));
    }
  }
  return {codes, scales, zeros};
}

torch::Tensor quarot_group_dequant(torch::Tensor codes, torch::Tensor scales, torch::Tensor zeros, int64_t group,
                                   bool symmetric) {
  auto q = codes.to(torch::kInt32).contiguous();
  auto s = f32c(scales), z = f32c(zeros);
  TORCH_CHECK(q.dim() == 2 && group > 0, "codes: [R, C]");
  const int64_t R = q.size(0), C = q.size(1);
  TORCH_CHECK(s.numel() >= (C + group - 1) / group && z.numel() == s.numel(), "scales / zeros: one per group");
  auto out = torch::empty({R, C}, torch::kFloat32);
  const int32_t* qp = q.data_ptr<int32_t>();
  const float *sp = s.data_ptr<float>(), *zp = z.data_ptr<float>();
  float* op = out.data_ptr<float>();
  for (int64_t r = 0; r < R; ++r)
    for (int64_t c = 0; c < C; ++c) {
      const int64_t g = c / group;
      op[r * C + c] = symmetric ? qp[r * C + c] * sp[g] : ((float)qp[r * C + c] - zp[g]) * sp[g];
    }
  return out;
}

// ---------------------------------------------------------------------------------- AdaRound
// One gradient step on the rounding variables V of AdaRound (Nagel et al. 2020, "Up or Down?"),
// weight-space objective: soft weight w~ = s (floor + h(V)) with the rectified sigmoid
// h(V) = clip(sigmoid(V) (zeta - gamma) + gamma, 0, 1) (zeta = 1.1, gamma = -0.1 in the paper),
// loss = 1/2 (w~ - w)^2 + lambda (1 - |2 h - 1|^beta). Returns V - lr dL/dV. (The reference's
// step uses a simplified sigmoid and regulariser; this is the published objective.)
torch::Tensor adaround_step(torch::Tensor v, torch::Tensor w, torch::Tensor w_floor, torch::Tensor scale, double lr,
                            double beta, double lambda_reg, double zeta, double gamma) {
  auto V = f32c(v).view({-1}).clone();
  auto W = f32c(w).view({-1}), F = f32c(w_floor).view({-1}), S = f32c(scale).view({-1});
  const int64_t n = V.numel();
  TORCH_CHECK(W.numel() == n && F.numel() == n && S.numel() == n, "v, w, w_floor, scale: same size");
  float* vp = V.data_ptr<float>();
  const float *wp = W.data_ptr<float>(), *fp = F.data_ptr<float>(), *sp = S.data_ptr<float>();
  const float zt = (float)zeta, gm = (float)gamma, b = (float)beta, lam = (float)lambda_reg, eta = (float)lr;
  for (int64_t i = 0; i < n; ++i) {
    const float sg = sigmoidf(vp[i]);
    const float raw = sg * (zt - gm) + gm;
    const float h = std::min(1.f, std::max(0.f, raw));
    const float dh = (raw > 0.f && raw < 1.f) ? sg * (1.f - sg) * (zt - gm) : 0.f;
    const float rec = (sp[i] * (fp[i] + h) - wp[i]) * sp[i];
    const float t = 2.f * h - 1.f;
    const float at = std::fabs(t);
    const float dreg = at > 0.f ? -b * std::pow(at, b - 1.f) * 2.f * (t > 0.f ? 1.f : -1.f) : 0.f;
    vp[i] -= eta * (rec + lam * dreg) * dh;
  }
  return V.view(v.sizes());
}

// ---------------------------------------------------------------------------------- FLUTE LUT
// Per column group g (group columns), each weight's code is its nearest entry (L1) of
// codebook[g] (any order; ties go to the lower index).
torch::Tensor flute_lut_encode(torch::Tensor w, torch::Tensor codebook, int64_t group) {
  auto x = f32c(w), cb = f32c(codebook);
  TORCH_CHECK(x.dim() == 2 && cb.dim() == 2 && group > 0 && cb.size(1) >= 1 && cb.size(1) <= 256,
              "w [R, C], codebook [G, <= 256]");
  const int64_t R = x.size(0), C = x.size(1), G = cb.size(0), K = cb.size(1);
  TORCH_CHECK(G * group >= C, "one codebook per column group");
  auto codes = torch::empty({R, C}, torch::kUInt8);
  const float *xp = x.data_ptr<float>(), *cbp = cb.data_ptr<float>();
  uint8_t* op = codes.data_ptr<uint8_t>();
  for (int64_t r = 0; r < R; ++r)
    for (int64_t c = 0; c < C; ++c) {
      const float* e = cbp + (c / group) * K;
      const float v = xp[r * C + c];
      int best = 0;
      float bd = std::fabs(v - e[0]);
      for (int64_t j = 1; j < K; ++j) {
        const float d = std::fabs(v - e[j]);
        if (d < bd) {
          bd = d;
          best = (int)j;
        }
      }
      op[r * C + c] = (uint8_t)best;
    }
  return codes;
}

torch::Tensor flute_lut_decode(torch::Tensor codes, torch::Tensor codebook, int64_t group) {
  auto q = codes.to(torch::kUInt8).contiguous();
  auto cb = f32c(codebook);
  TORCH_CHECK(q.dim() == 2 && cb.dim() == 2 && group > 0, "codes [R, C], codebook [G, K]");
  const int64_t R = q.size(0), C = q.size(1), K = cb.size(1);
  TORCH_CHECK(cb.size(0) * group >= C, "one codebook per column group");
  auto out = torch::empty({R, C}, torch::kFloat32);
  const uint8_t* qp = q.data_ptr<uint8_t>();
  const float* cbp = cb.data_ptr<float>();
  float* op = out.data_ptr<float>();
  for (int64_t r = 0; r < R; ++r)
    for (int64_t c = 0; c < C; ++c) {
      const int64_t j = qp[r * C + c];
      TORCH_CHECK(j < K, "code outside the codebook");
      op[r * C + c] = cbp[(c / group) * K + j];
    }
  return out;
}

// ---------------------------------------------------------------------------------- QMoE / PQ
// k-means (squared L2) over [N, D] rows. Start: k evenly spaced rows (seed < 0) or k rows drawn
// with a seeded splitmix64 (seed >= 0, PQ sub-codebooks); empty centroids keep their position.
// Returns (centroids [k, D], assignments int32 [N]).
std::tuple<torch::Tensor, torch::Tensor> kmeans_rows(torch::Tensor rows, int64_t k, int64_t n_iter, int64_t seed) {
  auto x = f32c(rows);
  TORCH_CHECK(x.dim() == 2 && k >= 1, "rows [N, D], k >= 1");
  const int64_t N = x.size(0), D = x.size(1);
  auto cb = torch::zeros({k, D}, torch::kFloat32);
  auto asg = torch::zeros({N}, torch::kInt32);
  if (N == 0) return {cb, asg};
  const float* xp = x.data_ptr<float>();
  float* cp = cb.data_ptr<float>();
  int32_t* ap = asg.data_ptr<int32_t>();
  uint64_t rng = (uint64_t)seed * 0x2545F4914F6CDD1Dull + 7;
  for (int64_t c = 0; c < k; ++c) {
    const int64_t src = seed < 0 ? std::min(N - 1, c * N / k) : (int64_t)(splitmix64(rng) % (uint64_t)N);
    std::copy(xp + src * D, xp + src * D + D, cp + c * D);
  }
  std::vector<double> sum(k * D);
  std::vector<int64_t> cnt(k);
  for (int64_t it = 0; it < n_iter; ++it) {
    bool changed = it == 0;
    for (int64_t i = 0; i < N; ++i) {
      int best = 0;
      float bd = INFINITY;
      for (int64_t c = 0; c < k; ++c) {
        float d = 0.f;
        for (int64_t j = 0; j < D; ++j) {
          const float t = xp[i * D + j] - cp[c * D + j];
          d += t * t;
        }
        if (d < bd) {
          bd = d;
          best = (int)c;
        }
      }
      changed |= ap[i] != best;
      ap[i] = best;
    }
    if (!changed) break;
    std::fill(sum.begin(), sum.end(), 0.0);
    std::fill(cnt.begin(), cnt.end(), 0);
    for (int64_t i = 0; i < N; ++i) {
      ++cnt[ap[i]];
      for (int64_t j = 0; j < D; ++j) sum[ap[i] * D + j] += xp[i * D + j];
    }
    for (int64_t c = 0; c < k; ++c)
      if (cnt[c])
        for (int64_t j = 0; j < D; ++j) cp[c * D + j] = (float)(sum[c * D + j] / (double)cnt[c]);
  }
  return {cb, asg};
}

// QMoE: block codebook of an expert's weights (evenly spaced start).
std::tuple<torch::Tensor, torch::Tensor> qmoe_compress(torch::Tensor blocks, int64_t k, int64_t n_iter) {
  return kmeans_rows(blocks, k, n_iter, -1);
}

// PQ cache: the centroids of one sub-space's sub-vectors [N, sub_dim] (seeded start).
torch::Tensor pq_cache_fit(torch::Tensor sub_vecs, int64_t k, int64_t n_iter, int64_t seed) {
  TORCH_CHECK(seed >= 0, "seed >= 0");
  return std::get<0>(kmeans_rows(sub_vecs, k, n_iter, seed));
}

// ---------------------------------------------------------------------------------- BitDistiller / GGUF
// Per-row groups of `group` columns, min/max asymmetric: scale = (max - min) / (2^bits - 1),
// code = round((w - min) / scale) in [0, 2^bits - 1] (unsigned, so 8-bit codes fit), zero =
// -min / scale. Returns (codes uint8 [R, C], scales [R, G], zeros [R, G]).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> bit_distiller_quant(torch::Tensor w, int64_t bits,
                                                                            int64_t group) {
  auto x = f32c(w);
  TORCH_CHECK(x.dim() == 2 && bits >= 2 && bits <= 8 && group > 0, "w [R, C], 2 <= bits <= 8");
  const int64_t R = x.size(0), C = x.size(1), G = (C + group - 1) / group;
  const float L = (float)((1 << bits) - 1);
  auto codes = torch::empty({R, C}, torch::kUInt8);
  auto scales = torch::empty({R, G}, torch::kFloat32), zeros = torch::empty({R, G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  uint8_t* cp = codes.data_ptr<uint8_t>();
  float *sp = scales.data_ptr<float>(), *zp = zeros.data_ptr<float>();
  for (int64_t r = 0; r < R; ++r)
    for (int64_t g = 0; g < G; ++g) {
      const int64_t c0 = g * group, c1 = std::min(C, c0 + group);
      float mn = INFINITY, mx = -INFINITY;
      for (int64_t c = c0; c < c1; ++c) {
        mn = std::min(mn, xp[r * C + c]);
        mx = std::max(mx, xp[r * C + c]);
      }
      const float range = std::max(mx - mn, 1e-8f), s = range / L;
      sp[r * G + g] = s;
      zp[r * G + g] = -mn / s;
      for (int64_t c = c0; c < c1; ++c)
        cp[r * C + c] = (uint8_t)std::min(L, std::max(0.f, std::nearbyint((xp[r * C + c] - mn) / range * L)));
    }
  return {codes, scales, zeros};
}

// BitDistiller-style teacher-guided grid refinement: per row group, the importance of each
// weight is p = softmax(teacher / temperature) over the group (the teacher's soft targets);
// among n_grid grids shrinking [min, max] about its midpoint by factors 1 .. 1/2, keep the one
// with the least p-weighted squared reconstruction error. Returns (scales [R, G], zeros [R, G])
// for codes round(w / scale + zero) in [0, 2^bits - 1]. (The reference's refinement is a
// different heuristic over the same inputs.)
std::tuple<torch::Tensor, torch::Tensor> bit_distiller_refine(torch::Tensor w, torch::Tensor teacher, int64_t bits,
                                                              int64_t group, int64_t n_grid, double temperature) {
  auto x = f32c(w), t = f32c(teacher);
  TORCH_CHECK(x.dim() == 2 && t.sizes() == x.sizes() && bits >= 2 && bits <= 8 && group > 0 && n_grid >= 1 &&
                  temperature > 0,
              "w / teacher [R, C], 2 <= bits <= 8, group > 0, n_grid >= 1, temperature > 0");
  const int64_t R = x.size(0), C = x.size(1), G = (C + group - 1) / group;
  const float L = (float)((1 << bits) - 1);
  auto scales = torch::empty({R, G}, torch::kFloat32), zeros = torch::empty({R, G}, torch::kFloat32);
  float *sp = scales.data_ptr<float>(), *zp = zeros.data_ptr<float>();
  const float *xp = x.data_ptr<float>(), *tp = t.data_ptr<float>();
  std::vector<float> p(group);
  for (int64_t r = 0; r < R; ++r)
    for (int64_t g = 0; g < G; ++g) {
      const int64_t c0 = g * group, c1 = std::min(C, c0 + group), n = c1 - c0;
      float mn = INFINITY, mx = -INFINITY, tm = -INFINITY;
      for (int64_t c = c0; c < c1; ++c) {
        mn = std::min(mn, xp[r * C + c]);
        mx = std::max(mx, xp[r * C + c]);
        tm = std::max(tm, tp[r * C + c]);
      }
      double z = 0;
      for (int64_t i = 0; i < n; ++i) z += (p[i] = std::exp((tp[r * C + c0 + i] - tm) / (float)temperature));
      const float mid = 0.5f * (mn + mx), half = 0.5f * (mx - mn);
      float best_e = INFINITY, best_s = 1.f, best_z = 0.f;
      for (int64_t k = 0; k < n_grid; ++k) {
        const float f = n_grid > 1 ? 1.f - 0.5f * (float)k / (float)(n_grid - 1) : 1.f;
        const float lo = mid - half * f, s = std::max(2.f * half * f, 1e-8f) / L, zz = -lo / s;
        double e = 0;
        for (int64_t i = 0; i < n; ++i) {
          const float v = xp[r * C + c0 + i];
          const float q = std::min(L, std::max(0.f, std::nearbyint(v / s + zz)));
          const float d = (q - zz) * s - v;
          e += p[i] / z * d * d;
        }
        if (e < best_e) {
          best_e = (float)e;
          best_s = s;
          best_z = zz;
        }
      }
      sp[r * G + g] = best_s;
      zp[r * G + g] = best_z;
    }
  return {scales, zeros};
}

// GGUF-style blocks: the same per-block min / scale codes, plus one super-block scale per 8
// consecutive blocks (row-major block order) = the mean of their scales. Returns (codes uint8,
// scales [R * G], mins [R * G], super_scales [ceil(R G / 8)]).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor> gguf_mixed_quant(torch::Tensor w,
                                                                                        int64_t bits,
                                                                                        int64_t group) {
  auto [codes, scales, zeros] = bit_distiller_quant(w, bits, group);
  auto s = scales.view({-1}).contiguous();
  auto mins = (-zeros * scales).view({-1}).contiguous();
  const int64_t nb = s.numel(), ns = (nb + 7) / 8;
  auto sup = torch::empty({ns}, torch::kFloat32);
  const float* sp = s.data_ptr<float>();
  float* up = sup.data_ptr<float>();
  for (int64_t i = 0; i < ns; ++i) {
    double a = 0.0;
    const int64_t b1 = std::min(nb, i * 8 + 8);
    for (int64_t j = i * 8; j < b1; ++j) a += sp[j];
    up[i] = (float)(a / (double)(b1 - i * 8));
  }
  return {codes, s, mins, sup};
}

// ---------------------------------------------------------------------------------- predictors
// GRU cell from pre-multiplied gates (PyTorch gate order r, z, n):
// r = sigmoid(gx_r + gh_r), z = sigmoid(gx_z + gh_z), n = tanh(gx_n + r gh_n), h' = (1 - z) n + z h.
torch::Tensor gru_step(torch::Tensor gates_x, torch::Tensor gates_h, torch::Tensor h) {
  auto gx = f32c(gates_x).view({-1}), gh = f32c(gates_h).view({-1}), hv = f32c(h).view({-1});
  const int64_t H = hv.numel();
  TORCH_CHECK(gx.numel() == 3 * H && gh.numel() == 3 * H, "gates: [3 H]");
  auto out = torch::empty({H}, torch::kFloat32);
  const float *x = gx.data_ptr<float>(), *g = gh.data_ptr<float>(), *hp = hv.data_ptr<float>();
  float* op = out.data_ptr<float>();
  for (int64_t i = 0; i < H; ++i) {
    const float r = sigmoidf(x[i] + g[i]);
    const float z = sigmoidf(x[H + i] + g[H + i]);
    const float nn = std::tanh(x[2 * H + i] + r * g[2 * H + i]);
    op[i] = (1.f - z) * nn + z * hp[i];
  }
  return out;
}

// [Ta, D] x [Tb, D] -> [Ta, Tb] cosine similarities (a zero row gives 0)
torch::Tensor batched_cosine_similarity(torch::Tensor a, torch::Tensor b) {
  auto x = f32c(a), y = f32c(b);
  TORCH_CHECK(x.dim() == 2 && y.dim() == 2 && x.size(1) == y.size(1), "a [Ta, D], b [Tb, D]");
  const int64_t Ta = x.size(0), Tb = y.size(0), D = x.size(1);
  const float *xp = x.data_ptr<float>(), *yp = y.data_ptr<float>();
  std::vector<double> ny(Tb);
  for (int64_t j = 0; j < Tb; ++j) {
    double s = 0;
    for (int64_t d = 0; d < D; ++d) s += (double)yp[j * D + d] * yp[j * D + d];
    ny[j] = std::sqrt(s);
  }
  auto out = torch::empty({Ta, Tb}, torch::kFloat32);
  float* op = out.data_ptr<float>();
  for (int64_t i = 0; i < Ta; ++i) {
    double nx = 0;
    for (int64_t d = 0; d < D; ++d) nx += (double)xp[i * D + d] * xp[i * D + d];
    nx = std::sqrt(nx);
    for (int64_t j = 0; j < Tb; ++j) {
      double dot = 0;
      for (int64_t d = 0; d < D; ++d) dot += (double)xp[i * D + d] * yp[j * D + d];
      const double den = nx * ny[j];
      op[i * Tb + j] = den > 0 ? (float)(dot / den) : 0.f;
    }
  }
  return out;
}

// logistic regression: y_hat = sigmoid(w . x), error = y - y_hat
std::tuple<double, double> logistic_step(torch::Tensor w, torch::Tensor x, double y) {
  auto wv = f32c(w).view({-1}), xv = f32c(x).view({-1});
  TORCH_CHECK(wv.numel() == xv.numel(), "w and x: same length");
  double z = 0;
  for (int64_t i = 0; i < wv.numel(); ++i) z += (double)wv.data_ptr<float>()[i] * xv.data_ptr<float>()[i];
  const double yh = 1.0 / (1.0 + std::exp(-z));
  return {yh, y - yh};
}

// w + lr * error * x (the logistic log-likelihood gradient step)
torch::Tensor sgd_weight_update(torch::Tensor w, torch::Tensor x, double error, double lr) {
  auto wv = f32c(w).view({-1}).clone(), xv = f32c(x).view({-1});
  TORCH_CHECK(wv.numel() == xv.numel(), "w and x: same length");
  float* wp = wv.data_ptr<float>();
  const float* xp = xv.data_ptr<float>();
  for (int64_t i = 0; i < wv.numel(); ++i) wp[i] += (float)(lr * error) * xp[i];
  return wv;
}

void register_research(pybind11::module& c) {
  c.def("any4_lloyd", &any4_lloyd, pybind11::arg("values"), pybind11::arg("init"), pybind11::arg("n_iter") = 100,
        pybind11::arg("seed") = 0);
  c.def("any4_quantize", &any4_quantize, pybind11::arg("w"), pybind11::arg("group"), pybind11::arg("n_iter") = 30,
        pybind11::arg("seed") = 0);
  c.def("quarot_group_quant", &quarot_group_quant);
  c.def("quarot_group_dequant", &quarot_group_dequant);
  c.def("adaround_step", &adaround_step, pybind11::arg("v"), pybind11::arg("w"), pybind11::arg("w_floor"),
        pybind11::arg("scale"), pybind11::arg("lr"), pybind11::arg("beta"), pybind11::arg("lambda_reg"),
        pybind11::arg("zeta") = 1.1, pybind11::arg("gamma") = -0.1);
  c.def("flute_lut_encode", &flute_lut_encode);
  c.def("flute_lut_decode", &flute_lut_decode);
  c.def("qmoe_compress", &qmoe_compress);
  c.def("pq_cache_fit", &pq_cache_fit, pybind11::arg("sub_vecs"), pybind11::arg("k"), pybind11::arg("n_iter") = 20,
        pybind11::arg("seed") = 0);
  c.def("bit_distiller_refine", &bit_distiller_refine, pybind11::arg("w"), pybind11::arg("teacher"),
        pybind11::arg("bits"), pybind11::arg("group"), pybind11::arg("n_grid") = 16,
        pybind11::arg("temperature") = 1.0);
  c.def("bit_distiller_quant", &bit_distiller_quant);
  c.def("gguf_mixed_quant", &gguf_mixed_quant);
  c.def("gru_step", &gru_step);
  c.def("batched_cosine_similarity", &batched_cosine_similarity);
  c.def("logistic_step", &logistic_step);
  c.def("sgd_weight_update", &sgd_weight_update);
}

}  // namespace sqcpu
