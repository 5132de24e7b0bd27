// recurrent.cpp — host C++ kernels for linear-recurrence sequence mixers and sparse GEMVs
// (float32, CPU): the Mamba-2 state-space scan, the Hawk real-gated linear recurrence, the
// DeltaNet delta-rule scan, a ternary-weight GEMV and an activation-sparse GEMV.
//
// The reference ships these as Rust functions of squish_quant_rs with no model that uses them
// (src/lib.rs:3331 mamba2_ssm_scan, 3378 mamba2_ssm_decode, 3525 hawk_rglr_scan, 3889 delta_net_scan, 3646
// ternary_gemv, 3158 sparse_act_gemv); they are kept here as library kernels with the same
// math, stated per function.
#include <torch/extension.h>

#include <cmath>
#include <cstdint>
#include <tuple>
#include <vector>

namespace sqcpu {

namespace {
torch::Tensor f32(const torch::Tensor& t) { return t.to(torch::kCPU, torch::kFloat32).contiguous(); }
inline float softplus(float x) { return x > 20.f ? x : std::log1p(std::exp(x)); }
}  // namespace

// Mamba-2 scan of one head: h_{t+1} = exp(a_t) h_t + B_t x_t, y_t = C_t . h_{t+1}.
// a [T] (log decay, <= 0 for stability), B / C [T, N], x [T], h0 [N] -> (y [T], h_T [N]).
std::tuple<torch::Tensor, torch::Tensor> mamba2_scan(torch::Tensor a, torch::Tensor b, torch::Tensor c,
                                                     torch::Tensor x, torch::Tensor h0) {
  auto A = f32(a).view({-1}), B = f32(b), Cm = f32(c), X = f32(x).view({-1});
  auto h = f32(h0).view({-1}).clone();
  const int64_t T = A.numel(), N = h.numel();
  TORCH_CHECK(B.dim() == 2 && B.size(0) == T && B.size(1) == N && Cm.sizes() == B.sizes() && X.numel() == T,
              "a [T], B / C [T, N], x [T], h0 [N]");
  auto y = torch::empty({T}, torch::kFloat32);
  float* hp = h.data_ptr<float>();
  const float *ap = A.data_ptr<float>(), *bp = B.data_ptr<float>(), *cp = Cm.data_ptr<float>(),
              *xp = X.data_ptr<float>();
  float* yp = y.data_ptr<float>();
  for (int64_t t = 0; t < T; ++t) {
    const float da = std::exp(ap[t]);
    double acc = 0;
    for (int64_t n = 0; n < N; ++n) {
      hp[n] = da * hp[n] + bp[t * N + n] * xp[t];
      acc += (double)cp[t * N + n] * hp[n];
    }
    yp[t] = (float)acc;
  }
  return {y, h};
}

// One Mamba-2 decode step (the scan at T = 1): h' = exp(a) h + B x, y = C . h'.
// a, x scalars; B / C / h [N] -> (y, h').
std::tuple<double, torch::Tensor> mamba2_step(double a, torch::Tensor b, torch::Tensor c, double x, torch::Tensor h) {
  auto B = f32(b).view({-1}), Cv = f32(c).view({-1});
  auto hn = f32(h).view({-1}).clone();
  const int64_t N = hn.numel();
  TORCH_CHECK(B.numel() == N && Cv.numel() == N, "B, C and h: [N]");
  float* hp = hn.data_ptr<float>();
  const float *bp = B.data_ptr<float>(), *cp = Cv.data_ptr<float>();
  const float da = std::exp((float)a);
  double y = 0;
  for (int64_t n = 0; n < N; ++n) {
    hp[n] = da * hp[n] + bp[n] * (float)x;
    y += (double)cp[n] * hp[n];
  }
  return {y, hn};
}

// Hawk real-gated linear recurrence, elementwise over the state:
// f_t = exp(-exp(lambda_log) softplus(dt_t)), h_t = f_t h_{t-1} + sqrt(1 - f_t^2) x_t.
// x / dt [T, N], lambda_log [N], h0 [N] -> (h [T, N], h_T [N]).
std::tuple<torch::Tensor, torch::Tensor> hawk_scan(torch::Tensor x, torch::Tensor dt, torch::Tensor lambda_log,
                                                   torch::Tensor h0) {
  auto X = f32(x), DT = f32(dt), L = f32(lambda_log).view({-1});
  auto h = f32(h0).view({-1}).clone();
  TORCH_CHECK(X.dim() == 2 && DT.sizes() == X.sizes() && L.numel() == X.size(1) && h.numel() == X.size(1),
              "x / dt [T, N], lambda_log [N], h0 [N]");
  const int64_t T = X.size(0), N = X.size(1);
  auto out = torch::empty({T, N}, torch::kFloat32);
  float *hp = h.data_ptr<float>(), *op = out.data_ptr<float>();
  const float *xp = X.data_ptr<float>(), *dp = DT.data_ptr<float>(), *lp = L.data_ptr<float>();
  for (int64_t t = 0; t < T; ++t)
    for (int64_t n = 0; n < N; ++n) {
      const float f = std::exp(-std::exp(lp[n]) * softplus(dp[t * N + n]));
      hp[n] = f * hp[n] + std::sqrt(std::max(0.f, 1.f - f * f)) * xp[t * N + n];
      op[t * N + n] = hp[n];
    }
  return {out, h};
}

// DeltaNet delta rule per head with state S [D, D] (from zero): k^ = k / |k|,
// S <- S + beta (v - S k^) k^T, y_t = S q_t. q / k / v [T, H, D], beta [T, H] -> y [T, H, D].
torch::Tensor delta_net_scan(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor beta) {
  auto Q = f32(q), K = f32(k), V = f32(v), Bt = f32(beta);
  TORCH_CHECK(Q.dim() == 3 && K.sizes() == Q.sizes() && V.sizes() == Q.sizes() && Bt.dim() == 2 &&
                  Bt.size(0) == Q.size(0) && Bt.size(1) == Q.size(1),
              "q / k / v [T, H, D], beta [T, H]");
  const int64_t T = Q.size(0), H = Q.size(1), D = Q.size(2);
  auto y = torch::zeros({T, H, D}, torch::kFloat32);
  float* yp = y.data_ptr<float>();
  const float *qp = Q.data_ptr<float>(), *kp = K.data_ptr<float>(), *vp = V.data_ptr<float>(),
              *bp = Bt.data_ptr<float>();
  std::vector<float> S(D * D), kh(D), u(D);
  for (int64_t h = 0; h < H; ++h) {
    std::fill(S.begin(), S.end(), 0.f);
    for (int64_t t = 0; t < T; ++t) {
      const float* kr = kp + (t * H + h) * D;
      double nn = 0;
      for (int64_t j = 0; j < D; ++j) nn += (double)kr[j] * kr[j];
      const float inv = nn > 0 ? (float)(1.0 / std::sqrt(nn)) : 0.f;
      for (int64_t j = 0; j < D; ++j) kh[j] = kr[j] * inv;
      const float* vr = vp + (t * H + h) * D;
      const float be = bp[t * H + h];
      for (int64_t i = 0; i < D; ++i) {  // u = beta (v - S k^)
        float sk = 0.f;
        for (int64_t j = 0; j < D; ++j) sk += S[i * D + j] * kh[j];
        u[i] = be * (vr[i] - sk);
      }
      for (int64_t i = 0; i < D; ++i)
        for (int64_t j = 0; j < D; ++j) S[i * D + j] += u[i] * kh[j];
      const float* qr = qp + (t * H + h) * D;
      float* yr = yp + (t * H + h) * D;
      for (int64_t i = 0; i < D; ++i) {
        float s = 0.f;
        for (int64_t j = 0; j < D; ++j) s += S[i * D + j] * qr[j];
        yr[i] = s;
      }
    }
  }
  return y;
}

// Ternary GEMV: y = scale * W x with W int8 in {-1, 0, +1} [O, I] (adds and subtractions only).
torch::Tensor ternary_gemv(torch::Tensor w, torch::Tensor x, double scale) {
  auto W = w.to(torch::kCPU, torch::kInt8).contiguous();
  auto X = f32(x).view({-1});
  TORCH_CHECK(W.dim() == 2 && W.size(1) == X.numel(), "w [O, I] int8, x [I]");
  const int64_t O = W.size(0), I = W.size(1);
  auto y = torch::empty({O}, torch::kFloat32);
  const int8_t* wp = W.data_ptr<int8_t>();
  const float* xp = X.data_ptr<float>();
  float* yp = y.data_ptr<float>();
  for (int64_t o = 0; o < O; ++o) {
    float acc = 0.f;
    for (int64_t i = 0; i < I; ++i) {
      const int8_t t = wp[o * I + i];
      TORCH_CHECK(t >= -1 && t <= 1, "ternary weights are -1, 0 or +1");
      if (t > 0) acc += xp[i];
      else if (t < 0) acc -= xp[i];
    }
    yp[o] = (float)scale * acc;
  }
  return y;
}

// Activation-sparse GEMV: y = W x over the inputs with |x_i| > threshold only.
torch::Tensor sparse_act_gemv(torch::Tensor w, torch::Tensor x, double threshold) {
  auto W = f32(w), X = f32(x).view({-1});
  TORCH_CHECK(W.dim() == 2 && W.size(1) == X.numel(), "w [O, I], x [I]");
  const int64_t O = W.size(0), I = W.size(1);
  std::vector<int64_t> nz;
  const float* xp = X.data_ptr<float>();
  for (int64_t i = 0; i < I; ++i)
    if (std::fabs(xp[i]) > threshold) nz.push_back(i);
  auto y = torch::empty({O}, torch::kFloat32);
  const float* wp = W.data_ptr<float>();
  float* yp = y.data_ptr<float>();
  for (int64_t o = 0; o < O; ++o) {
    double acc = 0;
    for (int64_t i : nz) acc += (double)wp[o * I + i] * xp[i];
    yp[o] = (float)acc;
  }
  return y;
}

void register_recurrent(pybind11::module& c) {
  c.def("mamba2_scan", &mamba2_scan);
  c.def("mamba2_step", &mamba2_step);
  c.def("hawk_scan", &hawk_scan);
  c.def("delta_net_scan", &delta_net_scan);
  c.def("ternary_gemv", &ternary_gemv, pybind11::arg("w"), pybind11::arg("x"), pybind11::arg("scale") = 1.0);
  c.def("sparse_act_gemv", &sparse_act_gemv, pybind11::arg("w"), pybind11::arg("x"), pybind11::arg("threshold") = 0.0);
}

}  // namespace sqcpu
