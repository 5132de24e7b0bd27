// cpu_ref.cpp — C++ CPU library restating the reference's native quantization kernels
// (squish_quant_rs/src/lib.rs, Rust + Rayon) with ATen's parallel_for. These serve three roles:
// the convert-time quantizers of `squish compress` on hosts without a GPU, the CPU
// oracle for the CUDA kernels' numerics tests, and the timed CPU baseline.
//
// Semantics follow the Rust source line by line where the format is defined by it:
//   quantize_int8_f32 (lib.rs:56), quantize_int8_grouped (121), quantize_int4_grouped (259),
//   quantize_int4_asymmetric_grouped (402) / dequantize (490), NF4 (742-890),
//   pack_int3_grouped_f32 (1125) / unpack_int3_grouped (1200), quantize_int2_grouped_f32 (1440)
//   / dequantize (1510), quantized_matmul_int4 (5511).
// Rust's f32::round rounds half away from zero; std::round does the same.
#include <torch/extension.h>
#include <ATen/Parallel.h>
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <vector>

#include "cpu_ref.h"

namespace sqcpu {

namespace {

void check_cpu_f32_2d(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(!t.is_cuda(), name, " must be a CPU tensor");
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.scalar_type() == torch::kFloat32, name, " must be float32");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

template <class F>
void prange(int64_t n, F&& f) {
  at::parallel_for(0, n, 1, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) f(i);
  });
}

inline float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

const float kNF4[16] = {-1.0f,
                        -0.6961928009986877f,
                        -0.5250730514526367f,
                        -0.39491748809814453f,
                        -0.28444138169288635f,
                        -0.18477343022823334f,
                        -0.09105003625154495f,
                        0.0f,
                        0.07958029955625534f,
                        0.16093020141124725f,
                        0.24611230194568634f,
                        0.33791524171829224f,
                        0.44070982933044434f,
                        0.5626170039176941f,
                        0.7229568362236023f,
                        1.0f};

// ---------------------------------------------------------------- INT8 symmetric
std::vector<torch::Tensor> quantize_int8(torch::Tensor x, int64_t group) {
  check_cpu_f32_2d(x, "x");
  const int64_t N = x.size(0), D = x.size(1);
  const int64_t g = group <= 0 ? D : group;
  TORCH_CHECK(D % g == 0, "group must divide columns");
  const int64_t G = D / g;
  auto q = torch::empty({N, D}, torch::kInt8);
  auto s = torch::empty({N, G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  int8_t* qp = q.data_ptr<int8_t>();
  float* sp = s.data_ptr<float>();
  prange(N, [&](int64_t r) {
    for (int64_t j = 0; j < G; ++j) {
      const float* row = xp + r * D + j * g;
      float am = 0.f;
      for (int64_t i = 0; i < g; ++i) am = std::max(am, std::fabs(row[i]));
      const float sc = am == 0.f ? 1.f : am / 127.f;
      sp[r * G + j] = sc;
      const float inv = 1.f / sc;
      for (int64_t i = 0; i < g; ++i) qp[r * D + j * g + i] = (int8_t)clampf(std::round(row[i] * inv), -127.f, 127.f);
    }
  });
  return {q, s};
}

torch::Tensor dequantize_int8(torch::Tensor q, torch::Tensor s) {
  const int64_t N = q.size(0), D = q.size(1), G = s.size(1), g = D / G;
  auto out = torch::empty({N, D}, torch::kFloat32);
  const int8_t* qp = q.contiguous().data_ptr<int8_t>();
  const float* sp = s.contiguous().data_ptr<float>();
  float* op = out.data_ptr<float>();
  prange(N, [&](int64_t r) {for (int64_t c = 0; c < D; ++c) op[r * D + c] = (float)qp[r * D + c] * sp[r * G + c / g];});
  return out;
}

// ---------------------------------------------------------------- INT4 asymmetric (primary weight format)
std::vector<torch::Tensor> quantize_int4_asym(torch::Tensor x, int64_t group) {
  check_cpu_f32_2d(x, "x");
  const int64_t N = x.size(0), D = x.size(1);
  TORCH_CHECK(D % group == 0 && D % 2 == 0, "columns must be even and divisible by group");
  const int64_t G = D / group;
  auto packed = torch::empty({N, D / 2}, torch::kUInt8);
  auto scales = torch::empty({N, G}, torch::kFloat32);
  auto offsets = torch::empty({N, G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  uint8_t* pp = packed.data_ptr<uint8_t>();
  float* sp = scales.data_ptr<float>();
  float* op = offsets.data_ptr<float>();
  prange(N, [&](int64_t r) {
    const float* row = xp + r * D;
    for (int64_t g = 0; g < G; ++g) {
      float mn = INFINITY, mx = -INFINITY;
      for (int64_t i = g * group; i < (g + 1) * group; ++i) {
        mn = std::min(mn, row[i]);
        mx = std::max(mx, row[i]);
      }
      sp[r * G + g] = (mx == mn) ? 1.f : (mx - mn) / 15.f;
      op[r * G + g] = mn;
    }
    for (int64_t i = 0; i < D / 2; ++i) {
      const int64_t j0 = 2 * i, j1 = j0 + 1;
      const int64_t g0 = j0 / group, g1 = j1 / group;
      const uint8_t q0 = (uint8_t)clampf(std::round((row[j0] - op[r * G + g0]) / sp[r * G + g0]), 0.f, 15.f);
      const uint8_t q1 = (uint8_t)clampf(std::round((row[j1] - op[r * G + g1]) / sp[r * G + g1]), 0.f, 15.f);
      pp[r * (D / 2) + i] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
    }
  });
  return {packed, scales, offsets};
}

// Per-group MSE clip search (8 candidates beta in [0, 0.1]) then the plain quantizer,
// as squish/quant/quantizer.py:500-605 does in numpy ahead of the Rust call.
std::vector<torch::Tensor> quantize_int4_asym_mse(torch::Tensor x, int64_t group, int64_t n_clip) {
  check_cpu_f32_2d(x, "x");
  const int64_t N = x.size(0), D = x.size(1);
  TORCH_CHECK(D % group == 0, "group must divide columns");
  if (N == 1) return quantize_int4_asym(x, group);
  auto clipped = x.clone();
  float* cp = clipped.data_ptr<float>();
  const int64_t G = N * (D / group);
  std::vector<float> betas(n_clip);
  for (int64_t i = 0; i < n_clip; ++i) betas[i] = n_clip == 1 ? 0.f : 0.10f * (float)i / (float)(n_clip - 1);
  prange(G, [&](int64_t gi) {
    float* grp = cp + gi * group;
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t i = 0; i < group; ++i) {
      mn = std::min(mn, grp[i]);
      mx = std::max(mx, grp[i]);
    }
    const float rng = mx - mn;
    float best = INFINITY, blo = mn, bhi = mx;
    for (float beta : betas) {
      const float lo = mn + beta * rng, hi = mx - beta * rng;
      if (lo >= hi) continue;
      const float sc = (hi - lo) > 0 ? (hi - lo) / 15.f : 1.f;
      double mse = 0.0;
      for (int64_t i = 0; i < group; ++i) {
        const float v = clampf(grp[i], lo, hi);
        const float q = clampf(std::nearbyint((v - lo) / sc), 0.f, 15.f);
        const float d = grp[i] - (lo + q * sc);
        mse += (double)d * d;
      }
      mse /= (double)group;
      if (mse < best) {
        best = (float)mse;
        blo = lo;
        bhi = hi;
      }
    }
    for (int64_t i = 0; i < group; ++i) grp[i] = clampf(grp[i], blo, bhi);
  });
  return quantize_int4_asym(clipped, group);
}

torch::Tensor dequantize_int4_asym(torch::Tensor packed, torch::Tensor scales, torch::Tensor offsets, int64_t group) {
  const int64_t N = packed.size(0), D = packed.size(1) * 2, G = scales.size(1);
  auto out = torch::empty({N, D}, torch::kFloat32);
  const uint8_t* pp = packed.contiguous().data_ptr<uint8_t>();
  const float* sp = scales.contiguous().data_ptr<float>();
  const float* op = offsets.contiguous().data_ptr<float>();
  float* o = out.data_ptr<float>();
  prange(N, [&](int64_t r) {for (int64_t c = 0; c < D; ++c) {
      const uint8_t b = pp[r * (D / 2) + c / 2];
      const float q = (float)((c & 1) ? (b >> 4) : (b & 0xF));
      const int64_t g = c / group;
      o[r * D + c] = op[r * G + g] + q * sp[r * G + g];
    }});
  return out;
}

// out[b, i] = sum_j x[b, j] * (offset[i, g(j)] + q[i, j] * scale[i, g(j)])  (fp32 accumulation)
torch::Tensor quantized_matmul_int4(torch::Tensor packed, torch::Tensor scales, torch::Tensor offsets, torch::Tensor x,
                                    int64_t group) {
  check_cpu_f32_2d(x, "x");
  const int64_t O = packed.size(0), K = packed.size(1) * 2, B = x.size(0), G = scales.size(1);
  TORCH_CHECK(x.size(1) == K, "x.size(1) must equal packed.size(1)*2");
  auto out = torch::empty({B, O}, torch::kFloat32);
  const uint8_t* pp = packed.contiguous().data_ptr<uint8_t>();
  const float* sp = scales.contiguous().data_ptr<float>();
  const float* op = offsets.contiguous().data_ptr<float>();
  const float* xp = x.data_ptr<float>();
  float* o = out.data_ptr<float>();
  at::parallel_for(0, O, 1, [&](int64_t i0, int64_t i1) {
    std::vector<float> wrow(K);
    for (int64_t i = i0; i < i1; ++i) {
      for (int64_t c = 0; c < K; ++c) {
        const uint8_t b = pp[i * (K / 2) + c / 2];
        const float q = (float)((c & 1) ? (b >> 4) : (b & 0xF));
        wrow[c] = op[i * G + c / group] + q * sp[i * G + c / group];
      }
      for (int64_t bb = 0; bb < B; ++bb) {
        const float* xr = xp + bb * K;
        float acc = 0.f;
        for (int64_t c = 0; c < K; ++c) acc += xr[c] * wrow[c];
        o[bb * O + i] = acc;
      }
    }
  });
  return out;
}

// ---------------------------------------------------------------- INT4 symmetric legacy (__q4/__s4)
std::vector<torch::Tensor> quantize_int4_sym(torch::Tensor x, int64_t group) {
  check_cpu_f32_2d(x, "x");
  const int64_t N = x.size(0), D = x.size(1), G = D / group;
  auto packed = torch::empty({N, D / 2}, torch::kUInt8);
  auto scales = torch::empty({N, G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  uint8_t* pp = packed.data_ptr<uint8_t>();
  float* sp = scales.data_ptr<float>();
  prange(N, [&](int64_t r) {
    for (int64_t g = 0; g < G; ++g) {
      float am = 0.f;
      for (int64_t i = g * group; i < (g + 1) * group; ++i) am = std::max(am, std::fabs(xp[r * D + i]));
      sp[r * G + g] = am == 0.f ? 1.f : am / 7.f;
    }
    for (int64_t i = 0; i < D / 2; ++i) {
      uint8_t qq[2];
      for (int k = 0; k < 2; ++k) {
        const int64_t j = 2 * i + k;
        const float q = clampf(std::round(xp[r * D + j] / sp[r * G + j / group]), -7.f, 7.f);
        qq[k] = (uint8_t)((int)q + 7);
      }
      pp[r * (D / 2) + i] = (uint8_t)((qq[0] & 0xF) | ((qq[1] & 0xF) << 4));
    }
  });
  return {packed, scales};
}

torch::Tensor dequantize_int4_sym(torch::Tensor packed, torch::Tensor scales, int64_t group) {
  const int64_t N = packed.size(0), D = packed.size(1) * 2, G = scales.size(1);
  auto out = torch::empty({N, D}, torch::kFloat32);
  const uint8_t* pp = packed.contiguous().data_ptr<uint8_t>();
  const float* sp = scales.contiguous().data_ptr<float>();
  float* o = out.data_ptr<float>();
  prange(N, [&](int64_t r) {for (int64_t c = 0; c < D; ++c) {
      const uint8_t b = pp[r * (D / 2) + c / 2];
      const int q = (int)((c & 1) ? (b >> 4) : (b & 0xF)) - 7;
      o[r * D + c] = (float)q * sp[r * G + c / group];
    }});
  return out;
}

// ---------------------------------------------------------------- NF4
std::vector<torch::Tensor> quantize_nf4(torch::Tensor x, int64_t group) {
  check_cpu_f32_2d(x, "x");
  const int64_t N = x.size(0), D = x.size(1), G = D / group;
  auto packed = torch::empty({N, D / 2}, torch::kUInt8);
  auto scales = torch::empty({N, G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  uint8_t* pp = packed.data_ptr<uint8_t>();
  float* sp = scales.data_ptr<float>();
  prange(N, [&](int64_t r) {
    for (int64_t g = 0; g < G; ++g) {
      float am = 0.f;
      for (int64_t i = g * group; i < (g + 1) * group; ++i) am = std::max(am, std::fabs(xp[r * D + i]));
      sp[r * G + g] = am == 0.f ? 1.f : am;
    }
    for (int64_t i = 0; i < D / 2; ++i) {
      uint8_t qq[2];
      for (int k = 0; k < 2; ++k) {
        const int64_t j = 2 * i + k;
        const float v = xp[r * D + j] / sp[r * G + j / group];
        int best = 0;
        float bd = INFINITY;
        for (int l = 0; l < 16; ++l) {
          const float d = std::fabs(v - kNF4[l]);
          if (d < bd) {
            bd = d;
            best = l;
          }
        }
        qq[k] = (uint8_t)best;
      }
      pp[r * (D / 2) + i] = (uint8_t)(qq[0] | (qq[1] << 4));
    }
  });
  return {packed, scales};
}

torch::Tensor dequantize_nf4(torch::Tensor packed, torch::Tensor scales, int64_t group) {
  const int64_t N = packed.size(0), D = packed.size(1) * 2, G = scales.size(1);
  auto out = torch::empty({N, D}, torch::kFloat32);
  const uint8_t* pp = packed.contiguous().data_ptr<uint8_t>();
  const float* sp = scales.contiguous().data_ptr<float>();
  float* o = out.data_ptr<float>();
  prange(N, [&](int64_t r) {for (int64_t c = 0; c < D; ++c) {
      const uint8_t b = pp[r * (D / 2) + c / 2];
      o[r * D + c] = kNF4[(c & 1) ? (b >> 4) : (b & 0xF)] * sp[r * G + c / group];
    }});
  return out;
}

// ---------------------------------------------------------------- INT3 symmetric, 8 values per 3 bytes
std::vector<torch::Tensor> pack_int3(torch::Tensor x, int64_t group) {
  check_cpu_f32_2d(x, "x");
  const int64_t N = x.size(0), D = x.size(1), G = D / group;
  TORCH_CHECK(D % group == 0, "group must divide columns");
  const int64_t padded = (D + 7) / 8 * 8, NP = padded * 3 / 8;
  auto packed = torch::zeros({N, NP}, torch::kUInt8);
  auto scales = torch::empty({N, G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  uint8_t* pp = packed.data_ptr<uint8_t>();
  float* sp = scales.data_ptr<float>();
  prange(N, [&](int64_t r) {
    for (int64_t g = 0; g < G; ++g) {
      float am = 0.f;
      for (int64_t i = g * group; i < (g + 1) * group; ++i) am = std::max(am, std::fabs(xp[r * D + i]));
      sp[r * G + g] = am == 0.f ? 1.f : am / 3.f;
    }
    for (int64_t ch = 0; ch < (D + 7) / 8; ++ch) {
      uint32_t bits = 0;
      for (int b = 0; b < 8; ++b) {
        const int64_t j = ch * 8 + b;
        uint32_t v = 0;
        if (j < D) v = (uint32_t)((int)clampf(std::round(xp[r * D + j] / sp[r * G + j / group]), -3.f, 3.f) & 7);
        bits |= v << (3 * b);
      }
      for (int k = 0; k < 3; ++k) pp[r * NP + ch * 3 + k] = (uint8_t)((bits >> (8 * k)) & 0xFF);
    }
  });
  return {packed, scales};
}

torch::Tensor unpack_int3(torch::Tensor packed, torch::Tensor scales, int64_t group, int64_t n_cols) {
  const int64_t N = packed.size(0), NP = packed.size(1), G = scales.size(1);
  auto out = torch::empty({N, n_cols}, torch::kFloat32);
  const uint8_t* pp = packed.contiguous().data_ptr<uint8_t>();
  const float* sp = scales.contiguous().data_ptr<float>();
  float* o = out.data_ptr<float>();
  prange(N, [&](int64_t r) {for (int64_t j = 0; j < n_cols; ++j) {
      const int64_t ch = j / 8, b = j % 8;
      uint32_t bits = 0;
      for (int k = 0; k < 3; ++k) {
        const int64_t idx = ch * 3 + k;
        bits |= (uint32_t)(idx < NP ? pp[r * NP + idx] : 0) << (8 * k);
      }
      int v = (int)((bits >> (3 * b)) & 7);
      if (v & 4) v -= 8;  // sign-extend 3-bit two's complement
      o[r * n_cols + j] = (float)v * sp[r * G + j / group];
    }});
  (void)G;
  return out;
}

// ---------------------------------------------------------------- INT2 asymmetric, 4 per byte
std::vector<torch::Tensor> quantize_int2(torch::Tensor x, int64_t group) {
  check_cpu_f32_2d(x, "x");
  const int64_t N = x.size(0), D = x.size(1), G = D / group;
  TORCH_CHECK(D % group == 0 && D % 4 == 0, "columns must be divisible by group and 4");
  auto packed = torch::empty({N, D / 4}, torch::kUInt8);
  auto scales = torch::empty({N, G}, torch::kFloat32);
  auto offsets = torch::empty({N, G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  uint8_t* pp = packed.data_ptr<uint8_t>();
  float* sp = scales.data_ptr<float>();
  float* op = offsets.data_ptr<float>();
  prange(N, [&](int64_t r) {
    for (int64_t g = 0; g < G; ++g) {
      float mn = INFINITY, mx = -INFINITY;
      for (int64_t i = g * group; i < (g + 1) * group; ++i) {
        mn = std::min(mn, xp[r * D + i]);
        mx = std::max(mx, xp[r * D + i]);
      }
      sp[r * G + g] = mx == mn ? 1.f : (mx - mn) / 3.f;
      op[r * G + g] = mn;
    }
    for (int64_t i = 0; i < D / 4; ++i) {
      uint8_t byte = 0;
      for (int b = 0; b < 4; ++b) {
        const int64_t j = i * 4 + b, g = j / group;
        const uint8_t q = (uint8_t)clampf(std::round((xp[r * D + j] - op[r * G + g]) / sp[r * G + g]), 0.f, 3.f);
        byte |= (uint8_t)((q & 3) << (2 * b));
      }
      pp[r * (D / 4) + i] = byte;
    }
  });
  return {packed, scales, offsets};
}

torch::Tensor dequantize_int2(torch::Tensor packed, torch::Tensor scales, torch::Tensor offsets, int64_t group) {
  const int64_t N = packed.size(0), D = packed.size(1) * 4, G = scales.size(1);
  auto out = torch::empty({N, D}, torch::kFloat32);
  const uint8_t* pp = packed.contiguous().data_ptr<uint8_t>();
  const float* sp = scales.contiguous().data_ptr<float>();
  const float* op = offsets.contiguous().data_ptr<float>();
  float* o = out.data_ptr<float>();
  prange(N, [&](int64_t r) {for (int64_t c = 0; c < D; ++c) {
      const uint8_t q = (pp[r * (D / 4) + c / 4] >> (2 * (c % 4))) & 3;
      o[r * D + c] = op[r * G + c / group] + (float)q * sp[r * G + c / group];
    }});
  return out;
}

// ---------------------------------------------------------------- KV page codecs (oracle for kv_write.cu)
// x: [rows, D] -> codes [rows, D*bits/8] u8, scales [rows, nscale] f32 (fp16-rounded like the kernel)
// fp16_scales (the paged device pools' layout): scales are rounded to fp16 before the codes
// are chosen, so every code is the nearest under the scale that is stored. fp16_scales false:
// float32 scales with the reference numpy codecs' arithmetic (squish/kv/kv_cache.py:78-375,
// squish/kv/k8v4_codec.py:64-137), code for code: INT8 q = round(x / absmax * 127), stored
// scale absmax / 127; INT4 / INT2 round(x / (absmax / L) + L); k8v4 round((x - lo) / scale).
std::vector<torch::Tensor> kv_quantize(torch::Tensor x, int64_t fmt, int64_t group, bool fp16_scales = true) {
  check_cpu_f32_2d(x, "x");
  TORCH_CHECK(fmt >= 1 && fmt <= 5, "kv format must be int8 / int4 / int2 / k8 / v4 (1..5)");
  TORCH_CHECK(group > 0 && x.size(1) % group == 0, "group must divide the row length");
  const int64_t R = x.size(0), D = x.size(1), NG = D / group;
  const bool asym = (fmt == 4 || fmt == 5);
  const int bits = fmt == 1 || fmt == 4 ? 8 : fmt == 2 || fmt == 5 ? 4 : 2;
  TORCH_CHECK((D * bits) % 8 == 0, "row length must fill whole bytes of codes (D * bits % 8 == 0)");
  const float qmax = fmt == 1 ? 127.f : fmt == 2 ? 7.5f : fmt == 3 ? 1.5f : fmt == 4 ? 255.f : 15.f;
  auto codes = torch::zeros({R, D * bits / 8}, torch::kUInt8);
  auto scales = torch::zeros({R, NG * (asym ? 2 : 1)}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  uint8_t* cp = codes.data_ptr<uint8_t>();
  float* sp = scales.data_ptr<float>();
  const int64_t CB = D * bits / 8, NS = NG * (asym ? 2 : 1);
  auto h16 = [fp16_scales](float v) { return fp16_scales ? c10::Half(v).operator float() : v; };
  prange(R, [&](int64_t r) {
    for (int64_t g = 0; g < NG; ++g) {
      const float* v = xp + r * D + g * group;
      float lo = INFINITY, hi = -INFINITY, am = 0.f;
      for (int64_t i = 0; i < group; ++i) {
        lo = std::min(lo, v[i]);
        hi = std::max(hi, v[i]);
        am = std::max(am, std::fabs(v[i]));
      }
      float s, z = 0.f;
      if (asym) {
        s = (hi - lo) / qmax;
        if (s == 0.f) s = 1.f;
        s = h16(s);
        z = h16(lo);
        sp[r * NS + 2 * g] = s;
        sp[r * NS + 2 * g + 1] = z;
      } else {
        s = h16(std::max(am, 1e-8f) / qmax);
        if (s == 0.f) s = 6e-8f;
        sp[r * NS + g] = s;
      }
      const float am_safe = std::max(am, 1e-8f);
      for (int64_t i = 0; i < group; ++i) {
        float t;
        if (asym) t = std::nearbyint((v[i] - z) / s);
        else if (fmt == 1 && !fp16_scales) t = std::nearbyint(v[i] / am_safe * 127.f);
        else if (fmt == 1) t = std::nearbyint(v[i] / s);
        else t = std::nearbyint(v[i] / s + qmax);
        int q;
        if (fmt == 1) q = (int)clampf(t, -128.f, 127.f);
        else if (fmt == 4) q = (int)clampf(t, 0.f, 255.f);
        else if (bits == 4) q = (int)clampf(t, 0.f, 15.f);
        else q = (int)clampf(t, 0.f, 3.f);
        const int64_t d = g * group + i;
        if (bits == 8) cp[r * CB + d] = (uint8_t)(q & 0xFF);
        else if (bits == 4) cp[r * CB + d / 2] |= (uint8_t)((q & 0xF) << (4 * (d & 1)));
        else cp[r * CB + d / 4] |= (uint8_t)((q & 3) << (2 * (d & 3)));
      }
    }
  });
  return {codes, scales};
}

torch::Tensor kv_dequantize(torch::Tensor codes, torch::Tensor scales, int64_t fmt, int64_t group, int64_t D) {
  TORCH_CHECK(fmt >= 1 && fmt <= 5, "kv format must be int8 / int4 / int2 / k8 / v4 (1..5)");
  TORCH_CHECK(group > 0 && D % group == 0, "group must divide D");
  TORCH_CHECK(codes.dim() == 2 && scales.dim() == 2 && codes.size(0) == scales.size(0), "codes / scales: [rows, ...]");
  TORCH_CHECK(codes.scalar_type() == torch::kUInt8 && codes.is_contiguous() && !codes.is_cuda(), "codes: uint8 CPU");
  TORCH_CHECK(scales.scalar_type() == torch::kFloat32 && scales.is_contiguous() && !scales.is_cuda(),
              "scales: float32 CPU");
  {
    const int bits = fmt == 1 || fmt == 4 ? 8 : fmt == 2 || fmt == 5 ? 4 : 2;
    TORCH_CHECK(D > 0 && (D * bits) % 8 == 0, "D must fill whole bytes of codes (D * bits % 8 == 0)");
    TORCH_CHECK(codes.size(1) == D * bits / 8, "codes row length does not match D and the format");
    TORCH_CHECK(scales.size(1) >= (D / group) * ((fmt == 4 || fmt == 5) ? 2 : 1), "too few scales per row");
  }
  const int64_t R = codes.size(0), CB = codes.size(1), NS = scales.size(1);
  const bool asym = (fmt == 4 || fmt == 5);
  const int bits = fmt == 1 || fmt == 4 ? 8 : fmt == 2 || fmt == 5 ? 4 : 2;
  auto out = torch::empty({R, D}, torch::kFloat32);
  const uint8_t* cp = codes.contiguous().data_ptr<uint8_t>();
  const float* sp = scales.contiguous().data_ptr<float>();
  float* o = out.data_ptr<float>();
  prange(R, [&](int64_t r) {for (int64_t d = 0; d < D; ++d) {
      const int64_t g = d / group;
      int q;
      if (bits == 8) q = (fmt == 1) ? (int)(int8_t)cp[r * CB + d] : (int)cp[r * CB + d];
      else if (bits == 4) q = (cp[r * CB + d / 2] >> (4 * (d & 1))) & 0xF;
      else q = (cp[r * CB + d / 4] >> (2 * (d & 3))) & 3;
      float v;
      if (asym) v = (float)q * sp[r * NS + 2 * g] + sp[r * NS + 2 * g + 1];
      else if (fmt == 1) v = (float)q * sp[r * NS + g];
      else if (fmt == 2) v = ((float)q - 7.5f) * sp[r * NS + g];
      else v = ((float)q - 1.5f) * sp[r * NS + g];
      o[r * D + d] = v;
    }});
  return out;
}

// ---- FP8 (OCP 8-bit floating point, E4M3 "fn" and E5M2), software codec ------------------
// The reference's experimental FP8 pair (lib.rs:960-1100) truncates the mantissa and flushes
// subnormals; this codec rounds to nearest even, keeps subnormals and saturates to the largest
// finite value, i.e. the conversion the sm_100a `cvt.rn.satfinite.e4m3x2/e5m2x2` instructions
// perform, so CPU and GPU codes agree bit for bit. Scale: absmax / largest finite per group, or
// one caller-given scale for every group (the reference's per-tensor form).
struct Fp8Fmt {
  int mbits, bias, maxcode;
  float maxval;
};
const Fp8Fmt kE4M3{3, 7, 0x7E, 448.f}, kE5M2{2, 15, 0x7B, 57344.f};

uint8_t fp8_encode(float v, const Fp8Fmt& f) {
  const uint8_t sign = std::signbit(v) ? 0x80 : 0;
  if (std::isnan(v)) return sign | 0x7F;
  const float a = std::fabs(v);
  if (a == 0.f) return sign;
  if (std::isinf(a)) return sign | (uint8_t)f.maxcode;
  int e2;
  std::frexp(a, &e2);
  const int ex = e2 - 1;          // a in [2^ex, 2^(ex+1))
  const int emin = 1 - f.bias;    // smallest normal exponent
  long code;
  if (ex < emin) {
    // subnormal: integer multiples of 2^(emin - mbits); a count of 2^mbits is the smallest normal
    code = (long)std::nearbyint(std::ldexp(a, f.mbits - emin));
  } else {
    const float m = std::ldexp(a, -ex) - 1.f;  // exact, in [0, 1)
    code = ((long)(ex + f.bias) << f.mbits) + (long)std::nearbyint(std::ldexp(m, f.mbits));  // carry rolls into the exponent
  }
  if (code > f.maxcode) code = f.maxcode;
  return sign | (uint8_t)code;
}

float fp8_decode(uint8_t c, const Fp8Fmt& f) {
  const int mag = c & 0x7F;
  const float sg = (c & 0x80) ? -1.f : 1.f;
  const int field = mag >> f.mbits, mant = mag & ((1 << f.mbits) - 1);
  if (f.mbits == 3 && mag == 0x7F) return std::nanf("");
  if (f.mbits == 2 && field == 31) return mant ? std::nanf("") : sg * INFINITY;
  if (field == 0) return sg * std::ldexp((float)mant, 1 - f.bias - f.mbits);
  return sg * std::ldexp(1.f + std::ldexp((float)mant, -f.mbits), field - f.bias);
}

std::vector<torch::Tensor> quantize_fp8(torch::Tensor x, int64_t fmt, int64_t group, double fixed_scale) {
  check_cpu_f32_2d(x, "x");
  TORCH_CHECK(fmt == 0 || fmt == 1, "fmt: 0 e4m3, 1 e5m2");
  const Fp8Fmt& f = fmt == 0 ? kE4M3 : kE5M2;
  const int64_t N = x.size(0), D = x.size(1), g = group <= 0 ? D : group;
  TORCH_CHECK(D % g == 0, "group must divide columns");
  const int64_t G = D / g;
  auto codes = torch::empty({N, D}, torch::kUInt8);
  auto scales = torch::empty({N, G}, torch::kFloat32);
  const float* xp = x.data_ptr<float>();
  uint8_t* cp = codes.data_ptr<uint8_t>();
  float* sp = scales.data_ptr<float>();
  prange(N * G, [&](int64_t i) {
    const int64_t r = i / G, gi = i % G;
    const float* src = xp + r * D + gi * g;
    float sc = (float)fixed_scale;
    if (!(sc > 0.f)) {
      float am = 0.f;
      for (int64_t j = 0; j < g; ++j) am = std::max(am, std::fabs(src[j]));
      sc = am == 0.f ? 1.f : am / f.maxval;
    }
    sp[i] = sc;
    for (int64_t j = 0; j < g; ++j) cp[r * D + gi * g + j] = fp8_encode(src[j] / sc, f);
  });
  return {codes, scales};
}

torch::Tensor dequantize_fp8(torch::Tensor codes, torch::Tensor scales, int64_t fmt) {
  TORCH_CHECK(codes.scalar_type() == torch::kUInt8 && codes.dim() == 2 && codes.is_contiguous(),
              "codes: contiguous uint8 [N, D]");
  check_cpu_f32_2d(scales, "scales");
  TORCH_CHECK(fmt == 0 || fmt == 1, "fmt: 0 e4m3, 1 e5m2");
  const Fp8Fmt& f = fmt == 0 ? kE4M3 : kE5M2;
  const int64_t N = codes.size(0), D = codes.size(1), G = scales.size(1);
  TORCH_CHECK(scales.size(0) == N && G > 0 && D % G == 0, "scales: [N, groups] with groups dividing D");
  const int64_t g = D / G;
  auto out = torch::empty({N, D}, torch::kFloat32);
  const uint8_t* cp = codes.data_ptr<uint8_t>();
  const float* sp = scales.data_ptr<float>();
  float* o = out.data_ptr<float>();
  prange(N, [&](int64_t r) {
    for (int64_t d = 0; d < D; ++d) o[r * D + d] = fp8_decode(cp[r * D + d], f) * sp[r * G + d / g];
  });
  return out;
}

// ---- FP6 (1 sign + e exponent + m mantissa bits, e + m = 5), 4 values per 3 bytes ----------
// Packing of the reference's fp6_encode_f32 / fp6_decode (lib.rs:2410-2470): the four 6-bit
// codes a, b, c, d form the 24-bit word a<<18 | b<<12 | c<<6 | d, stored most significant byte
// first. Values (the OCP MX FP6 convention, no infinities or NaNs): exponent field 0 holds
// subnormals man * 2^(1 - bias - m), others (1 + man / 2^m) * 2^(field - bias), bias =
// 2^(e-1) - 1. Encoding rounds to nearest even and saturates to the largest magnitude (the
// reference truncates the mantissa and flushes subnormals to zero; its codes decode the same).
struct Fp6Fmt {
  int e, m, bias;
  float maxval;
};
Fp6Fmt fp6_fmt(int64_t e, int64_t m) {
  TORCH_CHECK(e >= 1 && m >= 0 && e + m == 5, "FP6 needs exponent + mantissa bits = 5 (exponent >= 1)");
  const int bias = (1 << (e - 1)) - 1;
  const float maxv = std::ldexp(1.f + (float)((1 << m) - 1) / (float)(1 << m), (1 << e) - 1 - bias);
  return {(int)e, (int)m, bias, maxv};
}
uint8_t fp6_encode1(float v, const Fp6Fmt& f) {
  const uint8_t sign = std::signbit(v) ? 0x20 : 0;
  float a = std::fabs(v);
  if (std::isnan(a)) return 0;  // as the reference: NaN encodes as +0
  if (a == 0.f) return sign;
  const long maxcode = (1L << 5) - 1;  // all exponent and mantissa bits set
  if (std::isinf(a) || a >= f.maxval) return sign | (uint8_t)maxcode;
  int e2;
  std::frexp(a, &e2);
  const int ex = e2 - 1, emin = 1 - f.bias;
  long code;
  if (ex < emin) {
    code = (long)std::nearbyint(std::ldexp(a, f.m - emin));
  } else {
    const float mm = std::ldexp(a, -ex) - 1.f;
    code = ((long)(ex + f.bias) << f.m) + (long)std::nearbyint(std::ldexp(mm, f.m));
  }
  if (code > maxcode) code = maxcode;
  return sign | (uint8_t)code;
}
float fp6_decode1(uint8_t c, const Fp6Fmt& f) {
  const float sg = (c & 0x20) ? -1.f : 1.f;
  const int field = (c & 0x1F) >> f.m, man = c & ((1 << f.m) - 1);
  if (field == 0) return sg * std::ldexp((float)man, 1 - f.bias - f.m);
  return sg * std::ldexp(1.f + std::ldexp((float)man, -f.m), field - f.bias);
}

torch::Tensor fp6_encode(torch::Tensor x, int64_t exp_bits, int64_t man_bits) {
  TORCH_CHECK(!x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.is_contiguous(), "x: contiguous float32 (CPU)");
  TORCH_CHECK(x.numel() % 4 == 0, "length must be a multiple of 4");
  const Fp6Fmt f = fp6_fmt(exp_bits, man_bits);
  const int64_t packs = x.numel() / 4;
  auto out = torch::empty({packs * 3}, torch::kUInt8);
  const float* xp = x.data_ptr<float>();
  uint8_t* o = out.data_ptr<uint8_t>();
  prange(packs, [&](int64_t i) {
    const uint32_t w = ((uint32_t)fp6_encode1(xp[4 * i], f) << 18) | ((uint32_t)fp6_encode1(xp[4 * i + 1], f) << 12) |
                       ((uint32_t)fp6_encode1(xp[4 * i + 2], f) << 6) | (uint32_t)fp6_encode1(xp[4 * i + 3], f);
    o[3 * i] = (uint8_t)(w >> 16);
    o[3 * i + 1] = (uint8_t)(w >> 8);
    o[3 * i + 2] = (uint8_t)w;
  });
  return out;
}

torch::Tensor fp6_decode(torch::Tensor packed, int64_t n, int64_t exp_bits, int64_t man_bits) {
  TORCH_CHECK(!packed.is_cuda() && packed.scalar_type() == torch::kUInt8 && packed.is_contiguous(),
              "packed: contiguous uint8 (CPU)");
  TORCH_CHECK(n % 4 == 0 && packed.numel() >= n / 4 * 3, "n must be a multiple of 4 covered by the packed bytes");
  const Fp6Fmt f = fp6_fmt(exp_bits, man_bits);
  auto out = torch::empty({n}, torch::kFloat32);
  const uint8_t* p = packed.data_ptr<uint8_t>();
  float* o = out.data_ptr<float>();
  prange(n / 4, [&](int64_t i) {
    const uint32_t w = ((uint32_t)p[3 * i] << 16) | ((uint32_t)p[3 * i + 1] << 8) | (uint32_t)p[3 * i + 2];
    for (int j = 0; j < 4; ++j) o[4 * i + j] = fp6_decode1((uint8_t)((w >> (18 - 6 * j)) & 0x3F), f);
  });
  return out;
}

}  // namespace

void register_entropy(pybind11::module& c);   // entropy.cpp
void register_research(pybind11::module& c);  // quant_research.cpp
void register_kv_research(pybind11::module& c);  // kv_research.cpp
void register_recurrent(pybind11::module& c);    // recurrent.cpp

void register_cpu(pybind11::module& m) {
  auto c = m.def_submodule("cpu", "C++ CPU reference kernels (restating squish_quant_rs)");
  register_entropy(c);
  register_research(c);
  register_kv_research(c);
  register_recurrent(c);
  c.def("quantize_int8", &quantize_int8);
  c.def("dequantize_int8", &dequantize_int8);
  c.def("quantize_int4_asym", &quantize_int4_asym);
  c.def("quantize_int4_asym_mse", &quantize_int4_asym_mse);
  c.def("dequantize_int4_asym", &dequantize_int4_asym);
  c.def("quantized_matmul_int4", &quantized_matmul_int4);
  c.def("quantize_int4_sym", &quantize_int4_sym);
  c.def("dequantize_int4_sym", &dequantize_int4_sym);
  c.def("quantize_nf4", &quantize_nf4);
  c.def("dequantize_nf4", &dequantize_nf4);
  c.def("pack_int3", &pack_int3);
  c.def("unpack_int3", &unpack_int3);
  c.def("quantize_int2", &quantize_int2);
  c.def("dequantize_int2", &dequantize_int2);
  c.def("kv_quantize", &kv_quantize, pybind11::arg("x"), pybind11::arg("fmt"), pybind11::arg("group"),
        pybind11::arg("fp16_scales") = true);
  c.def("kv_dequantize", &kv_dequantize);
  c.def("quantize_fp8", &quantize_fp8, pybind11::arg("x"), pybind11::arg("fmt"), pybind11::arg("group"),
        pybind11::arg("fixed_scale") = 0.0);
  c.def("dequantize_fp8", &dequantize_fp8);
  c.def("fp6_encode", &fp6_encode);
  c.def("fp6_decode", &fp6_decode);
}

}  // namespace sqcpu
