// quantize.cu — weight quantizers on the GPU (the CUDA counterpart of the reference's
// squish_quant_rs kernels used by `squish compress`).
//
// quantize_int4_asym: per (row, group) scale = (max-min)/15 (1 if max == min), offset =
// min, q = clamp(round((x - offset)/scale), 0, 15) with round-half-away-from-zero, nibbles
// packed low = even column — the semantics of quantize_int4_asymmetric_grouped
// (squish_quant_rs/src/lib.rs:402). With n_clip > 1 each group first searches the
// inward clip fraction beta in linspace(0, 0.1, n_clip) that minimises the
// reconstruction MSE (squish/quant/quantizer.py:500-605).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace sq {

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

__device__ __forceinline__ float round_away(float x) { return roundf(x); }

// One thread per (row, group). group <= 256.
template <typename T>
__global__ void quantize_int4_asym_kernel(const T* __restrict__ x, uint8_t* __restrict__ packed,
                                          float* __restrict__ scales, float* __restrict__ offsets, int rows,
                                          int cols, int group, int n_clip) {
  const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int G = cols / group;
  if (gid >= (long)rows * G) return;
  const int r = (int)(gid / G), g = (int)(gid % G);
  const T* src = x + (size_t)r * cols + (size_t)g * group;
  float mn = 3.4e38f, mx = -3.4e38f;
  for (int i = 0; i < group; ++i) {
    const float v = to_f(src[i]);
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  float lo = mn, hi = mx;
  if (n_clip > 1 && rows > 1) {
    const float rng = mx - mn;
    float best = 3.4e38f;
    for (int c = 0; c < n_clip; ++c) {
      const float beta = 0.10f * (float)c / (float)(n_clip - 1);
      const float clo = mn + beta * rng, chi = mx - beta * rng;
      if (clo >= chi) continue;
      const float sc = (chi - clo) / 15.f;
      float mse = 0.f;
      for (int i = 0; i < group; ++i) {
        const float v = to_f(src[i]);
        const float vc = fminf(fmaxf(v, clo), chi);
        const float q = fminf(fmaxf(rintf((vc - clo) / sc), 0.f), 15.f);
        const float d = v - (clo + q * sc);
        mse += d * d;
      }
      if (mse < best) {
        best = mse;
        lo = clo;
        hi = chi;
      }
    }
  }
  const float scale = (hi == lo) ? 1.f : (hi - lo) / 15.f;
  scales[(size_t)r * G + g] = scale;
  offsets[(size_t)r * G + g] = lo;
  uint8_t* dst = packed + (size_t)r * (cols / 2) + (size_t)g * group / 2;
  for (int i = 0; i < group; i += 2) {
    const float v0 = fminf(fmaxf(to_f(src[i]), lo), hi);
    const float v1 = fminf(fmaxf(to_f(src[i + 1]), lo), hi);
    const int q0 = (int)fminf(fmaxf(round_away((v0 - lo) / scale), 0.f), 15.f);
    const int q1 = (int)fminf(fmaxf(round_away((v1 - lo) / scale), 0.f), 15.f);
    dst[i / 2] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
  }
}

}  // namespace

cudaError_t quantize_int4_asym_launch(const void* x, bool bf16, uint8_t* packed, float* scales, float* offsets,
                                      int rows, int cols, int group, int n_clip, cudaStream_t s) {
  const long total = (long)rows * (cols / group);
  const int threads = 256;
  const unsigned blocks = (unsigned)((total + threads - 1) / threads);
  if (bf16)
    quantize_int4_asym_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), packed, scales, offsets, rows, cols, group, n_clip);
  else
    quantize_int4_asym_kernel<float><<<blocks, threads, 0, s>>>(reinterpret_cast<const float*>(x), packed, scales,
                                                                offsets, rows, cols, group, n_clip);
  return cudaGetLastError();
}

}  // namespace sq
