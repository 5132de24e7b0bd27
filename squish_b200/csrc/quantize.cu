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
#include <cuda_fp8.h>
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

// ------------------------------------------------------------------ other codecs
// One thread per (row, group); the arithmetic mirrors the C++ CPU library (cpu_ref.cpp), which
// restates squish_quant_rs: quantize_int8_grouped (lib.rs:121), quantize_int4_grouped (259),
// NF4 (742-890), pack_int3_grouped_f32 (1125), quantize_int2_grouped_f32 (1440).
__constant__ float kNf4Lv[16] = {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
                                 -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
                                 0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f,
                                 0.33791524171829224f, 0.44070982933044434f, 0.5626170039176941f,
                                 0.7229568362236023f, 1.0f};

__device__ __forceinline__ float clampf_d(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }

template <typename T>
__device__ __forceinline__ float group_absmax(const T* src, int n) {
  float am = 0.f;
  for (int i = 0; i < n; ++i) am = fmaxf(am, fabsf(to_f(src[i])));
  return am;
}

// codec: 0 INT8 sym (q int8, s = absmax/127, x * (1/s)), 1 INT4 sym (q+7 nibbles, s = absmax/7),
// 2 NF4 (nearest level of x/absmax), 3 INT3 sym (s = absmax/3, 3-bit two's complement, 8 values
// per 3 bytes of the row), 4 INT2 asym (s = (max-min)/3, offset min, 4 values per byte)
template <typename T>
__global__ void quantize_codec_kernel(const T* __restrict__ x, uint8_t* __restrict__ codes,
                                      float* __restrict__ scales, float* __restrict__ offsets, int rows, int cols,
                                      int group, int codec, int code_ld, float fixed_scale) {
  const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int G = cols / group;
  if (gid >= (long)rows * G) return;
  const int r = (int)(gid / G), g = (int)(gid % G);
  const T* src = x + (size_t)r * cols + (size_t)g * group;
  uint8_t* row = codes + (size_t)r * code_ld;
  const size_t si = (size_t)r * G + g;
  if (codec == 4) {
    float mn = INFINITY, mx = -INFINITY;
    for (int i = 0; i < group; ++i) {
      const float v = to_f(src[i]);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    const float sc = mx == mn ? 1.f : (mx - mn) / 3.f;
    scales[si] = sc;
    offsets[si] = mn;
    for (int i = 0; i < group; i += 4) {
      uint8_t byte = 0;
      for (int b = 0; b < 4; ++b) {
        const uint8_t q = (uint8_t)clampf_d(roundf((to_f(src[i + b]) - mn) / sc), 0.f, 3.f);
        byte |= (uint8_t)((q & 3) << (2 * b));
      }
      row[(g * group + i) / 4] = byte;
    }
    return;
  }
  if (codec == 5 || codec == 6) {
    // FP8 (OCP E4M3 / E5M2): s = absmax / largest finite (or one scale for the whole tensor),
    // codes = cvt.rn.satfinite(x / s)
    const float fmax = codec == 5 ? 448.f : 57344.f;
    float sc = fixed_scale;
    if (!(sc > 0.f)) {
      const float am = group_absmax(src, group);
      sc = am == 0.f ? 1.f : am / fmax;
    }
    scales[si] = sc;
    const __nv_fp8_interpretation_t kind = codec == 5 ? __NV_E4M3 : __NV_E5M2;
    for (int i = 0; i < group; ++i)
      row[(size_t)g * group + i] = (uint8_t)__nv_cvt_float_to_fp8(to_f(src[i]) / sc, __NV_SATFINITE, kind);
    return;
  }
  const float am = group_absmax(src, group);
  if (codec == 0) {
    const float sc = am == 0.f ? 1.f : am / 127.f;
    scales[si] = sc;
    const float inv = 1.f / sc;
    int8_t* q = reinterpret_cast<int8_t*>(row) + (size_t)g * group;
    for (int i = 0; i < group; ++i) q[i] = (int8_t)clampf_d(roundf(to_f(src[i]) * inv), -127.f, 127.f);
  } else if (codec == 1) {
    const float sc = am == 0.f ? 1.f : am / 7.f;
    scales[si] = sc;
    for (int i = 0; i < group; i += 2) {
      const int q0 = (int)clampf_d(roundf(to_f(src[i]) / sc), -7.f, 7.f) + 7;
      const int q1 = (int)clampf_d(roundf(to_f(src[i + 1]) / sc), -7.f, 7.f) + 7;
      row[(g * group + i) / 2] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
    }
  } else if (codec == 2) {
    const float sc = am == 0.f ? 1.f : am;
    scales[si] = sc;
    for (int i = 0; i < group; i += 2) {
      uint8_t qq[2];
      for (int k = 0; k < 2; ++k) {
        const float v = to_f(src[i + k]) / sc;
        int best = 0;
        float bd = INFINITY;
        for (int l = 0; l < 16; ++l) {
          const float d = fabsf(v - kNf4Lv[l]);
          if (d < bd) {
            bd = d;
            best = l;
          }
        }
        qq[k] = (uint8_t)best;
      }
      row[(g * group + i) / 2] = (uint8_t)(qq[0] | (qq[1] << 4));
    }
  } else {  // codec 3: INT3; a group covers whole 8-value chunks (group % 8 == 0)
    const float sc = am == 0.f ? 1.f : am / 3.f;
    scales[si] = sc;
    for (int ch = 0; ch < group / 8; ++ch) {
      uint32_t bits = 0;
      for (int b = 0; b < 8; ++b) {
        const uint32_t v = (uint32_t)((int)clampf_d(roundf(to_f(src[ch * 8 + b]) / sc), -3.f, 3.f) & 7);
        bits |= v << (3 * b);
      }
      const int c3 = ((g * group) / 8 + ch) * 3;
      for (int k = 0; k < 3; ++k) row[c3 + k] = (uint8_t)((bits >> (8 * k)) & 0xFF);
    }
  }
}

}  // namespace

cudaError_t quantize_codec_launch(const void* x, bool bf16, int codec, uint8_t* codes, int code_ld, float* scales,
                                  float* offsets, int rows, int cols, int group, float fixed_scale, cudaStream_t s) {
  const long total = (long)rows * (cols / group);
  if (total == 0) return cudaSuccess;
  const int threads = 128;
  const unsigned blocks = (unsigned)((total + threads - 1) / threads);
  if (bf16)
    quantize_codec_kernel<__nv_bfloat16><<<blocks, threads, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x), codes, scales, offsets, rows, cols, group, codec, code_ld,
        fixed_scale);
  else
    quantize_codec_kernel<float><<<blocks, threads, 0, s>>>(reinterpret_cast<const float*>(x), codes, scales, offsets,
                                                           rows, cols, group, codec, code_ld, fixed_scale);
  return cudaGetLastError();
}

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

// ------------------------------------------------------------------ HQQ
// Half-quadratic quantization (Badri & Shaji, arXiv:2309.15531), the calibration-free refinement
// of squish/quant/hqq.py:195-222: from the min/max affine grid (scale = span / qmax, zero = min),
// `iters` alternating steps of
//   scale <- (sum q (w - zero) + lambda scale) / (sum q^2 + lambda)
//   zero  <- mean(w - q scale)
//   q     <- clamp(rint((w - zero) / max(|scale|, 1e-8)), 0, qmax)
// One warp per (row, group); a lane holds group/32 values in registers (group <= 512).
namespace {

constexpr int kHqqPerLane = 16;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__global__ void __launch_bounds__(256) hqq_kernel(const T* __restrict__ x, uint8_t* __restrict__ codes,
                                                  float* __restrict__ scales, float* __restrict__ zeros, int rows,
                                                  int cols, int group, float qmax, float lam, int iters) {
  const long warp = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int G = cols / group;
  if (warp >= (long)rows * G) return;  // uniform per warp
  const int r = (int)(warp / G), g = (int)(warp % G);
  const T* src = x + (size_t)r * cols + (size_t)g * group;
  float w[kHqqPerLane], q[kHqqPerLane];
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kHqqPerLane; ++j) {
    const int i = j * 32 + lane;
    w[j] = i < group ? to_f(src[i]) : 0.f;
    if (i < group) {
      mn = fminf(mn, w[j]);
      mx = fmaxf(mx, w[j]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  float sc = fmaxf(mx - mn, 1e-6f) / qmax, z = mn;
#pragma unroll
  for (int j = 0; j < kHqqPerLane; ++j) q[j] = clampf_d(rintf((w[j] - z) / sc), 0.f, qmax);
  const float inv_n = 1.f / (float)group;
  for (int it = 0; it < iters; ++it) {
    float c2 = 0.f, cw = 0.f;
#pragma unroll
    for (int j = 0; j < kHqqPerLane; ++j)
      if (j * 32 + lane < group) {
        c2 += q[j] * q[j];
        cw += q[j] * (w[j] - z);
      }
    c2 = warp_sum(c2) + lam;
    cw = warp_sum(cw) + lam * sc;
    sc = cw / c2;
    float rz = 0.f;
#pragma unroll
    for (int j = 0; j < kHqqPerLane; ++j)
      if (j * 32 + lane < group) rz += w[j] - q[j] * sc;
    z = warp_sum(rz) * inv_n;
    const float d = fmaxf(fabsf(sc), 1e-8f);
#pragma unroll
    for (int j = 0; j < kHqqPerLane; ++j) q[j] = clampf_d(rintf((w[j] - z) / d), 0.f, qmax);
  }
  uint8_t* dst = codes + (size_t)r * cols + (size_t)g * group;
#pragma unroll
  for (int j = 0; j < kHqqPerLane; ++j)
    if (j * 32 + lane < group) dst[j * 32 + lane] = (uint8_t)q[j];
  if (lane == 0) {
    scales[(size_t)r * G + g] = sc;
    zeros[(size_t)r * G + g] = z;
  }
}

// AWQ calibration statistics (squish/quant/awq.py:239-260): acc[c] += mean over rows of |x[:, c]|.
// Blocks own 256 columns x a slab of rows; the slab's partial mean is added to acc with one
// double atomic per column.
template <typename T>
__global__ void __launch_bounds__(256) channel_abs_mean_kernel(const T* __restrict__ x, double* __restrict__ acc,
                                                               int rows, int cols, int rows_per_block) {
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c >= cols) return;
  const int r0 = blockIdx.y * rows_per_block, r1 = min(rows, r0 + rows_per_block);
  float s = 0.f;
  for (int r = r0; r < r1; ++r) s += fabsf(to_f(x[(size_t)r * cols + c]));
  atomicAdd(acc + c, (double)s / (double)rows);
}

}  // namespace

cudaError_t hqq_launch(const void* x, bool bf16, uint8_t* codes, float* scales, float* zeros, int rows, int cols,
                       int group, int levels, float lam, int iters, cudaStream_t s) {
  if (group > 32 * kHqqPerLane || group <= 0 || cols % group != 0) return cudaErrorInvalidValue;
  const long warps = (long)rows * (cols / group);
  if (warps == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  const float qmax = (float)(levels - 1);
  if (bf16)
    hqq_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), codes, scales,
                                                     zeros, rows, cols, group, qmax, lam, iters);
  else
    hqq_kernel<float><<<blocks, 256, 0, s>>>(reinterpret_cast<const float*>(x), codes, scales, zeros, rows, cols,
                                             group, qmax, lam, iters);
  return cudaGetLastError();
}

cudaError_t channel_abs_mean_launch(const void* x, bool bf16, double* acc, int rows, int cols, cudaStream_t s) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  const int rpb = 64;
  const dim3 grid((cols + 255) / 256, (rows + rpb - 1) / rpb);
  if (bf16)
    channel_abs_mean_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(x), acc, rows,
                                                                cols, rpb);
  else
    channel_abs_mean_kernel<float><<<grid, 256, 0, s>>>(reinterpret_cast<const float*>(x), acc, rows, cols, rpb);
  return cudaGetLastError();
}

}  // namespace sq
