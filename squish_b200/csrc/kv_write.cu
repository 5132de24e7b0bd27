// kv_write.cu — fused RoPE + KV quantize + paged write, and RMSNorm.
//
// rope_kv_write: for every token of the step, rotate q and k (neox "rotate half" form,
// as in HF Llama/Qwen2), write q to a dense [T, Hq, D] buffer, and quantize k and v
// into their page slot with the layer's KV formats (kv_format.cuh). This replaces the
// reference's per-chunk numpy codecs applied after attention (squish/kv/kv_cache.py:
// 78-375, squish/kv/k8v4_codec.py:64) with quantize-on-write: a token's KV is stored
// once, already compressed, and never materialised in fp16.
#include "kv_format.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace sq {

namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Quantize the D values held by this warp (v[jj] = dim lane + 32*jj) into one row.
template <int D>
__device__ void quant_row(const float (&v)[D / 32], int fmt, int G, uint8_t* codes, __half* scales) {
  const int lane = threadIdx.x & 31;
  constexpr int J = D / 32;
  if (fmt == KV_BF16) {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(codes);
#pragma unroll
    for (int jj = 0; jj < J; ++jj) o[lane + 32 * jj] = __float2bfloat16(v[jj]);
    return;
  }
  const bool asym = kv_asym(fmt);
  const float qmax = kv_qmax(fmt);
  const int per_group = G / 32;  // jj indices per group (G >= 32)
  int idx[J];
#pragma unroll
  for (int jj = 0; jj < J; ++jj) idx[jj] = 0;
  for (int g = 0; g < D / G; ++g) {
    float lo = 3.4e38f, hi = -3.4e38f, am = 0.f;
#pragma unroll
    for (int jj = 0; jj < J; ++jj) {
      if (jj / per_group == g) {
        lo = fminf(lo, v[jj]);
        hi = fmaxf(hi, v[jj]);
        am = fmaxf(am, fabsf(v[jj]));
      }
    }
    float s, z = 0.f;
    if (asym) {
      lo = warp_min(lo);
      hi = warp_max(hi);
      s = (hi - lo) / qmax;
      if (s == 0.f) s = 1.f;
      s = __half2float(__float2half_rn(s));
      z = __half2float(__float2half_rn(lo));
      if (lane == 0) {
        scales[2 * g] = __float2half_rn(s);
        scales[2 * g + 1] = __float2half_rn(z);
      }
    } else {
      am = warp_max(am);
      s = __half2float(__float2half_rn(fmaxf(am, 1e-8f) / qmax));
      if (s == 0.f) s = 6e-8f;
      if (lane == 0) scales[g] = __float2half_rn(s);
    }
#pragma unroll
    for (int jj = 0; jj < J; ++jj) {
      if (jj / per_group == g) {
        float t;
        if (asym) t = rintf((v[jj] - z) / s);
        else if (fmt == KV_INT8) t = rintf(v[jj] / s);
        else t = rintf(v[jj] / s + qmax);  // INT4: +7.5, INT2: +1.5
        if (fmt == KV_INT8) t = fminf(fmaxf(t, -128.f), 127.f);
        else if (fmt == KV_K8) t = fminf(fmaxf(t, 0.f), 255.f);
        else if (fmt == KV_INT4 || fmt == KV_V4) t = fminf(fmaxf(t, 0.f), 15.f);
        else t = fminf(fmaxf(t, 0.f), 3.f);
        idx[jj] = (int)t;
      }
    }
  }
  const int bits = kv_bits(fmt);
#pragma unroll
  for (int jj = 0; jj < J; ++jj) {
    const int d = lane + 32 * jj;
    if (bits == 8) {
      codes[d] = (uint8_t)(idx[jj] & 0xFF);
    } else if (bits == 4) {
      const int nb = __shfl_down_sync(0xffffffffu, idx[jj], 1);
      if ((lane & 1) == 0) codes[d / 2] = (uint8_t)((idx[jj] & 0xF) | ((nb & 0xF) << 4));
    } else {
      const int n1 = __shfl_down_sync(0xffffffffu, idx[jj], 1);
      const int n2 = __shfl_down_sync(0xffffffffu, idx[jj], 2);
      const int n3 = __shfl_down_sync(0xffffffffu, idx[jj], 3);
      if ((lane & 3) == 0)
        codes[d / 4] = (uint8_t)((idx[jj] & 3) | ((n1 & 3) << 2) | ((n2 & 3) << 4) | ((n3 & 3) << 6));
    }
  }
}

// In-warp fast Walsh-Hadamard transform of the D values held as v[jj] = x[lane + 32 * jj],
// scaled by 1 / sqrt(D) (orthonormal): index bits 0-4 are lane bits (butterflies through
// shuffles), bits 5.. are register bits.
template <int D>
__device__ __forceinline__ void fwht_warp(float (&v)[D / 32]) {
  constexpr int J = D / 32;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int jj = 0; jj < J; ++jj) {
      const float o = __shfl_xor_sync(0xffffffffu, v[jj], h);
      v[jj] = (lane & h) ? o - v[jj] : v[jj] + o;
    }
  }
#pragma unroll
  for (int h = 1; h < J; h <<= 1) {
#pragma unroll
    for (int jj = 0; jj < J; ++jj) {
      if ((jj & h) == 0) {
        const float a = v[jj], b = v[jj + h];
        v[jj] = a + b;
        v[jj + h] = a - b;
      }
    }
  }
  constexpr float kScale = D == 32 ? 0.17677669529663688f : D == 64 ? 0.125f : D == 128 ? 0.08838834764831845f
                                                                                         : 0.0625f;
#pragma unroll
  for (int jj = 0; jj < J; ++jj) v[jj] *= kScale;
}

template <int D>
__global__ void rope_kv_write_kernel(RopeKvParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int J = D / 32;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = p.positions[t];
  const int slot = p.slot_mapping ? p.slot_mapping[t] : -1;
  const __nv_bfloat16* row = p.qkv + (size_t)t * p.ld_qkv;
  const float* cs = p.cos_sin + (size_t)pos * D;  // [cos(D/2) | sin(D/2)]
  const int jobs = p.Hq + 2 * p.Hkv;
  {
    // one warp per (token, head): grid (T, ceil(jobs / warps per block))
    const int j = blockIdx.y * (blockDim.x >> 5) + warp;
    if (j >= jobs) return;
    float v[J];
    const __nv_bfloat16* src = row + (size_t)j * D;
#pragma unroll
    for (int jj = 0; jj < J; ++jj) v[jj] = __bfloat162float(src[lane + 32 * jj]);
    if (j < p.Hq + p.Hkv) {  // (optional per-head RMSNorm, Qwen3) then rotate q and k
      const __nv_bfloat16* nw = (j < p.Hq) ? p.q_norm : p.k_norm;
      if (nw != nullptr) {
        float ss = 0.f;
#pragma unroll
        for (int jj = 0; jj < J; ++jj) ss += v[jj] * v[jj];
        ss = warp_sum(ss);
        const float inv = rsqrtf(ss / (float)D + p.norm_eps);
#pragma unroll
        for (int jj = 0; jj < J; ++jj) v[jj] = v[jj] * inv * __bfloat162float(nw[lane + 32 * jj]);
      }
      if constexpr (J == 1) {
        // D = 32: dims i and i+16 sit in lanes i and i+16
        const float other = __shfl_xor_sync(0xffffffffu, v[0], 16);
        const int i = lane & 15;
        const float c = cs[i], s = cs[D / 2 + i];
        v[0] = (lane < 16) ? v[0] * c - other * s : v[0] * c + other * s;
      } else {
        float r[J];
#pragma unroll
        for (int jj = 0; jj < J / 2; ++jj) {
          const int i = lane + 32 * jj;
          const float c = cs[i], s = cs[D / 2 + i];
          r[jj] = v[jj] * c - v[jj + J / 2] * s;
          r[jj + J / 2] = v[jj + J / 2] * c + v[jj] * s;
        }
#pragma unroll
        for (int jj = 0; jj < J; ++jj) v[jj] = r[jj];
      }
      if (p.had_k != nullptr) {  // rotated scores basis: H (s_k * x)
#pragma unroll
        for (int jj = 0; jj < J; ++jj) v[jj] *= p.had_k[lane + 32 * jj];
        fwht_warp<D>(v);
      }
    } else if (p.had_v != nullptr) {  // v: s_v * (H v)
      fwht_warp<D>(v);
#pragma unroll
      for (int jj = 0; jj < J; ++jj) v[jj] *= p.had_v[lane + 32 * jj];
    }
    if (j < p.Hq) {
      __nv_bfloat16* dst = p.q_out + ((size_t)t * p.Hq + j) * D;
#pragma unroll
      for (int jj = 0; jj < J; ++jj) dst[lane + 32 * jj] = __float2bfloat16(v[jj]);
    } else if (slot >= 0 && kv_index_ok(slot, (long long)p.num_pages * p.page_size, p.status)) {
      const bool is_k = j < p.Hq + p.Hkv;
      const int h = is_k ? j - p.Hq : j - p.Hq - p.Hkv;
      const int fmt = is_k ? p.fmt_k : p.fmt_v;
      const int page = slot / p.page_size, off = slot % p.page_size;
      const size_t rowid = ((size_t)page * p.Hkv + h) * p.page_size + off;
      uint8_t* codes = (is_k ? p.k_codes : p.v_codes) + rowid * kv_code_bytes(fmt, D);
      __half* scales = (is_k ? p.k_scales : p.v_scales) + rowid * kv_nscale(fmt, D, p.group);
      quant_row<D>(v, fmt, p.group, codes, scales);
    }
  }
}

// One CTA (128 threads) per row, the row held in registers (H % 8 == 0, H <= 8192):
// y[i] = x[row_idx[i]] * rsqrt(mean(x^2) + eps) * w.
template <int MAXV>
__global__ void __launch_bounds__(128) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      __nv_bfloat16* __restrict__ y, const int* __restrict__ row_idx,
                                                      int rows, int H, int ldx, int ldy, float eps) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[4];
  const int r = blockIdx.x;
  const int src = row_idx ? row_idx[r] : r;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)src * ldx);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)r * ldy);
  const int nv = H / 8;
  uint4 v[MAXV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int idx = threadIdx.x + i * 128;
    if (idx < nv) {
      v[i] = xr[idx];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = red[0] + red[1] + red[2] + red[3];
  const float inv = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int idx = threadIdx.x + i * 128;
    if (idx < nv) {
      const uint4 wu = wr[idx];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[i]);
      const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&wu);
      uint4 o;
      uint32_t* oo = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        const float2 gw = __bfloat1622float2(g[k]);
        __nv_bfloat162 r2 = __floats2bfloat162_rn(f.x * inv * gw.x, f.y * inv * gw.y);
        oo[k] = *reinterpret_cast<uint32_t*>(&r2);
      }
      yr[idx] = o;
    }
  }
}

}  // namespace

cudaError_t rope_kv_write_launch(const RopeKvParams& p, int T, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  const int threads = 128;
  const dim3 grid(T, (p.Hq + 2 * p.Hkv + 3) / 4);
  switch (p.D) {
    case 32: SQ_LAUNCH(rope_kv_write_kernel<32>, dim3(grid), dim3(threads), 0, s, 1, p); break;
    case 64: SQ_LAUNCH(rope_kv_write_kernel<64>, dim3(grid), dim3(threads), 0, s, 1, p); break;
    case 128: SQ_LAUNCH(rope_kv_write_kernel<128>, dim3(grid), dim3(threads), 0, s, 1, p); break;
    case 256: SQ_LAUNCH(rope_kv_write_kernel<256>, dim3(grid), dim3(threads), 0, s, 1, p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t rmsnorm_launch(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, const int* row_idx,
                           int rows, int H, int ldx, int ldy, float eps, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const int nv = H / 8;
  if (nv <= 128) SQ_LAUNCH(rmsnorm_kernel<1>, dim3(rows), dim3(128), 0, s, 1, x, w, y, row_idx, rows, H, ldx, ldy, eps);
  else if (nv <= 256) SQ_LAUNCH(rmsnorm_kernel<2>, dim3(rows), dim3(128), 0, s, 1, x, w, y, row_idx, rows, H, ldx, ldy, eps);
  else if (nv <= 512) SQ_LAUNCH(rmsnorm_kernel<4>, dim3(rows), dim3(128), 0, s, 1, x, w, y, row_idx, rows, H, ldx, ldy, eps);
  else if (nv <= 1024) SQ_LAUNCH(rmsnorm_kernel<8>, dim3(rows), dim3(128), 0, s, 1, x, w, y, row_idx, rows, H, ldx, ldy, eps);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace sq
