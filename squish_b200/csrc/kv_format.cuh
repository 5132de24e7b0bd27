// kv_format.cuh — quantized KV page formats shared by the KV-write and attention kernels.
//
// A layer's KV cache is two code pools and two scale pools:
//   codes  [num_pages][Hkv][page_size][code_bytes]     uint8
//   scales [num_pages][Hkv][page_size][n_scale]        fp16
// one row per (page, kv head, token slot). Formats follow the reference codecs:
//   KV_INT4 : symmetric 16 levels, x = (idx - 7.5) * absmax/7.5 per (token, head, group)
//             (squish/kv/kv_cache.py:297-375, generalised from whole-head to group G)
//   KV_INT2 : symmetric 4 levels {-1.5,-0.5,0.5,1.5} * absmax/1.5 (kv_cache.py:159-240)
//   KV_INT8 : symmetric, x = q * absmax/127 (kv_cache.py:78-119)
//   KV_K8 / KV_V4 : the k8v4 codec, asymmetric affine per group, keys 8-bit (255 levels),
//             values 4-bit (15 levels), scale = (hi-lo)/qmax, zero = lo (squish/kv/k8v4_codec.py:64-137)
//   KV_BF16 : unquantized bf16.
// Nibble order: low nibble = even dim (as in the reference packers); 2-bit: dim 4i+j at bits 2j.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace sq {

enum KvFmt : int { KV_BF16 = 0, KV_INT8 = 1, KV_INT4 = 2, KV_INT2 = 3, KV_K8 = 4, KV_V4 = 5 };

__host__ __device__ constexpr int kv_bits(int f) {
  return f == KV_BF16 ? 16 : (f == KV_INT8 || f == KV_K8) ? 8 : (f == KV_INT4 || f == KV_V4) ? 4 : 2;
}
__host__ __device__ constexpr bool kv_asym(int f) { return f == KV_K8 || f == KV_V4; }
__host__ __device__ constexpr int kv_code_bytes(int f, int D) { return D * kv_bits(f) / 8; }
__host__ __device__ constexpr int kv_nscale(int f, int D, int G) {
  return f == KV_BF16 ? 0 : (D / G) * (kv_asym(f) ? 2 : 1);
}
__host__ __device__ constexpr float kv_qmax(int f) {
  return f == KV_INT8 ? 127.f : f == KV_INT4 ? 7.5f : f == KV_INT2 ? 1.5f : f == KV_K8 ? 255.f : 15.f;
}

// KV pool index check shared by the kernels that read or write pages: true when `idx` lies in
// [0, limit); otherwise the first failing thread records SQ_ERR_BOUNDS (6, sm100.cuh) in
// *status and the caller skips the access. limit <= 0 disables the check.
__device__ __forceinline__ bool kv_index_ok(long long idx, long long limit, int* status) {
  if (limit <= 0 || (idx >= 0 && idx < limit)) return true;
  if (status != nullptr) atomicCAS(status, 0, 6);
  return false;
}

struct KvLayer {
  const uint8_t* codes;
  const __half* scales;
};

__device__ __forceinline__ uint32_t bf2u(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// Dequantize 8 consecutive dims [d8, d8+8) of one (page, head, token) row into 8 bf16.
template <int FMT>
__device__ __forceinline__ uint4 kv_dequant8(const uint8_t* __restrict__ row_codes,
                                             const __half* __restrict__ row_scales, int d8, int G) {
  if constexpr (FMT == KV_BF16) {
    return *reinterpret_cast<const uint4*>(row_codes + d8 * 2);
  } else if constexpr (FMT == KV_INT4 || FMT == KV_V4) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(row_codes + d8 / 2);
    const int g = d8 / G;
    float s, z;
    if constexpr (FMT == KV_INT4) {
      s = __half2float(row_scales[g]);
      z = -7.5f * s;
    } else {
      s = __half2float(row_scales[2 * g]);
      z = __half2float(row_scales[2 * g + 1]);
    }
    const __nv_bfloat162 s2 = __floats2bfloat162_rn(s, s), z2 = __floats2bfloat162_rn(z, z);
    const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t b = (w >> (8 * i)) & 0xFFu;
      uint32_t t = (b & 0xFu) | ((b >> 4) << 16) | 0x43004300u;
      __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t);
      v = __hfma2(__hsub2(v, k128), s2, z2);
      o[i] = bf2u(v);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  } else if constexpr (FMT == KV_INT2) {
    const uint32_t w = *reinterpret_cast<const uint16_t*>(row_codes + d8 / 4);
    const float s = __half2float(row_scales[d8 / G]);
    const __nv_bfloat162 s2 = __floats2bfloat162_rn(s, s), z2 = __floats2bfloat162_rn(-1.5f * s, -1.5f * s);
    const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = (w >> (4 * i)) & 0x3u, hi = (w >> (4 * i + 2)) & 0x3u;
      uint32_t t = lo | (hi << 16) | 0x43004300u;
      __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t);
      v = __hfma2(__hsub2(v, k128), s2, z2);
      o[i] = bf2u(v);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  } else {  // KV_INT8 (signed) or KV_K8 (unsigned, asymmetric)
    const uint2 w = *reinterpret_cast<const uint2*>(row_codes + d8);
    const int g = d8 / G;
    float s, z;
    if constexpr (FMT == KV_INT8) {
      s = __half2float(row_scales[g]);
      z = 0.f;
    } else {
      s = __half2float(row_scales[2 * g]);
      z = __half2float(row_scales[2 * g + 1]);
    }
    const uint32_t ww[2] = {w.x, w.y};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t word = ww[i >> 1];
      const int sh = (i & 1) * 16;
      float a, b;
      if constexpr (FMT == KV_INT8) {
        a = (float)(int8_t)((word >> sh) & 0xFF);
        b = (float)(int8_t)((word >> (sh + 8)) & 0xFF);
      } else {
        a = (float)((word >> sh) & 0xFF);
        b = (float)((word >> (sh + 8)) & 0xFF);
      }
      o[i] = bf2u(__floats2bfloat162_rn(fmaf(a, s, z), fmaf(b, s, z)));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Raw (still quantized) codes and scales of one contiguous part (D/P dims) of one
// (page, head, token) row, held in registers so the load of the next tile can be in
// flight while the current one is computed; dequant() turns 8 dims into 8 bf16.
// Requires a KV group size >= 32 (so a part holds at most D/P/32 scale groups).
template <int D, int FMT, int P>
struct RowPart {
  static constexpr int DIMS = D / P;
  static constexpr int BYTES = DIMS * kv_bits(FMT) / 8;
  static constexpr int WORDS = BYTES / 4;
  static constexpr int CHUNKS = DIMS / 8;
  static constexpr int NG = DIMS >= 32 ? DIMS / 32 : 1;
  static_assert(BYTES % 4 == 0, "row part must be a whole number of 32-bit words");
  static constexpr int NZ = kv_asym(FMT) ? NG : 1;  // symmetric formats derive the zero from the scale
  uint32_t w[WORDS];
  float s[NG], z[NZ];

  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int i = 0; i < WORDS; ++i) w[i] = 0u;
#pragma unroll
    for (int i = 0; i < NG; ++i) s[i] = 0.f;
#pragma unroll
    for (int i = 0; i < NZ; ++i) z[i] = 0.f;
  }

  // NC: read-only global loads (__ldg); false: generic loads (e.g. a shared-memory staging copy)
  template <bool NC = true, class T>
  static __device__ __forceinline__ T ld(const T* p) {
    if constexpr (NC) return __ldg(p);
    else return *p;
  }

  template <bool NC = true>
  __device__ __forceinline__ void load(const uint8_t* __restrict__ row_codes, const __half* __restrict__ row_scales,
                                       int part, int G) {
    const uint8_t* src = row_codes + part * BYTES;
    if constexpr (BYTES % 16 == 0 && (D * kv_bits(FMT) / 8) % 16 == 0) {
#pragma unroll
      for (int i = 0; i < WORDS / 4; ++i) {
        const uint4 v = ld<NC>(reinterpret_cast<const uint4*>(src) + i);
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < WORDS; ++i) w[i] = ld<NC>(reinterpret_cast<const uint32_t*>(src) + i);
    }
    if constexpr (FMT != KV_BF16) {
      // scale groups of this part: DIMS / G of them (one, shared with the neighbour part,
      // when the group is wider than the part)
      const int ng = DIMS >= G ? DIMS / G : 1;
#pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        if (gi >= ng) break;
        const int g = (part * DIMS) / G + gi;
        if constexpr (kv_asym(FMT)) {
          s[gi] = __half2float(ld<NC>(row_scales + 2 * g));
          z[gi] = __half2float(ld<NC>(row_scales + 2 * g + 1));
        } else {
          s[gi] = __half2float(ld<NC>(row_scales + g));
        }
      }
    }
  }

  // 8 dims starting at c*8 within the part -> 8 bf16
  __device__ __forceinline__ uint4 dequant(int c, int G) const {
    if constexpr (FMT == KV_BF16) {
      return make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    } else {
      const int gi = (NG == 1 || DIMS < G) ? 0 : (c * 8) / G;
      // select, not index: a runtime index would move s[] / z[] to local memory
      float sc = s[0], ze = z[0];
#pragma unroll
      for (int i = 1; i < NG; ++i)
        if (gi == i) {
          sc = s[i];
          if constexpr (kv_asym(FMT)) ze = z[i];
        }
      if constexpr (!kv_asym(FMT)) ze = (FMT == KV_INT4) ? -7.5f * sc : (FMT == KV_INT2) ? -1.5f * sc : 0.f;
      if constexpr (FMT == KV_INT4 || FMT == KV_V4 || FMT == KV_INT2) {
        const __nv_bfloat162 s2 = __floats2bfloat162_rn(sc, sc), z2 = __floats2bfloat162_rn(ze, ze);
        const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
        uint32_t o[4];
        if constexpr (FMT == KV_INT2) {
          const uint32_t word = (w[c >> 1] >> ((c & 1) * 16)) & 0xFFFFu;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t lo = (word >> (4 * i)) & 0x3u, hi = (word >> (4 * i + 2)) & 0x3u;
            uint32_t t = lo | (hi << 16) | 0x43004300u;
            __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t);
            o[i] = bf2u(__hfma2(__hsub2(v, k128), s2, z2));
          }
        } else {
          const uint32_t word = w[c];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint32_t b = (word >> (8 * i)) & 0xFFu;
            uint32_t t = (b & 0xFu) | ((b >> 4) << 16) | 0x43004300u;
            __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t);
            o[i] = bf2u(__hfma2(__hsub2(v, k128), s2, z2));
          }
        }
        return make_uint4(o[0], o[1], o[2], o[3]);
      } else {  // 8-bit: KV_INT8 signed symmetric, KV_K8 unsigned asymmetric
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t word = w[2 * c + (i >> 1)];
          const int sh = (i & 1) * 16;
          float a, b;
          if constexpr (FMT == KV_INT8) {
            a = (float)(int8_t)((word >> sh) & 0xFF);
            b = (float)(int8_t)((word >> (sh + 8)) & 0xFF);
          } else {
            a = (float)((word >> sh) & 0xFF);
            b = (float)((word >> (sh + 8)) & 0xFF);
          }
          o[i] = bf2u(__floats2bfloat162_rn(fmaf(a, sc, ze), fmaf(b, sc, ze)));
        }
        return make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }

  __device__ __forceinline__ void store(__nv_bfloat16* dst, int G) const {
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) *reinterpret_cast<uint4*>(dst + c * 8) = dequant(c, G);
  }
};

}  // namespace sq
