// hadamard.cu — randomized block Walsh–Hadamard rotation of activation rows.
//
// y[r, blk*b + i] = (1/sqrt(b)) * sum_j H_b[i, j] * s[blk*b + j] * x[r, blk*b + j]
// with H_b the Sylvester-ordered Hadamard matrix of size b (a power of two) and s a +-1 sign
// vector: the input side of an SQINT2 linear layer, whose weights were stored rotated by the
// same orthogonal map (W_rot = W R^T, so W x = W_rot (R x)). The reference rotates with dense
// matrices in NumPy at load time (squish/quant/sqint2.py:384-470); here the rotation is an
// O(b log b) butterfly per block applied to the activations, so the weights stay 2-bit.
//
// 512-wide blocks (the SQINT2 block of 3584- and 18944-wide inputs): see hadamard512_kernel.
// Other blocks up to 1024 wide: one warp per (row, block). Lane l holds the b/32 consecutive values
// l*b/32 .. (l+1)*b/32 - 1 in registers: the butterfly stages over the low index bits run inside
// each lane, the stages over the high (lane) bits exchange registers with __shfl_xor_sync --
// no shared memory, no barriers; loads and stores are 16-byte vectors covering the block.
// Wider blocks (2048, 4096) use a shared-memory CTA per (block, row).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"
#include "launch.cuh"

namespace sq {

namespace {

__global__ void __launch_bounds__(512) hadamard_rows_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                            __nv_bfloat16* __restrict__ y, int ldy,
                                                            const float* __restrict__ signs, int b, float scale) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float v[];
  const int blk = blockIdx.x, row = blockIdx.y;
  const int nt = blockDim.x, tid = threadIdx.x;
  const __nv_bfloat16* xr = x + (size_t)row * ldx + (size_t)blk * b;
  const float* sr = signs + (size_t)blk * b;
  for (int i = tid; i < b; i += nt) v[i] = __bfloat162float(xr[i]) * sr[i];
  __syncthreads();
  for (int h = 1; h < b; h <<= 1) {
    for (int p = tid; p < (b >> 1); p += nt) {
      const int i = (p / h) * (h << 1) + (p % h);
      const float a = v[i], c = v[i + h];
      v[i] = a + c;
      v[i + h] = a - c;
    }
    __syncthreads();
  }
  __nv_bfloat16* yr = y + (size_t)row * ldy + (size_t)blk * b;
  for (int i = tid; i < b; i += nt) yr[i] = __float2bfloat16(v[i] * scale);
}

template <int VPL>  // values per lane: b = 32 * VPL
__global__ void __launch_bounds__(256) hadamard_warp_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                            __nv_bfloat16* __restrict__ y, int ldy,
                                                            const float* __restrict__ signs, int nblk, int rows,
                                                            float scale) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long w = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= (long)rows * nblk) return;  // uniform per warp
  const int row = (int)(w / nblk), blk = (int)(w % nblk);
  const int col0 = blk * 32 * VPL + lane * VPL;
  const __nv_bfloat16* xr = x + (size_t)row * ldx + col0;
  float v[VPL];
  if constexpr (VPL >= 8) {
#pragma unroll
    for (int c = 0; c < VPL / 8; ++c) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + 8 * c);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        v[8 * c + 2 * e] = f.x;
        v[8 * c + 2 * e + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int r = 0; r < VPL; ++r) v[r] = __bfloat162float(xr[r]);
  }
#pragma unroll
  for (int r = 0; r < VPL; ++r) v[r] *= signs[col0 + r];
#pragma unroll
  for (int h = 1; h < VPL; h <<= 1) {
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (i & h) continue;
      const float a = v[i], c = v[i + h];
      v[i] = a + c;
      v[i + h] = a - c;
    }
  }
#pragma unroll
  for (int hl = 1; hl < 32; hl <<= 1) {
    const bool upper = lane & hl;
#pragma unroll
    for (int r = 0; r < VPL; ++r) {
      const float o = __shfl_xor_sync(0xffffffffu, v[r], hl);
      v[r] = upper ? o - v[r] : v[r] + o;
    }
  }
  __nv_bfloat16* yr = y + (size_t)row * ldy + col0;
  if constexpr (VPL >= 8) {
#pragma unroll
    for (int c = 0; c < VPL / 8; ++c) {
      uint4 u;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * c + 2 * e] * scale, v[8 * c + 2 * e + 1] * scale);
      *reinterpret_cast<uint4*>(yr + 8 * c) = u;
    }
  } else {
#pragma unroll
    for (int r = 0; r < VPL; ++r) yr[r] = __float2bfloat16(v[r] * scale);
  }
}

// b = 512: lane L holds i = L*16 + r for bits 0-3 in registers; a padded shared-memory transpose
// (address i + i/16: both access patterns below hit 32 distinct banks) gives lane L = b8*16 + l4
// the values i = b8*256 + r*16 + l4, so bits 4-7 are in registers too and only bit 8 (lane bit 4)
// needs a shuffle: 16 shuffles per lane instead of 80. A second transpose restores the
// contiguous layout for 16-byte stores.
__global__ void __launch_bounds__(256) hadamard512_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                          __nv_bfloat16* __restrict__ y, int ldy,
                                                          const float* __restrict__ signs, int nblk, int rows,
                                                          float scale) {
  pdl_wait();
  pdl_trigger();
  __shared__ float sbuf[8][544];
  const int lane = threadIdx.x & 31, wi = threadIdx.x >> 5;
  const long w = (long)blockIdx.x * 8 + wi;
  if (w >= (long)rows * nblk) return;  // uniform per warp; no block-wide barriers below
  float* sb = sbuf[wi];
  const int row = (int)(w / nblk), blk = (int)(w % nblk);
  const int col0 = blk * 512 + lane * 16;
  const __nv_bfloat16* xr = x + (size_t)row * ldx + col0;
  float v[16];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + 8 * c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      v[8 * c + 2 * e] = f.x;
      v[8 * c + 2 * e + 1] = f.y;
    }
  }
  const float4* s4 = reinterpret_cast<const float4*>(signs + col0);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 sg = s4[c];
    v[4 * c] *= sg.x;
    v[4 * c + 1] *= sg.y;
    v[4 * c + 2] *= sg.z;
    v[4 * c + 3] *= sg.w;
  }
  auto butterfly16 = [&]() {
#pragma unroll
    for (int h = 1; h < 16; h <<= 1) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (i & h) continue;
        const float a = v[i], c = v[i + h];
        v[i] = a + c;
        v[i + h] = a - c;
      }
    }
  };
  butterfly16();  // index bits 0-3
#pragma unroll
  for (int r = 0; r < 16; ++r) sb[lane * 17 + r] = v[r];  // i = lane*16 + r at i + i/16
  __syncwarp();
  const int b8 = lane >> 4, l4 = lane & 15;
#pragma unroll
  for (int r = 0; r < 16; ++r) v[r] = sb[b8 * 272 + r * 17 + l4];  // i = b8*256 + r*16 + l4
  butterfly16();  // index bits 4-7
#pragma unroll
  for (int r = 0; r < 16; ++r) {  // index bit 8 = lane bit 4
    const float o = __shfl_xor_sync(0xffffffffu, v[r], 16);
    v[r] = b8 ? o - v[r] : v[r] + o;
  }
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 16; ++r) sb[b8 * 272 + r * 17 + l4] = v[r];
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 16; ++r) v[r] = sb[lane * 17 + r];
  __nv_bfloat16* yr = y + (size_t)row * ldy + col0;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[8 * c + 2 * e] * scale, v[8 * c + 2 * e + 1] * scale);
    *reinterpret_cast<uint4*>(yr + 8 * c) = u;
  }
}

template <int VPL>
cudaError_t launch_warp(const __nv_bfloat16* x, int ldx, __nv_bfloat16* y, int ldy, const float* signs, int M, int K,
                        cudaStream_t s) {
  const int b = 32 * VPL, nblk = K / b;
  const long warps = (long)M * nblk;
  const unsigned blocks = (unsigned)((warps + 7) / 8);
  SQ_LAUNCH(hadamard_warp_kernel<VPL>, dim3(blocks), dim3(256), 0, s, 1, x, ldx, y, ldy, signs, nblk, M,
            1.0f / sqrtf((float)b));
  return cudaGetLastError();
}

}  // namespace

cudaError_t hadamard_rows_launch(const __nv_bfloat16* x, int ldx, __nv_bfloat16* y, int ldy, const float* signs,
                                 int M, int K, int b, cudaStream_t s) {
  if (M == 0 || K == 0) return cudaSuccess;
  if (b < 2 || b > 4096 || (b & (b - 1)) != 0 || K % b != 0) return cudaErrorInvalidValue;
  // the register path needs 16-byte aligned rows for its vector accesses (from 256-wide blocks)
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0 &&
                      ldx % 8 == 0 && ldy % 8 == 0;
  switch (b) {
    case 32: return launch_warp<1>(x, ldx, y, ldy, signs, M, K, s);
    case 64: return launch_warp<2>(x, ldx, y, ldy, signs, M, K, s);
    case 128: return launch_warp<4>(x, ldx, y, ldy, signs, M, K, s);
    case 256: if (vec_ok) return launch_warp<8>(x, ldx, y, ldy, signs, M, K, s); break;
    case 512:
      if (vec_ok && (reinterpret_cast<uintptr_t>(signs) & 15) == 0) {
        const int nblk = K / 512;
        const long warps = (long)M * nblk;
        SQ_LAUNCH(hadamard512_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, s, 1, x, ldx, y, ldy, signs,
                  nblk, M, 1.0f / sqrtf(512.f));
        return cudaGetLastError();
      }
      if (vec_ok) return launch_warp<16>(x, ldx, y, ldy, signs, M, K, s);
      break;
    case 1024: if (vec_ok) return launch_warp<32>(x, ldx, y, ldy, signs, M, K, s); break;
    default: break;
  }
  const dim3 grid(K / b, M);
  const int threads = b / 2 < 512 ? b / 2 : 512;
  SQ_LAUNCH(hadamard_rows_kernel, grid, dim3(threads), sizeof(float) * (size_t)b, s, 1, x, ldx, y, ldy, signs, b,
            1.0f / sqrtf((float)b));
  return cudaGetLastError();
}

}  // namespace sq
