// hadamard.cu — randomized block Walsh–Hadamard rotation of activation rows.
//
// y[r, blk*b + i] = (1/sqrt(b)) * sum_j H_b[i, j] * s[blk*b + j] * x[r, blk*b + j]
// with H_b the Sylvester-ordered Hadamard matrix of size b (a power of two) and s a +-1 sign
// vector: the input side of an SQINT2 linear layer, whose weights were stored rotated by the
// same orthogonal map (W_rot = W R^T, so W x = W_rot (R x)). The reference rotates with dense
// matrices in NumPy at load time (squish/quant/sqint2.py:384-470); here the rotation is an
// O(b log b) butterfly per block applied to the activations, so the weights stay 2-bit.
//
// One CTA per (block, row): the b values (times their signs) go to shared memory in fp32,
// log2(b) butterfly stages run with a barrier between stages, and the scaled result is stored
// as bf16. Up to 4096-wide blocks (16 KiB of shared memory).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

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

}  // namespace

cudaError_t hadamard_rows_launch(const __nv_bfloat16* x, int ldx, __nv_bfloat16* y, int ldy, const float* signs,
                                 int M, int K, int b, cudaStream_t s) {
  if (M == 0 || K == 0) return cudaSuccess;
  if (b < 2 || b > 4096 || (b & (b - 1)) != 0 || K % b != 0) return cudaErrorInvalidValue;
  const dim3 grid(K / b, M);
  const int threads = b / 2 < 512 ? b / 2 : 512;
  SQ_LAUNCH(hadamard_rows_kernel, grid, dim3(threads), sizeof(float) * (size_t)b, s, 1, x, ldx, y, ldy, signs, b,
            1.0f / sqrtf((float)b));
  return cudaGetLastError();
}

}  // namespace sq
