// kmeans.cu — convert-time vector quantization on the GPU: Lloyd k-means (AQLM codebooks,
// product quantization, vector k-means) and product-quantization ADC scoring.
//
// The reference runs these on the CPU with Rayon (squish_quant_rs/src/lib.rs:1836-1960:
// pq_kmeans_fit, pq_encode_batch, pq_adc_search; aqlm_kmeans_f32 at 4858). Here:
//   assign:   one thread per vector, its D values in registers; centroids stream through
//             shared memory in tiles and every thread of a warp reads the same centroid word
//             (a broadcast); squared L2 distance, the lowest index wins ties. Optionally counts
//             the vectors whose assignment changed (Lloyd's stopping test).
//   update:   per-block partial sums and counts in shared memory when k x D fits, flushed with
//             one atomic per entry; global atomics otherwise. Empty clusters keep their centroid.
//   ADC:      the [M, K] lookup table of query-subvector-to-centroid distances in shared
//             memory; one thread per database vector sums its M table entries.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace sq {

namespace {

constexpr int kSmemFloats = 12288;  // 48 KiB of centroids per tile

template <int D>
__global__ void __launch_bounds__(256) kmeans_assign_kernel(const float* __restrict__ x, int n,
                                                            const float* __restrict__ c, int k,
                                                            int* __restrict__ assign, float* __restrict__ dist,
                                                            int* __restrict__ changed) {
  extern __shared__ float sc[];
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  float xv[D];
#pragma unroll
  for (int e = 0; e < D; ++e) xv[e] = i < n ? x[(size_t)i * D + e] : 0.f;
  float best = INFINITY;
  int bi = 0;
  const int tile = kSmemFloats / D;
  for (int t0 = 0; t0 < k; t0 += tile) {
    const int tn = min(tile, k - t0);
    __syncthreads();
    for (int j = threadIdx.x; j < tn * D; j += blockDim.x) sc[j] = c[(size_t)t0 * D + j];
    __syncthreads();
    for (int j = 0; j < tn; ++j) {
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < D; ++e) {
        const float df = xv[e] - sc[j * D + e];
        d = fmaf(df, df, d);
      }
      if (d < best) {
        best = d;
        bi = t0 + j;
      }
    }
  }
  if (i < n) {
    if (changed != nullptr && assign[i] != bi) atomicAdd(changed, 1);
    assign[i] = bi;
    if (dist != nullptr) dist[i] = best;
  }
}

// rows [blockIdx.x * per_block, ...) accumulated into shared partials, then flushed
__global__ void __launch_bounds__(256) kmeans_accum_smem_kernel(const float* __restrict__ x, int n, int d,
                                                                const int* __restrict__ assign, int k,
                                                                float* __restrict__ sums, int* __restrict__ counts,
                                                                int per_block) {
  extern __shared__ float ps[];
  int* pc = reinterpret_cast<int*>(ps + (size_t)k * d);
  for (int j = threadIdx.x; j < k * d; j += blockDim.x) ps[j] = 0.f;
  for (int j = threadIdx.x; j < k; j += blockDim.x) pc[j] = 0;
  __syncthreads();
  const long r0 = (long)blockIdx.x * per_block, r1 = min((long)n, r0 + per_block);
  for (long t = r0 * d + threadIdx.x; t < r1 * d; t += blockDim.x) {
    const long i = t / d;
    const int e = (int)(t - i * d);
    const int a = assign[i];
    atomicAdd(&ps[a * d + e], x[t]);
    if (e == 0) atomicAdd(&pc[a], 1);
  }
  __syncthreads();
  for (int j = threadIdx.x; j < k * d; j += blockDim.x)
    if (ps[j] != 0.f) atomicAdd(&sums[j], ps[j]);
  for (int j = threadIdx.x; j < k; j += blockDim.x)
    if (pc[j] != 0) atomicAdd(&counts[j], pc[j]);
}

__global__ void kmeans_accum_global_kernel(const float* __restrict__ x, int n, int d, const int* __restrict__ assign,
                                           float* __restrict__ sums, int* __restrict__ counts) {
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long)n * d) return;
  const long i = t / d;
  const int e = (int)(t - i * d);
  const int a = assign[i];
  atomicAdd(&sums[(size_t)a * d + e], x[t]);
  if (e == 0) atomicAdd(&counts[a], 1);
}

__global__ void kmeans_finalize_kernel(float* __restrict__ c, const float* __restrict__ sums,
                                       const int* __restrict__ counts, int k, int d) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= k * d) return;
  const int cnt = counts[t / d];
  if (cnt > 0) c[t] = sums[t] / (float)cnt;
}

__global__ void __launch_bounds__(256) pq_adc_kernel(const uint8_t* __restrict__ codes, int n, int m,
                                                     const float* __restrict__ lut, int k, float* __restrict__ out) {
  extern __shared__ float sl[];
  for (int j = threadIdx.x; j < m * k; j += blockDim.x) sl[j] = lut[j];
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint8_t* ci = codes + (size_t)i * m;
  float s = 0.f;
  for (int j = 0; j < m; ++j) s += sl[j * k + ci[j]];
  out[i] = s;
}

}  // namespace

cudaError_t kmeans_assign_launch(const float* x, int n, int d, const float* c, int k, int* assign, float* dist,
                                 int* changed, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  const size_t smem = sizeof(float) * (size_t)(kSmemFloats / d) * d;
  switch (d) {
    case 1: kmeans_assign_kernel<1><<<blocks, 256, smem, s>>>(x, n, c, k, assign, dist, changed); break;
    case 2: kmeans_assign_kernel<2><<<blocks, 256, smem, s>>>(x, n, c, k, assign, dist, changed); break;
    case 4: kmeans_assign_kernel<4><<<blocks, 256, smem, s>>>(x, n, c, k, assign, dist, changed); break;
    case 8: kmeans_assign_kernel<8><<<blocks, 256, smem, s>>>(x, n, c, k, assign, dist, changed); break;
    case 16: kmeans_assign_kernel<16><<<blocks, 256, smem, s>>>(x, n, c, k, assign, dist, changed); break;
    case 32: kmeans_assign_kernel<32><<<blocks, 256, smem, s>>>(x, n, c, k, assign, dist, changed); break;
    case 64: kmeans_assign_kernel<64><<<blocks, 256, smem, s>>>(x, n, c, k, assign, dist, changed); break;
    default: return cudaErrorInvalidValue;  // callers zero-pad to a supported width
  }
  return cudaGetLastError();
}

cudaError_t kmeans_update_launch(const float* x, int n, int d, const int* assign, float* c, int k, float* sums,
                                 int* counts, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(sums, 0, sizeof(float) * (size_t)k * d, s);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(counts, 0, sizeof(int) * (size_t)k, s);
  if (e != cudaSuccess) return e;
  const size_t part = sizeof(float) * (size_t)k * d + sizeof(int) * (size_t)k;
  if (n > 0) {
    if (part <= 48 * 1024) {
      const int per_block = 4096;
      const unsigned blocks = (unsigned)((n + per_block - 1) / per_block);
      kmeans_accum_smem_kernel<<<blocks, 256, part, s>>>(x, n, d, assign, k, sums, counts, per_block);
    } else {
      const long total = (long)n * d;
      kmeans_accum_global_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(x, n, d, assign, sums, counts);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  kmeans_finalize_kernel<<<(unsigned)((k * d + 255) / 256), 256, 0, s>>>(c, sums, counts, k, d);
  return cudaGetLastError();
}

cudaError_t pq_adc_launch(const uint8_t* codes, int n, int m, const float* lut, int k, float* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if ((size_t)m * k > (size_t)kSmemFloats) return cudaErrorInvalidValue;
  pq_adc_kernel<<<(unsigned)((n + 255) / 256), 256, sizeof(float) * (size_t)m * k, s>>>(codes, n, m, lut, k, out);
  return cudaGetLastError();
}

}  // namespace sq
