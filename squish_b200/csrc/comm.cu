// comm.cu — tensor-parallel collectives over NVLink peer memory (no NCCL on the hot path).
//
// Fused GEMM -> all-reduce (row-parallel o_proj / down_proj): the INT4 GEMM runs in push
// mode (w4a16_gemm.cu): each CTA stores its bf16 partial output tile straight into every
// rank's receive buffer slot for this source rank (P2P stores over NVLink) and bumps that
// tile's flag on every rank. tp_reduce (below) then runs on each rank: one CTA per GEMM
// output tile waits until the tile's flag from every source rank reached its expected
// count, sums the tp partials in rank order (the same order on every rank, so every rank
// holds bit-identical results), adds the residual and writes the hidden state in place.
// The transfer of early tiles overlaps the GEMM of later ones.
//
// Buffers alternate by parity (bit 0 of a device-side op counter) so a fast rank can push
// op s+1 while a slow one still reads op s; a rank can only reach op s+2 after every peer
// pushed op s+1, which each peer does only after finishing its read of op s. The consumer
// clears its flags after reading; the last CTA to finish advances the counter. Every wait
// is bounded: on timeout the status word gets SQ_ERR_TIMEOUT_PEER and the kernel goes on.
//
// tp_gather: each rank stores its column block (vocab shard of the logits) into every
// rank's full-width output (P2P stores), then bumps a per-source flag on every rank; a
// one-warp kernel waits for all sources. The output has no parity copy: between two
// gathers every rank passes at least one tp_reduce, which needs every peer's next push,
// which a peer issues only after it finished reading the previous gather's output.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

#include "comm.h"
#include "sm100.cuh"
#include "launch.cuh"

namespace sq {

namespace {

constexpr long long kPeerSpin = 1LL << 22;  // ~seconds of polling, then report and go on

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// wait until *f >= want (bounded); returns false on timeout
__device__ bool wait_flag(const int* f, int want, int* status) {
  for (long long i = 0; i < kPeerSpin; ++i) {
    if (ld_acquire_sys(f) >= want) return true;
    if ((i & 4095) == 4095 && *reinterpret_cast<volatile int*>(status) != 0) return false;
  }
  atomicCAS(status, 0, SQ_ERR_TIMEOUT_PEER);
  return false;
}

__global__ void __launch_bounds__(256) tp_reduce_kernel(const TpReduceParams p) {
  pdl_wait();
  pdl_trigger();
  const int tile = blockIdx.x * gridDim.y + blockIdx.y;  // same numbering as the GEMM grid
  const int par = *reinterpret_cast<volatile const int*>(p.seq) & 1;
  const int tp = p.tp;
  int* flags = p.flags + (size_t)par * p.flag_stride;
  if ((int)threadIdx.x < tp) wait_flag(flags + (size_t)threadIdx.x * p.flag_src_stride + tile, p.expect, p.status);
  __syncthreads();
  __threadfence();
  const int n0 = blockIdx.x * p.tile_n, m0 = blockIdx.y * p.tile_m;
  const int n1 = min(p.N, n0 + p.tile_n), m1 = min(p.M, m0 + p.tile_m);
  const __nv_bfloat16* recv = p.recv + (size_t)par * p.recv_stride;
  const int w = n1 - n0;
  // each thread handles pairs of columns
  for (int idx = threadIdx.x * 2; idx < (m1 - m0) * w; idx += blockDim.x * 2) {
    const int m = m0 + idx / w, n = n0 + idx % w;
    const bool two = (idx % w) + 1 < w;
    float a0 = 0.f, a1 = 0.f;
    for (int r = 0; r < tp; ++r) {
      const __nv_bfloat16* src = recv + (size_t)r * p.src_stride + (size_t)m * p.ld + n;
      a0 += __bfloat162float(src[0]);
      if (two) a1 += __bfloat162float(src[1]);
    }
    __nv_bfloat16* o = p.out + (size_t)m * p.ld_out + n;
    if (p.residual_in_out) {
      a0 += __bfloat162float(o[0]);
      if (two) a1 += __bfloat162float(o[1]);
    }
    o[0] = __float2bfloat16(a0);
    if (two) o[1] = __float2bfloat16(a1);
  }
  __syncthreads();
  if ((int)threadIdx.x < tp) flags[(size_t)threadIdx.x * p.flag_src_stride + tile] = 0;
  // the last CTA advances the op counter
  __shared__ int last;
  if (threadIdx.x == 0) {
    __threadfence();
    last = (atomicAdd(p.done, 1) == (int)(gridDim.x * gridDim.y) - 1);
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    *p.done = 0;
    __threadfence();
    atomicAdd(p.seq, 1);
  }
}

__global__ void __launch_bounds__(256) tp_push_kernel(const TpPushParams p) {
  pdl_wait();
  pdl_trigger();
  const int par = *reinterpret_cast<volatile const int*>(p.seq) & 1;
  const int n0 = blockIdx.x * 128, m0 = blockIdx.y * p.tile_m;
  const int n1 = min(p.N, n0 + 128), m1 = min(p.M, m0 + p.tile_m);
  const int w = n1 - n0;
  for (int idx = threadIdx.x; idx < (m1 - m0) * w; idx += blockDim.x) {
    const int m = m0 + idx / w, n = n0 + idx % w;
    const __nv_bfloat16 v = p.src[(size_t)m * p.ld_src + n];
    for (int r = 0; r < p.tp; ++r) p.dst[r][(size_t)par * p.parity_stride + (size_t)m * p.ld_dst + n] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int tile = blockIdx.x * gridDim.y + blockIdx.y;
    for (int r = 0; r < p.tp; ++r) {
      int* f = p.flags[r] + (size_t)par * p.flag_stride + tile;
      asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(f), "r"(1) : "memory");
    }
  }
}

// src [rows, cols] is written into every rank's dst at rows row0.., columns col0..
__global__ void __launch_bounds__(256) tp_gather_push_kernel(const TpGatherParams p) {
  pdl_wait();
  pdl_trigger();
  const int par = __ldg(p.seq) & 1;
  const int vec = p.cols / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < p.rows * vec; i += gridDim.x * blockDim.x) {
    const int r = i / vec, c = i % vec;
    const uint4 v = reinterpret_cast<const uint4*>(p.src + (size_t)r * p.ld_src)[c];
    for (int k = 0; k < p.tp; ++k)
      reinterpret_cast<uint4*>(p.dst[k] + (size_t)(p.row0 + r) * p.ld_dst + p.col0)[c] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int k = 0; k < p.tp; ++k) {
      int* f = p.flags[k] + (size_t)par * p.flag_stride + p.rank;
      asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(f), "r"(1) : "memory");
    }
}

__global__ void tp_gather_wait_kernel(const TpGatherParams p) {
  pdl_wait();
  pdl_trigger();
  const int par = __ldg(p.seq) & 1;
  int* flags = p.local_flags + (size_t)par * p.flag_stride;
  if ((int)threadIdx.x < p.tp) {
    wait_flag(flags + threadIdx.x, p.expect, p.status);
    flags[threadIdx.x] = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.seq, 1);
  }
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 t = __bfloat1622float2(h[k]);
    f[2 * k] = t.x;
    f[2 * k + 1] = t.y;
  }
}

// One CTA per owned row (grid = rows_per_rank on every rank, so every source signals the same
// count); the row lives in registers, kRsNormMaxChunks chunks of 8 columns per thread.
__global__ void __launch_bounds__(1024) tp_rs_norm_ag_kernel(const TpRsNormParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  const int par = *reinterpret_cast<volatile const int*>(p.seq) & 1;
  int* flags = p.rs_flags + par * p.tp;
  if ((int)threadIdx.x < p.tp) wait_flag(flags + threadIdx.x, p.rs_expect, p.status);
  __syncthreads();
  __threadfence();
  const int lr = blockIdx.x;
  const int own = min(p.rows_per_rank, p.T - p.rank * p.rows_per_rank);
  if (lr < own) {  // (uniform over the CTA)
    const int m = p.rank * p.rows_per_rank + lr;
    __nv_bfloat16* hr = p.h + (size_t)m * p.ldh;
    float v[kRsNormMaxChunks][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kRsNormMaxChunks; ++k) {
      const int c = (threadIdx.x + k * blockDim.x) * 8;
      if (c >= p.N) break;
      float t[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(hr + c), v[k]);  // residual + partials in source order
      for (int s2 = 0; s2 < p.tp; ++s2) {
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(p.recv + s2 * p.src_stride + (size_t)lr * p.ld_recv + c), t);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] += t[e];
      }
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o2[e] = __floats2bfloat162_rn(v[k][2 * e], v[k][2 * e + 1]);
        const float2 r2 = __bfloat1622float2(o2[e]);  // the norm sees the stored (rounded) values
        v[k][2 * e] = r2.x;
        v[k][2 * e + 1] = r2.y;
        ss += r2.x * r2.x + r2.y * r2.y;
      }
      *reinterpret_cast<uint4*>(hr + c) = o;
    }
    ss = warp_sum_f(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = (int)threadIdx.x < (int)(blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      t = warp_sum_f(t);
      if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(red[0] / (float)p.N + p.eps);
#pragma unroll
    for (int k = 0; k < kRsNormMaxChunks; ++k) {
      const int c = (threadIdx.x + k * blockDim.x) * 8;
      if (c >= p.N) break;
      float g[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(p.w + c), g);
      uint4 o;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o2[e] = __floats2bfloat162_rn(v[k][2 * e] * inv * g[2 * e], v[k][2 * e + 1] * inv * g[2 * e + 1]);
      if (p.local_only)
        *reinterpret_cast<uint4*>(p.ag_dst[p.rank] + (size_t)m * p.ld_ag + c) = o;
      else
        for (int r = 0; r < p.tp; ++r) *reinterpret_cast<uint4*>(p.ag_dst[r] + (size_t)m * p.ld_ag + c) = o;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!p.local_only)
      for (int r = 0; r < p.tp; ++r)
        asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p.ag_flags[r]), "r"(1) : "memory");
    __threadfence();
    if (atomicAdd(p.done, 1) == (int)gridDim.x - 1) {
      for (int s2 = 0; s2 < p.tp; ++s2) flags[s2] = 0;
      *p.done = 0;
      __threadfence();
      atomicAdd(p.seq, 1);
    }
  }
}

// chunk of CTA b: 8-element vectors [b * per, (b + 1) * per) of the row-major [M, N] output
__global__ void __launch_bounds__(kOneshotThreads) tp_oneshot_kernel(const TpOneshotParams p) {
  pdl_wait();  // the partial (previous kernel) is complete
  pdl_trigger();
  const int s = *reinterpret_cast<volatile const int*>(p.seq);
  const int par = s & 1, val = s + 1;
  const int vecs_row = p.N / 8;
  const long long total = (long long)p.M * vecs_row;
  const long long per = (total + gridDim.x - 1) / gridDim.x;
  const long long v0 = blockIdx.x * per, v1 = min(total, v0 + per);
  __nv_bfloat16* mine = p.part[p.rank] + (size_t)par * p.par_stride;
  for (long long v = v0 + threadIdx.x; v < v1; v += blockDim.x) {  // own chunk into the peer-visible slot
    const int m = (int)(v / vecs_row), n = (int)(v % vecs_row) * 8;
    *reinterpret_cast<uint4*>(mine + (size_t)m * p.N + n) =
        *reinterpret_cast<const uint4*>(p.src + (size_t)m * p.ld_src + n);
  }
  // The CTA barrier orders every thread's chunk stores before the publishing threads'
  // system-scope release stores (release is cumulative), so no per-thread system fence.
  __syncthreads();
  const int b = blockIdx.x;
  if ((int)threadIdx.x < p.tp) {  // publish chunk b on every rank, then wait for every peer's
    int* f = p.flags[threadIdx.x] + b * p.tp + p.rank;
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f), "r"(val) : "memory");
    wait_flag(p.flags[p.rank] + b * p.tp + threadIdx.x, val, p.status);
  }
  __syncthreads();
  for (long long v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const int m = (int)(v / vecs_row), n = (int)(v % vecs_row) * 8;
    float acc[8], t[8];
    __nv_bfloat16* o = p.out + (size_t)m * p.ld_out + n;
    if (p.residual_in_out) {
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(o), acc);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.f;
    }
    for (int r = 0; r < p.tp; ++r) {  // rank order: the same sum on every rank
      // (peer memory: load through L2 only)
      bf16x8_to_f32(__ldcg(reinterpret_cast<const uint4*>(p.part[r] + (size_t)par * p.par_stride + (size_t)m * p.N + n)),
                    t);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += t[e];
    }
    uint4 w;
    __nv_bfloat162* w2 = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) w2[e] = __floats2bfloat162_rn(acc[2 * e], acc[2 * e + 1]);
    *reinterpret_cast<uint4*>(o) = w;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.done, 1) == (int)gridDim.x - 1) {
      *p.done = 0;
      __threadfence();
      atomicAdd(p.seq, 1);
    }
  }
}

__global__ void tp_ag_wait_kernel(int* ag_flags, int expect, int tp, int* status) {
  pdl_wait();
  pdl_trigger();
  if ((int)threadIdx.x < tp) wait_flag(ag_flags + threadIdx.x, expect, status);
  __syncthreads();
  __threadfence();
  if ((int)threadIdx.x < tp) ag_flags[threadIdx.x] = 0;
}

}  // namespace

cudaError_t tp_rs_norm_ag_launch(const TpRsNormParams& p, cudaStream_t s) {
  if (p.tp > 32 || p.N % 8 || p.ldh % 8 || p.ld_ag % 8 || p.ld_recv % 8 || p.N > 8 * 1024 * kRsNormMaxChunks)
    return cudaErrorInvalidValue;
  const int grid = p.rows_per_rank;  // one CTA per owned row
  if (grid == 0) return cudaSuccess;
  const int threads = min(1024, (p.N / 8 + 31) / 32 * 32);  // one 8-column chunk per thread up to N = 8192
  SQ_LAUNCH(tp_rs_norm_ag_kernel, dim3(grid), dim3(threads), 0, s, 1, p);
  return cudaGetLastError();
}

cudaError_t tp_oneshot_launch(const TpOneshotParams& p, cudaStream_t s) {
  if (p.M == 0) return cudaSuccess;
  if (p.tp > 32 || p.N % 8 || p.ld_src % 8 || p.ld_out % 8 || p.par_stride < (long long)p.M * p.N)
    return cudaErrorInvalidValue;
  const long long vecs = (long long)p.M * (p.N / 8);
  // one 8-element vector per thread up to kOneshotMaxCtas CTAs (latency bound: spread the
  // chunks); every rank computes the same grid (same M, N)
  const int grid = (int)std::min<long long>(kOneshotMaxCtas, (vecs + kOneshotThreads - 1) / kOneshotThreads);
  SQ_LAUNCH(tp_oneshot_kernel, dim3(grid), dim3(kOneshotThreads), 0, s, 1, p);
  return cudaGetLastError();
}

cudaError_t tp_ag_wait_launch(int* ag_flags, int expect, int tp, int* status, cudaStream_t s) {
  if (tp > 32) return cudaErrorInvalidValue;
  SQ_LAUNCH(tp_ag_wait_kernel, dim3(1), dim3(32), 0, s, 1, ag_flags, expect, tp, status);
  return cudaGetLastError();
}

cudaError_t tp_reduce_launch(const TpReduceParams& p, int grid_x, int grid_y, cudaStream_t s) {
  if (p.tp > 256) return cudaErrorInvalidValue;
  SQ_LAUNCH(tp_reduce_kernel, dim3(dim3(grid_x, grid_y)), dim3(256), 0, s, 1, p);
  return cudaGetLastError();
}

cudaError_t tp_push_launch(const TpPushParams& p, int grid_x, int grid_y, cudaStream_t s) {
  if (p.M == 0) return cudaSuccess;
  SQ_LAUNCH(tp_push_kernel, dim3(grid_x, grid_y), dim3(256), 0, s, 1, p);
  return cudaGetLastError();
}

cudaError_t tp_gather_launch(const TpGatherParams& p, cudaStream_t s) {
  if (p.cols % 8 || p.ld_src % 8 || p.ld_dst % 8 || p.col0 % 8) return cudaErrorInvalidValue;
  SQ_LAUNCH(tp_gather_push_kernel, dim3(p.expect), dim3(256), 0, s, 1, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  SQ_LAUNCH(tp_gather_wait_kernel, dim3(1), dim3(32), 0, s, 1, p);
  return cudaGetLastError();
}

}  // namespace sq
