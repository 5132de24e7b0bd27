// moe.cu — mixture-of-experts routing, dispatch layout, gather and combine for sm_100a.
//
// A Qwen3-MoE block (softmax router, top-k experts, renormalised weights; the reference's
// router top-k is squish_quant_rs/src/lib.rs:2688,2727) runs as
//
//   logits = x . Wg^T                      (bf16 library GEMM, E = 128 columns)
//   route    : softmax -> top-k -> renorm  (one warp per token)
//   align    : per-expert counts, offsets padded to the GEMM token tile, the sorted slot
//              list and each token tile's expert (one CTA; no host round trip, graph-safe)
//   gather   : X_sorted[row] = x[token(row)] (zero rows for padding)
//   grouped INT4 GEMMs (w4a16_gemm.cu grouped mode): gate_up with SiLU*up, then down
//   combine  : h[t] += sum_k w[t,k] * out_sorted[pos(t,k)]  (k in order: deterministic)
//
// Expert parallelism splits the slot list by owner rank before the gather; the same align
// kernel runs over the slots a rank receives (local expert ids).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "kernels.h"
#include "launch.cuh"
#include "moe_route.cuh"
#include "sm100.cuh"

namespace sq {

namespace {

template <int EPL>
__global__ void __launch_bounds__(256) moe_route_kernel(const __nv_bfloat16* __restrict__ logits, int ld, int T,
                                                        int E, int K, int renorm, int* __restrict__ topk_ids,
                                                        float* __restrict__ topk_w) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  if (t >= T) return;
  route_row_warp<EPL>(logits + (size_t)t * ld, E, K, renorm, lane, topk_ids + (size_t)t * K, topk_w + (size_t)t * K);
}

// Bounded wait (one thread per source) until every source's dispatch counter reached `expect`,
// then clear it: the expert-parallel receiver's arrival check, fused into the align kernel.
__device__ __forceinline__ void wait_dispatch(int* flags, int n, int expect, int* status) {
  if ((int)threadIdx.x < n) {
    int* f = flags + threadIdx.x;
    bool ok = false;
    for (long long i = 0; i < (1LL << 22); ++i) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (v >= expect) {
        ok = true;
        break;
      }
      if ((i & 4095) == 4095 && *reinterpret_cast<volatile int*>(status) != 0) break;
    }
    if (!ok) atomicCAS(status, 0, SQ_ERR_TIMEOUT_PEER);
    *f = 0;
  }
  __syncthreads();
  __threadfence();
}

__global__ void __launch_bounds__(1024) moe_align_kernel(const int* __restrict__ ids, int TK, int E, int bn,
                                                         int max_tiles, int* __restrict__ sorted_slot,
                                                         int* __restrict__ slot_pos, int* __restrict__ tile_expert,
                                                         int* __restrict__ num_tiles, int* __restrict__ counts,
                                                         int* wait_flags, int wait_n, int wait_expect, int* status) {
  pdl_wait();
  pdl_trigger();
  if (wait_flags != nullptr) wait_dispatch(wait_flags, wait_n, wait_expect, status);
  extern __shared__ int sh[];
  int* cnt = sh;           // [E]
  int* off = sh + E;       // [E + 1]
  int* cur = off + E + 1;  // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    cnt[e] = 0;
    cur[e] = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < TK; i += blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = o;
      o += (cnt[e] + bn - 1) / bn * bn;
    }
    off[E] = o;
    *num_tiles = o / bn;
  }
  __syncthreads();
  const int ntile = off[E] / bn;
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (counts) counts[e] = cnt[e];
  for (int tile = threadIdx.x; tile < max_tiles; tile += blockDim.x) {
    int lo = 0, hi = E - 1, r = tile * bn;  // last expert whose offset <= r
    if (tile >= ntile) {
      tile_expert[tile] = 0;
      continue;
    }
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (off[mid] <= r) lo = mid;
      else hi = mid - 1;
    }
    // skip experts with zero rows that share the same offset
    while (lo + 1 < E && off[lo + 1] <= r) ++lo;
    tile_expert[tile] = lo;
  }
  for (int r = threadIdx.x; r < off[E]; r += blockDim.x) sorted_slot[r] = -1;
  __syncthreads();
  for (int i = threadIdx.x; i < TK; i += blockDim.x) {
    const int e = ids[i];
    if (e < 0 || e >= E) {
      slot_pos[i] = -1;
      continue;
    }
    const int pos = off[e] + atomicAdd(&cur[e], 1);
    sorted_slot[pos] = i;
    slot_pos[i] = pos;
  }
}

// one CTA of 128 threads per 4 sorted rows; each thread moves 16-byte vectors
__global__ void __launch_bounds__(128) moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                         const int* __restrict__ sorted_slot,
                                                         const int* __restrict__ num_tiles, int bn, int K, int H,
                                                         __nv_bfloat16* __restrict__ xs, int ldxs) {
  pdl_wait();
  pdl_trigger();
  const int rows = __ldg(num_tiles) * bn;
  const int vec = H / 8;
  for (int rr = 0; rr < 4; ++rr) {
    const int r = blockIdx.x * 4 + rr;
    if (r >= rows) return;
    const int slot = sorted_slot[r];
    uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)r * ldxs);
    if (slot < 0) {
      for (int c = threadIdx.x; c < vec; c += blockDim.x) dst[c] = make_uint4(0, 0, 0, 0);
    } else {
      const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(slot / K) * ldx);
      for (int c = threadIdx.x; c < vec; c += blockDim.x) dst[c] = src[c];
    }
  }
}

__global__ void __launch_bounds__(256) moe_combine_kernel(const __nv_bfloat16* __restrict__ ys, int ldys,
                                                          const int* __restrict__ slot_pos,
                                                          const float* __restrict__ topk_w, int K, int H,
                                                          __nv_bfloat16* __restrict__ h, int ldh) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int vec = H / 8;
  for (int c = threadIdx.x; c < vec; c += blockDim.x) {
    float acc[8];
    const uint4 hv = reinterpret_cast<const uint4*>(h + (size_t)t * ldh)[c];
    const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hv);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(hp[j]);
      acc[2 * j] = f.x;
      acc[2 * j + 1] = f.y;
    }
    float moe[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k = 0; k < K; ++k) {
      const int pos = slot_pos[t * K + k];
      if (pos < 0) continue;
      const float w = topk_w[t * K + k];
      const uint4 yv = reinterpret_cast<const uint4*>(ys + (size_t)pos * ldys)[c];
      const __nv_bfloat162* yp = reinterpret_cast<const __nv_bfloat162*>(&yv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(yp[j]);
        moe[2 * j] = fmaf(w, f.x, moe[2 * j]);
        moe[2 * j + 1] = fmaf(w, f.y, moe[2 * j + 1]);
      }
    }
    uint4 ov;
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
    for (int j = 0; j < 4; ++j) op[j] = __floats2bfloat162_rn(acc[2 * j] + moe[2 * j], acc[2 * j + 1] + moe[2 * j + 1]);
    reinterpret_cast<uint4*>(h + (size_t)t * ldh)[c] = ov;
  }
}

}  // namespace

cudaError_t moe_route_launch(const __nv_bfloat16* logits, int ld, int T, int E, int K, bool renorm, int* topk_ids,
                             float* topk_w, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (E > 256 || K > 32 || K > E) return cudaErrorInvalidValue;
  const dim3 grid((T + 7) / 8);
  if (E <= 64) SQ_LAUNCH(moe_route_kernel<2>, dim3(grid), dim3(256), 0, s, 1, logits, ld, T, E, K, renorm, topk_ids, topk_w);
  else if (E <= 128) SQ_LAUNCH(moe_route_kernel<4>, dim3(grid), dim3(256), 0, s, 1, logits, ld, T, E, K, renorm, topk_ids, topk_w);
  else SQ_LAUNCH(moe_route_kernel<8>, dim3(grid), dim3(256), 0, s, 1, logits, ld, T, E, K, renorm, topk_ids, topk_w);
  return cudaGetLastError();
}

cudaError_t moe_align_launch(const int* ids, int TK, int E, int bn, int max_tiles, int* sorted_slot, int* slot_pos,
                             int* tile_expert, int* num_tiles, int* counts, cudaStream_t s, int* wait_flags,
                             int wait_n, int wait_expect, int* status) {
  if (wait_flags != nullptr && (wait_n > 32 || status == nullptr)) return cudaErrorInvalidValue;
  const size_t smem = (size_t)(3 * E + 1) * sizeof(int);
  SQ_LAUNCH(moe_align_kernel, dim3(1), dim3(1024), smem, s, 1, ids, TK, E, bn, max_tiles, sorted_slot, slot_pos, tile_expert, num_tiles,
                                         counts, wait_flags, wait_n, wait_expect, status);
  return cudaGetLastError();
}

cudaError_t moe_gather_launch(const __nv_bfloat16* x, int ldx, const int* sorted_slot, const int* num_tiles,
                              int max_rows, int bn, int K, int H, __nv_bfloat16* xs, int ldxs, cudaStream_t s) {
  if (H % 8 || ldx % 8 || ldxs % 8) return cudaErrorInvalidValue;
  if (max_rows == 0) return cudaSuccess;
  SQ_LAUNCH(moe_gather_kernel, dim3((max_rows + 3) / 4), dim3(128), 0, s, 1, x, ldx, sorted_slot, num_tiles, bn, K, H, xs, ldxs);
  return cudaGetLastError();
}

cudaError_t moe_combine_launch(const __nv_bfloat16* ys, int ldys, const int* slot_pos, const float* topk_w, int T,
                               int K, int H, __nv_bfloat16* h, int ldh, cudaStream_t s) {
  if (H % 8 || ldys % 8 || ldh % 8) return cudaErrorInvalidValue;
  if (T == 0) return cudaSuccess;
  SQ_LAUNCH(moe_combine_kernel, dim3(T), dim3(256), 0, s, 1, ys, ldys, slot_pos, topk_w, K, H, h, ldh);
  return cudaGetLastError();
}

}  // namespace sq
