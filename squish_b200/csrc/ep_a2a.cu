// ep_a2a.cu — expert-parallel all-to-all (dispatch / combine) over NVLink peer memory.
//
// Layout: sequence parallel. Rank r owns token rows [r R, r R + own) of a step (R = ceil(T /
// tp)); its experts are [r E_local, (r + 1) E_local). A MoE layer runs as
//
//   owner:    h_own += attention partials; xn_own = RMSNorm(h_own)     (tp_rs_norm_ag, local only)
//             router logits = xn_own . Wg^T                              (bf16 library GEMM)
//             ep_dispatch: route each row (softmax, top-K, renorm) and store it once into every
//             rank that holds one of its experts (P2P stores), with the row's
//             (local id | -1, weight) list
//   receiver: align waits for R arrivals per source, then builds the expert-sorted layout;
//             gather / grouped INT4 gate_up + down over the tp x R received rows (moe.cu,
//             w4a16_gemm.cu)
//             ep_combine: the weighted expert sum of each received row goes back to the row
//             owner's reduce-scatter block (P2P stores) + one arrival per row
//   owner:    tp_rs_norm_ag adds the tp partial rows to the residual, applies the next
//             RMSNorm and all-gathers for the next layer's attention.
//
// NVLink bytes per rank and layer: at most (tp - 1) / tp of the owned rows x the number of
// distinct peer ranks their experts live on for the dispatch, and (tp - 1) R rows for the
// combine -- against 2 (tp - 1) / tp T rows of a reduce-scatter + all-gather of the
// full-token partial output that the all-reduce formulation needs.
//
// Buffer reuse needs no parity: a source dispatches layer l + 1 only after its
// tp_rs_norm_ag of layer l, which waits for every receiver's combine of layer l, which each
// receiver issues after it has gathered (finished reading) the dispatched rows of layer l.
// The receivers' dispatch counters are cleared by the waiting kernel before the same stream
// issues the combine that lets any source move on. The reference routes on the host with
// numpy / Rust top-k (squish_quant_rs/src/lib.rs:2688,2727) and has no expert parallelism.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "comm.h"
#include "launch.cuh"
#include "moe_route.cuh"

namespace sq {

namespace {

constexpr int kEpThreads = 256;
constexpr int kEpMaxK = 32;
constexpr int kEpRouteEpl = 8;  // router logits per lane: E <= 256

__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(const EpDispatchParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ int sid[kEpMaxK];
  __shared__ float sw[kEpMaxK];
  __shared__ unsigned mask;  // bit d: some expert of the row lives on rank d
  const int t = blockIdx.x;
  const bool valid = t < p.own;
  if (threadIdx.x == 0) mask = 0u;
  if (p.logits != nullptr && valid && threadIdx.x < 32)  // fused routing of this row
    route_row_warp<kEpRouteEpl>(p.logits + (size_t)t * p.ld_logits, p.E, p.K, p.renorm, threadIdx.x, sid, sw);
  __syncthreads();
  if ((int)threadIdx.x < p.K) {
    const size_t i = (size_t)t * p.K + threadIdx.x;
    int e = -1;
    float wt = 0.f;
    if (valid && p.logits != nullptr) {
      e = sid[threadIdx.x];
      wt = sw[threadIdx.x];
      p.ids[i] = e;
      p.w[i] = wt;
    } else if (valid) {
      e = p.ids[i];
      wt = p.w[i];
    }
    sid[threadIdx.x] = e;
    sw[threadIdx.x] = wt;
    const int d = e >= 0 ? e / p.E_local : -1;
    if (d >= 0 && d < p.tp) atomicOr(&mask, 1u << d);
  }
  __syncthreads();
  const unsigned m = mask;
  const size_t slot = (size_t)p.rank * p.R + t;
  // the row, once per destination rank that holds one of its experts
  const int vec = p.H / 8;
  const uint4* src = reinterpret_cast<const uint4*>(p.x + (size_t)t * p.ldx);
  for (int c = threadIdx.x; c < vec; c += blockDim.x) {
    if (!m) break;
    const uint4 v = src[c];
    for (int d = 0; d < p.tp; ++d)
      if (m >> d & 1u) reinterpret_cast<uint4*>(p.recv_x[d] + slot * p.H)[c] = v;
  }
  // the (local id | -1, weight) list on every rank
  for (int i = threadIdx.x; i < p.tp * p.K; i += blockDim.x) {
    const int d = i / p.K, k = i % p.K;
    const int e = sid[k];
    const bool here = e >= 0 && e / p.E_local == d;
    p.recv_ids[d][slot * p.K + k] = here ? e - d * p.E_local : -1;
    p.recv_w[d][slot * p.K + k] = sw[k];
  }
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < p.tp)
    asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p.flags[threadIdx.x]), "r"(1) : "memory");
}

__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(const EpCombineParams p) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  const int s = b / p.R, t = b % p.R;  // owner rank, its row slot
  const int par = *reinterpret_cast<volatile const int*>(p.seq) & 1;
  const bool live = s * p.R + t < p.T;  // rows past the step are not read by the owner
  const int vec = p.H / 8;
  const size_t slot0 = ((size_t)s * p.R + t) * p.K;
  for (int c = threadIdx.x; c < vec && live; c += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < p.K; ++k) {  // K in order: the same rounding on every run
      const int pos = p.slot_pos[slot0 + k];
      if (pos < 0) continue;
      const float w = p.w[slot0 + k];
      const uint4 yv = reinterpret_cast<const uint4*>(p.ys + (size_t)pos * p.ldys)[c];
      const __nv_bfloat162* y2 = reinterpret_cast<const __nv_bfloat162*>(&yv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(y2[j]);
        acc[2 * j] = fmaf(w, f.x, acc[2 * j]);
        acc[2 * j + 1] = fmaf(w, f.y, acc[2 * j + 1]);
      }
    }
    uint4 o;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) o2[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    reinterpret_cast<uint4*>(p.dst[s] + (size_t)t * p.ld_dst)[c] = o;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* f = p.flags[s] + (size_t)par * p.flag_stride;
    asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(f), "r"(1) : "memory");
  }
}

}  // namespace

cudaError_t ep_dispatch_launch(const EpDispatchParams& p, cudaStream_t s) {
  if (p.R == 0) return cudaSuccess;
  if (p.tp > 32 || p.K > kEpMaxK || p.K < 1 || p.E_local < 1 || p.H % 8 || p.ldx % 8 || p.own > p.R || p.own < 0)
    return cudaErrorInvalidValue;
  if (p.logits != nullptr && (p.E > 32 * kEpRouteEpl || p.E < p.K || p.E > p.E_local * p.tp))
    return cudaErrorInvalidValue;
  SQ_LAUNCH(ep_dispatch_kernel, dim3(p.R), dim3(kEpThreads), 0, s, 1, p);
  return cudaGetLastError();
}

cudaError_t ep_combine_launch(const EpCombineParams& p, cudaStream_t s) {
  if (p.R == 0) return cudaSuccess;
  if (p.tp > 32 || p.K > kEpMaxK || p.K < 1 || p.H % 8 || p.ldys % 8 || p.ld_dst % 8) return cudaErrorInvalidValue;
  SQ_LAUNCH(ep_combine_kernel, dim3(p.tp * p.R), dim3(kEpThreads), 0, s, 1, p);
  return cudaGetLastError();
}

}  // namespace sq
