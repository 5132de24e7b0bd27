// moe_route.cuh — router top-k of one token by one warp (shared by the MoE routing kernel and
// the expert-parallel dispatch kernel, which routes and sends a row in one launch).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace sq {

// Softmax over the E (<= 32 * EPL) router logits of one token, the top K probabilities (the
// lower expert index wins a tie), renormalised over the K picks when renorm != 0. Lane 0
// writes ids[k] / w[k] in rank order; after a warp barrier lanes < K renormalise their weight.
// Every lane of the warp must call it.
template <int EPL>
__device__ __forceinline__ void route_row_warp(const __nv_bfloat16* __restrict__ row, int E, int K, int renorm,
                                               int lane, int* __restrict__ ids, float* __restrict__ w) {
  float v[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? __bfloat162float(row[e]) : -INFINITY;
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    v[i] = (lane + 32 * i) < E ? __expf(v[i] - m) : -1.f;
    s += v[i] > 0.f ? v[i] : 0.f;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float inv = 1.f / s;
  float picked = 0.f;
  for (int k = 0; k < K; ++k) {
    float bv = -2.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (v[i] > bv) {  // strict: the lower index wins ties within a lane
        bv = v[i];
        bi = lane + 32 * i;
      }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (lane + 32 * i == bi) v[i] = -1.f;
    const float pr = bv * inv;
    picked += pr;
    if (lane == 0) {
      ids[k] = bi;
      w[k] = pr;
    }
  }
  __syncwarp();
  if (renorm && lane < K) w[lane] /= picked;
}

}  // namespace sq
