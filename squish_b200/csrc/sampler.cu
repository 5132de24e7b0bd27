// sampler.cu — batched fused sampler: one CTA per row, per-row parameters.
//
// Order of operations follows the reference FusedSampler._compute_probs
// (squish/hardware/fused_sampler.py:226-310): repetition penalty (x/p if x>0 else x*p,
// once per distinct id) -> temperature -> softmax -> min-p (p >= min_p * p_max) ->
// top-k -> top-p (smallest prefix of the sorted kept probabilities, normalised over the
// full softmax, whose mass reaches top_p) -> renormalise -> draw. An optional grammar
// bitmask (bit set = allowed) is applied first, as the reference's grammar engine does
// with its token bitmask (squish/grammar/grammar_engine.py:220-254).
//
// Instead of sorting the vocabulary, every filter becomes a logit threshold:
//   min-p: tau_m = max + log(min_p);  top-k: tau_k = k-th largest logit (4-pass radix
//   select on the order-preserving bit pattern); top-p: bisection on tau for the mass of
//   kept tokens above tau. The draw is Gumbel-max over the kept set, which samples exactly
//   from the renormalised distribution. Temperature <= 0 means greedy (argmax).
#include "kernels.h"
#include "launch.cuh"

namespace sq {

namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  // SplitMix64 finaliser (Steele, Lea, Flood 2014): a bijective avalanche mix.
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float uniform01(uint64_t seed, uint64_t row, uint64_t step, uint64_t tok) {
  const uint64_t h = mix64(seed ^ mix64(row * 0x100000001B3ull + mix64(step ^ (tok << 20))));
  return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
}

__device__ __forceinline__ uint32_t f2ord(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T, typename Op>
__device__ T block_reduce(T v, Op op, T* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = (lane < (int)(blockDim.x >> 5)) ? sh[lane] : sh[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}

struct ArgMax {
  float v;
  int i;
};

__global__ void __launch_bounds__(kThreads) sampler_kernel(const SamplerParams p, float* __restrict__ work) {
  pdl_wait();
  pdl_trigger();
  __shared__ float shf[32];
  __shared__ int shi[32];
  __shared__ unsigned int hist[256];
  const int row = blockIdx.x;
  const int V = p.V;
  float* x = work + (size_t)row * V;
  const __nv_bfloat16* lg = p.logits + (size_t)row * p.ld;
  const float temp = p.temperature ? p.temperature[row] : 0.f;
  const bool greedy = !(temp > 0.f);
  const float inv_t = greedy ? 1.f : 1.f / temp;

  const uint32_t* mask = p.allow_mask ? p.allow_mask + (size_t)row * ((V + 31) / 32) : nullptr;
  const float rp0 = p.rep_penalty ? p.rep_penalty[row] : 1.f;
  const bool fused_greedy = greedy && !(rp0 != 1.f && p.hist);
  // pass 0: load + mask (greedy rows without a penalty: straight to the argmax, no fp32 copy)
  for (int i = threadIdx.x; i < V && !fused_greedy; i += kThreads) {
    float v = __bfloat162float(lg[i]);
    if (mask && !((mask[i >> 5] >> (i & 31)) & 1u)) v = -INFINITY;
    x[i] = v;
  }
  __syncthreads();
  // repetition penalty, once per distinct id in the history window
  const float rp = p.rep_penalty ? p.rep_penalty[row] : 1.f;
  if (rp != 1.f && p.hist) {
    const int* hr = p.hist + (size_t)row * p.hist_stride;
    for (int j = threadIdx.x; j < p.hist_stride; j += kThreads) {
      const int id = hr[j];
      if (id < 0 || id >= V) continue;
      bool first = true;
      for (int k = 0; k < j; ++k)
        if (hr[k] == id) {
          first = false;
          break;
        }
      if (first) {
        const float v = x[id];
        x[id] = v > 0.f ? v / rp : v * rp;
      }
    }
    __syncthreads();
  }
  // pass 1: temperature + max/argmax
  float mv = -INFINITY;
  int mi = 0;
  if (fused_greedy) {
    for (int i = threadIdx.x; i < V; i += kThreads) {
      float v = __bfloat162float(lg[i]);
      if (mask && !((mask[i >> 5] >> (i & 31)) & 1u)) v = -INFINITY;
      if (v > mv) {
        mv = v;
        mi = i;
      }
    }
  } else {
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const float v = x[i] * inv_t;
      if (!greedy) x[i] = v;
      if (v > mv) {
        mv = v;
        mi = i;
      }
    }
  }
  {
    // argmax reduce (lowest index wins ties)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, mv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, mi, o);
      if (ov > mv || (ov == mv && oi < mi)) {
        mv = ov;
        mi = oi;
      }
    }
    __syncthreads();
    if (lane == 0) {
      shf[warp] = mv;
      shi[warp] = mi;
    }
    __syncthreads();
    if (warp == 0) {
      mv = shf[lane];
      mi = shi[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, mv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, mi, o);
        if (ov > mv || (ov == mv && oi < mi)) {
          mv = ov;
          mi = oi;
        }
      }
      if (lane == 0) {
        shf[0] = mv;
        shi[0] = mi;
      }
    }
    __syncthreads();
    mv = shf[0];
    mi = shi[0];
  }
  if (greedy || mv == -INFINITY) {
    if (threadIdx.x == 0) {
      p.out_tokens[row] = mi;
      if (p.out_logprob) p.out_logprob[row] = 0.f;
    }
    return;
  }
  const float xmax = mv;
  // softmax normaliser
  float z = 0.f;
  for (int i = threadIdx.x; i < V; i += kThreads) z += __expf(x[i] - xmax);
  z = block_reduce(z, [](float a, float b) { return a + b; }, shf);

  float tau = -INFINITY;
  const float min_p = p.min_p ? p.min_p[row] : 0.f;
  if (min_p > 0.f) tau = fmaxf(tau, xmax + __logf(min_p));
  const int top_k = p.top_k ? p.top_k[row] : 0;
  if (top_k > 0 && top_k < V) {
    // radix select the k-th largest ordered key, 8 bits per pass from the top
    uint32_t prefix = 0, pmask = 0;
    int k = top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = threadIdx.x; i < 256; i += kThreads) hist[i] = 0;
      __syncthreads();
      for (int i = threadIdx.x; i < V; i += kThreads) {
        const uint32_t key = f2ord(x[i]);
        if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFF], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int acc = 0, bin = 255;
        for (; bin > 0; --bin) {
          if (acc + (int)hist[bin] >= k) break;
          acc += hist[bin];
        }
        shi[0] = bin;
        shi[1] = k - acc;
      }
      __syncthreads();
      prefix |= (uint32_t)shi[0] << shift;
      pmask |= 0xFFu << shift;
      k = shi[1];
      __syncthreads();
    }
    const uint32_t u = (prefix & 0x80000000u) ? (prefix & 0x7FFFFFFFu) : ~prefix;
    tau = fmaxf(tau, __uint_as_float(u));
  }
  const float top_p = p.top_p ? p.top_p[row] : 1.f;
  if (top_p < 1.f) {
    // largest t with sum_{x_i >= max(t, tau)} p_i >= top_p  (p normalised over the full softmax)
    float lo = (tau == -INFINITY) ? xmax - 40.f : tau, hi = xmax;
    auto mass = [&](float t) {
      float m = 0.f;
      for (int i = threadIdx.x; i < V; i += kThreads) {
        const float v = x[i];
        if (v >= t) m += __expf(v - xmax);
      }
      return block_reduce(m, [](float a, float b) { return a + b; }, shf) / z;
    };
    if (mass(lo) >= top_p) {
      for (int it = 0; it < 24; ++it) {
        const float mid = 0.5f * (lo + hi);
        if (mass(mid) >= top_p) lo = mid;
        else hi = mid;
      }
      tau = fmaxf(tau, lo);
    }
  }
  // Gumbel-max draw over the kept set
  const uint64_t step = p.step ? (uint64_t)p.step[row] : 0ull;
  float best = -INFINITY;
  int bi = mi;
  for (int i = threadIdx.x; i < V; i += kThreads) {
    const float v = x[i];
    if (v >= tau && v > -INFINITY) {
      const float u = uniform01(p.seed, (uint64_t)row, step, (uint64_t)i);
      const float gsc = v - __logf(-__logf(u));
      if (gsc > best) {
        best = gsc;
        bi = i;
      }
    }
  }
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    __syncthreads();
    if (lane == 0) {
      shf[warp] = best;
      shi[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
      best = shf[lane];
      bi = shi[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) {
          best = ov;
          bi = oi;
        }
      }
      if (lane == 0) shi[0] = bi;
    }
    __syncthreads();
    bi = shi[0];
  }
  float zk = 0.f;
  if (p.out_logprob) {
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const float v = x[i];
      if (v >= tau) zk += __expf(v - xmax);
    }
    zk = block_reduce(zk, [](float a, float b) { return a + b; }, shf);
  }
  if (threadIdx.x == 0) {
    p.out_tokens[row] = bi;
    if (p.out_logprob) p.out_logprob[row] = (x[bi] - xmax) - __logf(zk);
  }
}

}  // namespace

cudaError_t sampler_launch(const SamplerParams& p, float* work, cudaStream_t s) {
  if (p.B == 0) return cudaSuccess;
  SQ_LAUNCH(sampler_kernel, dim3(p.B), dim3(kThreads), 0, s, 1, p, work);
  return cudaGetLastError();
}

}  // namespace sq
