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
//   min-p: tau_m = max + log(min_p);  top-k: tau_k = k-th largest logit;  top-p: the last logit
//   of the shortest sorted head whose mass reaches top_p. Both are exact radix selections on
//   the order-preserving bit pattern (8 passes of 4 bits, weighted by 1 or by exp(x - max)).
//   The draw is Gumbel-max over the kept set, which samples exactly from the renormalised
//   distribution. Temperature <= 0 means greedy (argmax).
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

__device__ __forceinline__ float ord2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

struct RadixSmem {
  float part[32][16];  // per-warp bin sums
  float tot[16];
  float above;
  uint32_t prefix;
};

// Largest order key T such that the weight of the elements with key >= T (among keys >= lo) is
// at least `target`; weight 1 per element (counting: the k-th largest) or exp(x - xmax) (mass).
// Radix descent 4 bits per pass from the top: each thread sums its elements into 16 bin
// registers (no shared-memory atomics, so no contention when the logits crowd a few bins), the
// block adds the bins, and the bin where the running weight from the top reaches the target
// extends the prefix. If the candidates weigh less than the target, every one is kept (T = the
// smallest key present).
template <bool kMass>
__device__ uint32_t radix_select(const float* __restrict__ x, int V, uint32_t lo, float target, float xmax,
                                 RadixSmem& rs) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    rs.prefix = 0u;
    rs.above = 0.f;
  }
  __syncthreads();
  uint32_t prefix = 0u, pmask = 0u;
  for (int shift = 28; shift >= 0; shift -= 4) {
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.f;
#pragma unroll 4
    for (int i = threadIdx.x; i < V; i += kThreads) {
      const float v = x[i];
      const uint32_t key = f2ord(v);
      if (key >= lo && (key & pmask) == prefix) {
        const uint32_t b = (key >> shift) & 15u;
        const float w = kMass ? __expf(v - xmax) : 1.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] += (b == (uint32_t)j) ? w : 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < 16; ++j) rs.part[warp][j] = acc[j];
    }
    __syncthreads();
    if (threadIdx.x < 16) {
      float t = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += rs.part[w][threadIdx.x];
      rs.tot[threadIdx.x] = t;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float above = rs.above;
      int b = 15;
      for (; b > 0; --b) {
        if (above + rs.tot[b] >= target) break;
        above += rs.tot[b];
      }
      rs.above = above;
      rs.prefix = prefix | ((uint32_t)b << shift);
    }
    __syncthreads();
    prefix = rs.prefix;
    pmask |= 15u << shift;
    __syncthreads();  // rs is rewritten by the next pass
  }
  return prefix;
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
  __shared__ RadixSmem rs;
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
  if (top_k > 0 && top_k < V) tau = fmaxf(tau, ord2f(radix_select<false>(x, V, f2ord(tau), (float)top_k, xmax, rs)));
  const float top_p = p.top_p ? p.top_p[row] : 1.f;
  // the smallest head of the sorted kept logits whose mass (normalised over the full softmax)
  // reaches top_p: its last key is the threshold
  if (top_p < 1.f) tau = fmaxf(tau, ord2f(radix_select<true>(x, V, f2ord(tau), top_p * z, xmax, rs)));
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
