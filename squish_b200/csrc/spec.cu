// spec.cu — speculative decoding on the device: token-tree verification and KV compaction.
//
// tree_verify: one CTA per sequence walks its draft tree (<= 32 nodes, node 0 = the last
// committed token, parents before children) against the target logits of every node.
//
//   greedy (temperature <= 0): follow the child whose token is the target argmax; the first
//     node without such a child emits the argmax as the correction token.
//   sampling: multi-draft rejection sampling (SpecInfer, Miao et al. 2024): at node u with
//     target p = softmax(l_u / T), try the children in order; child c with token x drawn
//     from q_c is accepted with probability min(1, r(x) / q_c(x)), where r is the current
//     residual (p at first); on rejection r <- norm(max(0, r - q_c)). If every child is
//     rejected the correction token is drawn from r; at a leaf the bonus token is drawn
//     from p. q_c is the draft model's softmax(logits / T) row, or a point mass on x for
//     deterministic drafts (prompt lookup, Jacobi), for which r <- r with x removed.
//   The emitted sequence has exactly the target distribution (greedy: the target argmax
//   chain). The reference restates this per branch in tree_verify_softmax_f32
//   (squish_quant_rs/src/lib.rs:4111); here branches share prefixes and the walk runs on
//   the device, so only (accepted path, final token) returns to the host.
//
// Draws use a SplitMix64 counter hash (seed, step, node, child / vocab index): Gumbel-max
// over the residual for the correction token, one uniform per acceptance test.
//
// kv_compact: after a branch other than the first-index chain is accepted, the accepted
// nodes' KV rows (written at chunk slots start + node) move to start + depth, for every
// layer; copies run in increasing depth so no source is overwritten before it is read.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "kernels.h"
#include "launch.cuh"

namespace sq {

namespace {

constexpr int kVThreads = 512;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float uni(uint64_t seed, uint64_t a, uint64_t b, uint64_t c) {
  const uint64_t h = mix64(seed ^ mix64(a * 0x100000001B3ull + mix64(b ^ (c << 24))));
  return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a;
}

__device__ ArgMax block_argmax(ArgMax a, ArgMax* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, b);
  }
  __syncthreads();
  if (lane == 0) sh[warp] = a;
  __syncthreads();
  if (warp == 0) {
    a = lane < (int)(blockDim.x >> 5) ? sh[lane] : ArgMax{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
      a = better(a, b);
    }
    if (lane == 0) sh[0] = a;
  }
  __syncthreads();
  const ArgMax r = sh[0];
  __syncthreads();
  return r;
}

__device__ float block_sum(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? sh[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  const float r = sh[0];
  __syncthreads();
  return r;
}

__device__ float block_max(float v, float* sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? sh[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  const float r = sh[0];
  __syncthreads();
  return r;
}

// softmax(row / T): returns (max of row/T, sum of exp(row/T - max))
__device__ float2 softmax_stats(const __nv_bfloat16* row, int V, float invT, float* shf) {
  float m = -INFINITY;
  for (int v = threadIdx.x; v < V; v += blockDim.x) m = fmaxf(m, __bfloat162float(row[v]) * invT);
  m = block_max(m, shf);
  float s = 0.f;
  for (int v = threadIdx.x; v < V; v += blockDim.x) s += __expf(__bfloat162float(row[v]) * invT - m);
  s = block_sum(s, shf);
  return make_float2(m, s);
}

__global__ void __launch_bounds__(kVThreads) tree_verify_kernel(const TreeVerifyParams p) {
  pdl_wait();
  pdl_trigger();
  __shared__ ArgMax sha[32];
  __shared__ float shf[32];
  __shared__ int children[kMaxTreeNodes];
  const int g = blockIdx.x;
  const int* meta = p.meta + (size_t)g * kTreeMetaInts;
  const int row0 = meta[0], n = min(meta[1], kMaxTreeNodes);
  const int* parent = meta + 2;
  const int* token = parent + kMaxTreeNodes;
  const int* qrow = token + kMaxTreeNodes;
  const float T = p.temperature[g];
  const uint64_t step = (uint64_t)(uint32_t)p.step[g];
  int* out = p.out + (size_t)g * (2 + kMaxTreeNodes);
  float* res = p.scratch + (size_t)g * p.V;
  const int V = p.V;
  int u = 0, nacc = 0, final_tok = 0;
  for (int guard = 0; guard < kMaxTreeNodes + 1; ++guard) {
    __syncthreads();  // every thread is done with the previous node's child list
    // children of u, in index order
    int nc = 0;
    for (int c = 1; c < n; ++c)
      if (parent[c] == u) {
        if (threadIdx.x == 0) children[nc] = c;
        ++nc;
      }
    __syncthreads();
    const __nv_bfloat16* lrow = p.logits + (size_t)(row0 + u) * p.ld;
    if (T <= 0.f) {
      ArgMax a{-INFINITY, 0x7fffffff};
      for (int v = threadIdx.x; v < V; v += blockDim.x) a = better(a, ArgMax{__bfloat162float(lrow[v]), v});
      a = block_argmax(a, sha);
      int next = -1;
      for (int j = 0; j < nc; ++j)
        if (token[children[j]] == a.i) {
          next = children[j];
          break;
        }
      if (next < 0) {
        final_tok = a.i;
        break;
      }
      if (threadIdx.x == 0) out[2 + nacc] = next;
      ++nacc;
      u = next;
      continue;
    }
    const float invT = 1.f / T;
    const float2 st = softmax_stats(lrow, V, invT, shf);
    bool have_res = false;  // res[] holds the (unnormalised) residual
    float rsum = 1.f;
    int next = -1;
    for (int j = 0; j < nc; ++j) {
      const int c = children[j];
      const int x = token[c];
      const float px = have_res ? res[x] / rsum : __expf(__bfloat162float(lrow[x]) * invT - st.x) / st.y;
      float qx = 1.f;
      float2 qs = make_float2(0.f, 1.f);
      const __nv_bfloat16* qr = nullptr;
      if (qrow[c] >= 0 && p.draft_logits != nullptr) {
        qr = p.draft_logits + (size_t)qrow[c] * p.ld_draft;
        qs = softmax_stats(qr, V, invT, shf);
        qx = __expf(__bfloat162float(qr[x]) * invT - qs.x) / qs.y;
      }
      const float ur = uni(p.seed, step, (uint64_t)u * 64 + c, 0x5eedull);
      if (ur < fminf(1.f, px / fmaxf(qx, 1e-30f))) {
        next = c;
        break;
      }
      // rejected: residual <- max(0, residual - q)
      if (!have_res) {
        for (int v = threadIdx.x; v < V; v += blockDim.x) res[v] = __expf(__bfloat162float(lrow[v]) * invT - st.x) / st.y;
        have_res = true;
        rsum = 1.f;
      }
      __syncthreads();
      float part = 0.f;
      if (qr != nullptr) {
        for (int v = threadIdx.x; v < V; v += blockDim.x) {
          const float q = __expf(__bfloat162float(qr[v]) * invT - qs.x) / qs.y;
          const float r = fmaxf(0.f, res[v] / rsum - q);
          res[v] = r;
          part += r;
        }
      } else {
        for (int v = threadIdx.x; v < V; v += blockDim.x) {
          const float r = (v == x) ? 0.f : res[v] / rsum;
          res[v] = r;
          part += r;
        }
      }
      rsum = block_sum(part, shf);
      if (!(rsum > 0.f)) {  // nothing left (numerically): fall back to the target itself
        have_res = false;
        rsum = 1.f;
      }
    }
    if (next >= 0) {
      if (threadIdx.x == 0) out[2 + nacc] = next;
      ++nacc;
      u = next;
      __syncthreads();
      continue;
    }
    // correction / bonus token: Gumbel-max over log(residual) or over the target logits
    ArgMax a{-INFINITY, 0x7fffffff};
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
      const float gum = -__logf(-__logf(uni(p.seed, step, 0x10000ull + (uint64_t)u, (uint64_t)v)));
      float key;
      if (have_res) {
        const float r = res[v];
        key = r > 0.f ? __logf(r) + gum : -INFINITY;
      } else {
        key = __bfloat162float(lrow[v]) * invT + gum;
      }
      a = better(a, ArgMax{key, v});
    }
    a = block_argmax(a, sha);
    final_tok = a.i;
    break;
  }
  if (threadIdx.x == 0) {
    out[0] = nacc;
    out[1] = final_tok;
  }
}

__global__ void kv_compact_kernel(const KvCompactParams p) {
  pdl_wait();
  pdl_trigger();
  // grid (layers, Hkv); pairs copied in order
  const int layer = blockIdx.x, h = blockIdx.y;
  const KvLayerPtrs L = p.layers[layer];
  for (int i = 0; i < p.n_pairs; ++i) {
    const int src = p.src[i], dst = p.dst[i];
    if (src == dst || src < 0 || dst < 0) continue;
    const size_t rs = ((size_t)(src / p.page_size) * p.Hkv + h) * p.page_size + src % p.page_size;
    const size_t rd = ((size_t)(dst / p.page_size) * p.Hkv + h) * p.page_size + dst % p.page_size;
    for (int b = threadIdx.x; b < p.kc_bytes; b += blockDim.x) L.kc[rd * p.kc_bytes + b] = L.kc[rs * p.kc_bytes + b];
    for (int b = threadIdx.x; b < p.vc_bytes; b += blockDim.x) L.vc[rd * p.vc_bytes + b] = L.vc[rs * p.vc_bytes + b];
    for (int b = threadIdx.x; b < p.ks_n; b += blockDim.x) L.ks[rd * p.ks_n + b] = L.ks[rs * p.ks_n + b];
    for (int b = threadIdx.x; b < p.vs_n; b += blockDim.x) L.vs[rd * p.vs_n + b] = L.vs[rs * p.vs_n + b];
    __syncthreads();
  }
}

}  // namespace

cudaError_t tree_verify_launch(const TreeVerifyParams& p, int groups, cudaStream_t s) {
  if (groups == 0) return cudaSuccess;
  SQ_LAUNCH(tree_verify_kernel, dim3(groups), dim3(kVThreads), 0, s, 1, p);
  return cudaGetLastError();
}

cudaError_t kv_compact_launch(const KvCompactParams& p, int layers, cudaStream_t s) {
  if (p.n_pairs == 0 || layers == 0) return cudaSuccess;
  SQ_LAUNCH(kv_compact_kernel, dim3(dim3(layers, p.Hkv)), dim3(128), 0, s, 1, p);
  return cudaGetLastError();
}

}  // namespace sq
