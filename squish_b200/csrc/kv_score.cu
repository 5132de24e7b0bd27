// kv_score.cu — attention mass per KV page, for heavy-hitter (H2O-style) page eviction.
//
// For every decode row b and KV head h, the attention probabilities of the GQA group's query
// heads over the row's kept keys (softmax over all of them, scale sm_scale) are summed per page
// and added to mass[page] (float, indexed by the physical page id). A CTA owns one (row, KV
// head): pass 1 computes each query head's running max and normaliser over the keys, pass 2
// recomputes the scores and accumulates exp(s - m) / l per page in shared memory, then one
// atomic add per page goes to global memory. Keys are dequantized with the page format's
// helpers (kv_format.cuh), 8 dims per lane; D / 8 lanes share a key.
//
// The reference scores tokens by accumulated attention on the host after each step
// (squish/kv/kv_cache.py:3590-3735, H2O); here the scores come from the cache on the device,
// page granular, and only on the steps that refresh them.
#include "kernels.h"
#include "kv_format.cuh"
#include "launch.cuh"

namespace sq {

namespace {

constexpr int kScoreThreads = 128;
constexpr int kMaxScorePages = 4096;  // kept pages per row held in shared memory

template <int D, int FMT, int GQ>
__global__ void __launch_bounds__(kScoreThreads) page_mass_kernel(const PageMassParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int LPK = D / 8;          // lanes per key
  constexpr int KPW = 32 / LPK;       // keys per warp and iteration
  constexpr int NW = kScoreThreads / 32;
  __shared__ float page_acc[kMaxScorePages];
  __shared__ float red_m[NW * KPW][GQ], red_l[NW * KPW][GQ];
  __shared__ float fin_m[GQ], fin_l[GQ];
  const int b = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane / LPK, part = lane % LPK;  // key slot within the warp, 8-dim chunk of the key
  const int n = p.seq_lens[b];
  const int npages = (n + p.page_size - 1) / p.page_size;
  if (n <= 0 || npages > kMaxScorePages) return;
  // this lane's 8 dims of every query head of the group
  float q[GQ][8];
#pragma unroll
  for (int g = 0; g < GQ; ++g) {
    const __nv_bfloat16* qr = p.q + (size_t)b * p.ld_q + (size_t)(h * GQ + g) * D + part * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(qr);
    const __nv_bfloat162* v2 = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(v2[i]);
      q[g][2 * i] = f.x * p.sm_scale;
      q[g][2 * i + 1] = f.y * p.sm_scale;
    }
  }
  const int cb = kv_code_bytes(FMT, D), ns = kv_nscale(FMT, D, p.group);
  const int* bt = p.block_tables + (size_t)b * p.bt_stride;
  // scores of key j for every head of the group, reduced over the LPK lanes of the key
  // (every lane runs the shuffles: a slot past the row or on a bad page computes on page 0 and
  // reports false)
  auto scores = [&](int j, float (&s)[GQ]) -> bool {
    const bool in = j < n;
    int page = bt[(in ? j : 0) / p.page_size];
    const bool ok = in && kv_index_ok(page, p.num_pages, p.status);
    if (!ok) page = 0;
    const size_t row = ((size_t)page * p.Hkv + h) * p.page_size + (in ? j : 0) % p.page_size;
    const uint4 kv = kv_dequant8<FMT>(p.k_codes + row * cb, p.k_scales + row * ns, part * 8, p.group);
    const __nv_bfloat162* k2 = reinterpret_cast<const __nv_bfloat162*>(&kv);
    float k[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(k2[i]);
      k[2 * i] = f.x;
      k[2 * i + 1] = f.y;
    }
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) a = fmaf(q[g][i], k[i], a);
#pragma unroll
      for (int o = LPK / 2; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      s[g] = a;
    }
    return ok;
  };
  // pass 1: per-head max and normaliser (online), per key slot
  float m[GQ], l[GQ];
#pragma unroll
  for (int g = 0; g < GQ; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
  }
  const int slot = warp * KPW + sub;
  for (int j0 = 0; j0 < n; j0 += NW * KPW) {
    const int j = j0 + slot;
    float s[GQ];
    if (scores(j, s)) {
#pragma unroll
      for (int g = 0; g < GQ; ++g) {
        const float mn = fmaxf(m[g], s[g]);
        l[g] = l[g] * __expf(m[g] - mn) + __expf(s[g] - mn);
        m[g] = mn;
      }
    }
  }
  for (int i = threadIdx.x; i < npages; i += kScoreThreads) page_acc[i] = 0.f;
  if (part == 0) {
#pragma unroll
    for (int g = 0; g < GQ; ++g) {
      red_m[slot][g] = m[g];
      red_l[slot][g] = l[g];
    }
  }
  __syncthreads();
  if (threadIdx.x < GQ) {
    const int g = threadIdx.x;
    float mm = -INFINITY, ll = 0.f;
    for (int t = 0; t < NW * KPW; ++t) {
      const float mt = red_m[t][g];
      if (mt == -INFINITY) continue;
      const float mn = fmaxf(mm, mt);
      ll = ll * __expf(mm - mn) + red_l[t][g] * __expf(mt - mn);
      mm = mn;
    }
    fin_m[g] = mm;
    fin_l[g] = ll > 0.f ? ll : 1.f;
  }
  __syncthreads();
  // pass 2: probability mass per page, summed over the group's heads
  for (int j0 = 0; j0 < n; j0 += NW * KPW) {
    const int j = j0 + slot;
    float s[GQ];
    const bool ok = scores(j, s);
    if (ok && part == 0) {
      float pm = 0.f;
#pragma unroll
      for (int g = 0; g < GQ; ++g) pm += __expf(s[g] - fin_m[g]) / fin_l[g];
      atomicAdd(&page_acc[j / p.page_size], pm);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < npages; i += kScoreThreads) {
    const int page = bt[i];
    if (page >= 0 && page < p.num_pages) atomicAdd(p.mass + page, page_acc[i]);
  }
}

template <int D, int FMT>
cudaError_t launch_d_f(const PageMassParams& p, int gq, cudaStream_t s) {
  const dim3 grid(p.B, p.Hkv);
  switch (gq) {
    case 1: SQ_LAUNCH((page_mass_kernel<D, FMT, 1>), grid, dim3(kScoreThreads), 0, s, 1, p); break;
    case 2: SQ_LAUNCH((page_mass_kernel<D, FMT, 2>), grid, dim3(kScoreThreads), 0, s, 1, p); break;
    case 4: SQ_LAUNCH((page_mass_kernel<D, FMT, 4>), grid, dim3(kScoreThreads), 0, s, 1, p); break;
    case 5: SQ_LAUNCH((page_mass_kernel<D, FMT, 5>), grid, dim3(kScoreThreads), 0, s, 1, p); break;
    case 6: SQ_LAUNCH((page_mass_kernel<D, FMT, 6>), grid, dim3(kScoreThreads), 0, s, 1, p); break;
    case 7: SQ_LAUNCH((page_mass_kernel<D, FMT, 7>), grid, dim3(kScoreThreads), 0, s, 1, p); break;
    case 8: SQ_LAUNCH((page_mass_kernel<D, FMT, 8>), grid, dim3(kScoreThreads), 0, s, 1, p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_d(const PageMassParams& p, int gq, cudaStream_t s) {
  switch (p.fmt_k) {
    case KV_BF16: return launch_d_f<D, KV_BF16>(p, gq, s);
    case KV_INT8: return launch_d_f<D, KV_INT8>(p, gq, s);
    case KV_INT4: return launch_d_f<D, KV_INT4>(p, gq, s);
    case KV_INT2: return launch_d_f<D, KV_INT2>(p, gq, s);
    case KV_K8: return launch_d_f<D, KV_K8>(p, gq, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t page_mass_launch(const PageMassParams& p, cudaStream_t s) {
  if (p.B == 0) return cudaSuccess;
  if (p.Hkv <= 0 || p.Hq % p.Hkv != 0 || p.group < 32 || p.D % p.group != 0 || p.ld_q < p.Hq * p.D ||
      p.ld_q % 8 != 0)
    return cudaErrorInvalidValue;
  const int gq = p.Hq / p.Hkv;
  switch (p.D) {
    case 32: return launch_d<32>(p, gq, s);
    case 64: return launch_d<64>(p, gq, s);
    case 128: return launch_d<128>(p, gq, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace sq
