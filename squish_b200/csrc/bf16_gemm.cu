// bf16_gemm.cu — persistent tcgen05 GEMM y[M, N] = x[M, K] . W[N, K]^T for bf16 operands.
//
// The large-M (prefill) path of the weight-only quantized linear layers: the weight codes are
// first expanded to bf16 (dequant_weight_launch), then this kernel runs at tensor-core rate,
// instead of dequantizing every weight tile once per token tile inside the GEMM.
//
// One CTA per SM loops over 128 x 256 output tiles (128 tokens = MMA M = TMEM lanes, 256
// features = MMA N = TMEM columns), tile t -> (m = t % Mt, n = t / Mt) so CTAs running at the
// same time share a weight block in L2:
//
//   warp 0     TMA producer: x tile [128 x 64] and W tile [256 x 64] per stage (128B swizzle)
//   warp 1     MMA issuer: 4 x tcgen05.mma (K = 16) per stage into one of two TMEM accumulators
//   warp 2     TMEM allocator (512 columns = two 128 x 256 fp32 accumulators)
//   warps 4-7  epilogue: TMEM lane quarter (warp & 3) -> bias / residual / SwiGLU -> bf16 stores
//
// The epilogue of tile i runs while the MMAs of tile i+1 accumulate into the other buffer.
// Every wait is bounded; a timeout records an error code in p.status and the CTA leaves
// (freeing its tensor memory).
#include "bf16_gemm.h"
#include "launch.cuh"
#include "sm100.cuh"
#include "w4a16_gemm.h"

namespace sq {
namespace {

constexpr int TM = 128;
constexpr int TN = 256;
constexpr int TK = 64;
constexpr int kStages = 4;
constexpr int kABytes = TM * TK * 2;
constexpr int kBBytes = TN * TK * 2;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 2 * TN;
constexpr int kBarBytes = 256;
constexpr size_t kSmem = (size_t)kStages * kStageBytes + kBarBytes + 1024;

struct Ring {
  int s = 0;
  uint32_t ph = 0;
  __device__ __forceinline__ void next() {
    if (++s == kStages) {
      s = 0;
      ph ^= 1u;
    }
  }
};

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 32 consecutive outputs of row m starting at column n (vectorised when the whole run is in
// range and p.vec allows 16-byte accesses).
__device__ __forceinline__ void store_run(const Bf16GemmParams& p, int m, int n, int ncols, float (&v)[32],
                                          bool add_bias_res) {
  if (add_bias_res) {
    if (p.vec && n + 32 <= ncols) {
      if (p.bias != nullptr) {
        const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + n);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 b = __ldg(b4 + q);
          const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[q * 8 + j] += __bfloat162float(bb[j]);
        }
      }
      if (p.residual != nullptr) {
        const uint4* r4 = reinterpret_cast<const uint4*>(p.residual + (size_t)m * p.ldr + n);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 r = r4[q];
          const __nv_bfloat16* rr = reinterpret_cast<const __nv_bfloat16*>(&r);
#pragma unroll
          for (int j = 0; j < 8; ++j) v[q * 8 + j] += __bfloat162float(rr[j]);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (n + j < ncols) {
          if (p.bias != nullptr) v[j] += __bfloat162float(p.bias[n + j]);
          if (p.residual != nullptr) v[j] += __bfloat162float(p.residual[(size_t)m * p.ldr + n + j]);
        }
      }
    }
  }
  __nv_bfloat16* dst = p.y + (size_t)m * p.ldy + n;
  if (p.vec && n + 32 <= ncols) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      d4[q] = make_uint4(pack_bf2(v[8 * q], v[8 * q + 1]), pack_bf2(v[8 * q + 2], v[8 * q + 3]),
                         pack_bf2(v[8 * q + 4], v[8 * q + 5]), pack_bf2(v[8 * q + 6], v[8 * q + 7]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n + j < ncols) dst[j] = __float2bfloat16(v[j]);
  }
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The epilogue of one 128 x 256 tile for this thread's row m; get(col, v) yields the 32 fp32
// sums of columns [col, col + 32) of the tile (from TMEM, or the split-K partials).
template <class Get>
__device__ __forceinline__ void epilogue_tile(const Bf16GemmParams& p, int m, int n0, Get&& get) {
  if (p.epilogue == EPI_SILU_MUL) {
    // rows of W: [gate 64 | up 64] blocks -> output columns n0/2 + [0, 128)
#pragma unroll 1
    for (int g = 0; g < TN / 128; ++g) {
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float gv[32], uv[32];
        get(g * 128 + h * 32, gv);
        get(g * 128 + 64 + h * 32, uv);
        if (m < p.M) {
#pragma unroll
          for (int j = 0; j < 32; ++j) gv[j] = silu_f(gv[j]) * uv[j];
          store_run(p, m, n0 / 2 + g * 64 + h * 32, p.N / 2, gv, false);
        }
      }
    }
  } else {
#pragma unroll 1
    for (int c0 = 0; c0 < TN; c0 += 32) {
      float v[32];
      get(c0, v);
      if (m < p.M && n0 + c0 < p.N) store_run(p, m, n0 + c0, p.N, v, true);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    bf16_gemm_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                     const Bf16GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  __shared__ int last_split;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (p.M + TM - 1) / TM;
  const int S = p.splits;
  const int items = mt * ((p.N + TN - 1) / TN) * S;
  const int nkb_all = (p.K + TK - 1) / TK;
  int* status = p.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrive per epilogue warp
    }
    fence_mbar_init();
    prefetch_tmap(&amap);
    prefetch_tmap(&bmap);
  }
  if (warp == 2) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    pdl_wait();  // x (and the expanded weights) come from earlier kernels
    Ring r;
    bool ok = true;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
      const int t = w / S, kb0 = (w % S) * p.kb_per_split;
      const int m0 = (t % mt) * TM, n0 = (t / mt) * TN;
      const int nkb = min(nkb_all - kb0, p.kb_per_split);
      for (int i = 0; i < nkb; ++i) {
        const int kb = kb0 + i;
        if (!mbar_wait(&empty[r.s], r.ph ^ 1u, status, SQ_ERR_TIMEOUT_W)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          uint8_t* st = smem + r.s * kStageBytes;
          mbar_expect_tx(&full[r.s], kStageBytes);
          tma_load_2d(st, &amap, kb * TK, m0, &full[r.s]);
          tma_load_2d(st + kABytes, &bmap, kb * TK, n0, &full[r.s]);
        }
        __syncwarp();
        r.next();
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_bf16_f32(TM, TN);
    Ring r;
    int it = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t ph = (uint32_t)(it >> 1) & 1u;
      const int nkb = min(nkb_all - (w % S) * p.kb_per_split, p.kb_per_split);
      if (!mbar_wait(&acc_empty[buf], ph ^ 1u, status, SQ_ERR_TIMEOUT_ACC)) break;
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(buf * TN);
      for (int kb = 0; kb < nkb; ++kb) {
        if (!mbar_wait(&full[r.s], r.ph, status, SQ_ERR_TIMEOUT_X)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
          const uint32_t a = smem_u32(smem + r.s * kStageBytes), b = a + kABytes;
#pragma unroll
          for (int k = 0; k < TK / 16; ++k)
            mma_bf16_ss(d, sdesc_sw128(a + k * 32), sdesc_sw128(b + k * 32), idesc, (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[r.s]);
        }
        __syncwarp();
        r.next();
      }
      if (!ok) break;
      if (elect_one()) mma_commit(&acc_full[buf]);
      __syncwarp();
    }
  } else if (warp >= 4) {
    // ------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int it = 0;
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t ph = (uint32_t)(it >> 1) & 1u;
      const int t = w / S;
      if (!mbar_wait(&acc_full[buf], ph, status, SQ_ERR_TIMEOUT_ACC)) break;
      tc_fence_after();
      const int m = (t % mt) * TM + row, n0 = (t / mt) * TN;
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * TN);
      if (S == 1) {
        epilogue_tile(p, m, n0, [&](int col, float(&v)[32]) {
          uint32_t u[32];
          tmem_ld32(base + (uint32_t)col, u);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(u[j]);
        });
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        continue;
      }
      // split-K: partial -> ws (column-major: a warp stores 128 contiguous bytes per column)
      float* part = p.ws + (size_t)w * (TM * TN);
#pragma unroll 1
      for (int c0 = 0; c0 < TN; c0 += 32) {
        uint32_t u[32];
        tmem_ld32(base + (uint32_t)c0, u);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) __stcg(part + (c0 + j) * TM + row, __uint_as_float(u[j]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);  // the accumulator is free again
      __threadfence();
      epi_sync();
      if (threadIdx.x == 128) last_split = (atomicAdd(p.counters + t, 1) == S - 1);
      epi_sync();
      if (!last_split) continue;
      __threadfence();
      const float* parts = p.ws + (size_t)t * S * (TM * TN);
      epilogue_tile(p, m, n0, [&](int col, float(&v)[32]) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
        for (int sp = 0; sp < S; ++sp) {  // split order: deterministic
          const float* src = parts + (size_t)sp * (TM * TN) + col * TM + row;
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += __ldcg(src + j * TM);
        }
      });
      if (threadIdx.x == 128) p.counters[t] = 0;
      epi_sync();  // last_split is rewritten by the next item
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

cudaError_t bf16_gemm_launch(const CUtensorMap& amap, const CUtensorMap& bmap, Bf16GemmParams p, int num_sms,
                             long long ws_floats, int n_counters, cudaStream_t s) {
  if (p.M <= 0 || p.N <= 0) return cudaSuccess;
  if (p.epilogue == EPI_SILU_MUL && p.N % 128 != 0) return cudaErrorInvalidValue;
  const int tiles = ((p.M + TM - 1) / TM) * ((p.N + TN - 1) / TN);
  const int nkb = (p.K + TK - 1) / TK;
  // split K when the tiles fill less than ~2/3 of the SMs and K is long: the last split of a
  // tile sums all partials alone, which only pays off at >= 32 k-blocks per split (measured:
  // K = 18944 gains 2x at 28 tiles, K = 3584 loses)
  int S = 1;
  if (3 * tiles < 2 * num_sms && p.ws != nullptr && p.counters != nullptr && tiles <= n_counters) {
    S = min(min(num_sms / tiles, nkb / 32), 16);
    while (S > 1 && (long long)tiles * S * TM * TN > ws_floats) --S;
    S = max(S, 1);
  }
  p.kb_per_split = (nkb + S - 1) / S;
  p.splits = (nkb + p.kb_per_split - 1) / p.kb_per_split;
  const int items = tiles * p.splits;
  cudaError_t e = cudaFuncSetAttribute(bf16_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  if (e != cudaSuccess) return e;
  SQ_LAUNCH(bf16_gemm_kernel, dim3(items < num_sms ? items : num_sms), dim3(kThreads), kSmem, s, 1u, amap, bmap, p);
  return cudaSuccess;
}

}  // namespace sq
