// attention_tc.cu — causal prefill attention over the paged, quantized KV cache on the
// Blackwell tensor cores (tcgen05), head dim 128.
//
// A CTA computes 128 rows = P query positions x HS head slots of one KV head (HS = the query
// heads per KV head rounded up to a power of two, P = 128 / HS), so each K/V tile it
// dequantizes serves all query heads of the group. Per tile of 128 keys:
//
//   S  = Q . K^T         tcgen05.mma  A = Q (smem, TMA)  B = K (smem, K-major)  D = TMEM
//   P  = 2^(S' - m)      softmax warps: TMEM -> registers -> bf16 pairs -> TMEM
//   O += P . V           tcgen05.mma  A = P (TMEM)       B = V (smem, d-major)  D = TMEM
//
// S is double-buffered in TMEM, so the tensor core computes S(j+1) while the softmax warps
// turn S(j) into P(j). The running row max is raised (and O rescaled through registers)
// only when it grows by more than 2^8; P and the row sum always use the same stale max, so
// the result is exact and most tiles skip the O round trip.
//
// TMEM columns: O [0,128)  S0 [128,256)  S1 [256,384)  P0 [384,448)  P1 [448,512).
// Warps: 0 = TMEM allocation, Q load and MMA issue; 4-11 = softmax and epilogue (thread = row =
// TMEM lane; two warpgroups split each row's 128 keys / 128 output dims; a warp reaches only
// the TMEM lanes of its rank mod 4); 1 = page loader (bulk copies of the tile's pages into a
// shared-memory staging slot); 12-15 = K/V producers (thread = key: dequantize its staged
// rows, store in the 128-byte-swizzled operand layout); 2-3 idle.
//
// Every wait is bounded; a timeout records an error code in *status and the CTA leaves
// through the common teardown (freeing its tensor memory).
#include "kernels.h"
#include "kv_format.cuh"
#include "launch.cuh"
#include "sm100.cuh"

namespace sq {
namespace {

constexpr int TD = 128;                  // head dim
constexpr int TR = 128;                  // rows per CTA
constexpr int TKEYS = 128;               // keys per tile
constexpr int kAtomBytes = 128 * 128;    // 128 rows x 64 bf16 (one 128-byte swizzle column)
constexpr int kTileBytes = 2 * kAtomBytes;
constexpr int kThreadsT = 512;
constexpr uint32_t kTmemT = 512;
constexpr uint32_t kColO = 0, kColS = 128, kColP = 384;

struct TcAttnArgs {
  AttnParams p;
  int hs;      // head slots per CTA (power of two >= Gq)
  int npos;    // query positions per CTA (128 / hs)
  int sub;     // CTAs per 32-position host tile
  int* status;
  // optional pipeline trace of CTA (0, 0): clock64() per event and tile (< 32), [16][32]
  unsigned long long* trace;
};

// trace events: 0 loader issued, 1 staged data arrived, 2 K stored, 3 V stored, 4 S issued,
// 5 S ready (softmax), 6 P ready, 7 PV issued, 8 O rescaled, 9 setup done, 10 epilogue done
__device__ __forceinline__ void tmark(unsigned long long* tr, int ev, int j) {
  if (tr != nullptr && j < 32) tr[ev * 32 + j] = clock64();
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// named barrier of the two softmax warpgroups (warps 4-11)
__device__ __forceinline__ void softmax_sync() { asm volatile("bar.sync 2, 256;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// B operand stored d-major (rows = keys, 128 bytes = 64 dims per row, swizzled): leading
// byte offset = next 64-dim column (16 KiB), stride byte offset = next 8 keys (1 KiB).
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)(kAtomBytes >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Operand offset of 16-dim K step kk (0..7) of a K-major 128-dim tile: two 64-dim columns.
__device__ __forceinline__ uint32_t kmajor_step(uint32_t base, int kk) {
  return base + (uint32_t)((kk >> 2) * kAtomBytes + (kk & 3) * 32);
}

// K/V staging: per tile of 128 keys, the raw codes and scales of its pages are brought into a
// shared-memory slot by 1-D bulk copies (one elected lane per page issues four: K codes,
// K scales, V codes, V scales, each a contiguous run of page_size rows in the pool), so the
// producer threads dequantize from shared memory with no global latency on their path.
template <int FK, int FV>
struct Stage {
  static constexpr int kCBK = kv_code_bytes(FK, TD), kCBV = kv_code_bytes(FV, TD);
  static constexpr int kScaleRow = 16;  // bytes reserved per row for scales (<= 8 fp16)
  static constexpr int kKC = 0, kKS = kKC + TKEYS * kCBK, kVC = kKS + TKEYS * kScaleRow,
                       kVS = kVC + TKEYS * kCBV;
  static constexpr int kBytes = kVS + TKEYS * kScaleRow;
  static constexpr int kFixed = 5 * kTileBytes + 256 + 1024;  // Q, K[2], V[2], barriers, alignment
  static constexpr int kSlots = kFixed + 2 * kBytes <= 220 * 1024 ? 2 : 1;
  static constexpr size_t kSmem = (size_t)kFixed + (size_t)kSlots * kBytes;
};

// One staged K or V row (128 dims) in registers, with its scale / zero per 32-dim quarter
// already converted, so dequantizing a chunk of 8 dims is a few bit operations and two
// bf16x2 FMAs (no per-chunk group arithmetic).
template <int FMT>
struct FastRow {
  static constexpr int kWords = kv_code_bytes(FMT, TD) / 4;
  static constexpr bool k8bit = (FMT == KV_INT8 || FMT == KV_K8);
  uint32_t w[kWords];
  uint32_t s2[4], z2[4];  // bf16x2 (4/2-bit formats)
  float sf[4], zf[4];     // fp32 (8-bit formats)

  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int i = 0; i < kWords; ++i) w[i] = 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      s2[q] = z2[q] = 0u;
      sf[q] = zf[q] = 0.f;
    }
  }

  // codes / scales: this row in the staging slot; gshift = log2(group / 32)
  __device__ __forceinline__ void load(const uint8_t* codes, const __half* scales, int gshift) {
#pragma unroll
    for (int i = 0; i < kWords / 4; ++i) {
      const uint4 v = *reinterpret_cast<const uint4*>(codes + 16 * i);
      w[4 * i] = v.x;
      w[4 * i + 1] = v.y;
      w[4 * i + 2] = v.z;
      w[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int g = q >> gshift;
      float sc, ze;
      if constexpr (kv_asym(FMT)) {
        sc = __half2float(scales[2 * g]);
        ze = __half2float(scales[2 * g + 1]);
      } else {
        sc = __half2float(scales[g]);
        ze = FMT == KV_INT4 ? -7.5f * sc : FMT == KV_INT2 ? -1.5f * sc : 0.f;
      }
      if constexpr (k8bit) {
        sf[q] = sc;
        zf[q] = ze;
      } else {
        s2[q] = pack_bf2(sc, sc);
        z2[q] = pack_bf2(ze, ze);
      }
    }
  }

  __device__ __forceinline__ uint4 dequant(int c) const {
    const int q = c >> 2;  // 32-dim quarter (static in unrolled loops)
    uint32_t o[4];
    if constexpr (FMT == KV_INT4 || FMT == KV_V4) {
      // byte i of the word = dims (2i, 2i+1) as (low, high) nibble
      const uint32_t lo = w[c] & 0x0F0F0F0Fu, hi = (w[c] >> 4) & 0x0F0F0F0Fu;
      const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t t = (__byte_perm(lo, hi, (uint32_t)(i | ((4 + i) << 8))) & 0x00FF00FFu) | 0x43004300u;
        const __nv_bfloat162 v = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&t), k128);  // exact q
        const __nv_bfloat162 r = __hfma2(v, *reinterpret_cast<const __nv_bfloat162*>(&s2[q]),
                                         *reinterpret_cast<const __nv_bfloat162*>(&z2[q]));
        o[i] = *reinterpret_cast<const uint32_t*>(&r);
      }
    } else if constexpr (FMT == KV_INT2) {
      // 16 bits per chunk: dim 4i+j at bits 2j of nibble i
      const uint32_t word = (w[c >> 1] >> ((c & 1) * 16)) & 0xFFFFu;
      const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = (word >> (4 * i)) & 0x3u, hi = (word >> (4 * i + 2)) & 0x3u;
        uint32_t t = lo | (hi << 16) | 0x43004300u;
        const __nv_bfloat162 v = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&t), k128);
        const __nv_bfloat162 r = __hfma2(v, *reinterpret_cast<const __nv_bfloat162*>(&s2[q]),
                                         *reinterpret_cast<const __nv_bfloat162*>(&z2[q]));
        o[i] = *reinterpret_cast<const uint32_t*>(&r);
      }
    } else {  // 8-bit
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t word = w[2 * c + (i >> 1)];
        const int sh = (i & 1) * 16;
        float a, b;
        if constexpr (FMT == KV_INT8) {
          a = (float)(int8_t)((word >> sh) & 0xFF);
          b = (float)(int8_t)((word >> (sh + 8)) & 0xFF);
        } else {
          a = (float)((word >> sh) & 0xFF);
          b = (float)((word >> (sh + 8)) & 0xFF);
        }
        o[i] = pack_bf2(fmaf(a, sf[q], zf[q]), fmaf(b, sf[q], zf[q]));
      }
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
  }
};

template <int FMT>
__device__ __forceinline__ void store_row(const FastRow<FMT>& rp, uint8_t* dst, int sw) {
#pragma unroll
  for (int c = 0; c < TD / 8; ++c)
    *reinterpret_cast<uint4*>(dst + (c >> 3) * kAtomBytes + (((c & 7) ^ sw) << 4)) = rp.dequant(c);
}

// Loader (one warp): for every tile, wait for a free staging slot and issue its bulk copies.
template <int FK, int FV>
__device__ __forceinline__ void load_stages(const AttnParams& p, uint8_t* stg, uint64_t* stg_full,
                                            uint64_t* stg_empty, int h, int b, int nt, int kv_end, int* status,
                                            unsigned long long* tr) {
  using St = Stage<FK, FV>;
  const int lane = threadIdx.x & 31;
  const int PS = p.page_size;
  const int ppt = TKEYS / PS;
  const int nsk = kv_nscale(FK, TD, p.group), nsv = kv_nscale(FV, TD, p.group);
  const int* bt = p.block_tables + (size_t)b * p.bt_stride;
  for (int j = 0; j < nt; ++j) {
    const int slot = j % St::kSlots;
    const uint32_t par = ((uint32_t)(j / St::kSlots) & 1u) ^ 1u;
    if (!mbar_wait(&stg_empty[slot], par, status, SQ_ERR_TIMEOUT_W)) break;
    const int np = min(ppt, (kv_end - j * TKEYS + PS - 1) / PS);
    uint8_t* st = stg + slot * St::kBytes;
    if (lane == 0)
    {
      mbar_expect_tx(&stg_full[slot], (uint32_t)(np * PS * (St::kCBK + St::kCBV + 2 * nsk + 2 * nsv)));
      tmark(tr, 0, j);
    }
    __syncwarp();
    if (lane < np) {
      int page = __ldg(bt + j * ppt + lane);
      // an entry outside the pool is recorded and read as page 0 (the expected byte count of
      // the stage barrier stays the same, so the pipeline does not stall)
      if (!kv_index_ok(page, p.num_pages, p.status)) page = 0;
      const size_t row0 = ((size_t)page * p.Hkv + h) * PS;
      const int r0 = lane * PS;
      bulk_g2s(st + St::kKC + r0 * St::kCBK, p.k_codes + row0 * St::kCBK, (uint32_t)(PS * St::kCBK), &stg_full[slot]);
      bulk_g2s(st + St::kKS + r0 * 2 * nsk, p.k_scales + row0 * nsk, (uint32_t)(PS * 2 * nsk), &stg_full[slot]);
      bulk_g2s(st + St::kVC + r0 * St::kCBV, p.v_codes + row0 * St::kCBV, (uint32_t)(PS * St::kCBV), &stg_full[slot]);
      bulk_g2s(st + St::kVS + r0 * 2 * nsv, p.v_scales + row0 * nsv, (uint32_t)(PS * 2 * nsv), &stg_full[slot]);
    }
    __syncwarp();
  }
}

// Producers (thread = key kk of the tile): staged codes -> bf16 K / V operand tiles.
template <int FK, int FV>
__device__ __forceinline__ void produce_kv(const AttnParams& p, const uint8_t* stg, uint64_t* stg_full,
                                           uint64_t* stg_empty, uint8_t* Ks, uint8_t* Vs, uint64_t* k_full,
                                           uint64_t* k_empty, uint64_t* v_full, uint64_t* v_empty, int kk, int nt,
                                           int kv_end, int* status, unsigned long long* tr) {
  if (kk != 0) tr = nullptr;
  using St = Stage<FK, FV>;
  const int lane = threadIdx.x & 31;
  const int nsk = kv_nscale(FK, TD, p.group), nsv = kv_nscale(FV, TD, p.group);
  const int sw = kk & 7;
  const uint32_t roff = (uint32_t)kk * 128u;
  const int gshift = p.group >= 128 ? 2 : p.group >= 64 ? 1 : 0;
  for (int j = 0; j < nt; ++j) {
    const int cur = j & 1;
    const uint32_t par = ((uint32_t)(j >> 1) & 1u) ^ 1u;
    const int slot = j % St::kSlots;
    const bool valid = j * TKEYS + kk < kv_end;
    if (!mbar_wait(&stg_full[slot], (uint32_t)(j / St::kSlots) & 1u, status, SQ_ERR_TIMEOUT_W)) break;
    tmark(tr, 1, j);
    const uint8_t* st = stg + slot * St::kBytes;
    FastRow<FK> kr;
    FastRow<FV> vr;
    if (valid) {
      kr.load(st + St::kKC + kk * St::kCBK, reinterpret_cast<const __half*>(st + St::kKS + kk * 2 * nsk), gshift);
      vr.load(st + St::kVC + kk * St::kCBV, reinterpret_cast<const __half*>(st + St::kVS + kk * 2 * nsv), gshift);
    } else {
      kr.clear();
      vr.clear();
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&stg_empty[slot]);  // the slot's codes are in registers now
    if (!mbar_wait(&k_empty[cur], par, status, SQ_ERR_TIMEOUT_W)) break;
    store_row<FK>(kr, Ks + cur * kTileBytes + roff, sw);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&k_full[cur]);
    tmark(tr, 2, j);
    if (!mbar_wait(&v_empty[cur], par, status, SQ_ERR_TIMEOUT_W)) break;
    store_row<FV>(vr, Vs + cur * kTileBytes + roff, sw);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&v_full[cur]);
    tmark(tr, 3, j);
  }
}

template <int FK, int FV>
__global__ void __launch_bounds__(kThreadsT, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ TcAttnArgs a) {
  const AttnParams& p = a.p;
  // heavier (later) query tiles first
  const int item = (int)(gridDim.x - 1 - blockIdx.x);
  const int tile = item / a.sub;
  const int b = __ldg(p.tile_seq + tile);
  const int qlen = __ldg(p.q_len + b);
  const int q0 = __ldg(p.tile_q0 + tile) + (item % a.sub) * a.npos;
  if (q0 >= qlen) return;  // whole CTA, before any setup
  const int h = blockIdx.y;
  const int Gq = p.Hq / p.Hkv;
  const int ctx = __ldg(p.ctx_len + b);
  const int qn = min(a.npos, qlen - q0);
  const int pos0 = ctx - qlen + q0;
  const int kv_end = pos0 + qn;
  const int nt = (kv_end + TKEYS - 1) / TKEYS;
  int* status = a.status;
  unsigned long long* tr = (a.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0) ? a.trace : nullptr;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Qs = smem;
  uint8_t* Ks = smem + kTileBytes;          // [2] tiles
  uint8_t* Vs = smem + 3 * kTileBytes;      // [2] tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 5 * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* k_empty = bars + 3;
  uint64_t* v_full = bars + 5;
  uint64_t* v_empty = bars + 7;
  uint64_t* s_full = bars + 9;
  uint64_t* p_full = bars + 11;
  // PV(j) completes o_done[j & 1]: a waiter never lags two phases behind one of them (the
  // softmax has seen S(j), committed after PV(j-2)), so parity waits stay unambiguous
  uint64_t* o_done = bars + 13;
  uint64_t* stg_full = bars + 15;
  uint64_t* stg_empty = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  uint8_t* stg = smem + 5 * kTileBytes + 256;  // staging slots (16-byte aligned)

  __shared__ float row_max[6 * TR];  // [tile parity][group][row] partial maxima; [4 + group][row] row sums
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 4);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 4);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);  // both softmax warpgroups
      mbar_init(&o_done[i], 1);
      mbar_init(&stg_full[i], 1);
      mbar_init(&stg_empty[i], 4);
    }
    fence_mbar_init();
    prefetch_tmap(&qmap);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q and the KV pages are written by the preceding kernels
  pdl_trigger();
  if (threadIdx.x == 0) tmark(tr, 9, 0);

  if (warp == 0) {
    // ------------------------------------------------ Q load + MMA issue
    constexpr uint32_t idesc_s = idesc_bf16_f32(TR, TKEYS);
    constexpr uint32_t idesc_pv = idesc_bf16_f32(TR, TD) | (1u << 16);  // B (V) is d-major
    const int qrow0 = __ldg(p.q_start + b) + q0;
    if (elect_one()) {
      mbar_expect_tx(q_full, kTileBytes);
      tma_load_3d(Qs, &qmap, 0, h * Gq, qrow0, q_full);
      tma_load_3d(Qs + kAtomBytes, &qmap, 64, h * Gq, qrow0, q_full);
    }
    __syncwarp();
    bool ok = mbar_wait(q_full, 0, status, SQ_ERR_TIMEOUT_X);
    const uint32_t qa = smem_u32(Qs);
    // Issue S(s) once K(s) is staged and S buffer s & 1 is free (PV(s-2) issued), and PV(j) once
    // P(j) and V(j) are ready, whichever comes first: polling both keeps PV off the path of
    // the K producers. Idle polls sleep briefly (this warp shares its sub-partition with a
    // producer and two softmax warps) and are bounded.
    int s_next = 0, pv_next = 0;
    uint32_t idle = 0;
    while (ok && pv_next < nt) {
      bool prog = false;
      if (s_next < nt && s_next <= pv_next + 1) {
        const int sl = s_next & 1;
        if (__shfl_sync(0xffffffffu, mbar_test(&k_full[sl], (uint32_t)(s_next >> 1) & 1u), 0)) {
          tc_fence_after();
          if (elect_one()) {
            const uint32_t ka = smem_u32(Ks + sl * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < TD / 16; ++kk)
              mma_bf16_ss(tmem + kColS + (uint32_t)(sl * 128), sdesc_sw128(kmajor_step(qa, kk)),
                          sdesc_sw128(kmajor_step(ka, kk)), idesc_s, kk > 0 ? 1u : 0u);
            mma_commit(&k_empty[sl]);
            mma_commit(&s_full[sl]);
            tmark(tr, 4, s_next);
          }
          __syncwarp();
          ++s_next;
          prog = true;
        }
      }
      if (pv_next < s_next) {
        const int j = pv_next, sl = j & 1;
        const uint32_t par = (uint32_t)(j >> 1) & 1u;
        if (__shfl_sync(0xffffffffu, mbar_test(&p_full[sl], par) && mbar_test(&v_full[sl], par), 0)) {
          tc_fence_after();
          if (elect_one()) {
            const uint32_t va = smem_u32(Vs + sl * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < TKEYS / 16; ++kk)
              mma_bf16_ts(tmem + kColO, tmem + kColP + (uint32_t)(sl * 64 + kk * 8), sdesc_mn_sw128(va + kk * 2048),
                          idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
            mma_commit(&v_empty[sl]);
            mma_commit(&o_done[sl]);
            tmark(tr, 7, j);
          }
          __syncwarp();
          ++pv_next;
          prog = true;
        }
      }
      if (prog) {
        idle = 0;
      } else if (++idle >= (1u << 24)) {  // ~seconds without progress
        atomicCAS(status, SQ_OK, SQ_ERR_TIMEOUT_A);
        ok = false;
      } else {
        if ((idle & 255u) == 0 && *reinterpret_cast<volatile int*>(status) != SQ_OK) ok = false;
        __nanosleep(64);
      }
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------ softmax + epilogue
    // Two warpgroups share each row (thread = row = TMEM lane): group g takes key columns
    // [64g, 64g + 64) of S and dims [64g, 64g + 64) of O; the row max and the final row sum
    // are exchanged through shared memory.
    const int g = (warp - 4) >> 2;
    const int w = warp & 3;
    const int r = w * 32 + lane;
    const int pl = r / a.hs, hs = r % a.hs;
    const int pos = pos0 + pl;
    const bool row_ok = pl < qn && hs < Gq;
    const float scale = p.sm_scale * 1.4426950408889634f;
    const uint32_t lane_base = tmem + ((uint32_t)(w * 32) << 16);
    const uint32_t ocol = lane_base + kColO + (uint32_t)(g * 64);
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int sl = j & 1;
      // warp-uniform outcome: the tcgen05 loads / stores below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&s_full[sl], (uint32_t)(j >> 1) & 1u, status, SQ_ERR_TIMEOUT_ACC))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (threadIdx.x == 128) tmark(tr, 5, j);
      const uint32_t sb = lane_base + kColS + (uint32_t)(sl * 128 + g * 64);
      const int kbase = j * TKEYS + g * 64;     // key of this group's first column
      const int lim = row_ok ? pos - kbase : -1;  // columns c <= lim are visible
      const bool diag = kbase + 63 > pos0;      // some column is in some row's future
      // this group's 64 columns of S: one TMEM round trip, kept in registers
      uint32_t u0[32], u1[32];
      tmem_ld32(sb, u0);
      tmem_ld32(sb + 32u, u1);
      tmem_wait_ld();
      float mt;
      {
        float m[32];
        if (diag) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float a0 = i <= lim ? __uint_as_float(u0[i]) : -INFINITY;
            const float a1 = 32 + i <= lim ? __uint_as_float(u1[i]) : -INFINITY;
            m[i] = fmaxf(a0, a1);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) m[i] = fmaxf(__uint_as_float(u0[i]), __uint_as_float(u1[i]));
        }
#pragma unroll
        for (int st = 16; st >= 1; st >>= 1)
#pragma unroll
          for (int i = 0; i < st; ++i) m[i] = fmaxf(m[i], m[i + st]);
        mt = m[0];
      }
      if (!row_ok) mt = -INFINITY;
      float* xm = row_max + (sl * 2 + g) * TR;
      xm[r] = mt;
      softmax_sync();
      mt = fmaxf(mt, row_max[(sl * 2 + (g ^ 1)) * TR + r]) * scale;
      const bool raise = mt > m_used + 8.f;  // false for fully masked rows (mt = -inf)
      const float m_new = raise ? mt : m_used;
      const float alpha = raise ? ex2(m_used - m_new) : 1.f;  // 0 when m_used was -inf
      m_used = m_new;
      const float base = (m_used == -INFINITY) ? 0.f : m_used;
      // P = 2^(s * scale - m) as bf16 pairs into TMEM; row sum
      const uint32_t pb = lane_base + kColP + (uint32_t)(sl * 64 + g * 32);
      const bool masked = diag || !row_ok;
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t* uc = c == 0 ? u0 : u1;
        float e[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          e[i] = ex2(fmaf(__uint_as_float(uc[i]), scale, -base));
          if (masked && c * 32 + i > lim) e[i] = 0.f;  // lim = -1 for rows that are not computed
        }
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) pk[i] = pack_bf2(e[2 * i], e[2 * i + 1]);
        tmem_st16(pb + (uint32_t)(c * 16), pk);
#pragma unroll
        for (int st = 16; st >= 1; st >>= 1)
#pragma unroll
          for (int i = 0; i < st; ++i) e[i] += e[i + st];
        rs += e[0];
      }
      l = l * alpha + rs;
      // O *= alpha (only when some row of this warp raised its max; O holds PV(j-1))
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&o_done[(j - 1) & 1], (uint32_t)((j - 1) >> 1) & 1u, status,
                                               SQ_ERR_TIMEOUT_ACC))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t u[32];
          tmem_ld32(ocol + (uint32_t)(c * 32), u);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * alpha);
          tmem_st32(ocol + (uint32_t)(c * 32), u);
        }
        if (threadIdx.x == 128) tmark(tr, 8, j);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sl]);
      if (threadIdx.x == 128) tmark(tr, 6, j);
    }
    // epilogue: O / l -> bf16 (this group's 64 dims of the row)
    row_max[(4 + g) * TR + r] = l;
    softmax_sync();
    l += row_max[(4 + (g ^ 1)) * TR + r];
    if (ok && __all_sync(0xffffffffu, mbar_wait(&o_done[(nt - 1) & 1], (uint32_t)((nt - 1) >> 1) & 1u, status,
                                                SQ_ERR_TIMEOUT_ACC))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst =
          p.out + (size_t)(__ldg(p.q_start + b) + q0 + pl) * p.ld_out + (size_t)(h * Gq + hs) * TD + g * 64;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t u[32];
        tmem_ld32(ocol + (uint32_t)(c * 32), u);
        tmem_wait_ld();
        if (row_ok) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const float* f = reinterpret_cast<const float*>(u + 8 * v);
            d4[v] = make_uint4(pack_bf2(f[0] * inv, f[1] * inv), pack_bf2(f[2] * inv, f[3] * inv),
                               pack_bf2(f[4] * inv, f[5] * inv), pack_bf2(f[6] * inv, f[7] * inv));
          }
        }
      }
    }
    if (threadIdx.x == 128) tmark(tr, 10, 0);
  } else if (warp == 1) {
    // ------------------------------------------------ page loader (bulk copies)
    load_stages<FK, FV>(p, stg, stg_full, stg_empty, h, b, nt, kv_end, status, lane == 0 ? tr : nullptr);
  } else if (warp >= 12) {
    // ------------------------------------------------ K / V producers (thread = key)
    produce_kv<FK, FV>(p, stg, stg_full, stg_empty, Ks, Vs, k_full, k_empty, v_full, v_empty, threadIdx.x - 384, nt,
                       kv_end, status, tr);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemT);
}

template <int FK, int FV>
cudaError_t launch_tc(const CUtensorMap& qmap, const TcAttnArgs& a, cudaStream_t s) {
  auto k = prefill_tc_kernel<FK, FV>;
  constexpr size_t smem = Stage<FK, FV>::kSmem;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  SQ_LAUNCH(k, dim3(a.p.n_tiles * a.sub, a.p.Hkv), dim3(kThreadsT), smem, s, 1u, qmap, a);
  return cudaSuccess;
}

}  // namespace

bool prefill_tc_supported(const AttnParams& p) {
  const int gq = p.Hkv > 0 ? p.Hq / p.Hkv : 0;
  const bool fmt_ok = (p.fmt_k == KV_INT4 && p.fmt_v == KV_INT4) || (p.fmt_k == KV_INT8 && p.fmt_v == KV_INT8) ||
                      (p.fmt_k == KV_INT2 && p.fmt_v == KV_INT2) || (p.fmt_k == KV_K8 && p.fmt_v == KV_V4);
  const int nsk = kv_nscale(p.fmt_k, TD, p.group), nsv = kv_nscale(p.fmt_v, TD, p.group);
  const bool pages_ok = p.page_size >= 4 && TKEYS % p.page_size == 0 && (p.page_size * 2 * nsk) % 16 == 0 &&
                        (p.page_size * 2 * nsv) % 16 == 0 && nsk <= 8 && nsv <= 8;
  return p.D == TD && p.tree_mask == nullptr && gq >= 3 && gq <= 16 && p.Hq % p.Hkv == 0 && fmt_ok &&
         (p.group == 32 || p.group == 64 || p.group == 128) && p.ld_q % 8 == 0 && p.ld_out % 8 == 0 && pages_ok;
}

int prefill_tc_head_slots(int gq) { return gq <= 4 ? 4 : gq <= 8 ? 8 : 16; }

cudaError_t paged_prefill_attn_tc_launch(const CUtensorMap& qmap, const AttnParams& p, int* status,
                                         unsigned long long* trace, cudaStream_t s) {
  if (p.n_tiles == 0) return cudaSuccess;
  TcAttnArgs a{};
  a.p = p;
  a.hs = prefill_tc_head_slots(p.Hq / p.Hkv);
  a.npos = TR / a.hs;
  a.sub = 32 / a.npos;
  a.status = status;
  a.trace = trace;
  if (p.fmt_k == KV_INT4 && p.fmt_v == KV_INT4) return launch_tc<KV_INT4, KV_INT4>(qmap, a, s);
  if (p.fmt_k == KV_INT8 && p.fmt_v == KV_INT8) return launch_tc<KV_INT8, KV_INT8>(qmap, a, s);
  if (p.fmt_k == KV_INT2 && p.fmt_v == KV_INT2) return launch_tc<KV_INT2, KV_INT2>(qmap, a, s);
  if (p.fmt_k == KV_K8 && p.fmt_v == KV_V4) return launch_tc<KV_K8, KV_V4>(qmap, a, s);
  return cudaErrorInvalidValue;
}

}  // namespace sq
