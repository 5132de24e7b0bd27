// w4a16_gemm.cu — weight-only INT4 (asymmetric, group-scaled) GEMM for sm_100a.
//
//   Y[M, N] = X[M, K] (bf16) . dequant(W)[N, K]^T  (+ bias) (+ residual)
//   or, for a fused gate/up projection, Y[M, N/2] = silu(gate) * up.
//
// The math this replaces is the reference's fused INT4 matmul
// (squish_quant_rs/src/lib.rs:5511 `quantized_matmul_int4`, numpy oracle
// squish/quant/quantizer.py:632 `_quantized_matmul_int4_numpy`): W_hat = offset + q*scale
// per (row, group), q the unsigned nibble. Here it runs on the 5th-generation tensor cores:
//
//  * swap-AB: weight rows are the MMA M side (128 per tile = one TMEM lane each), tokens
//    the MMA N side (16..256), so a decode batch of 1-64 tokens still fills the M side;
//  * each (128 rows x 64 columns) weight tile is one contiguous block on the device —
//    4 KiB of interleaved nibbles followed by its (scale, zero) bf16 pairs — streamed with
//    one 1-D bulk copy per stage into a shared-memory ring (L2 evict-first);
//  * activations arrive by TMA (2-D tensor map, 128-byte swizzle, zero fill past M and K);
//  * dequant warps turn nibbles into bf16 with the 0x4300 exponent trick plus one bf16x2
//    subtract and one bf16x2 FMA per pair, and write the canonical SWIZZLE_128B K-major
//    operand layout; they signal per warp (one mbarrier arrive per warp, not per thread);
//  * one thread issues tcgen05.mma (kind::f16, fp32 accumulators in TMEM) and retires ring
//    slots with tcgen05.commit;
//  * epilogue warps read TMEM with tcgen05.ld. With split-K (decode shapes with too few
//    output tiles to fill the SMs) the split CTAs of a tile form a thread-block cluster:
//    each stages its fp32 partial in its own shared memory and, after a cluster barrier,
//    reduces a slice of the tile by reading all partials over distributed shared memory
//    in split order (deterministic, no global workspace).
//
// Decode shapes (BN <= 64) run two CTAs per SM (small rings), so two independent
// pipelines hide each other's hand-off latency. Every wait is bounded (sm100.cuh); on
// timeout *status is set and the kernel still releases its TMEM before exiting.
#include <cuda_fp8.h>
#include <cuda_fp16.h>
#include <cstdio>
#include <cstdlib>

#include "sm100.cuh"
#include "w4a16_gemm.h"
#include "launch.cuh"

namespace sq {

namespace {

constexpr int BM = 128;                    // weight rows per MMA tile
constexpr int BK = 64;                     // K per stage = one 128-byte bf16 swizzle row
constexpr int W_TILE_BYTES = BM * BK / 2;  // 4096 nibble bytes per tile
constexpr int A_TILE_BYTES = BM * BK * 2;  // 16384

template <int BN_, int NT_, int MINB_, int DQW_ = 8, bool ASMEM_ = false>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int NT = NT_;          // 128-row weight tiles per CTA
  static constexpr int kMinBlocks = MINB_;
  static constexpr int kDqWarps = DQW_;   // dequant warps 4..; thread -> (row, 1/(DQW/4) of the 64 columns)
  static constexpr int kWpt = 32 / DQW_;  // 32-bit nibble words per thread and tile (8 nibbles each)
  static constexpr int kThreads = 128 + 32 * kDqWarps;
  static constexpr int kXBytes = BN * 128;
  // Single weight tile per CTA: the dequantized A operand goes to tensor memory (tcgen05.st)
  // instead of shared memory; columns [kA0, kA0 + 32 * ring_a) hold the A ring.
  static constexpr bool AT = (NT == 1) && !ASMEM_;
  static constexpr int kA0 = AT ? (NT * BN < 32 ? 32 : NT * BN) : 0;
  // CTAs per SM share 512 TMEM columns: 3+ -> 2 A stages, 2 -> 4, one CTA -> what is left (<= 12)
  // (two CTAs: the A stages fill the 256 columns each CTA allocates anyway, 6 for 64 tokens)
  static constexpr int kMaxRingA = MINB_ >= 3 ? 2 : MINB_ == 2 ? ((256 - kA0) / 32 > 4 ? (256 - kA0) / 32 : 4)
                                                     : ((512 - kA0) / 32 < 12 ? (512 - kA0) / 32 : 12);
  static constexpr int kCols = AT ? kA0 + 32 * kMaxRingA : NT * BN;
  static constexpr int kTmemCols = (kCols <= 32) ? 32 : (kCols <= 64) ? 64 : (kCols <= 128) ? 128 : (kCols <= 256) ? 256 : 512;
  // static shared table for NF4 levels / AQLM codebooks: only the 8-dequant-warp configurations
  // decode those formats (the 4-warp decode configurations are INT4 only), so the others keep
  // their 8 KiB for the rings: several CTAs per SM must fit 228 KiB including it
  static constexpr int kFmtTab = DQW_ == 4 ? 1 : 512;
};

__host__ __device__ constexpr int code_bytes(int wfmt) {
  return (wfmt == WF_INT8 || wfmt == WF_FP8)    ? 2 * W_TILE_BYTES
         : (wfmt == WF_INT2 || wfmt == WF_AQLM) ? W_TILE_BYTES / 2
         : wfmt == WF_INT3                      ? 3 * W_TILE_BYTES / 4
                                                : W_TILE_BYTES;
}
__host__ __device__ constexpr int tile_bytes(int gpk, int wfmt = WF_INT4) { return code_bytes(wfmt) + gpk * BM * 4; }

struct Layout {
  uint32_t x_off, w_off, w_stage, bar_off, trace_off, total;
};

// rw / rx count ring stages of wg weight k-blocks / xg activation k-blocks (one bulk copy / one
// TMA load each).
__host__ __device__ inline Layout make_layout(int bn, int nt, int gpk, int rw, int rx, int ra, bool trace,
                                              bool a_in_tmem, int wfmt, int wg = 1, int xg = 1) {
  Layout L;
  L.x_off = a_in_tmem ? 0u : (uint32_t)(ra * nt * A_TILE_BYTES);
  L.w_off = L.x_off + (uint32_t)(rx * xg * bn * 128);
  L.w_stage = (uint32_t)(nt * wg * tile_bytes(gpk, wfmt));
  L.bar_off = L.w_off + (uint32_t)rw * L.w_stage;
  L.bar_off = (L.bar_off + 15u) & ~15u;
  L.trace_off = L.bar_off + (uint32_t)(2 * rw + 2 * rx + 2 * ra + 1) * 8u + 16u;
  L.trace_off = (L.trace_off + 7u) & ~7u;
  L.total = L.trace_off + (trace ? 16u * 64u * 8u : 0u);
  return L;
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t*>(&v); }

// 8 nibbles of one 32-bit word (interleaved so that (w >> 4e) & 0x000F000F holds columns
// 2e and 2e+1) -> 8 bf16 = one 16-byte operand chunk.
__device__ __forceinline__ uint4 dq_word(uint32_t w, __nv_bfloat162 s2, __nv_bfloat162 z2) {
  const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    uint32_t t = ((w >> (4 * e)) & 0x000F000Fu) | 0x43004300u;  // bf16(128 + q)
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t);
    v = __hsub2(v, k128);   // exact q
    v = __hfma2(v, s2, z2); // q*scale + zero, one rounding
    o[e] = bf2_bits(v);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// NF4: 8 level indices of one word (same interleaved order as INT4) -> 8 bf16 = level * absmax.
// lut[(q_even) | (q_odd << 4)] holds the two levels as a bf16 pair.
// The NormalFloat-4 levels (QLoRA, Dettmers et al. 2023), as the npy-dir __nf4 format stores them.
__constant__ float kNf4Levels[16] = {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
                                     -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
                                     0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f,
                                     0.33791524171829224f, 0.44070982933044434f, 0.5626170039176941f,
                                     0.7229568362236023f, 1.0f};

__device__ __forceinline__ uint4 dq_nf4(uint32_t w, __nv_bfloat162 s2, const uint32_t* lut) {
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t t = (w >> (4 * e)) & 0x000F000Fu;
    uint32_t pr = lut[(t & 0xFu) | ((t >> 12) & 0xF0u)];
    __nv_bfloat162 v = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&pr), s2);
    o[e] = bf2_bits(v);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// INT2: half h of a word of 16 codes (value 2e at bits 2e, value 2e+1 at bits 16+2e) -> 8 bf16.
__device__ __forceinline__ uint4 dq_int2(uint32_t w, int h, __nv_bfloat162 s2, __nv_bfloat162 z2) {
  const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    uint32_t t = ((w >> (2 * (4 * h + e))) & 0x00030003u) | 0x43004300u;  // bf16(128 + q)
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t);
    v = __hfma2(__hsub2(v, k128), s2, z2);
    o[e] = bf2_bits(v);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// INT8: 8 signed bytes (little-endian in two words) -> 8 bf16 = q * scale.
__device__ __forceinline__ uint4 dq_int8(uint32_t a, uint32_t b, float s) {
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t w = e < 2 ? a : b;
    const int sh = (e & 1) * 16;
    const float f0 = (float)((int)(w << (24 - sh)) >> 24) * s;
    const float f1 = (float)((int)(w << (16 - sh)) >> 24) * s;
    o[e] = bf2_bits(__floats2bfloat162_rn(f0, f1));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// FP8 E4M3: 8 bytes (column order, little-endian) -> 8 bf16 values * s, two per cvt.
__device__ __forceinline__ uint4 dq_fp8(uint32_t a, uint32_t b, float s) {
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t w = e < 2 ? a : b;
    const __nv_fp8x2_storage_t pr = (__nv_fp8x2_storage_t)((w >> ((e & 1) * 16)) & 0xFFFFu);
    const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pr, __NV_E4M3);
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
    o[e] = bf2_bits(__floats2bfloat162_rn(f.x * s, f.y * s));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// INT3: 32 codes u = q + 4 in three words. Pair p < 15 (values 2p, 2p+1) sits in word p / 5 at
// bits 3*(p%5) and 16 + 3*(p%5); pair 15 is spread over bits 15 (even value) and 31 (odd
// value) of words 0, 1, 2 (its bits 0, 1, 2).
__device__ __forceinline__ uint32_t int3_pair(const uint32_t (&ww)[8], int p) {
  if (p < 15) return (ww[p / 5] >> (3 * (p % 5))) & 0x00070007u;
  return ((ww[0] >> 15) & 0x00010001u) | ((ww[1] >> 14) & 0x00020002u) | ((ww[2] >> 13) & 0x00040004u);
}
__device__ __forceinline__ uint4 dq_int3(const uint32_t (&ww)[8], int ch, __nv_bfloat162 s2, __nv_bfloat162 z2) {
  const __nv_bfloat162 k132 = __floats2bfloat162_rn(132.f, 132.f);
  uint32_t o[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    uint32_t t = int3_pair(ww, ch * 4 + e) | 0x43004300u;  // bf16(128 + u)
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&t);
    v = __hfma2(__hsub2(v, k132), s2, z2);  // exact q, then q * scale + zero
    o[e] = bf2_bits(v);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// AQLM: one 8-column group from its codebook indices (book k's index in byte k of idx).
__device__ __forceinline__ uint4 dq_aqlm(uint32_t idx, int n_books, const uint4* books, __nv_bfloat162 s2) {
  uint4 a = books[idx & 0xFFu];
  if (n_books > 1) {
    const uint4 b = books[256 + ((idx >> 8) & 0xFFu)];
    __nv_bfloat162* pa = reinterpret_cast<__nv_bfloat162*>(&a);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
    for (int e = 0; e < 4; ++e) pa[e] = __hadd2(pa[e], pb[e]);
  }
  __nv_bfloat162* pa = reinterpret_cast<__nv_bfloat162*>(&a);
#pragma unroll
  for (int e = 0; e < 4; ++e) pa[e] = __hmul2(pa[e], s2);
  return a;
}

// The 32 K values (4 chunks of 8) of row r, part c of a tile in a non-INT4 format.
__device__ __forceinline__ void dq_other(const uint8_t* tb, int fmt, int r, int c, int gpk, const uint32_t* lut,
                                         int n_books, uint4 (&o)[4]) {
  const uint32_t* szt = reinterpret_cast<const uint32_t*>(tb + code_bytes(fmt));
  uint32_t ww[8];
  if (fmt == WF_INT8 || fmt == WF_FP8) {
    const uint4 a = *reinterpret_cast<const uint4*>(tb + (c * BM + r) * 32);
    const uint4 b = *reinterpret_cast<const uint4*>(tb + (c * BM + r) * 32 + 16);
    ww[0] = a.x; ww[1] = a.y; ww[2] = a.z; ww[3] = a.w; ww[4] = b.x; ww[5] = b.y; ww[6] = b.z; ww[7] = b.w;
  } else if (fmt == WF_INT2 || fmt == WF_AQLM) {
    const uint2 a = *reinterpret_cast<const uint2*>(tb + (c * BM + r) * 8);
    ww[0] = a.x; ww[1] = a.y;
  } else if (fmt == WF_INT3) {
    const uint32_t* a = reinterpret_cast<const uint32_t*>(tb + (c * BM + r) * 12);
    ww[0] = a[0]; ww[1] = a[1]; ww[2] = a[2];
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(tb + (c * BM + r) * 16);
    ww[0] = a.x; ww[1] = a.y; ww[2] = a.z; ww[3] = a.w;
  }
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t szw = szt[(((c * 4 + w) * gpk) >> 3) * BM + r];
    const __nv_bfloat16 sc = __ushort_as_bfloat16((unsigned short)(szw & 0xFFFFu));
    const __nv_bfloat16 ze = __ushort_as_bfloat16((unsigned short)(szw >> 16));
    if (fmt == WF_NF4) o[w] = dq_nf4(ww[w], __bfloat162bfloat162(sc), lut);
    else if (fmt == WF_INT2) o[w] = dq_int2(ww[w >> 1], w & 1, __bfloat162bfloat162(sc), __bfloat162bfloat162(ze));
    else if (fmt == WF_INT3) o[w] = dq_int3(ww, w, __bfloat162bfloat162(sc), __bfloat162bfloat162(ze));
    else if (fmt == WF_AQLM)
      o[w] = dq_aqlm((ww[w >> 1] >> (16 * (w & 1))) & 0xFFFFu, n_books, reinterpret_cast<const uint4*>(lut),
                     __bfloat162bfloat162(sc));
    else if (fmt == WF_FP8) o[w] = dq_fp8(ww[2 * w], ww[2 * w + 1], __bfloat162float(sc));
    else o[w] = dq_int8(ww[2 * w], ww[2 * w + 1], __bfloat162float(sc));
  }
}

__device__ __forceinline__ float silu(float g) { return g / (1.f + __expf(-g)); }

// Optional pipeline trace (p.trace != nullptr): CTA (0,0,0) stamps clock64() per role and
// k-block into shared memory (no global traffic inside the pipeline) and copies the
// 16 x 64 table to p.trace at exit.
__device__ __forceinline__ void trace_mark(unsigned long long* smem_tr, int slot, int i) {
  if (smem_tr != nullptr && i < 64) smem_tr[slot * 64 + i] = clock64();
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Store one output element locally, or (push mode) into every rank's receive buffer.
__device__ __forceinline__ void store_out(const W4A16Params& p, int par, int m, int n, float v) {
  const __nv_bfloat16 b = __float2bfloat16(v);
  if (p.push_dst == nullptr) {
    p.y[(size_t)m * p.ldy + n] = b;
    return;
  }
  if (p.push_rows > 0) {  // reduce-scatter: only the owner of token row m receives it
    const int owner = m / p.push_rows;
    p.push_dst[owner][(size_t)par * p.push_stride + (size_t)(m - owner * p.push_rows) * p.ldy + n] = b;
    return;
  }
  const size_t off = (size_t)par * p.push_stride + (size_t)m * p.ldy + n;
  for (int r = 0; r < p.tp; ++r) p.push_dst[r][off] = b;
}

// After this CTA's stores of an output tile: make them visible system-wide, then bump the
// tile's arrival flag on every rank (release at system scope).
__device__ __forceinline__ void push_signal(const W4A16Params& p, int par, int tile) {
  if (p.push_rows > 0) tile = 0;  // reduce-scatter: one arrival counter per (parity, source)
  for (int r = 0; r < p.tp; ++r) {
    int* f = p.push_flags[r] + (size_t)par * p.flag_stride + tile;
    asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(f), "r"(1) : "memory");
  }
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ring position: stage index and phase parity, advanced without division
struct Ring {
  int s = 0;
  uint32_t ph = 0;
  int n;
  __device__ explicit Ring(int n_) : n(n_) {}
  __device__ __forceinline__ void next() {
    if (++s == n) {
      s = 0;
      ph ^= 1u;
    }
  }
};

template <class C>
__global__ void __launch_bounds__(C::kThreads, C::kMinBlocks)
    w4a16_gemm_kernel(const __grid_constant__ CUtensorMap xmap, const W4A16Params p) {
  constexpr int BN = C::BN;
  constexpr int NT = C::NT;
  const uint8_t* wbase = reinterpret_cast<const uint8_t*>(p.wq);
  // Programmatic dependent launch: weights are static, so the plain mode streams them before
  // waiting for the previous kernel; only the activation loads (warp 1) and the epilogue
  // wait. Grouped and push modes read predecessor data (tile table, op counter) up front.
  const bool early_wait = (p.tile_expert != nullptr) || (p.push_dst != nullptr);
  if (early_wait) pdl_wait();
  if (p.tile_expert != nullptr) {  // grouped mode: whole CTA leaves before any setup
    if ((int)blockIdx.y >= __ldg(p.num_tiles)) return;
    wbase += (size_t)__ldg(p.tile_expert + blockIdx.y) * (size_t)p.expert_stride;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int gpk = p.gpk;
  const int ring_w = p.ring_w, ring_x = p.ring_x, ring_a = p.ring_a;
  // k-blocks per weight bulk copy / per activation TMA load
  const int wg = p.wg > 1 ? p.wg : 1;
  const int xg = p.xg > 1 ? p.xg : 1;
  const int ag = (C::AT && p.ag > 1) ? p.ag : 1;  // k-blocks per tensor-memory A stage (one hand-off)
  const uint32_t xstage = (uint32_t)(xg * C::kXBytes);
  const Layout L = make_layout(BN, NT, gpk, ring_w, ring_x, ring_a, p.trace != nullptr, C::AT, p.wfmt, wg, xg);
  uint8_t* a_ring = smem;  // (shared-memory A ring; with C::AT the region starts the X ring)
  uint8_t* x_ring = smem + L.x_off;
  uint8_t* w_ring = smem + L.w_off;
  uint64_t* w_full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
  uint64_t* w_empty = w_full + ring_w;
  uint64_t* x_full = w_empty + ring_w;
  uint64_t* x_empty = x_full + ring_x;
  uint64_t* a_full = x_empty + ring_x;
  uint64_t* a_empty = a_full + ring_a;
  uint64_t* acc_full = a_empty + ring_a;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  unsigned long long* str = nullptr;
  if (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
    str = reinterpret_cast<unsigned long long*>(smem + L.trace_off);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nblk = blockIdx.x;
  const int mblk = blockIdx.y;
  const int split = blockIdx.z;
  const int kb0 = split * p.kb_per_split;
  const int kb1 = min(p.kb_total, kb0 + p.kb_per_split);
  const int nkb = max(0, kb1 - kb0);
  int* status = p.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ring_w; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], C::kDqWarps);
    }
    for (int i = 0; i < ring_x; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < ring_a; ++i) {
      mbar_init(&a_full[i], C::kDqWarps);
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
    prefetch_tmap(&xmap);
  }
  if (warp == 3) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  // format table: NF4 (level[q0], level[q1]) bf16 pairs, or the AQLM codebooks (<= 2 x 256 x 8 bf16)
  __shared__ uint4 fmt_tab[C::kFmtTab];
  uint32_t* nf4_lut = reinterpret_cast<uint32_t*>(fmt_tab);
  if constexpr (C::kFmtTab >= 512) {
    if (p.wfmt == WF_NF4) {  // NormalFloat-4 levels, or a learned 16-level table (any4) in codebook
      for (int i = threadIdx.x; i < 256; i += blockDim.x)
        nf4_lut[i] = bf2_bits(p.codebook != nullptr
                                  ? __halves2bfloat162(p.codebook[i & 15], p.codebook[i >> 4])
                                  : __floats2bfloat162_rn(kNf4Levels[i & 15], kNf4Levels[i >> 4]));
    } else if (p.wfmt == WF_AQLM) {
      for (int i = threadIdx.x; i < 256 * p.n_books; i += blockDim.x)
        fmt_tab[i] = reinterpret_cast<const uint4*>(p.codebook)[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int tbytes = tile_bytes(gpk, p.wfmt);
  if (threadIdx.x == 0) trace_mark(str, 14, 0);  // setup done
  pdl_trigger();

  // Warps 0-2 run converged: every lane waits, one elected lane issues (tensor-core and
  // bulk-copy instructions are issued by one thread of a converged warp).
  if (warp == 0) {
    // ------------------------------------------------ weight producer: one bulk copy per tile
    const uint64_t pol = policy_evict_first();
    Ring r(ring_w);
    for (int i = 0; i < nkb; i += wg) {
      if (!mbar_wait(&w_empty[r.s], r.ph ^ 1u, status, SQ_ERR_TIMEOUT_W)) break;
      if (elect_one()) {
        // wg consecutive k-blocks of a 128-row block are contiguous (tile-major layout): one copy
        const int cnt = min(wg, nkb - i);
        uint8_t* dst = w_ring + r.s * L.w_stage;
        mbar_expect_tx(&w_full[r.s], (uint32_t)(NT * cnt * tbytes));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const size_t tile = ((size_t)nblk * NT + t) * p.kb_total + kb0 + i;
          bulk_g2s_hint(dst + (size_t)t * wg * tbytes, wbase + tile * tbytes, (uint32_t)(cnt * tbytes),
                        &w_full[r.s], pol);
        }
        trace_mark(str, 0, i);
      }
      __syncwarp();
      r.next();
    }
  } else if (warp == 1) {
    // ------------------------------------------------ activation producer (TMA)
    pdl_wait();  // activations come from the previous kernel
    if (p.ag_flags != nullptr && lane < p.tp) {
      // all-gathered X: every source rank's rows have landed in this rank's buffer
      for (long long it = 0;; ++it) {
        int v;
        asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p.ag_flags + lane) : "memory");
        if (v >= p.ag_expect) break;
        if (it > (1LL << 22) || *reinterpret_cast<volatile int*>(status) != 0) {
          atomicCAS(status, 0, SQ_ERR_TIMEOUT_PEER);
          break;
        }
      }
    }
    __syncwarp();
    Ring r(ring_x);
    for (int i = 0; i < nkb; i += xg) {
      if (!mbar_wait(&x_empty[r.s], r.ph ^ 1u, status, SQ_ERR_TIMEOUT_X)) break;
      if (elect_one()) {
        mbar_expect_tx(&x_full[r.s], xstage);  // (a 3-D box always transfers all xg k-blocks)
        if (xg > 1)  // 3-D map {64 columns, rows, k-block}: xg consecutive k-blocks in one load
          tma_load_3d(x_ring + r.s * xstage, &xmap, 0, mblk * BN, kb0 + i, &x_full[r.s]);
        else
          tma_load_2d(x_ring + r.s * xstage, &xmap, (kb0 + i) * BK, mblk * BN, &x_full[r.s]);
        trace_mark(str, 1, i);
      }
      __syncwarp();
      r.next();
    }
  } else if (warp == 2) {
    // ------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
    Ring rx(ring_x), ra(ring_a);
    for (int i = 0; i < nkb; ++i) {
      const int xsub = i % xg;
      if (xsub == 0 && !mbar_wait(&x_full[rx.s], rx.ph, status, SQ_ERR_TIMEOUT_X)) break;
      if (lane == 0) trace_mark(str, 2, i);
      const int asub = i % ag;
      if (asub == 0 && !mbar_wait(&a_full[ra.s], ra.ph, status, SQ_ERR_TIMEOUT_A)) break;
      if (lane == 0) trace_mark(str, 3, i);
      tc_fence_after();
      if (elect_one()) {
        const uint32_t xa = smem_u32(x_ring + rx.s * xstage + xsub * C::kXBytes);
        if (p.dbg & 2) {
          // (timing experiment: no MMA)
        } else if constexpr (C::AT) {
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_bf16_ts(tmem, tmem + (uint32_t)(C::kA0 + (ra.s * ag + asub) * 32 + k * 8), sdesc_sw128(xa + k * 32),
                        idesc, (i > 0 || k > 0) ? 1u : 0u);
        } else {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint32_t aa = smem_u32(a_ring + (ra.s * NT + t) * A_TILE_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              mma_bf16_ss(tmem + t * BN, sdesc_sw128(aa + k * 32), sdesc_sw128(xa + k * 32), idesc,
                          (i > 0 || k > 0) ? 1u : 0u);
          }
        }
        if (xsub == xg - 1 || i == nkb - 1) mma_commit(&x_empty[rx.s]);
        if (asub == ag - 1 || i == nkb - 1) mma_commit(&a_empty[ra.s]);
        trace_mark(str, 12, i);
      }
      __syncwarp();
      if (xsub == xg - 1 || i == nkb - 1) rx.next();
      if (asub == ag - 1 || i == nkb - 1) ra.next();
    }
    if (elect_one()) mma_commit(acc_full);
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------ dequant warps
    const int d = threadIdx.x - 128;
    const int r = d & (BM - 1);
    constexpr int WPT = C::kWpt;
    const int c = d >> 7;  // which part of the 64-column tile: words [c*WPT, c*WPT + WPT) of the row
    const int sw_row = r & 7;
    const uint32_t row_off = (uint32_t)((r >> 3) * 1024 + sw_row * 128);
    Ring rw(ring_w), ra(ring_a);
    // Dequantize the next raw weight stage into o (waits for it, releases it); false on timeout.
    auto dq_stage = [&](int i, uint4 (&o)[NT][WPT]) -> bool {
      const int wsub = i % wg;
      if (wsub == 0 && !mbar_wait(&w_full[rw.s], rw.ph, status, SQ_ERR_TIMEOUT_W)) return false;
      if (d == 0) trace_mark(str, 4, i);
      const uint8_t* wst = w_ring + rw.s * L.w_stage;
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint8_t* tb = wst + (size_t)(t * wg + wsub) * tbytes;
        if constexpr (WPT == 4) {
          if (p.wfmt != WF_INT4) {
            dq_other(tb, p.wfmt, r, c, gpk, nf4_lut, p.n_books, o[t]);
            continue;
          }
        }
        // nibble words of a row: [2 halves][128 rows][4 words]
        uint32_t ww[WPT];
        if constexpr (WPT == 8) {  // the whole row: both 32-column halves
          const uint4 a = *reinterpret_cast<const uint4*>(tb + r * 16);
          const uint4 b = *reinterpret_cast<const uint4*>(tb + (BM + r) * 16);
          ww[0] = a.x; ww[1] = a.y; ww[2] = a.z; ww[3] = a.w;
          ww[4] = b.x; ww[5] = b.y; ww[6] = b.z; ww[7] = b.w;
        } else if constexpr (WPT == 4) {
          const uint4 wv = *reinterpret_cast<const uint4*>(tb + (c * BM + r) * 16);
          ww[0] = wv.x;
          ww[1] = wv.y;
          ww[2] = wv.z;
          ww[3] = wv.w;
        } else {
          const uint2 wv = *reinterpret_cast<const uint2*>(tb + ((c >> 1) * BM + r) * 16 + (c & 1) * 8);
          ww[0] = wv.x;
          ww[1] = wv.y;
        }
        const uint32_t* szt = reinterpret_cast<const uint32_t*>(tb + W_TILE_BYTES);
        if (p.dbg & 1) {
#pragma unroll
          for (int w = 0; w < WPT; ++w) o[t][w] = make_uint4(ww[w], ww[w] ^ 1u, ww[w] ^ 2u, ww[w] ^ 3u);
        } else if (gpk == 1) {  // one (scale, zero) group covers the whole 64-column k-block
          const uint32_t szw = szt[r];
          const __nv_bfloat162 s2 = __bfloat162bfloat162(__ushort_as_bfloat16((unsigned short)(szw & 0xFFFFu)));
          const __nv_bfloat162 z2 = __bfloat162bfloat162(__ushort_as_bfloat16((unsigned short)(szw >> 16)));
#pragma unroll
          for (int w = 0; w < WPT; ++w) o[t][w] = dq_word(ww[w], s2, z2);
        } else {
#pragma unroll
          for (int w = 0; w < WPT; ++w) {
            const uint32_t szw = szt[(((c * WPT + w) * gpk) >> 3) * BM + r];
            const __nv_bfloat16 sc = __ushort_as_bfloat16((unsigned short)(szw & 0xFFFFu));
            const __nv_bfloat16 ze = __ushort_as_bfloat16((unsigned short)(szw >> 16));
            o[t][w] = dq_word(ww[w], __bfloat162bfloat162(sc), __bfloat162bfloat162(ze));
          }
        }
      }
      if (wsub == wg - 1 || i == nkb - 1) {  // the copy's last tile consumed: release the slot
        __syncwarp();
        if (lane == 0) mbar_arrive(&w_empty[rw.s]);  // (one arrive per warp)
        rw.next();
      }
      return true;
    };
    // this thread's 8*WPT K values of row r = 4*WPT columns of its lane in the TMEM A stage
    auto st_tmem = [&](const uint4 (&o)[NT][WPT], int asub) {
      const uint32_t col =
          tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(C::kA0 + (ra.s * ag + asub) * 32 + c * WPT * 4);
      if constexpr (WPT == 8) {
        uint32_t regs[32];
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          regs[4 * w] = o[0][w].x;
          regs[4 * w + 1] = o[0][w].y;
          regs[4 * w + 2] = o[0][w].z;
          regs[4 * w + 3] = o[0][w].w;
        }
        tmem_st32(col, regs);
      } else if constexpr (WPT == 4) {
        const uint32_t regs[16] = {o[0][0].x, o[0][0].y, o[0][0].z, o[0][0].w, o[0][1].x, o[0][1].y,
                                   o[0][1].z, o[0][1].w, o[0][2].x, o[0][2].y, o[0][2].z, o[0][2].w,
                                   o[0][3].x, o[0][3].y, o[0][3].z, o[0][3].w};
        tmem_st16(col, regs);
      } else {
        const uint32_t regs[8] = {o[0][0].x, o[0][0].y, o[0][0].z, o[0][0].w,
                                  o[0][1].x, o[0][1].y, o[0][1].z, o[0][1].w};
        tmem_st8(col, regs);
      }
    };
    {
      for (int i = 0; i < nkb; ++i) {
        uint4 o[NT][WPT];
        if (!dq_stage(i, o)) break;
        const int asub = i % ag;
        const bool alast = asub == ag - 1 || i == nkb - 1;
        if (asub == 0 && !mbar_wait(&a_empty[ra.s], ra.ph ^ 1u, status, SQ_ERR_TIMEOUT_A)) break;
        if (d == 0) trace_mark(str, 5, i);
        if constexpr (C::AT) {
          if (asub == 0) tc_fence_after();
          st_tmem(o, asub);
          if (alast) {  // the stage's stores land before the MMA warp is told
            tmem_wait_st();
            tc_fence_before();
          }
        } else {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            uint8_t* adst = a_ring + (ra.s * NT + t) * A_TILE_BYTES + row_off;
#pragma unroll
            for (int w = 0; w < WPT; ++w)
              *reinterpret_cast<uint4*>(adst + (((c * WPT + w) ^ sw_row) << 4)) = o[t][w];
          }
          fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core (async proxy)
        }
        if (alast) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[ra.s]);
          if (lane == 0 && warp < 8) trace_mark(str, 4 + warp, i);  // trace slots 8-11: each warp's hand-off
          ra.next();
        }
        if (d == 0) trace_mark(str, 6, i);
      }
    }
  }

  pdl_wait();  // (already satisfied) residual reads and output writes follow
  // ------------------------------------------------ epilogue: warps 4..7 = TMEM lane quarters
  if (warp >= 4 && warp < 8) {
    const int q = warp & 3;
    const int row = q * 32 + lane;  // row within a 128-row weight tile
    const int m0 = mblk * BN;
    const bool single = (p.splits == 1);
    const bool silu_mode = (p.epilogue == EPI_SILU_MUL);
    const int par = p.push_dst != nullptr ? (__ldg(p.seq) & 1) : 0;
    float* xch = reinterpret_cast<float*>(a_ring);  // operand buffers are dead once acc_full fires

    // Emit 16 consecutive token columns of tile t for this thread's row.
    auto emit16 = [&](int t, int c0, const float(&val)[16]) {
      if (silu_mode) {
#pragma unroll
        for (int j = 0; j < 16; ++j) xch[j * 128 + row] = val[j];
        epi_bar();
        if (row < 64) {
          const int nn = (nblk * NT + t) * 64 + row;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            const float u = xch[j * 128 + row + 64];
            if (m < p.M && nn < (p.N >> 1)) p.y[(size_t)m * p.ldy + nn] = __float2bfloat16(silu(val[j]) * u);
          }
        }
        epi_bar();
      } else {
        const int n = (nblk * NT + t) * BM + row;
        if (n < p.N) {
          const float b = p.bias ? __bfloat162float(p.bias[n]) : 0.f;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (m < p.M) {
              float acc = val[j] + b;
              if (p.residual) acc += __bfloat162float(p.residual[(size_t)m * p.ldr + n]);
              store_out(p, par, m, n, acc);
            }
          }
        }
      }
    };

    const bool have_acc = (nkb > 0) && mbar_wait(acc_full, 0, status, SQ_ERR_TIMEOUT_ACC);
    if (threadIdx.x == 128) trace_mark(str, 7, 0);
    tc_fence_after();
#pragma unroll 1
    for (int t = 0; t < NT; ++t) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t v[16];
        if (have_acc) {
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(t * BN + c0), v);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0u;
        }
        if (single) {
          float val[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) val[j] = __uint_as_float(v[j]);
          emit16(t, c0, val);
        } else {
          // split-K: stage this CTA's fp32 partial in its own shared memory, [column][row]
#pragma unroll
          for (int j = 0; j < 16; ++j) xch[(c0 + j) * BM + row] = __uint_as_float(v[j]);
        }
      }
    }
    if (single && p.push_dst != nullptr) {
      __threadfence_system();
      epi_bar();
      if (threadIdx.x == 128) push_signal(p, par, nblk * gridDim.y + mblk);
    }
  }

  if constexpr (NT == 1) {
    if (p.splits > 1) {
      // The split CTAs of one output tile form a cluster along z. After a cluster barrier,
      // CTA r reduces columns [r*BN/S, (r+1)*BN/S) of the tile by reading every CTA's
      // partial through distributed shared memory, in split order (deterministic).
      cluster_sync();
      const int S = p.splits;
      const int jb = (BN + S - 1) / S;
      const int j0 = split * jb, j1 = min(BN, j0 + jb);
      const int m0 = mblk * BN;
      const uint32_t base = smem_u32(a_ring);
      // Remote partials are read with every split's load issued before any is consumed, so
      // the S distributed-shared-memory round trips overlap instead of chaining.
      auto ld_part = [&](int s, int idx) -> float {
        uint32_t ra, val;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(base + idx * 4), "r"(s));
        asm volatile("ld.shared::cluster.b32 %0, [%1];" : "=r"(val) : "r"(ra) : "memory");
        return __uint_as_float(val);
      };
      auto sum_parts = [&](int idx) -> float {
        float v[16];
#pragma unroll
        for (int s = 0; s < 16; ++s) v[s] = (s < S) ? ld_part(s, idx) : 0.f;
        float acc = 0.f;
#pragma unroll
        for (int s = 0; s < 16; ++s) acc += v[s];  // split order: deterministic
        return acc;
      };
      if (p.epilogue == EPI_SILU_MUL) {
        for (int idx = threadIdx.x; idx < (j1 - j0) * 64; idx += blockDim.x) {
          const int j = j0 + idx / 64, r = idx % 64;
          const int m = m0 + j, nn = nblk * 64 + r;
          const float g = sum_parts(j * BM + r);
          const float u = sum_parts(j * BM + r + 64);
          if (m < p.M && nn < (p.N >> 1)) p.y[(size_t)m * p.ldy + nn] = __float2bfloat16(silu(g) * u);
        }
      } else {
        for (int idx = threadIdx.x; idx < (j1 - j0) * BM; idx += blockDim.x) {
          const int j = j0 + idx / BM, r = idx % BM;
          const int m = m0 + j, n = nblk * BM + r;
          float acc = sum_parts(j * BM + r);
          if (m < p.M && n < p.N) {
            acc += p.bias ? __bfloat162float(p.bias[n]) : 0.f;
            if (p.residual) acc += __bfloat162float(p.residual[(size_t)m * p.ldr + n]);
            store_out(p, p.push_dst != nullptr ? (__ldg(p.seq) & 1) : 0, m, n, acc);
          }
        }
      }
      if (p.push_dst != nullptr) {
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x == 0) push_signal(p, __ldg(p.seq) & 1, nblk * gridDim.y + mblk);
      }
      cluster_sync();  // keep every CTA's shared memory alive until all remote reads are done
    }
  }

  tc_fence_before();
  __syncthreads();
  if (p.ag_flags != nullptr && threadIdx.x == 0) {
    // every CTA's producer has passed the wait once this counter reaches the grid size; no peer
    // can signal the next all-gather before this rank's next reduce-scatter push, which comes
    // after this kernel
    __threadfence();
    const int total = (int)(gridDim.x * gridDim.y * gridDim.z);
    if (atomicAdd(p.ag_done, 1) == total - 1) {
      for (int s2 = 0; s2 < p.tp; ++s2) p.ag_flags[s2] = 0;
      *p.ag_done = 0;
      __threadfence();
    }
  }
  if (threadIdx.x == 0) trace_mark(str, 15, 0);  // epilogue done
  __syncthreads();
  if (str != nullptr)
    for (int i = threadIdx.x; i < 16 * 64; i += blockDim.x) p.trace[i] = str[i];
  if (warp == 3) tmem_dealloc(tmem, C::kTmemCols);
}

template <class C>
cudaError_t launch_cfg(const CUtensorMap& xmap, W4A16Params p, int rw, int rx, int ra, cudaStream_t stream) {
  p.ring_w = rw;
  p.ring_x = rx;
  p.ring_a = ra;
  const Layout L = make_layout(C::BN, C::NT, p.gpk, rw, rx, ra, p.trace != nullptr, C::AT, p.wfmt,
                               p.wg > 1 ? p.wg : 1, p.xg > 1 ? p.xg : 1);
  if (p.wfmt != WF_INT4 && C::kWpt != 4) return cudaErrorInvalidConfiguration;
  if (p.xg > 1 && (C::NT != 1 || C::BN > 64)) return cudaErrorInvalidConfiguration;
  if (C::AT) {
    // the A ring lives in TMEM; the epilogue stages through the (then idle) X + W rings
    if (ra * (p.ag > 1 ? p.ag : 1) > C::kMaxRingA || L.bar_off < (uint32_t)(C::BN * BM * 4) ||
        L.bar_off < 16u * BM * 4u)
      return cudaErrorInvalidConfiguration;
  }
  const size_t smem = (size_t)L.total + 1024;  // + alignment slack
  if (smem + C::kFmtTab * sizeof(uint4) > 227 * 1024) return cudaErrorInvalidConfiguration;  // + static fmt_tab
  auto kern = w4a16_gemm_kernel<C>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  // all of the SM's unified L1/shared storage as shared memory, so kMinBlocks CTAs fit
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return e;
  dim3 grid((p.N + BM * C::NT - 1) / (BM * C::NT), (p.M + C::BN - 1) / C::BN, p.splits);
  if (p.splits > 1 && (C::NT != 1 || p.splits > 16)) return cudaErrorInvalidConfiguration;
  if (p.splits > 8) {  // clusters of 9..16 CTAs are outside the portable size
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  return launch_k(kern, grid, dim3(C::kThreads), smem, stream, (unsigned)p.splits, xmap, p);
}

}  // namespace

// Ring depths (stages): W = nt*(4 KiB + gpk*512 B), X = bn*128 B, A = nt*16 KiB (shared memory
// only when NT = 2; single-tile configs keep the A ring in tensor memory). Decode shapes
// (BN <= 64) and BN = 128 fit two CTAs per SM.
// Tuning override for experiments: SQ_GEMM_RINGS="w,x,a" replaces the decode (BN <= 64)
// ring depths; invalid or oversized settings fail the launch instead of running.
static bool ring_override(int* w, int* x, int* a) {
  static int v[3] = {-1, -1, -1};
  static bool read = false;
  if (!read) {
    read = true;
    if (const char* e = std::getenv("SQ_GEMM_RINGS")) {
      if (std::sscanf(e, "%d,%d,%d", &v[0], &v[1], &v[2]) != 3 || v[0] < 2 || v[1] < 2 || v[2] < 2) v[0] = -1;
    }
  }
  if (v[0] < 0) return false;
  *w = v[0];
  *x = v[1];
  *a = v[2];
  return true;
}

// Decode shapes, INT4 only: 4 dequant warps (a whole 64-column row per thread) and four CTAs
// per SM. SQ_GEMM_WIDE_DQ=1 selects the 8-warp, two-CTA configuration instead.
bool w4a16_decode_grouping(int bn, int wfmt, int gpk) {
  int ow, ox, oa;
  return bn <= 64 && w4a16_narrow(wfmt, gpk) && !ring_override(&ow, &ox, &oa);
}

bool w4a16_narrow(int wfmt, int gpk) {
  static const bool wide = [] {
    const char* e = std::getenv("SQ_GEMM_WIDE_DQ");
    return e != nullptr && e[0] == '1';
  }();
  return !wide && wfmt == WF_INT4 && gpk == 1;
}

static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Decode shapes stream their weights: a CTA keeps as many weight stages in flight as the
// shared memory its SM share allows. The launch's CTAs per SM decide that share: with two or
// fewer per SM each CTA takes half of the 228 KiB (deep rings, four TMEM A stages), otherwise
// a quarter (the four-CTA configuration).
template <int BN>
cudaError_t launch_decode_narrow(const CUtensorMap& xmap, W4A16Params p, cudaStream_t s) {
  const long ctas = (long)((p.N + BM - 1) / BM) * ((p.M + BN - 1) / BN) * p.splits;
  const int per_sm = (int)((ctas + sm_count() - 1) / sm_count());
  const bool tr = p.trace != nullptr;
  const int xg = p.xg > 1 ? p.xg : 1;
  auto fit = [&](int rx, int ra, int wg, size_t budget, int lo, int hi) {
    for (int rw = hi; rw > lo; --rw) {
      const Layout L = make_layout(BN, 1, p.gpk, rw, rx, ra, tr, true, p.wfmt, wg, xg);
      if ((size_t)L.total + 1024 <= budget) return rw;
    }
    return lo;
  };
  // shared-memory budgets per CTA: the SM's 228 KiB over the resident CTAs, less the 1 KiB the
  // hardware keeps per CTA (the budget covers the dynamic part + 1 KiB of alignment slack).
  // Ring depths count loads: a weight stage holds wg k-blocks, an activation stage xg.
  // k-blocks per weight copy (SQ_GEMM_WG overrides). Measured on B200 (Qwen2.5-7B shapes, 64
  // tokens): 4-k-block copies with 2-k-block activation loads take gate_up 48.6 -> 45.3 us,
  // down 33.0 -> 31.0, lm_head 193 -> 181 against one copy / one load per k-block.
  static const int wg_env = [] {
    const char* e = std::getenv("SQ_GEMM_WG");
    return e != nullptr ? std::max(1, std::min(8, std::atoi(e))) : 4;
  }();
  static const int rx_env = [] {  // activation ring stages (loads of xg k-blocks; SQ_GEMM_RX overrides)
    const char* e = std::getenv("SQ_GEMM_RX");
    return e != nullptr ? std::atoi(e) : 0;
  }();
  static const int ag_env = [] {  // k-blocks per A stage hand-off (SQ_GEMM_AG overrides)
    const char* e = std::getenv("SQ_GEMM_AG");
    return e != nullptr ? std::max(1, std::min(4, std::atoi(e))) : 2;  // (measured 47.2 -> 45.8 us gate_up)
  }();
  p.wg = wg_env;
  if (per_sm <= 2) {
    p.ag = ag_env;
    static const int ra_env = [] {  // A k-blocks in flight (SQ_GEMM_RA overrides; <= the TMEM room)
      const char* e = std::getenv("SQ_GEMM_RA");
      return e != nullptr ? std::atoi(e) : 4;
    }();
    const int ra = std::max(1, std::min(ra_env, Cfg<BN, 1, 2, 4>::kMaxRingA) / p.ag);
    const int rx = rx_env >= 2 && rx_env <= 16 ? rx_env : std::max(2, (BN >= 32 ? 4 : 6) / xg);
    return launch_cfg<Cfg<BN, 1, 2, 4>>(xmap, p, fit(rx, ra, p.wg, 112 * 1024, std::max(2, 4 / p.wg), 24 / p.wg + 1),
                                        rx, ra, s);
  }
  p.ag = 1;
  p.wg = std::min(p.wg > 1 ? p.wg : 1, 2);  // a quarter of the SM: two-k-block copies at most
  const int rx = std::max(2, (BN == 64 ? 3 : BN == 32 ? 4 : 6) / xg);
  return launch_cfg<Cfg<BN, 1, 4, 4>>(xmap, p, fit(rx, 2, p.wg, 55 * 1024, 2, 12 / p.wg + 1), rx, 2, s);
}

cudaError_t w4a16_gemm_launch(const CUtensorMap& xmap, const W4A16Params& p0, int bn, int nt, cudaStream_t s) {
  static const int dbg_env = [] {  // experiment: SQ_GEMM_DBG bit 0 = no dequant arithmetic, bit 1 = no MMA
    const char* e = std::getenv("SQ_GEMM_DBG");
    return e != nullptr ? std::atoi(e) : 0;
  }();
  W4A16Params p = p0;
  p.dbg = dbg_env;
  p.wg = 1;  // (the decode configuration groups weight copies and A stages)
  p.ag = 1;
  int ow, ox, oa;
  const bool ov = ring_override(&ow, &ox, &oa);
  if (nt == 1) {
    switch (bn) {
      case 16:
        if (!ov && w4a16_narrow(p.wfmt, p.gpk)) return launch_decode_narrow<16>(xmap, p, s);
        return ov ? launch_cfg<Cfg<16, 1, 2>>(xmap, p, ow, ox, oa, s) : launch_cfg<Cfg<16, 1, 2>>(xmap, p, 8, 8, 4, s);
      case 32:
        if (!ov && w4a16_narrow(p.wfmt, p.gpk)) return launch_decode_narrow<32>(xmap, p, s);
        return ov ? launch_cfg<Cfg<32, 1, 2>>(xmap, p, ow, ox, oa, s) : launch_cfg<Cfg<32, 1, 2>>(xmap, p, 8, 6, 4, s);
      case 64:
        if (ov) return launch_cfg<Cfg<64, 1, 2>>(xmap, p, ow, ox, oa, s);
        if (w4a16_narrow(p.wfmt, p.gpk)) return launch_decode_narrow<64>(xmap, p, s);
        return launch_cfg<Cfg<64, 1, 2>>(xmap, p, 8, 6, 4, s);
      case 128: return launch_cfg<Cfg<128, 1, 2>>(xmap, p, 8, 4, 4, s);
      case 256: return launch_cfg<Cfg<256, 1, 1>>(xmap, p, 6, 4, 4, s);
      default: return cudaErrorInvalidValue;
    }
  } else if (nt == 2) {
    switch (bn) {
      case 128: return launch_cfg<Cfg<128, 2, 1>>(xmap, p, 6, 4, 2, s);
      case 256: return launch_cfg<Cfg<256, 2, 1>>(xmap, p, 4, 3, 2, s);
      default: return cudaErrorInvalidValue;
    }
  }
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------------
// Repack the canonical npy-dir INT4 asymmetric layout into the tile-major device layout.
//   src: packed (N, K/2) u8 with lo nibble = even column; scales/zeros (N, G) fp32.
//   dst: per (128-row block rb, 64-column block kb) one contiguous tile of
//        1024 words of nibbles [2 halves][128 rows][4 words] followed by gpk*128 words of
//        (bf16 scale | bf16 zero << 16) [gpk][128 rows].
//   Np = N rounded up to 256, KB = ceil(K/64); padding rows/columns dequantize to 0.
__global__ void repack_int4_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ scales,
                                   const float* __restrict__ zeros, uint32_t* __restrict__ wt, int N, int K,
                                   int group, int kb_total, int n_pad, int gpk) {
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)n_pad * kb_total) return;
  const int n = (int)(idx % n_pad);
  const int kb = (int)(idx / n_pad);
  const int rb = n / 128, r = n % 128;
  const int G = (K + group - 1) / group;
  const int pos[8] = {0, 16, 4, 20, 8, 24, 12, 28};
  uint32_t* tile = wt + ((size_t)rb * kb_total + kb) * (1024 + gpk * 128);
  for (int c = 0; c < 2; ++c) {
    for (int w = 0; w < 4; ++w) {
      uint32_t word = 0;
      for (int e = 0; e < 8; ++e) {
        const int col = kb * 64 + c * 32 + w * 8 + e;
        uint32_t qv = 0;
        if (n < N && col < K) {
          const uint8_t b = packed[(size_t)n * (K / 2) + col / 2];
          qv = (col & 1) ? (b >> 4) : (b & 0xF);
        }
        word |= qv << pos[e];
      }
      tile[(c * 128 + r) * 4 + w] = word;
    }
  }
  uint32_t* st = tile + 1024;
  for (int j = 0; j < gpk; ++j) {
    const int col = kb * 64 + j * (64 / gpk);
    const int g = col / group;
    float sc = 0.f, ze = 0.f;
    if (n < N && col < K && g < G) {
      sc = scales[(size_t)n * G + g];
      ze = zeros[(size_t)n * G + g];
    }
    const uint32_t sb = __bfloat16_as_ushort(__float2bfloat16(sc));
    const uint32_t zb = __bfloat16_as_ushort(__float2bfloat16(ze));
    st[j * 128 + r] = sb | (zb << 16);
  }
}

cudaError_t repack_int4_launch(const uint8_t* packed, const float* scales, const float* zeros, uint32_t* wt, int N,
                               int K, int group, cudaStream_t s) {
  const int kb_total = (K + 63) / 64;
  const int n_pad = (N + 255) / 256 * 256;
  const int gpk = group >= 64 ? 1 : 64 / group;
  const long total = (long)n_pad * kb_total;
  repack_int4_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(packed, scales, zeros, wt, N, K, group,
                                                                     kb_total, n_pad, gpk);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ weight expansion
// Tile-major weight codes (any WF_* format) -> bf16 [N, ld] row-major, the values the fused
// GEMM computes (one rounding of q * scale + zero). Used by the large-M path, where a
// bf16 tensor-core GEMM over the expanded weights beats dequantizing every weight tile once
// per token tile.
namespace {
// INT4: thread (row lr, word w) of a 256-thread CTA expands 8 columns (one nibble word) of
// one row per k-block, so the 8 threads of a row store its 128 bytes contiguously.
constexpr int kDqKbPerCta = 8;
__global__ void __launch_bounds__(256) dequant_int4_kernel(const uint8_t* __restrict__ wq, int gpk, int kb_total,
                                                           int N, int ld, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  const int w = threadIdx.x & 7;
  const int row = blockIdx.y * 32 + (threadIdx.x >> 3);
  const int rb = row >> 7, r = row & (BM - 1);
  const int kb0 = blockIdx.x * kDqKbPerCta;
  const int tbytes = tile_bytes(gpk, WF_INT4);
  const uint8_t* base = wq + ((size_t)rb * kb_total) * tbytes;
  const int woff = ((w >> 2) * BM + r) * 16 + (w & 3) * 4;
  const int soff = W_TILE_BYTES + ((((w * gpk) >> 3) * BM + r) << 2);
  uint32_t code[kDqKbPerCta], szw[kDqKbPerCta];
#pragma unroll
  for (int j = 0; j < kDqKbPerCta; ++j) {
    const int kb = min(kb0 + j, kb_total - 1);
    code[j] = __ldg(reinterpret_cast<const uint32_t*>(base + (size_t)kb * tbytes + woff));
    szw[j] = __ldg(reinterpret_cast<const uint32_t*>(base + (size_t)kb * tbytes + soff));
  }
  pdl_wait();  // the output buffer may still be read by the previous kernel
  if (row >= N) return;
  __nv_bfloat16* dst = out + (size_t)row * ld + w * 8;
#pragma unroll
  for (int j = 0; j < kDqKbPerCta; ++j) {
    const int kb = kb0 + j;
    if (kb < kb_total) {
      const __nv_bfloat16 sc = __ushort_as_bfloat16((unsigned short)(szw[j] & 0xFFFFu));
      const __nv_bfloat16 ze = __ushort_as_bfloat16((unsigned short)(szw[j] >> 16));
      *reinterpret_cast<uint4*>(dst + kb * 64) = dq_word(code[j], __bfloat162bfloat162(sc), __bfloat162bfloat162(ze));
    }
  }
}

// Other formats: thread (r, c) expands row r, columns [32c, 32c + 32) of each k-block.
__global__ void __launch_bounds__(256) dequant_weight_kernel(const uint8_t* __restrict__ wq, int wfmt, int gpk,
                                                             int kb_total, int kb_per_cta, int N, int ld,
                                                             __nv_bfloat16* __restrict__ out,
                                                             const __nv_bfloat16* codebook, int n_books) {
  __shared__ uint4 fmt_tab[512];
  uint32_t* lut = reinterpret_cast<uint32_t*>(fmt_tab);
  if (wfmt == WF_NF4) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
      lut[i] = bf2_bits(codebook != nullptr ? __halves2bfloat162(codebook[i & 15], codebook[i >> 4])
                                            : __floats2bfloat162_rn(kNf4Levels[i & 15], kNf4Levels[i >> 4]));
  } else if (wfmt == WF_AQLM) {
    for (int i = threadIdx.x; i < 256 * n_books; i += blockDim.x) fmt_tab[i] = reinterpret_cast<const uint4*>(codebook)[i];
  }
  __syncthreads();
  pdl_trigger();
  const int r = threadIdx.x & (BM - 1), c = threadIdx.x >> 7;
  const int rb = blockIdx.y, row = rb * BM + r;
  const int kb0 = blockIdx.x * kb_per_cta, kb1 = min(kb_total, kb0 + kb_per_cta);
  const int tbytes = tile_bytes(gpk, wfmt);
  pdl_wait();
  for (int kb = kb0; kb < kb1; ++kb) {
    const uint8_t* tb = wq + ((size_t)rb * kb_total + kb) * tbytes;
    uint4 o[4];
    dq_other(tb, wfmt, r, c, gpk, lut, n_books, o);
    if (row < N) {
      uint4* dst = reinterpret_cast<uint4*>(out + (size_t)row * ld + kb * 64 + c * 32);
#pragma unroll
      for (int w = 0; w < 4; ++w) dst[w] = o[w];
    }
  }
}
}  // namespace

cudaError_t dequant_weight_launch(const uint32_t* wq, int wfmt, int N, int K, int group, int ld,
                                  __nv_bfloat16* out, const __nv_bfloat16* codebook, int n_books, int num_sms,
                                  cudaStream_t s) {
  const int gpk = group >= 64 ? 1 : 64 / group;
  const int kb_total = (K + 63) / 64;
  const uint8_t* w8 = reinterpret_cast<const uint8_t*>(wq);
  if (wfmt == WF_INT4) {
    dim3 grid((kb_total + kDqKbPerCta - 1) / kDqKbPerCta, (N + 31) / 32);
    SQ_LAUNCH(dequant_int4_kernel, grid, dim3(256), 0, s, 1u, w8, gpk, kb_total, N, ld, out);
    return cudaSuccess;
  }
  const int rbs = (N + BM - 1) / BM;
  // about four CTAs per SM in one wave; each CTA expands a run of k-blocks of one row block
  const int want = max(1, (4 * num_sms + rbs - 1) / rbs);
  const int kpc = (kb_total + min(want, kb_total) - 1) / min(want, kb_total);
  dim3 grid((kb_total + kpc - 1) / kpc, rbs);
  SQ_LAUNCH(dequant_weight_kernel, grid, dim3(256), 0, s, 1u, w8, wfmt, gpk, kb_total, kpc, N, ld, out, codebook,
            n_books);
  return cudaSuccess;
}

}  // namespace sq
