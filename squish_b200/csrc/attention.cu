// attention.cu — paged attention over quantized KV pages (decode and chunked prefill).
//
// Replaces the reference's attention paths: mx.fast.scaled_dot_product_attention and the
// Metal `fused_sdpa` shader (squish/hardware/fused_kernels.py:87-133, CPU restatement
// :218-224) and the split-KV decode kernel `flash_decode_split_f32`
// (squish_quant_rs/src/lib.rs:3056), which returns (out, lse, max) per split for a later
// merge. Here the cache is paged (page tables read in-kernel, no gather) and quantized;
// each 16-token tile is dequantized into shared memory (kv_format.cuh) and multiplied on
// the tensor cores with mma.sync m16n8k16 (GQA query heads of one KV head form the
// 16-row M side in decode; query tokens in prefill). Decode is HBM-bound: the roofline
// is the quantized KV bytes per step, not MMA rate.
//
// Softmax runs in the log2 domain (scores pre-multiplied by scale*log2(e), exp2f).
#include <cstdlib>

#include "kernels.h"
#include "kv_format.cuh"
#include "launch.cuh"

namespace sq {

namespace {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------------------- decode
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Half of one (page, head, token) row (D/2 dims) in registers, with its scale / zero per
// 32-dim quarter converted at load, so a chunk of 8 dims dequantizes in a few bit operations
// and two bf16x2 FMAs (4/2-bit codes) or eight fp32 FMAs (8-bit codes).
template <int D, int FMT>
struct FastHalf {
  static constexpr int DL = D / 2;
  static constexpr int kBytes = DL * kv_bits(FMT) / 8;
  static constexpr int kWords = kBytes / 4;
  static constexpr int NQ = DL >= 32 ? DL / 32 : 1;
  static_assert(kBytes % 4 == 0, "half rows are whole 32-bit words");
  uint32_t w[kWords];
  uint32_t s2[NQ], z2[NQ];
  float sf[NQ], zf[NQ];

  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int i = 0; i < kWords; ++i) w[i] = 0u;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      s2[q] = z2[q] = 0u;
      sf[q] = zf[q] = 0.f;
    }
  }

  __device__ __forceinline__ void load(const uint8_t* __restrict__ row_codes, const __half* __restrict__ row_scales,
                                       int part, int G) {
    const uint8_t* src = row_codes + part * kBytes;
    if constexpr (kBytes % 16 == 0) {
#pragma unroll
      for (int i = 0; i < kWords / 4; ++i) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + i);
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < kWords; ++i) w[i] = __ldg(reinterpret_cast<const uint32_t*>(src) + i);
    }
    if constexpr (FMT != KV_BF16) {
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const int g = (part * DL + q * 32) / G;
        float sc, ze;
        if constexpr (kv_asym(FMT)) {
          sc = __half2float(__ldg(row_scales + 2 * g));
          ze = __half2float(__ldg(row_scales + 2 * g + 1));
        } else {
          sc = __half2float(__ldg(row_scales + g));
          ze = FMT == KV_INT4 ? -7.5f * sc : FMT == KV_INT2 ? -1.5f * sc : 0.f;
        }
        sf[q] = sc;
        zf[q] = ze;
        s2[q] = pack_bf2(sc, sc);
        z2[q] = pack_bf2(ze, ze);
      }
    }
  }

  // dims [8c, 8c + 8) of the half row -> 8 bf16
  __device__ __forceinline__ uint4 dequant(int c) const {
    if constexpr (FMT == KV_BF16) {
      return make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    } else {
      const int q = NQ == 1 ? 0 : (c >> 2);
      uint32_t o[4];
      if constexpr (FMT == KV_INT4 || FMT == KV_V4 || FMT == KV_INT2) {
        const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
        const __nv_bfloat162 s = *reinterpret_cast<const __nv_bfloat162*>(&s2[q]);
        const __nv_bfloat162 z = *reinterpret_cast<const __nv_bfloat162*>(&z2[q]);
        if constexpr (FMT == KV_INT2) {
          const uint32_t word = (w[c >> 1] >> ((c & 1) * 16)) & 0xFFFFu;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t t = ((word >> (4 * i)) & 0x3u) | (((word >> (4 * i + 2)) & 0x3u) << 16) | 0x43004300u;
            const __nv_bfloat162 r = __hfma2(__hsub2(*reinterpret_cast<__nv_bfloat162*>(&t), k128), s, z);
            o[i] = *reinterpret_cast<const uint32_t*>(&r);
          }
        } else {
          // byte i of the word = dims (2i, 2i+1) as (low, high) nibble
          const uint32_t lo = w[c] & 0x0F0F0F0Fu, hi = (w[c] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t t = (__byte_perm(lo, hi, (uint32_t)(i | ((4 + i) << 8))) & 0x00FF00FFu) | 0x43004300u;
            const __nv_bfloat162 r = __hfma2(__hsub2(*reinterpret_cast<__nv_bfloat162*>(&t), k128), s, z);
            o[i] = *reinterpret_cast<const uint32_t*>(&r);
          }
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
  }

  __device__ __forceinline__ void store(__nv_bfloat16* dst) const {
#pragma unroll
    for (int c = 0; c < DL / 8; ++c) *reinterpret_cast<uint4*>(dst + c * 8) = dequant(c);
  }
};

// grid (B, Hkv, splits), 4 warps; warp w handles 16-token tiles t0+w, t0+w+4, ...
// M side of each MMA = the G_q query heads of this KV head (padded to 16), read from a
// shared-memory copy of Q by ldmatrix per tile (keeps 32 registers free for occupancy).
// The running max is raised, and O rescaled, only when it grows by more than 2^8.
template <int D, int FK, int FV>
__global__ void __launch_bounds__(128, (FK == KV_BF16 || kv_bits(FK) == 8) ? 3 : 4) decode_kernel(const AttnParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int LD = D + 8;
  constexpr int NWARP = 4;
  extern __shared__ __align__(16) uint8_t sm[];
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int Gq = p.Hq / p.Hkv;
  const int kv_len = p.seq_lens[b];
  const int n_tiles = (kv_len + 15) / 16;
  const int t0 = split * p.tiles_per_split;
  const int t1 = min(n_tiles, t0 + p.tiles_per_split);
  const int* bt = p.block_tables + (size_t)b * p.bt_stride;
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(sm);       // [16][LD]
  __nv_bfloat16* Ks = Qs + 16 * LD + warp * 2 * 16 * LD;           // per warp [16][LD]
  __nv_bfloat16* Vs = Ks + 16 * LD;
  const float scale = p.sm_scale * kLog2e;

  // Q rows (query heads of this KV head; rows >= Gq zero) -> shared memory
  {
    const __nv_bfloat16* qb = p.q + (size_t)b * p.ld_q + (size_t)h * Gq * D;
    for (int i = threadIdx.x; i < 16 * (D / 8); i += blockDim.x) {
      const int r = i / (D / 8), c = i % (D / 8);
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < Gq) v = *reinterpret_cast<const uint4*>(qb + (size_t)r * D + c * 8);
      *reinterpret_cast<uint4*>(Qs + r * LD + c * 8) = v;
    }
  }
  __syncthreads();
  const uint32_t qbase = smem_addr(Qs);
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  // Each lane owns half a row (token lane/2, dims [half*D/2, +D/2)) of the 16-token tile.
  // A tile never crosses a page (page_size % 16 == 0), so one page-table read per tile;
  // the next tile's raw codes are loaded into registers while this tile is computed.
  using RK = FastHalf<D, FK>;
  using RV = FastHalf<D, FV>;
  const int rr = lane >> 1, part = lane & 1;
  const int PS = p.page_size;
  constexpr int CBK = kv_code_bytes(FK, D), CBV = kv_code_bytes(FV, D);
  const int NSK = kv_nscale(FK, D, p.group), NSV = kv_nscale(FV, D, p.group);
  auto fetch = [&](int tile, RK& a, RV& c) {
    const int tok = tile * 16 + rr;
    const int page = (tile < t1 && tok < kv_len) ? __ldg(bt + (tile * 16) / PS) : -1;
    if (tile < t1 && tok < kv_len && kv_index_ok(page, p.num_pages, p.status)) {
      const size_t rowid = ((size_t)page * p.Hkv + h) * PS + ((tile * 16) % PS) + rr;
      a.load(p.k_codes + rowid * CBK, p.k_scales + rowid * NSK, part, p.group);
      c.load(p.v_codes + rowid * CBV, p.v_scales + rowid * NSV, part, p.group);
    } else {
      a.clear();
      c.clear();
    }
  };
  RK rk;
  RV rv;
  fetch(t0 + warp, rk, rv);
  for (int tile = t0 + warp; tile < t1; tile += NWARP) {
    const int tok0 = tile * 16;
    rk.store(Ks + rr * LD + part * RK::DL);
    rv.store(Vs + rr * LD + part * RV::DL);
    fetch(tile + NWARP, rk, rv);  // in flight during this tile's math
    __syncwarp();
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
    const uint32_t kbase = smem_addr(Ks);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(qbase + (((lane & 15) * LD) + ks * 16 + (lane >> 4) * 8) * 2, a0, a1, a2, a3);
      const int tok = (lane & 7) + ((lane >> 4) << 3);
      const int col = ks * 16 + ((lane >> 3) & 1) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kbase + (tok * LD + col) * 2, b0, b1, b2, b3);
      mma16816(s[0], a0, a1, a2, a3, b0, b1);
      mma16816(s[1], a0, a1, a2, a3, b2, b3);
    }
    // scale + mask + online softmax (rows g, g+8; columns = tokens)
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = tok0 + nt * 8 + 2 * t4 + (e & 1);
        float v = s[nt][e] * scale;
        if (tok >= kv_len) v = -INFINITY;
        s[nt][e] = v;
      }
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    // lazy max: raise only when the tile max exceeds the running one by > 2^8
    const bool r0 = mx0 > m0 + 8.f, r1 = mx1 > m1 + 8.f;
    const float a0 = r0 ? ex2f(m0 - mx0) : 1.f;  // 0 when m was -inf
    const float a1 = r1 ? ex2f(m1 - mx1) : 1.f;
    if (r0) m0 = mx0;
    if (r1) m1 = mx1;
    const float base0 = (m0 == -INFINITY) ? 0.f : m0, base1 = (m1 == -INFINITY) ? 0.f : m1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = ex2f(s[nt][0] - base0);
      s[nt][1] = ex2f(s[nt][1] - base0);
      s[nt][2] = ex2f(s[nt][2] - base1);
      s[nt][3] = ex2f(s[nt][3] - base1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * a0 + rs0;
    l1 = l1 * a1 + rs1;
    if (__any_sync(0xffffffffu, r0 || r1)) {
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[i][0] *= a0;
        o[i][1] *= a0;
        o[i][2] *= a1;
        o[i][3] *= a1;
      }
    }
    const uint32_t pa0 = pack_bf2(s[0][0], s[0][1]), pa1 = pack_bf2(s[0][2], s[0][3]);
    const uint32_t pa2 = pack_bf2(s[1][0], s[1][1]), pa3 = pack_bf2(s[1][2], s[1][3]);
    const uint32_t vbase = smem_addr(Vs);
#pragma unroll
    for (int dt = 0; dt < D / 16; ++dt) {
      const int tok = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int col = dt * 16 + (lane >> 4) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vbase + (tok * LD + col) * 2, b0, b1, b2, b3);
      mma16816(o[2 * dt], pa0, pa1, pa2, pa3, b0, b1);
      mma16816(o[2 * dt + 1], pa0, pa1, pa2, pa3, b2, b3);
    }
    __syncwarp();
  }
  // quad-reduce l
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  // cross-warp merge through shared memory: [warp][16 rows] m, l and [warp][16][D] o
  __syncthreads();
  float* mw = reinterpret_cast<float*>(sm);
  float* lw = mw + NWARP * 16;
  float* ow = lw + NWARP * 16;
  if (t4 == 0) {
    mw[warp * 16 + g] = m0;
    mw[warp * 16 + g + 8] = m1;
    lw[warp * 16 + g] = l0;
    lw[warp * 16 + g + 8] = l1;
  }
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int col = i * 8 + 2 * t4;
    ow[(warp * 16 + g) * D + col] = o[i][0];
    ow[(warp * 16 + g) * D + col + 1] = o[i][1];
    ow[(warp * 16 + g + 8) * D + col] = o[i][2];
    ow[(warp * 16 + g + 8) * D + col + 1] = o[i][3];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < Gq * D; idx += blockDim.x) {
    const int row = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) M = fmaxf(M, mw[w * 16 + row]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NWARP; ++w) {
        const float f = (mw[w * 16 + row] == -INFINITY) ? 0.f : exp2f(mw[w * 16 + row] - M);
        L += lw[w * 16 + row] * f;
        O += ow[(w * 16 + row) * D + d] * f;
      }
    }
    const int hq = h * Gq + row;
    if (p.splits == 1) {
      p.out[(size_t)b * p.ld_out + (size_t)hq * D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
    } else {
      const size_t base = ((size_t)b * p.Hq + hq) * p.splits + split;
      p.o_part[base * D + d] = (L > 0.f) ? O / L : 0.f;
      if (d == 0) p.lse_part[base] = (L > 0.f) ? M + log2f(L) : -INFINITY;
    }
  }
}

// ----------------------------------------------------------------------------- decode, token-major MMA
// Decode attention with the 16 keys of a tile on the MMA M side and the (<= 8) query heads of
// one KV head on the N side, so an m16n8k16 tile wastes nothing on a GQA group of 7-8
// heads, and with the keys multiplied in their quantized form:
//
//  * a key code c becomes the exact operand M0 + c by one byte permute with a constant
//    exponent byte (bf16 128 + c for 4-bit codes, fp16 1024 + c for 8-bit codes), straight
//    from global memory into the A fragment (no shared memory, no per-element scaling);
//    with key value v = s * c + z per (token, group), q . k over a group is
//    s * (q . (M0 + c)) + (z - M0 * s) * sum(q), so each group's MMA sum is scaled once per
//    (token, head) afterwards. Every MMA k-step takes its 16 dims from one scale group.
//    The sum(q) terms use the same rounded q values as the MMA, and the products are
//    exact in fp32, so the M0 offset cancels to fp32 rounding;
//  * values are dequantized once into a per-warp shared-memory tile (exact code, then one
//    bf16 FMA with the group's scale and zero, as in the prefill kernels), dims permuted
//    inside each 8-dim chunk to the order the byte permute produces; O^T = V^T P^T takes
//    V^T by ldmatrix.trans and P^T from the score accumulators by movmatrix.trans;
//  * softmax runs per head over the key axis (three shuffles), with the lazy running-max
//    raise of the other kernels (O is rescaled only when a head's max grows by > 2^8).
// Reference op: squish_quant_rs/src/lib.rs:3056 flash_decode_split_f32 (one split of
// per-head softmax(q K^T / sqrt(d)) V with (out, lse) for the merge).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}
__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}
__device__ __forceinline__ void mma16816_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// N consecutive fp16 values (a row's scales) in one vector load, as 32-bit words (two halves
// each, low half first); zeros when !ok
template <int N>
__device__ __forceinline__ void load_halves(const __half* src, bool ok, uint32_t (&w)[(N + 1) / 2]) {
  static_assert(N == 1 || N == 2 || N == 4 || N == 8, "scale row of 1, 2, 4 or 8 halves");
  if constexpr (N == 8) {
    const uint4 v = ok ? __ldg(reinterpret_cast<const uint4*>(src)) : make_uint4(0u, 0u, 0u, 0u);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (N == 4) {
    const uint2 v = ok ? __ldg(reinterpret_cast<const uint2*>(src)) : make_uint2(0u, 0u);
    w[0] = v.x; w[1] = v.y;
  } else if constexpr (N == 2) {
    w[0] = ok ? __ldg(reinterpret_cast<const unsigned int*>(src)) : 0u;
  } else {
    w[0] = ok ? (uint32_t)__half_as_ushort(__ldg(src)) : 0u;
  }
}
__device__ __forceinline__ float half_at(const uint32_t* w, int i) {
  return __half2float(__ushort_as_half((unsigned short)((w[i >> 1] >> ((i & 1) * 16)) & 0xFFFFu)));
}

// dims of the 8 positions of a value-tile chunk (the byte permute's order)
__device__ __forceinline__ int vperm(int col) { return (col & ~7) | ((col & 3) << 1) | ((col >> 2) & 1); }

template <int D, int FK, int FV, int NG>
__global__ void __launch_bounds__(128, 4) decode_tm_kernel(const AttnParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int NW = 4;
  constexpr bool K8 = (FK == KV_K8);      // 8-bit keys: fp16 operands (1024 + c is exact)
  constexpr int NS = D / 16;              // k-steps of the score MMA
  constexpr int SPG = NS / NG;            // k-steps per key scale group
  constexpr int KW = K8 ? D / 16 : D / 32;  // key code words a thread loads per token
  constexpr int LDV = D + 8;
  constexpr int CBK = kv_code_bytes(FK, D), CBV = kv_code_bytes(FV, D);
  constexpr int NSK = NG * (kv_asym(FK) ? 2 : 1), NSV = NG * (kv_asym(FV) ? 2 : 1);
  constexpr int G = D / NG;
  static_assert(FV == KV_INT4 || FV == KV_V4, "4-bit values");
  extern __shared__ __align__(16) uint8_t sm[];
  uint16_t* Qs = reinterpret_cast<uint16_t*>(sm);                       // [8][D] operand-type bits
  float* qsum = reinterpret_cast<float*>(sm + 8 * D * 2);               // [8][NG]
  __nv_bfloat16* Vt = reinterpret_cast<__nv_bfloat16*>(sm + 8 * D * 2 + 8 * NG * 4);  // [NW][16][LDV]
  const int b = blockIdx.x, h = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int Gq = p.Hq / p.Hkv;
  const int kv_len = p.seq_lens[b];
  const int n_tiles = (kv_len + 15) / 16;
  const int t0 = split * p.tiles_per_split;
  const int t1 = min(n_tiles, t0 + p.tiles_per_split);
  const int* bt = p.block_tables + (size_t)b * p.bt_stride;
  const int PS = p.page_size;
  const float scale = p.sm_scale * kLog2e;

  // Q rows of this KV head's query heads (rows >= Gq zero), converted to the key operand type
  {
    const __nv_bfloat16* qb = p.q + (size_t)b * p.ld_q + (size_t)h * Gq * D;
    for (int i = threadIdx.x; i < 8 * D / 2; i += blockDim.x) {
      const int r = i / (D / 2), c = 2 * (i % (D / 2));
      float2 f = make_float2(0.f, 0.f);
      if (r < Gq) f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(qb + (size_t)r * D + c));
      *reinterpret_cast<uint32_t*>(Qs + r * D + c) = K8 ? pack_h2(f.x, f.y) : pack_bf2(f.x, f.y);
    }
  }
  __syncthreads();
  if (threadIdx.x < 8 * NG) {  // per (head, group) sums of the rounded operand values
    const int r = threadIdx.x / NG, gg = threadIdx.x % NG;
    float acc = 0.f;
    for (int d = gg * G; d < gg * G + G; ++d) {
      const uint16_t u = Qs[r * D + d];
      acc += K8 ? __half2float(__ushort_as_half(u)) : __bfloat162float(__ushort_as_bfloat16(u));
    }
    qsum[r * NG + gg] = acc;
  }
  // B fragments of Q^T for every k-step: b0 = (Q[g][pi(2t4)], Q[g][pi(2t4+1)]),
  // b1 = (Q[g][pi(2t4+8)], Q[g][pi(2t4+9)]) in the dim order of this thread's key bytes
  uint32_t qf[NS][2];
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    int d0;
    if constexpr (K8) {
      d0 = 4 * (t4 + 4 * s);  // word t4 + 4s: dims d0 .. d0 + 3
      qf[s][0] = *reinterpret_cast<const uint32_t*>(Qs + g * D + d0);
      qf[s][1] = *reinterpret_cast<const uint32_t*>(Qs + g * D + d0 + 2);
    } else {
      const int i = s >> 1, e = s & 1;  // word t4 + 4i, low (e = 0) or high nibbles
      d0 = 8 * (t4 + 4 * i) + e;
      qf[s][0] = (uint32_t)Qs[g * D + d0] | ((uint32_t)Qs[g * D + d0 + 2] << 16);
      qf[s][1] = (uint32_t)Qs[g * D + d0 + 4] | ((uint32_t)Qs[g * D + d0 + 6] << 16);
    }
  }
  __syncthreads();
  float qs_a[NG], qs_b[NG];  // sums for this thread's two heads 2t4, 2t4 + 1
#pragma unroll
  for (int gg = 0; gg < NG; ++gg) {
    qs_a[gg] = qsum[(2 * t4) * NG + gg];
    qs_b[gg] = qsum[(2 * t4 + 1) * NG + gg];
  }

  float o[D / 16][4];
#pragma unroll
  for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  __nv_bfloat16* Vs = Vt + warp * 16 * LDV;
  const uint32_t vbase = smem_addr(Vs);

  // per tile: key words of tokens g and g + 8, their scales, and this lane's half value row
  uint32_t kw[2][KW];
  float ks[2][NG], kz[2][NG];
  uint32_t vw[D / 16];
  uint32_t vs2[NG > 1 ? NG / 2 : 1], vz2[NG > 1 ? NG / 2 : 1];  // bf16 pairs of scale / zero
  const int vr = lane >> 1, vhalf = lane & 1;
  constexpr int NGH = NG > 1 ? NG / 2 : 1;  // value scale groups in half a row
  auto fetch = [&](int tile) {
    int page = tile < t1 ? __ldg(bt + (tile * 16) / PS) : 0;
    const bool live = tile < t1 && kv_index_ok(page, p.num_pages, p.status);
    if (!live) page = 0;
    const size_t row0 = ((size_t)page * p.Hkv + h) * PS + ((tile * 16) % PS);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int tok = tile * 16 + g + 8 * j;
      const bool ok = live && tok < kv_len;
      const size_t row = row0 + g + 8 * j;
      const uint32_t* kc = reinterpret_cast<const uint32_t*>(p.k_codes + row * CBK);
#pragma unroll
      for (int i = 0; i < KW; ++i) kw[j][i] = ok ? __ldg(kc + t4 + 4 * i) : 0u;
      uint32_t sc[(NSK + 1) / 2];
      load_halves<NSK>(p.k_scales + row * NSK, ok, sc);
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) {
        const float s_ = half_at(sc, kv_asym(FK) ? 2 * gg : gg);
        const float z_ = kv_asym(FK) ? half_at(sc, 2 * gg + 1) : -7.5f * s_;
        // s * (q . (M0 + c)) + (z - M0 * s) * sum(q)
        ks[j][gg] = s_;
        kz[j][gg] = z_ - (K8 ? 1024.f : 128.f) * s_;
      }
    }
    {
      const int tok = tile * 16 + vr;
      const bool ok = live && tok < kv_len;
      const size_t row = row0 + vr;
      const uint4* vc = reinterpret_cast<const uint4*>(p.v_codes + row * CBV + vhalf * (CBV / 2));
#pragma unroll
      for (int i = 0; i < D / 64; ++i) {
        const uint4 u = ok ? __ldg(vc + i) : make_uint4(0u, 0u, 0u, 0u);
        vw[4 * i] = u.x;
        vw[4 * i + 1] = u.y;
        vw[4 * i + 2] = u.z;
        vw[4 * i + 3] = u.w;
      }
      uint32_t sc[(NSV + 1) / 2];
      load_halves<NSV>(p.v_scales + row * NSV, ok, sc);
#pragma unroll
      for (int q = 0; q < NGH; ++q) {
        const int gg = NG > 1 ? vhalf * NGH + q : 0;
        const float s_ = half_at(sc, kv_asym(FV) ? 2 * gg : gg);
        const float z_ = kv_asym(FV) ? half_at(sc, 2 * gg + 1) : -7.5f * s_;
        vs2[q] = pack_bf2(s_, s_);
        vz2[q] = pack_bf2(z_, z_);
      }
    }
  };

  fetch(t0 + warp);
  constexpr uint32_t kMagicB = 0x43434343u, kMagicH = 0x64646464u;
  for (int tile = t0 + warp; tile < t1; tile += NW) {
    // ---- values of this tile -> shared memory (exact code, one FMA with scale and zero)
    {
      const __nv_bfloat162 k128 = __floats2bfloat162_rn(128.f, 128.f);
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {  // 8-dim chunks of this lane's half row
        const int q = NG > 1 ? (c * 8) / G : 0;
        const __nv_bfloat162 s2 = *reinterpret_cast<const __nv_bfloat162*>(&vs2[q]);
        const __nv_bfloat162 z2 = *reinterpret_cast<const __nv_bfloat162*>(&vz2[q]);
        const uint32_t L = vw[c] & 0x0F0F0F0Fu, H = (vw[c] >> 4) & 0x0F0F0F0Fu;
        uint32_t t[4] = {prmt(L, kMagicB, 0x4140u), prmt(L, kMagicB, 0x4342u), prmt(H, kMagicB, 0x4140u),
                         prmt(H, kMagicB, 0x4342u)};
        uint32_t o4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __nv_bfloat162 v = __hfma2(__hsub2(*reinterpret_cast<__nv_bfloat162*>(&t[e]), k128), s2, z2);
          o4[e] = *reinterpret_cast<const uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(Vs + vr * LDV + vhalf * (D / 2) + c * 8) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
      }
    }
    // ---- scores S^T[token][head] = K Q^T, one scale group at a time
    float sc4[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t kcur[2][KW];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int i = 0; i < KW; ++i) kcur[j][i] = kw[j][i];
    float kss[2][NG], kzz[2][NG];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int gg = 0; gg < NG; ++gg) {
        kss[j][gg] = ks[j][gg];
        kzz[j][gg] = kz[j][gg];
      }
    fetch(tile + NW);  // the next tile's codes are in flight during this tile's math
    __syncwarp();
#pragma unroll
    for (int gg = 0; gg < NG; ++gg) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ss = 0; ss < SPG; ++ss) {
        const int s = gg * SPG + ss;
        uint32_t a0, a1, a2, a3;
        if constexpr (K8) {
          a0 = prmt(kcur[0][s], kMagicH, 0x4140u);
          a2 = prmt(kcur[0][s], kMagicH, 0x4342u);
          a1 = prmt(kcur[1][s], kMagicH, 0x4140u);
          a3 = prmt(kcur[1][s], kMagicH, 0x4342u);
          mma16816_f16(acc, a0, a1, a2, a3, qf[s][0], qf[s][1]);
        } else {
          const int i = s >> 1, e = s & 1;
          const uint32_t w0 = e ? (kcur[0][i] >> 4) & 0x0F0F0F0Fu : kcur[0][i] & 0x0F0F0F0Fu;
          const uint32_t w1 = e ? (kcur[1][i] >> 4) & 0x0F0F0F0Fu : kcur[1][i] & 0x0F0F0F0Fu;
          a0 = prmt(w0, kMagicB, 0x4140u);
          a2 = prmt(w0, kMagicB, 0x4342u);
          a1 = prmt(w1, kMagicB, 0x4140u);
          a3 = prmt(w1, kMagicB, 0x4342u);
          mma16816(acc, a0, a1, a2, a3, qf[s][0], qf[s][1]);
        }
      }
      // acc: (token g, head 2t4), (g, 2t4+1), (g+8, 2t4), (g+8, 2t4+1)
      sc4[0] = fmaf(kss[0][gg], acc[0], fmaf(kzz[0][gg], qs_a[gg], sc4[0]));
      sc4[1] = fmaf(kss[0][gg], acc[1], fmaf(kzz[0][gg], qs_b[gg], sc4[1]));
      sc4[2] = fmaf(kss[1][gg], acc[2], fmaf(kzz[1][gg], qs_a[gg], sc4[2]));
      sc4[3] = fmaf(kss[1][gg], acc[3], fmaf(kzz[1][gg], qs_b[gg], sc4[3]));
    }
    // ---- online softmax per head over the 16 keys (log2 domain)
    const int tok0 = tile * 16;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = tok0 + g + 8 * (e >> 1);
      sc4[e] = (tok < kv_len) ? sc4[e] * scale : -INFINITY;
    }
    float mx_a = fmaxf(sc4[0], sc4[2]), mx_b = fmaxf(sc4[1], sc4[3]);
#pragma unroll
    for (int off = 4; off <= 16; off <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
    }
    const bool ra = mx_a > m_a + 8.f, rb = mx_b > m_b + 8.f;
    if (__any_sync(0xffffffffu, ra || rb)) {
      const float al_a = ra ? ex2f(m_a - mx_a) : 1.f, al_b = rb ? ex2f(m_b - mx_b) : 1.f;
      if (ra) m_a = mx_a;
      if (rb) m_b = mx_b;
      l_a *= al_a;
      l_b *= al_b;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        o[i][0] *= al_a;
        o[i][1] *= al_b;
        o[i][2] *= al_a;
        o[i][3] *= al_b;
      }
    }
    const float base_a = (m_a == -INFINITY) ? 0.f : m_a, base_b = (m_b == -INFINITY) ? 0.f : m_b;
    const float p0 = ex2f(sc4[0] - base_a), p1 = ex2f(sc4[1] - base_b);
    const float p2 = ex2f(sc4[2] - base_a), p3 = ex2f(sc4[3] - base_b);
    l_a += p0 + p2;
    l_b += p1 + p3;
    // P^T as the B operand: transpose the two 8x8 (token x head) blocks in registers
    const uint32_t pb0 = movtrans(pack_bf2(p0, p1)), pb1 = movtrans(pack_bf2(p2, p3));
    // ---- O^T[dim][head] += V^T P^T
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      const int j = lane >> 3;
      const int tok = (lane & 7) + ((j >> 1) << 3);
      const int col = mt * 16 + ((j & 1) << 3);
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vbase + (tok * LDV + col) * 2, a0, a1, a2, a3);
      mma16816(o[mt], a0, a1, a2, a3, pb0, pb1);
    }
    __syncwarp();
  }
#pragma unroll
  for (int off = 4; off <= 16; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  // cross-warp merge through shared memory: m, l [warp][8 heads], O [warp][8 heads][D]
  __syncthreads();
  float* mw = reinterpret_cast<float*>(sm);
  float* lw = mw + NW * 8;
  float* ow = lw + NW * 8;
  if (g == 0) {
    mw[warp * 8 + 2 * t4] = m_a;
    mw[warp * 8 + 2 * t4 + 1] = m_b;
    lw[warp * 8 + 2 * t4] = l_a;
    lw[warp * 8 + 2 * t4 + 1] = l_b;
  }
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) {
    const int d0 = vperm(mt * 16 + g), d1 = vperm(mt * 16 + g + 8);
    ow[(warp * 8 + 2 * t4) * D + d0] = o[mt][0];
    ow[(warp * 8 + 2 * t4 + 1) * D + d0] = o[mt][1];
    ow[(warp * 8 + 2 * t4) * D + d1] = o[mt][2];
    ow[(warp * 8 + 2 * t4 + 1) * D + d1] = o[mt][3];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < Gq * D; idx += blockDim.x) {
    const int row = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, mw[w * 8 + row]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float f = (mw[w * 8 + row] == -INFINITY) ? 0.f : exp2f(mw[w * 8 + row] - M);
        L += lw[w * 8 + row] * f;
        O += ow[(w * 8 + row) * D + d] * f;
      }
    }
    const int hq = h * Gq + row;
    if (p.splits == 1) {
      p.out[(size_t)b * p.ld_out + (size_t)hq * D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
    } else {
      const size_t base = ((size_t)b * p.Hq + hq) * p.splits + split;
      p.o_part[base * D + d] = (L > 0.f) ? O / L : 0.f;
      if (d == 0) p.lse_part[base] = (L > 0.f) ? M + log2f(L) : -INFINITY;
    }
  }
}

// grid (B, Hq), D threads: combine split partials (log2-domain LSE weights).
__global__ void decode_merge_kernel(const AttnParams p) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x, hq = blockIdx.y, d = threadIdx.x;
  const int D = p.D, S = p.splits;
  const size_t base = ((size_t)b * p.Hq + hq) * S;
  float M = -INFINITY;
  for (int s = 0; s < S; ++s) M = fmaxf(M, p.lse_part[base + s]);
  float L = 0.f, O = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < S; ++s) {
      const float lse = p.lse_part[base + s];
      if (lse == -INFINITY) continue;
      const float f = exp2f(lse - M);
      L += f;
      O += p.o_part[(base + s) * D + d] * f;
    }
  }
  if (d < D) p.out[(size_t)b * p.ld_out + (size_t)hq * D + d] = __float2bfloat16(L > 0.f ? O / L : 0.f);
}

// ------------------------------------------------------------------------------- prefill
// grid (n_tiles, Hkv * head_blocks); warps = query heads of this KV head (<= 8 per block).
// Each warp owns 32 query rows (2 m16 tiles) of one head; K/V tiles of 32 tokens are
// dequantized once per block into shared memory and shared by all its warps.
constexpr int PQ = 32;  // query rows per block
constexpr int PK = 32;  // kv tokens per tile

template <int D, int FK, int FV>
__global__ void __launch_bounds__(256) prefill_kernel(const AttnParams p) {
  pdl_wait();
  pdl_trigger();
  constexpr int LD = D + 8;
  extern __shared__ __align__(16) uint8_t sm[];
  const int tile = blockIdx.x;
  const int Gq = p.Hq / p.Hkv;
  const int hblocks = (Gq + 7) / 8;
  const int h = blockIdx.y / hblocks;
  const int hq0 = h * Gq + (blockIdx.y % hblocks) * 8;
  const int nheads = min(8, h * Gq + Gq - hq0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int b = p.tile_seq[tile];
  const int q0 = p.tile_q0[tile];
  const int qlen = p.q_len[b];
  const int ctx = p.ctx_len[b];
  const int qn = min(PQ, qlen - q0);
  const int pos0 = ctx - qlen + q0;  // absolute position of query row 0
  const int kv_end = pos0 + qn;      // exclusive
  const int* bt = p.block_tables + (size_t)b * p.bt_stride;
  const float scale = p.sm_scale * kLog2e;

  __nv_bfloat16* Ks = reinterpret_cast<__nv_bfloat16*>(sm);
  __nv_bfloat16* Vs = Ks + PK * LD;
  __nv_bfloat16* Qs = Vs + PK * LD + warp * PQ * LD;
  const int hq = hq0 + warp;
  const bool active = warp < nheads;
  __shared__ int tmask[PQ];
  const int cstart = ctx - qlen;  // absolute position of chunk token 0
  if (threadIdx.x < PQ)
    tmask[threadIdx.x] = (p.tree_mask != nullptr && (int)threadIdx.x < qn)
                             ? p.tree_mask[p.q_start[b] + q0 + threadIdx.x] : 0;

  // stage Q rows of this warp's head
  if (active) {
    for (int it = lane; it < PQ * (D / 8); it += 32) {
      const int r = it / (D / 8), c = it % (D / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r < qn)
        v = *reinterpret_cast<const uint4*>(p.q + (size_t)(p.q_start[b] + q0 + r) * p.ld_q + (size_t)hq * D + c * 8);
      *reinterpret_cast<uint4*>(Qs + r * LD + c * 8) = v;
    }
  }
  float o[2][D / 8][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int i = 0; i < D / 8; ++i) o[mt][i][0] = o[mt][i][1] = o[mt][i][2] = o[mt][i][3] = 0.f;
  float mrow[2][2] = {{-INFINITY, -INFINITY}, {-INFINITY, -INFINITY}};
  float lrow[2][2] = {{0.f, 0.f}, {0.f, 0.f}};

  // K/V tile loader: items = (row, part of a row) of the 32-token tile, at most two per
  // thread; raw codes of tile kt+1 are fetched into registers while tile kt is computed.
  // parts per row: up to 4, but every part must hold whole 32-bit words of codes
  constexpr int WK = D * kv_bits(FK) / 32, WV = D * kv_bits(FV) / 32;
  constexpr int NP = (WK < WV ? WK : WV) >= 4 ? 4 : 2;
  using RK = RowPart<D, FK, NP>;
  using RV = RowPart<D, FV, NP>;
  constexpr int ITEMS = PK * NP;
  const int PS = p.page_size;
  constexpr int CBK = kv_code_bytes(FK, D), CBV = kv_code_bytes(FV, D);
  const int NSK = kv_nscale(FK, D, p.group), NSV = kv_nscale(FV, D, p.group);
  RK rk[2];
  RV rv[2];
  auto fetch = [&](int kt) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int it = threadIdx.x + i * blockDim.x;
      if (it >= ITEMS) continue;
      const int r = it / NP, part = it % NP;
      const int tok = kt * PK + r;
      const int page = tok < kv_end ? __ldg(bt + tok / PS) : -1;
      if (tok < kv_end && kv_index_ok(page, p.num_pages, p.status)) {
        const size_t rowid = ((size_t)page * p.Hkv + h) * PS + (tok % PS);
        rk[i].load(p.k_codes + rowid * CBK, p.k_scales + rowid * NSK, part, p.group);
        rv[i].load(p.v_codes + rowid * CBV, p.v_scales + rowid * NSV, part, p.group);
      } else {
        rk[i].clear();
        rv[i].clear();
      }
    }
  };
  const int n_kv_tiles = (kv_end + PK - 1) / PK;
  fetch(0);
  for (int kt = 0; kt < n_kv_tiles; ++kt) {
    const int tok0 = kt * PK;
    __syncthreads();  // previous tile fully consumed
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int it = threadIdx.x + i * blockDim.x;
      if (it >= ITEMS) continue;
      const int r = it / NP, part = it % NP;
      rk[i].store(Ks + r * LD + part * RK::DIMS, p.group);
      rv[i].store(Vs + r * LD + part * RV::DIMS, p.group);
    }
    if (kt + 1 < n_kv_tiles) fetch(kt + 1);
    __syncthreads();
    if (!active) continue;
    float s[2][PK / 8][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < PK / 8; ++nt) s[mt][nt][0] = s[mt][nt][1] = s[mt][nt][2] = s[mt][nt][3] = 0.f;
    const uint32_t qbase = smem_addr(Qs), kbase = smem_addr(Ks), vbase = smem_addr(Vs);
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t a[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const int row = mt * 16 + (lane & 15);
        const int col = ks * 16 + (lane >> 4) * 8;
        ldsm_x4(qbase + (row * LD + col) * 2, a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
      }
#pragma unroll
      for (int np = 0; np < PK / 16; ++np) {
        const int tok = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int col = ks * 16 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kbase + (tok * LD + col) * 2, b0, b1, b2, b3);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          mma16816(s[mt][2 * np], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b0, b1);
          mma16816(s[mt][2 * np + 1], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b2, b3);
        }
      }
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
      for (int nt = 0; nt < PK / 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qrow = mt * 16 + g + ((e >> 1) << 3);
          const int key = tok0 + nt * 8 + 2 * t4 + (e & 1);
          float v = s[mt][nt][e] * scale;
          if (key > pos0 + qrow || qrow >= qn) v = -INFINITY;
          else if (key >= cstart) {
            const int tm = tmask[qrow];
            if (tm != 0 && !((tm >> (key - cstart)) & 1)) v = -INFINITY;
          }
          s[mt][nt][e] = v;
          mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        const float mn = fmaxf(mrow[mt][r], mx[r]);
        const float alpha = (mrow[mt][r] == -INFINITY) ? 0.f : exp2f(mrow[mt][r] - mn);
        mrow[mt][r] = mn;
        mx[r] = alpha;  // reuse as the rescale factor
      }
      const float base0 = (mrow[mt][0] == -INFINITY) ? 0.f : mrow[mt][0];
      const float base1 = (mrow[mt][1] == -INFINITY) ? 0.f : mrow[mt][1];
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < PK / 8; ++nt) {
        s[mt][nt][0] = exp2f(s[mt][nt][0] - base0);
        s[mt][nt][1] = exp2f(s[mt][nt][1] - base0);
        s[mt][nt][2] = exp2f(s[mt][nt][2] - base1);
        s[mt][nt][3] = exp2f(s[mt][nt][3] - base1);
        rs0 += s[mt][nt][0] + s[mt][nt][1];
        rs1 += s[mt][nt][2] + s[mt][nt][3];
      }
      lrow[mt][0] = lrow[mt][0] * mx[0] + rs0;
      lrow[mt][1] = lrow[mt][1] * mx[1] + rs1;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        o[mt][i][0] *= mx[0];
        o[mt][i][1] *= mx[0];
        o[mt][i][2] *= mx[1];
        o[mt][i][3] *= mx[1];
      }
    }
#pragma unroll
    for (int kk = 0; kk < PK / 16; ++kk) {
      uint32_t pa[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        pa[mt][0] = pack_bf2(s[mt][2 * kk][0], s[mt][2 * kk][1]);
        pa[mt][1] = pack_bf2(s[mt][2 * kk][2], s[mt][2 * kk][3]);
        pa[mt][2] = pack_bf2(s[mt][2 * kk + 1][0], s[mt][2 * kk + 1][1]);
        pa[mt][3] = pack_bf2(s[mt][2 * kk + 1][2], s[mt][2 * kk + 1][3]);
      }
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        const int tok = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int col = dt * 16 + (lane >> 4) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vbase + (tok * LD + col) * 2, b0, b1, b2, b3);
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          mma16816(o[mt][2 * dt], pa[mt][0], pa[mt][1], pa[mt][2], pa[mt][3], b0, b1);
          mma16816(o[mt][2 * dt + 1], pa[mt][0], pa[mt][1], pa[mt][2], pa[mt][3], b2, b3);
        }
      }
    }
  }
  if (!active) return;
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float l = lrow[mt][r];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      lrow[mt][r] = (l > 0.f) ? 1.f / l : 0.f;
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int qrow = mt * 16 + g + r * 8;
      if (qrow >= qn) continue;
      __nv_bfloat16* dst = p.out + (size_t)(p.q_start[b] + q0 + qrow) * p.ld_out + (size_t)hq * D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        const int col = i * 8 + 2 * t4;
        *reinterpret_cast<uint32_t*>(dst + col) =
            pack_bf2(o[mt][i][2 * r] * lrow[mt][r], o[mt][i][2 * r + 1] * lrow[mt][r]);
      }
    }
  }
}

template <int D, int FK, int FV>
cudaError_t launch_decode(const AttnParams& p, cudaStream_t s) {
  constexpr int LD = D + 8;
  const size_t kv_bytes = (size_t)(1 + 4 * 2) * 16 * LD * 2;  // Q tile + per-warp K / V tiles
  const size_t merge_bytes = (size_t)4 * 16 * 2 * 4 + (size_t)4 * 16 * D * 4;
  const size_t smem = kv_bytes > merge_bytes ? kv_bytes : merge_bytes;
  auto k = decode_kernel<D, FK, FV>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaError_t le = launch_k(k, dim3(p.B, p.Hkv, p.splits), dim3(128), smem, s, 1, p);
  if (le != cudaSuccess) return le;
  e = cudaGetLastError();
  if (e != cudaSuccess || p.splits == 1) return e;
  le = launch_k(decode_merge_kernel, dim3(p.B, p.Hq), dim3(D), 0, s, 1, p);
  if (le != cudaSuccess) return le;
  return cudaGetLastError();
}

template <int D, int FK, int FV>
cudaError_t launch_prefill(const AttnParams& p, cudaStream_t s) {
  constexpr int LD = D + 8;
  const size_t smem = (size_t)(2 * PK + 8 * PQ) * LD * 2;
  auto k = prefill_kernel<D, FK, FV>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int Gq = p.Hq / p.Hkv;
  const int hblocks = (Gq + 7) / 8;
  const int warps = Gq < 8 ? Gq : 8;
  e = launch_k(k, dim3(p.n_tiles, p.Hkv * hblocks), dim3(warps * 32), smem, s, 1, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

#define SQ_ATTN_DISPATCH(FN)                                                   \
  template <int D>                                                             \
  cudaError_t FN##_fmt(const AttnParams& p, cudaStream_t s) {                  \
    if (p.fmt_k == KV_BF16 && p.fmt_v == KV_BF16) return FN<D, KV_BF16, KV_BF16>(p, s); \
    if (p.fmt_k == KV_INT8 && p.fmt_v == KV_INT8) return FN<D, KV_INT8, KV_INT8>(p, s); \
    if (p.fmt_k == KV_INT4 && p.fmt_v == KV_INT4) return FN<D, KV_INT4, KV_INT4>(p, s); \
    if (p.fmt_k == KV_INT2 && p.fmt_v == KV_INT2) return FN<D, KV_INT2, KV_INT2>(p, s); \
    if (p.fmt_k == KV_K8 && p.fmt_v == KV_V4) return FN<D, KV_K8, KV_V4>(p, s);         \
    return cudaErrorInvalidValue;                                              \
  }

SQ_ATTN_DISPATCH(launch_decode)
SQ_ATTN_DISPATCH(launch_prefill)

template <int D, int FK, int FV, int NG>
cudaError_t launch_decode_tm(const AttnParams& p, cudaStream_t s) {
  constexpr int LDV = D + 8;
  const size_t main_bytes = (size_t)8 * D * 2 + (size_t)8 * NG * 4 + (size_t)4 * 16 * LDV * 2;
  const size_t merge_bytes = (size_t)4 * 8 * 2 * 4 + (size_t)4 * 8 * D * 4;
  const size_t smem = main_bytes > merge_bytes ? main_bytes : merge_bytes;
  auto k = decode_tm_kernel<D, FK, FV, NG>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaError_t le = launch_k(k, dim3(p.B, p.Hkv, p.splits), dim3(128), smem, s, 1, p);
  if (le != cudaSuccess) return le;
  e = cudaGetLastError();
  if (e != cudaSuccess || p.splits == 1) return e;
  le = launch_k(decode_merge_kernel, dim3(p.B, p.Hq), dim3(D), 0, s, 1, p);
  if (le != cudaSuccess) return le;
  return cudaGetLastError();
}

template <int D, int FK, int FV>
cudaError_t launch_decode_tm_g(const AttnParams& p, cudaStream_t s) {
  const int ng = D / p.group;
  if (ng == 1) return launch_decode_tm<D, FK, FV, 1>(p, s);
  if (ng == 2) return launch_decode_tm<D, FK, FV, 2>(p, s);
  if (ng == 4) return launch_decode_tm<D, FK, FV, 4>(p, s);
  return cudaErrorInvalidValue;
}

// The token-major decode kernel covers 4-bit values with 4-bit symmetric or 8-bit
// asymmetric keys, up to 8 query heads per KV head, head dims 64 / 128, and 1, 2 or 4
// scale groups per row (group >= 32); other cases run decode_kernel.
bool decode_tm_supported(const AttnParams& p) {
  if (p.Hkv <= 0 || p.Hq % p.Hkv != 0 || p.Hq / p.Hkv > 8) return false;
  if (p.D != 128 && p.D != 64) return false;
  if (p.group < 32 || p.D % p.group != 0 || p.D / p.group > 4) return false;
  if (std::getenv("SQ_DECODE_LEGACY") != nullptr) return false;
  return (p.fmt_k == KV_INT4 && p.fmt_v == KV_INT4) || (p.fmt_k == KV_K8 && p.fmt_v == KV_V4);
}

cudaError_t launch_decode_tm_any(const AttnParams& p, cudaStream_t s) {
  if (p.fmt_k == KV_INT4) {
    return p.D == 128 ? launch_decode_tm_g<128, KV_INT4, KV_INT4>(p, s) : launch_decode_tm_g<64, KV_INT4, KV_INT4>(p, s);
  }
  return p.D == 128 ? launch_decode_tm_g<128, KV_K8, KV_V4>(p, s) : launch_decode_tm_g<64, KV_K8, KV_V4>(p, s);
}

}  // namespace

cudaError_t paged_decode_attn_launch(const AttnParams& p, cudaStream_t s) {
  if (p.B == 0) return cudaSuccess;
  if (decode_tm_supported(p)) return launch_decode_tm_any(p, s);
  if (p.D == 128) return launch_decode_fmt<128>(p, s);
  if (p.D == 64) return launch_decode_fmt<64>(p, s);
  if (p.D == 32) return launch_decode_fmt<32>(p, s);
  return cudaErrorInvalidValue;
}

cudaError_t paged_prefill_attn_launch(const AttnParams& p, cudaStream_t s) {
  if (p.n_tiles == 0) return cudaSuccess;
  if (p.D == 128) return launch_prefill_fmt<128>(p, s);
  if (p.D == 64) return launch_prefill_fmt<64>(p, s);
  if (p.D == 32) return launch_prefill_fmt<32>(p, s);
  return cudaErrorInvalidValue;
}

}  // namespace sq
