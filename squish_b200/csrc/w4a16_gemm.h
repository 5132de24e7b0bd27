// w4a16_gemm.h — host/device interface of the INT4 weight-only tcgen05 GEMM.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace sq {

enum : int { EPI_PLAIN = 0, EPI_SILU_MUL = 1 };
// Weight code formats of a (128 rows x 64 columns) tile; the (scale, zero) words follow the codes.
enum : int {
  WF_INT4 = 0,  // unsigned nibbles, x = zero + q * scale                    (4 KiB of codes)
  WF_NF4 = 1,   // NormalFloat-4 level index, x = level[q] * absmax          (4 KiB)
  WF_INT8 = 2,  // signed bytes, x = q * scale                                (8 KiB)
  WF_INT2 = 3,  // unsigned 2-bit codes, x = zero + q * scale                 (2 KiB)
  WF_INT3 = 4,  // 3-bit codes q + 4 (q in [-4, 3]), x = zero + q * scale      (3 KiB)
  WF_AQLM = 5,  // per 8 columns one index into each of <= 2 codebooks of 256 x 8 values,
                // x = scale * sum_k book_k[idx_k]                             (2 KiB)
  WF_FP8 = 6,   // OCP FP8 E4M3 bytes, x = fp8(q) * scale                       (8 KiB)
};

struct W4A16Params {
  const uint32_t* wq;             // tile-major weight tiles [N/128][KB][1024 + gpk*128] words (nibbles, then
                                  // (scale | zero<<16) bf16 pairs)
  const uint32_t* sz;             // unused (kept for layout compatibility)
  const __nv_bfloat16* bias;      // [N] or nullptr
  const __nv_bfloat16* residual;  // [M, ldr] added in the epilogue, or nullptr (may alias y)
  __nv_bfloat16* y;               // [M, ldy]
  float* ws;                      // split-K partials [splits][M][N] (splits > 1)
  int* counters;                  // per output tile arrival counters, zero on entry, reset on exit
  int* status;                    // device status word (0 = ok)
  int M, N, K;
  int ldy, ldr;
  int kb_total, kb_per_split, splits;
  int gpk;                        // (scale, zero) groups per 64-column k-block: 1, 2 or 4
  int epilogue;                   // EPI_PLAIN | EPI_SILU_MUL
  int wfmt;                       // WF_* code format of the weight tiles
  const __nv_bfloat16* codebook;  // WF_AQLM: [n_books][256][8] bf16
  int n_books;
  int ring_w, ring_x, ring_a;     // set by the launcher
  unsigned long long* trace;      // optional: per-k-block role timestamps of CTA (0,0,0), 16 x 64 entries
  // Grouped (mixture-of-experts) mode, when tile_expert != nullptr: the rows of X are sorted
  // by expert and padded so every BN-row token tile belongs to one expert; token tile y uses
  // the weights at wq + tile_expert[y] * expert_stride bytes, and tiles y >= *num_tiles exit.
  const int* tile_expert;
  const int* num_tiles;
  long long expert_stride;
  // Tensor-parallel push mode (fused GEMM -> all-reduce), when push_dst != nullptr: the
  // partial tile is stored into every rank's receive buffer (peer memory over NVLink) at
  // push_dst[r] + parity * push_stride, then each CTA adds 1 to its tile's flag on every
  // rank (push_flags[r] + parity * flag_stride + tile). parity = *seq & 1.
  __nv_bfloat16* const* push_dst;
  int* const* push_flags;
  long long push_stride;
  int flag_stride;
  const int* seq;
  int tp;
  // Reduce-scatter routing (push_rows > 0): row m goes only to rank m / push_rows (the owner of
  // that token), at push_dst[owner] + parity * push_stride + (m - owner * push_rows) * ldy, and
  // every CTA adds 1 to flag index 0 of its source row on every rank (the owners wait for the
  // launch's CTA count).
  int push_rows;
  // All-gather wait (ag_flags != nullptr): X was pushed into this rank's buffer by tp ranks;
  // before its first activation load the producer waits (bounded) until ag_flags[s] >= ag_expect
  // for every source s. The last CTA to finish clears the flags (ag_done counts finished CTAs).
  int* ag_flags;
  int* ag_done;
  int ag_expect;
  // timing experiments only (results are wrong when set): bit 0 skips the dequant arithmetic
  // (raw code words go to the operand), bit 1 skips the MMAs (the ring slots are still retired)
  int dbg;
  // k-blocks per weight bulk copy (wg, set by the launcher) and per activation TMA load (xg: the
  // caller's x map is then the 3-D {64, rows, k-block} view with box depth xg); 0 or 1 = one
  int wg, xg;
  // k-blocks per tensor-memory A stage (one dequant -> MMA hand-off), set by the launcher
  int ag;
};

// True when token tiles of <= 64 run the 4-dequant-warp configuration (four CTAs per SM):
// INT4 codes with one (scale, zero) group per 64-column k-block.
bool w4a16_narrow(int wfmt, int gpk);
// True when a launch with token tile bn runs the decode configuration, which takes an activation
// map of xg > 1 k-blocks per load (W4A16Params::xg).
bool w4a16_decode_grouping(int bn, int wfmt, int gpk);
cudaError_t w4a16_gemm_launch(const CUtensorMap& xmap, const W4A16Params& p, int bn, int nt, cudaStream_t s);
// Expand tile-major weight codes to bf16 [N, ld] (ld >= 64 * ceil(K / 64), a multiple of 8).
cudaError_t dequant_weight_launch(const uint32_t* wq, int wfmt, int N, int K, int group, int ld,
                                  __nv_bfloat16* out, const __nv_bfloat16* codebook, int n_books, int num_sms,
                                  cudaStream_t s);
cudaError_t repack_int4_launch(const uint8_t* packed, const float* scales, const float* zeros, uint32_t* wt, int N,
                               int K, int group, cudaStream_t s);

}  // namespace sq
