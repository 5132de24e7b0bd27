// bf16_gemm.h — persistent tcgen05 GEMM for bf16 operands: y = x . W^T (+ bias) (+ residual),
// or the SwiGLU epilogue over gate/up rows interleaved in blocks of 64.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace sq {

struct Bf16GemmParams {
  const __nv_bfloat16* bias;      // [N] or nullptr
  const __nv_bfloat16* residual;  // [M, ldr] or nullptr (may alias y)
  __nv_bfloat16* y;               // [M, ldy]; N / 2 columns with the SwiGLU epilogue
  int M, N, K;
  int ldy, ldr;
  int epilogue;                   // EPI_PLAIN | EPI_SILU_MUL
  int vec;                        // y / residual / bias rows allow 16-byte accesses
  int* status;                    // device status word (0 = ok)
  // split-K (few output tiles): work item = (tile, split); each split stores its fp32 partial
  // tile in ws, and the last split of a tile to finish (counters[tile]) sums them in split
  // order and runs the epilogue, then resets its counter to zero.
  int splits, kb_per_split;
  float* ws;                      // [tiles][splits][256 columns][128 rows]
  int* counters;                  // [tiles], zero on entry and exit
};

// amap: x [M, K] bf16, box 64 x 128 (128B swizzle); bmap: W [N, K] bf16, box 64 x 256.
// Launches with p.splits / p.kb_per_split chosen from the tile count (ws_floats / n_counters:
// capacities of p.ws and p.counters; splitting is skipped when they are too small).
cudaError_t bf16_gemm_launch(const CUtensorMap& amap, const CUtensorMap& bmap, Bf16GemmParams p, int num_sms,
                             long long ws_floats, int n_counters, cudaStream_t s);

}  // namespace sq
