// comm.h — tensor-parallel collectives over NVLink peer memory (see comm.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace sq {

struct TpReduceParams {
  const __nv_bfloat16* recv;  // local receive buffer [2 parity][tp src][rows][ld]
  long long recv_stride;      // elements per parity
  long long src_stride;       // elements per source rank
  int ld;
  int* flags;                 // local flags [2 parity][tp src][tiles]
  int flag_stride, flag_src_stride;
  int expect;                 // arrivals per (source, tile): the GEMM's split count
  __nv_bfloat16* out;         // [M, ld_out]: out = residual (its old value) + sum
  int ld_out;
  int residual_in_out;
  int M, N, tile_m, tile_n, tp;
  int* seq;                   // device op counter (parity = seq & 1)
  int* done;                  // CTA completion counter, zero between ops
  int* status;
};

struct TpGatherParams {
  const __nv_bfloat16* src;      // this rank's rows [rows, ld_src]
  int ld_src;
  __nv_bfloat16* const* dst;     // [tp] every rank's output base
  int ld_dst;
  int row0, col0, rows, cols;
  int* const* flags;             // [tp] every rank's gather flags [2 parity][tp src]
  int* local_flags;
  int flag_stride;
  int expect;                    // pushing CTAs per source
  int rank, tp;
  int* seq;
  int* status;
};

// Push a [M, N] bf16 partial into every rank's receive slot for this source, tile by tile
// (tile_m x 128 columns, the tp_reduce numbering), bumping each tile's flag on every rank.
struct TpPushParams {
  const __nv_bfloat16* src;
  int ld_src;
  __nv_bfloat16* const* dst;  // [tp] receive slot of this source on every rank (parity 0)
  long long parity_stride;    // elements
  int ld_dst;
  int* const* flags;          // [tp] this source's flag row on every rank (parity 0)
  int flag_stride;
  int M, N, tile_m, tp;
  const int* seq;
};
// Sequence-parallel collectives (reduce-scatter -> RMSNorm -> all-gather), one kernel.
// Rank r owns token rows [r * rows_per_rank, min(T, (r + 1) * rows_per_rank)). The row-parallel
// GEMM pushed each source's bf16 partial of the owned rows into recv (the GEMM's reduce-scatter
// routing); this kernel (one CTA per owned row, rows_per_rank CTAs on every rank) waits for
// every source's CTAs, adds the partials in source order to the residual rows of h (written
// back), RMS-normalises them with w and stores the normalised rows into every rank's all-gather
// buffer (P2P stores), then counts one arrival per CTA on every rank's ag counter for this
// source. The last CTA clears this rank's reduce-scatter counters of
// the parity it used and advances seq (parity = seq & 1 for the next round).
struct TpRsNormParams {
  const __nv_bfloat16* recv;     // [tp source][rows_per_rank][ld_recv] on this rank
  long long src_stride;          // elements per source block
  int ld_recv;
  int* rs_flags;                 // this rank's counters [2 parity][tp source]
  int rs_expect;                 // CTAs of the pushing GEMM launch (the same on every rank)
  __nv_bfloat16* h;              // residual stream [T, ldh]
  int ldh;
  const __nv_bfloat16* w;        // RMSNorm weight [N]
  float eps;
  __nv_bfloat16* const* ag_dst;  // [tp] every rank's all-gather buffer [T, ld_ag]
  int ld_ag;
  int* const* ag_flags;          // [tp] every rank's all-gather counter for this source
  int rank, tp, rows_per_rank, T, N;
  int* seq;
  int* done;
  int* status;
  // local_only != 0: the normalised rows go to this rank's buffer only (ag_dst[rank]) and no
  // all-gather arrival is counted (the input of an expert-parallel dispatch, which sends each
  // row only to the ranks that hold its experts)
  int local_only;
};
constexpr int kRsNormMaxChunks = 4;  // one CTA per row: <= 4 chunks of 8 columns per thread (N <= 32768)
cudaError_t tp_rs_norm_ag_launch(const TpRsNormParams& p, cudaStream_t s);
// Wait (one CTA, bounded) until ag_flags[s] >= expect for every source, then clear them.
cudaError_t tp_ag_wait_launch(int* ag_flags, int expect, int tp, int* status, cudaStream_t s);
// One-shot all-reduce over peer memory, for small row-parallel outputs (decode): CTA b copies
// chunk b of this rank's partial `src` [M, ld_src] into its own double-buffered peer-visible
// slot part[rank][parity], publishes chunk b (flag value seq + 1 in every rank's slot
// [b][rank]), waits (bounded) for chunk b of every peer, then out[chunk b] = residual + the tp
// partials summed in rank order (bit-identical on every rank). The last CTA advances seq.
struct TpOneshotParams {
  const __nv_bfloat16* src;
  int ld_src;
  __nv_bfloat16* const* part;  // [tp] every rank's slot base (parity 0); parity 1 at + par_stride
  long long par_stride;        // elements
  int* const* flags;           // [tp] every rank's flag array [kOneshotMaxCtas][tp]
  __nv_bfloat16* out;
  int ld_out;
  int residual_in_out;         // out += sum (out holds the residual) instead of out = sum
  int M, N, rank, tp;
  int* seq;
  int* done;
  int* status;
};
constexpr int kOneshotMaxCtas = 148;
constexpr int kOneshotThreads = 256;
cudaError_t tp_oneshot_launch(const TpOneshotParams& p, cudaStream_t s);
// Expert-parallel all-to-all over peer memory (sequence-parallel layout: rank r owns token rows
// [r R, r R + own)). Every receiver holds, per source rank s, R row slots of x, and R x K slots
// of (local expert id or -1, routing weight).
//
// Dispatch: one CTA per owned row slot t (R CTAs on every rank). The row's K routed experts
// name the ranks that hold them (expert e lives on rank e / E_local); the row is stored once
// into each such rank's x slot [rank][t], and every rank gets the K (id, weight) pairs of the
// row with the ids that are not its own set to -1 (rows past `own` send -1 everywhere). Then one
// arrival per CTA on every rank's dispatch counter for this source (receivers wait for R).
// With router logits given, warp 0 of each CTA first routes its row (softmax, top-K, renorm:
// the MoE routing kernel's warp routine) and writes ids / w; otherwise ids / w are read.
struct EpDispatchParams {
  const __nv_bfloat16* x;        // [own, ldx] this rank's normalised rows
  int ldx;
  const __nv_bfloat16* logits;   // [own, ld_logits] router logits, or nullptr
  int ld_logits, E, renorm;
  int* ids;                      // [own, K] global expert ids (router output / input)
  float* w;                      // [own, K] routing weights
  __nv_bfloat16* const* recv_x;  // [tp] every rank's x slots base [tp src][R][H]
  int* const* recv_ids;          // [tp] every rank's id slots [tp src][R][K]
  float* const* recv_w;          // [tp] every rank's weight slots [tp src][R][K]
  int* const* flags;             // [tp] every rank's dispatch counter for this source
  int own, R, H, K, E_local, rank, tp;
};
// Combine: one CTA per received row slot (s, t) (tp x R CTAs): the weighted sum of the local
// experts' outputs for the row's slots (K in order, zeros when none of its experts is here)
// goes to the row owner's reduce-scatter receive block for this source, dst[s] + t * ld_dst,
// and one arrival on the owner's reduce-scatter counter [parity][this source] (the owner
// waits for R arrivals per source in tp_rs_norm_ag, which adds the tp partial rows to the
// residual, normalises and all-gathers as after a row-parallel GEMM).
struct EpCombineParams {
  const __nv_bfloat16* ys;       // [P, ldys] local experts' outputs in sorted slot order
  int ldys;
  const int* slot_pos;           // [tp R K] position of each received slot in ys (-1: not here)
  const float* w;                // [tp R K] received routing weights
  __nv_bfloat16* const* dst;     // [tp] owner's receive block for this source
  int ld_dst;
  int* const* flags;             // [tp] owner's counter row for this source (parity 0)
  int flag_stride;               // elements between parities
  const int* seq;                // parity = seq & 1
  int R, H, K, tp, T;
};
cudaError_t ep_dispatch_launch(const EpDispatchParams& p, cudaStream_t s);
cudaError_t ep_combine_launch(const EpCombineParams& p, cudaStream_t s);
cudaError_t tp_push_launch(const TpPushParams& p, int grid_x, int grid_y, cudaStream_t s);
cudaError_t tp_reduce_launch(const TpReduceParams& p, int grid_x, int grid_y, cudaStream_t s);
cudaError_t tp_gather_launch(const TpGatherParams& p, cudaStream_t s);

}  // namespace sq
