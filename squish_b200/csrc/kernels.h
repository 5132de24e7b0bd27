// kernels.h — launch interfaces of the non-GEMM CUDA kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace sq {

struct RopeKvParams {
  const __nv_bfloat16* qkv;  // [T, ld_qkv]: Hq*D q | Hkv*D k | Hkv*D v
  int ld_qkv;
  const int* positions;      // [T]
  const float* cos_sin;      // [max_pos, D]: cos(D/2) | sin(D/2)
  __nv_bfloat16* q_out;      // [T, Hq, D]
  const int* slot_mapping;   // [T] page*page_size + offset, -1 = do not store
  uint8_t* k_codes;
  __half* k_scales;
  uint8_t* v_codes;
  __half* v_scales;
  int Hq, Hkv, D, page_size, group, fmt_k, fmt_v;
  const __nv_bfloat16* q_norm;  // [D] per-head RMSNorm weight applied before RoPE (Qwen3), or nullptr
  const __nv_bfloat16* k_norm;
  float norm_eps;
  int num_pages;  // pages in the pools: a slot at or past num_pages * page_size is not written and
  int* status;    // records SQ_ERR_BOUNDS here (num_pages 0 or status nullptr: unchecked)
  // Hadamard-rotated KV (nullptr: off): q and k are stored as H (had_k * x) / sqrt(D), v as
  // had_v * (H v) / sqrt(D), with H the Sylvester Hadamard matrix and had_* +-1 signs [D]. Scores
  // are unchanged (an orthogonal map on both sides); the attention output comes out rotated and
  // is mapped back with H (had_v * o) / sqrt(D) (hadamard_rows) before o_proj.
  const float* had_k;
  const float* had_v;
};

// Attention mass per KV page (kv_score.cu): for every decode row b, the softmax probabilities of
// its query heads over the row's keys (block table row b, seq_lens[b] keys) summed per page and
// added to mass[page].
struct PageMassParams {
  const __nv_bfloat16* q;  // [B, ld_q] (Hq * D per row)
  int ld_q;
  const uint8_t* k_codes;
  const __half* k_scales;
  const int* block_tables;  // [B, bt_stride]
  int bt_stride;
  const int* seq_lens;      // [B]
  float* mass;              // [num_pages], accumulated
  int B, Hq, Hkv, D, page_size, group, fmt_k, num_pages;
  float sm_scale;
  int* status;
};
cudaError_t page_mass_launch(const PageMassParams& p, cudaStream_t s);

struct AttnParams {
  const __nv_bfloat16* q;  // [rows, ld_q] (Hq*D per row)
  int ld_q;
  const uint8_t* k_codes;
  const __half* k_scales;
  const uint8_t* v_codes;
  const __half* v_scales;
  const int* block_tables;  // [B, bt_stride]
  int bt_stride;
  __nv_bfloat16* out;       // [rows, ld_out]
  int ld_out;
  int Hq, Hkv, D, page_size, group, fmt_k, fmt_v;
  float sm_scale;
  // decode: one query row per sequence b (row b of q/out)
  const int* seq_lens;      // [B] kv length including the current token
  int B;
  int splits, tiles_per_split;
  float* o_part;            // [B, Hq, splits, D]
  float* lse_part;          // [B, Hq, splits]
  // prefill (varlen, causal over the paged context)
  const int* tile_seq;      // [n_tiles] sequence index of the work tile
  const int* tile_q0;       // [n_tiles] first query (within the chunk) of the tile
  const int* q_start;       // [B] first row of the sequence's chunk in q/out
  const int* q_len;         // [B]
  const int* ctx_len;       // [B] kv length after this chunk
  int n_tiles;
  // optional token-tree masks (speculative verification), one per query row: bit j set =
  // the row may attend chunk token j; 0 = plain causal. A tree chunk is at most 32 tokens.
  const int* tree_mask;
  // page-index check: a block-table entry outside [0, num_pages) is read as an empty page and
  // records SQ_ERR_BOUNDS in *status (num_pages 0 or status nullptr: unchecked)
  int num_pages;
  int* status;
};

cudaError_t rope_kv_write_launch(const RopeKvParams& p, int T, cudaStream_t s);
cudaError_t rmsnorm_launch(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, const int* row_idx,
                           int rows, int H, int ldx, int ldy, float eps, cudaStream_t s);
cudaError_t paged_decode_attn_launch(const AttnParams& p, cudaStream_t s);
cudaError_t paged_prefill_attn_launch(const AttnParams& p, cudaStream_t s);
// tcgen05 prefill attention (head dim 128, 3..16 query heads per KV head, no token-tree
// masks, quantized KV): q is read through a 3-D tensor map {D, Hq, rows} with box
// {64, head slots, 128 / head slots} and 128-byte swizzle.
bool prefill_tc_supported(const AttnParams& p);
int prefill_tc_head_slots(int gq);
cudaError_t paged_prefill_attn_tc_launch(const CUtensorMap& qmap, const AttnParams& p, int* status,
                                         unsigned long long* trace, cudaStream_t s);

struct SamplerParams {
  const __nv_bfloat16* logits;  // [B, ld]
  int ld, V, B;
  const float* temperature;     // [B] (<= 0 -> greedy)
  const float* top_p;           // [B] (>= 1 -> off)
  const int* top_k;             // [B] (<= 0 -> off)
  const float* min_p;           // [B] (<= 0 -> off)
  const float* rep_penalty;     // [B] (== 1 -> off)
  const int* hist;              // [B, hist_stride] recent token ids for the repetition penalty, -1 padded
  int hist_stride;
  const uint32_t* allow_mask;   // [B, ceil(V/32)] grammar bitmask (bit set = allowed) or nullptr
  uint64_t seed;
  const int* step;              // [B] per-row counter mixed into the RNG stream
  int* out_tokens;              // [B]
  float* out_logprob;           // [B] log-probability of the chosen token (after processing) or nullptr
};
cudaError_t sampler_launch(const SamplerParams& p, float* work, cudaStream_t s);

// codec 0 INT8 sym, 1 INT4 sym, 2 NF4, 3 INT3 (group % 8 == 0), 4 INT2 asym (offsets used)
cudaError_t quantize_codec_launch(const void* x, bool bf16, int codec, uint8_t* codes, int code_ld, float* scales,
                                  float* offsets, int rows, int cols, int group, float fixed_scale, cudaStream_t s);
// HQQ refinement (one warp per group, group <= 512): codes [rows, cols] uint8 in [0, levels-1],
// scales / zeros [rows, cols / group]; x = zero + code * scale.
cudaError_t hqq_launch(const void* x, bool bf16, uint8_t* codes, float* scales, float* zeros, int rows, int cols,
                       int group, int levels, float lam, int iters, cudaStream_t s);
// acc[c] += mean_r |x[r, c]| (AWQ calibration statistics), double accumulator.
cudaError_t channel_abs_mean_launch(const void* x, bool bf16, double* acc, int rows, int cols, cudaStream_t s);
cudaError_t quantize_int4_asym_launch(const void* x, bool bf16, uint8_t* packed, float* scales, float* offsets,
                                      int rows, int cols, int group, int n_clip, cudaStream_t s);

// ---------------------------------------------------------------- speculative decoding
constexpr int kMaxTreeNodes = 32;
constexpr int kTreeMetaInts = 2 + 3 * kMaxTreeNodes;  // row0, n, parent[], token[], qrow[]
struct TreeVerifyParams {
  const __nv_bfloat16* logits;        // [rows, ld] target logits, node i of group g at row meta.row0 + i
  int ld, V;
  const __nv_bfloat16* draft_logits;  // [rows_q, ld_draft] or nullptr (deterministic drafts only)
  int ld_draft;
  const int* meta;                    // [G, kTreeMetaInts]
  const float* temperature;           // [G]
  const int* step;                    // [G]
  unsigned long long seed;
  float* scratch;                     // [G, V] residual distribution
  int* out;                           // [G, 2 + kMaxTreeNodes]: n_accepted, final token, accepted nodes
};
struct KvLayerPtrs {
  uint8_t* kc;
  __half* ks;
  uint8_t* vc;
  __half* vs;
};
struct KvCompactParams {
  const KvLayerPtrs* layers;  // [L] device array
  const int* src;             // [n] absolute cache slots (page * page_size + offset)
  const int* dst;
  int n_pairs;
  int Hkv, page_size;
  int kc_bytes, vc_bytes, ks_n, vs_n;  // per (token, head) row
};
cudaError_t tree_verify_launch(const TreeVerifyParams& p, int groups, cudaStream_t s);
cudaError_t kv_compact_launch(const KvCompactParams& p, int layers, cudaStream_t s);

cudaError_t moe_route_launch(const __nv_bfloat16* logits, int ld, int T, int E, int K, bool renorm, int* topk_ids,
                             float* topk_w, cudaStream_t s);
// wait_flags != nullptr: first wait (bounded, then clear) until wait_flags[s] >= wait_expect for
// s < wait_n -- the expert-parallel receiver's dispatch arrivals -- recording a timeout in status
cudaError_t moe_align_launch(const int* ids, int TK, int E, int bn, int max_tiles, int* sorted_slot, int* slot_pos,
                             int* tile_expert, int* num_tiles, int* counts, cudaStream_t s,
                             int* wait_flags = nullptr, int wait_n = 0, int wait_expect = 0, int* status = nullptr);
cudaError_t moe_gather_launch(const __nv_bfloat16* x, int ldx, const int* sorted_slot, const int* num_tiles,
                              int max_rows, int bn, int K, int H, __nv_bfloat16* xs, int ldxs, cudaStream_t s);
cudaError_t moe_combine_launch(const __nv_bfloat16* ys, int ldys, const int* slot_pos, const float* topk_w, int T,
                               int K, int H, __nv_bfloat16* h, int ldh, cudaStream_t s);

// k-means / product quantization (kmeans.cu); d in {1, 2, 4, 8, 16, 32, 64}
cudaError_t kmeans_assign_launch(const float* x, int n, int d, const float* c, int k, int* assign, float* dist,
                                 int* changed, cudaStream_t s);
cudaError_t kmeans_update_launch(const float* x, int n, int d, const int* assign, float* c, int k, float* sums,
                                 int* counts, cudaStream_t s);
cudaError_t pq_adc_launch(const uint8_t* codes, int n, int m, const float* lut, int k, float* out, cudaStream_t s);

// randomized block Walsh-Hadamard rotation of rows (hadamard.cu): y = blockdiag(H_b / sqrt(b)) (s * x)
cudaError_t hadamard_rows_launch(const __nv_bfloat16* x, int ldx, __nv_bfloat16* y, int ldy, const float* signs,
                                 int M, int K, int b, cudaStream_t s);

}  // namespace sq
