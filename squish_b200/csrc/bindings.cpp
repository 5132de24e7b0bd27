// bindings.cpp — Python bindings of the CUDA kernels and the C++ CPU reference library.
//
// Every CUDA entry point launches on the current torch stream, allocates nothing, and
// takes its workspaces from the caller, so the calls can be captured in CUDA graphs.
// Tensors are checked for device, dtype and contiguity; a failed launch raises.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include "kernels.h"
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "w4a16_gemm.h"
#include "bf16_gemm.h"
#include "comm.h"
#include "cpu_ref.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_DT(x, dt) TORCH_CHECK((x).scalar_type() == (dt), #x " has wrong dtype")
#define CUDA_OK(expr)                                                                       \
  do {                                                                                      \
    cudaError_t _e = (expr);                                                                \
    TORCH_CHECK(_e == cudaSuccess, std::string("squish_b200 kernel launch failed: ") + cudaGetErrorString(_e)); \
  } while (0)

template <typename T>
T* ptr(const torch::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
template <typename T>
T* optr(const c10::optional<torch::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    CUDA_OK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 row-major [rows, cols] (row stride ld elements), box [box_rows, 64], 128B swizzle.
CUtensorMap make_bf16_map(const void* base, int rows, int cols, int ld, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, std::string("cuTensorMapEncodeTiled failed (") + std::to_string((int)r) + ")");
  return m;
}

// Activation map of the INT4 GEMM. With xg > 1 k-blocks per load (K a multiple of 64): a 3-D
// view {64 columns, rows, k-block} (k-block stride 128 B) whose box {64, box_rows, xg} lands as
// xg consecutive [box_rows x 128 B] swizzled tiles, the layout of xg single-k-block loads.
CUtensorMap make_x_map(const torch::Tensor& x, int rows, int cols, int box_rows, int xg) {
  const int ld = (int)x.stride(0);
  if (xg <= 1 || cols % 64 != 0) return make_bf16_map(x.data_ptr(), rows, cols, ld, box_rows);
  CUtensorMap m;
  cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 2, 128};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)xg};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, x.data_ptr(), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, std::string("cuTensorMapEncodeTiled (3-D) failed (") + std::to_string((int)r) + ")");
  return m;
}

// k-blocks per activation load of the INT4 GEMM (SQ_GEMM_XG overrides; 1 when K is not a
// multiple of 64)
int gemm_xg(int64_t K, const sq::W4A16Params& p, int bn) {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("SQ_GEMM_XG");
    v = e != nullptr ? std::max(1, std::min(4, std::atoi(e))) : 2;
  }
  if (K % 64 != 0 || p.tile_expert != nullptr || !sq::w4a16_decode_grouping(bn, p.wfmt, p.gpk)) return 1;
  return std::max(1, std::min(v, p.kb_per_split));
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// ------------------------------------------------------------------ INT4 GEMM
std::vector<torch::Tensor> repack_int4(torch::Tensor packed, torch::Tensor scales, torch::Tensor zeros, int64_t K,
                                       int64_t group) {
  CHECK_CUDA(packed);
  CHECK_CONTIG(packed);
  CHECK_CONTIG(scales);
  CHECK_CONTIG(zeros);
  CHECK_DT(packed, torch::kUInt8);
  CHECK_DT(scales, torch::kFloat32);
  CHECK_DT(zeros, torch::kFloat32);
  TORCH_CHECK(group == 16 || group == 32 || group % 64 == 0, "INT4 group size must be 16, 32 or a multiple of 64");
  TORCH_CHECK(K % 2 == 0 && packed.size(1) * 2 == K, "packed width must be K/2");
  const c10::cuda::CUDAGuard g(packed.device());
  const int64_t N = packed.size(0);
  const int64_t kb = (K + 63) / 64;
  const int64_t npad = (N + 255) / 256 * 256;
  const int64_t gpk = group >= 64 ? 1 : 64 / group;
  auto opts = packed.options().dtype(torch::kInt32);
  torch::Tensor wt = torch::empty({npad / 128, kb, 1024 + gpk * 128}, opts);
  CUDA_OK(sq::repack_int4_launch(ptr<uint8_t>(packed), ptr<float>(scales), ptr<float>(zeros), ptr<uint32_t>(wt),
                                 (int)N, (int)K, (int)group, cur_stream()));
  return {wt, torch::empty({0}, opts)};
}

// Tile choice shared by the GEMM launch and the workspace sizing in Python.
std::vector<int64_t> gemm_plan(int64_t M, int64_t N, int64_t K, int64_t group = 64, int64_t wfmt = 0) {
  int bn, nt = 1;
  if (M <= 16) bn = 16;
  else if (M <= 32) bn = 32;
  else if (M <= 64) bn = 64;
  else if (M <= 128) bn = 128;
  else if (K <= 8192) {
    // 128-token tiles keep the A operand in tensor memory and run two CTAs per SM
    // (measured 8-13% faster than 256 x 2-tile CTAs for K <= 8192)
    bn = 128;
  } else {
    bn = 256;
    nt = (N % 256 == 0 && N >= 2048) ? 2 : 1;
  }
  // tuning override for experiments: SQ_GEMM_PLAN="bn,nt" fixes the tile for M > 128
  static int ov_bn = -1, ov_nt = -1;
  static bool ov_read = false;
  if (!ov_read) {
    ov_read = true;
    if (const char* e = std::getenv("SQ_GEMM_PLAN")) {
      if (std::sscanf(e, "%d,%d", &ov_bn, &ov_nt) != 2) ov_bn = -1;
    }
  }
  if (M > 128 && ov_bn > 0) {
    bn = ov_bn;
    nt = ov_nt;
  }
  const int64_t kb = (K + 63) / 64;
  const int64_t sms = num_sms();
  auto tiles_of = [&](int b, int t) { return ((N + 128 * t - 1) / (128 * t)) * ((M + b - 1) / b); };
  int64_t tiles = tiles_of(bn, nt);
  if (tiles * 2 <= sms && bn == 256) {  // too few tiles: smaller token tiles before splitting K
    bn = 128;
    nt = 1;
    tiles = tiles_of(bn, nt);
  }
  int64_t splits = 1;
  // decode shapes run two CTAs per SM, four with the 4-dequant-warp configuration
  const bool narrow = bn <= 64 && sq::w4a16_narrow((int)wfmt, group >= 64 ? 1 : (int)(64 / group));
  const int64_t slots = (bn <= 64) ? (narrow ? 4 : 2) * sms : sms;
  if (tiles * 2 < slots) {
    // split-K over a thread-block cluster: up to 8 CTAs (portable size), 16 for the narrow
    // configuration; at least 7 (narrow) / 4 k-blocks per split (measured on B200: qkv / o_proj
    // of a 7B model are fastest at 8 splits, down (K = 18944) at 16)
    const int64_t max_s = narrow ? 16 : 8, min_kps = narrow ? 7 : 4;
    splits = std::min<int64_t>({slots / tiles, std::max<int64_t>(1, kb / min_kps), max_s});
    splits = std::max<int64_t>(splits, 1);
  }
  static int ov_splits = -1;
  static bool ov_s_read = false;
  if (!ov_s_read) {  // tuning override for experiments: SQ_GEMM_SPLITS=n (1..16) for every NT=1 plan
    ov_s_read = true;
    if (const char* e = std::getenv("SQ_GEMM_SPLITS")) ov_splits = std::atoi(e);
  }
  if (ov_splits > 0 && nt == 1) splits = std::min<int64_t>({ov_splits, 16, kb});
  int64_t kps = (kb + splits - 1) / splits;
  splits = (kb + kps - 1) / kps;
  return {bn, nt, splits, kps, tiles};
}

// NF4-format weights may carry a learned 16-level table (any4) in place of the NormalFloat levels
static void check_level_table(int64_t wfmt, const c10::optional<torch::Tensor>& codebook) {
  if (wfmt == sq::WF_NF4 && codebook.has_value())
    TORCH_CHECK(codebook->scalar_type() == torch::kBFloat16 && codebook->is_cuda() && codebook->is_contiguous() &&
                    codebook->numel() == 16,
                "a 4-bit level table is 16 contiguous bf16 values on the device");
}

void w4a16_gemm(torch::Tensor x, torch::Tensor wq, torch::Tensor sz, int64_t N, int64_t K, int64_t group,
                torch::Tensor y, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> residual,
                int64_t epilogue, torch::Tensor ws, torch::Tensor counters, torch::Tensor status,
                c10::optional<torch::Tensor> trace, int64_t wfmt, c10::optional<torch::Tensor> codebook,
                c10::optional<torch::Tensor> ag_flags = c10::nullopt, c10::optional<torch::Tensor> ag_done = c10::nullopt,
                int64_t ag_expect = 0, int64_t ag_tp = 0) {
  TORCH_CHECK(wfmt >= 0 && wfmt <= 6, "unknown weight format");
  if (wfmt == sq::WF_AQLM) {
    TORCH_CHECK(codebook.has_value() && codebook->scalar_type() == torch::kBFloat16 && codebook->is_cuda() &&
                    codebook->is_contiguous() && codebook->numel() % (256 * 8) == 0 && codebook->numel() <= 2 * 256 * 8,
                "AQLM needs 1 or 2 contiguous bf16 codebooks of 256 x 8 on the device");
  }
  check_level_table(wfmt, codebook);
  CHECK_CUDA(x);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(y, torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be [M, K] with unit column stride");
  TORCH_CHECK(x.size(1) == K, "x.size(1) != K");
  TORCH_CHECK(y.stride(1) == 1, "y must have unit column stride");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) == 0,
              "x rows must be 16-byte aligned");
  const int64_t M = x.size(0);
  if (M == 0) return;
  const c10::cuda::CUDAGuard g(x.device());
  auto plan = gemm_plan(M, N, K, group, wfmt);
  const int bn = (int)plan[0], nt = (int)plan[1];
  sq::W4A16Params p{};
  p.wq = ptr<uint32_t>(wq);
  p.sz = ptr<uint32_t>(sz);
  p.bias = optr<__nv_bfloat16>(bias);
  p.residual = optr<__nv_bfloat16>(residual);
  p.y = ptr<__nv_bfloat16>(y);
  p.ws = ptr<float>(ws);
  p.counters = ptr<int>(counters);
  p.status = ptr<int>(status);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldy = (int)y.stride(0);
  p.ldr = residual.has_value() ? (int)residual->stride(0) : 0;
  p.kb_total = (int)((K + 63) / 64);
  p.splits = (int)plan[2];
  p.kb_per_split = (int)plan[3];
  p.gpk = group >= 64 ? 1 : (int)(64 / group);
  p.epilogue = (int)epilogue;
  p.wfmt = (int)wfmt;
  p.codebook = optr<__nv_bfloat16>(codebook);
  p.n_books = codebook.has_value() ? (int)(codebook->numel() / (256 * 8)) : 0;
  p.trace = optr<unsigned long long>(trace);
  if (ag_flags.has_value()) {  // all-gathered X: the activation producer waits for every source
    TORCH_CHECK(ag_done.has_value() && ag_tp > 0 && ag_tp <= 32 && ag_flags->numel() >= ag_tp,
                "all-gather wait needs ag_done, ag_expect and 1..32 sources");
    p.ag_flags = ptr<int>(*ag_flags);
    p.ag_done = ptr<int>(*ag_done);
    p.ag_expect = (int)ag_expect;
    p.tp = (int)ag_tp;
  }
  p.xg = gemm_xg(K, p, bn);
  const CUtensorMap xmap = make_x_map(x, (int)M, (int)K, bn, p.xg);
  CUDA_OK(sq::w4a16_gemm_launch(xmap, p, bn, nt, cur_stream()));
}

// Expand tile-major weight codes to bf16 out[N, ld] (columns >= K hold the padding codes).
void dequant_weight(torch::Tensor wq, int64_t N, int64_t K, int64_t group, int64_t wfmt,
                    c10::optional<torch::Tensor> codebook, torch::Tensor out) {
  CHECK_CUDA(wq);
  CHECK_CUDA(out);
  CHECK_DT(out, torch::kBFloat16);
  TORCH_CHECK(wfmt >= 0 && wfmt <= 6, "unknown weight format");
  const int64_t kpad = (K + 63) / 64 * 64;
  TORCH_CHECK(out.dim() == 2 && out.size(0) >= N && out.stride(1) == 1 && out.stride(0) >= kpad &&
                  out.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
              "out must be [>= N, >= 64 * ceil(K / 64)] bf16 with 16-byte aligned rows");
  if (wfmt == sq::WF_AQLM) TORCH_CHECK(codebook.has_value(), "AQLM weights need their codebooks");
  check_level_table(wfmt, codebook);
  const c10::cuda::CUDAGuard g(wq.device());
  CUDA_OK(sq::dequant_weight_launch(ptr<uint32_t>(wq), (int)wfmt, (int)N, (int)K, (int)group, (int)out.stride(0),
                                    ptr<__nv_bfloat16>(out), optr<__nv_bfloat16>(codebook),
                                    codebook.has_value() ? (int)(codebook->numel() / (256 * 8)) : 0, num_sms(),
                                    cur_stream()));
}

static bool al16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

// y = x . w^T (+ bias) (+ residual), bf16 operands, persistent tcgen05 kernel. w: [N, K] with
// unit column stride (row stride a multiple of 8 elements). With epilogue EPI_SILU_MUL the rows
// of w are [gate 64 | up 64] blocks and y = silu(gate) * up has N / 2 columns.
void bf16_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor y, c10::optional<torch::Tensor> bias,
               c10::optional<torch::Tensor> residual, int64_t epilogue, torch::Tensor ws, torch::Tensor counters,
               torch::Tensor status) {
  CHECK_CUDA(x);
  CHECK_CUDA(w);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(w, torch::kBFloat16);
  CHECK_DT(y, torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "x [M, K], w [N, K]");
  TORCH_CHECK(x.stride(1) == 1 && w.stride(1) == 1 && y.stride(1) == 1, "unit column strides");
  TORCH_CHECK(x.stride(0) % 8 == 0 && w.stride(0) % 8 == 0 && al16(x.data_ptr()) && al16(w.data_ptr()),
              "x / w rows must be 16-byte aligned");
  const int64_t M = x.size(0), N = w.size(0), K = x.size(1);
  const bool silu = epilogue == sq::EPI_SILU_MUL;
  TORCH_CHECK(y.size(0) >= M && y.size(1) >= (silu ? N / 2 : N), "y too small");
  TORCH_CHECK(!silu || (N % 128 == 0 && !bias.has_value() && !residual.has_value()),
              "SwiGLU epilogue: N a multiple of 128, no bias / residual");
  if (M == 0) return;
  const c10::cuda::CUDAGuard g(x.device());
  sq::Bf16GemmParams p{};
  p.bias = optr<__nv_bfloat16>(bias);
  p.residual = optr<__nv_bfloat16>(residual);
  p.y = ptr<__nv_bfloat16>(y);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldy = (int)y.stride(0);
  p.ldr = residual.has_value() ? (int)residual->stride(0) : 0;
  p.epilogue = (int)epilogue;
  p.vec = al16(p.y) && p.ldy % 8 == 0 && (!p.bias || al16(p.bias)) &&
          (!p.residual || (al16(p.residual) && p.ldr % 8 == 0 && residual->stride(1) == 1));
  p.status = ptr<int>(status);
  CHECK_DT(ws, torch::kFloat32);
  CHECK_DT(counters, torch::kInt32);
  p.ws = ptr<float>(ws);
  p.counters = ptr<int>(counters);
  const CUtensorMap amap = make_bf16_map(x.data_ptr(), (int)M, (int)K, (int)x.stride(0), 128);
  const CUtensorMap bmap = make_bf16_map(w.data_ptr(), (int)N, (int)K, (int)w.stride(0), 256);
  CUDA_OK(sq::bf16_gemm_launch(amap, bmap, p, num_sms(), (long long)ws.numel(), (int)counters.numel(),
                               cur_stream()));
}

// Grouped (mixture-of-experts) INT4 GEMM over expert-sorted, tile-padded rows of x.
void w4a16_grouped_gemm(torch::Tensor x, torch::Tensor wq, int64_t N, int64_t K, int64_t group, torch::Tensor y,
                        int64_t epilogue, torch::Tensor tile_expert, torch::Tensor num_tiles, int64_t bn,
                        torch::Tensor ws, torch::Tensor counters, torch::Tensor status) {
  CHECK_CUDA(x);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(y, torch::kBFloat16);
  CHECK_DT(tile_expert, torch::kInt32);
  CHECK_DT(num_tiles, torch::kInt32);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(1) == K, "x must be [rows, K]");
  TORCH_CHECK(wq.dim() == 2, "wq must be [experts, words per expert]");
  TORCH_CHECK(bn == 16 || bn == 32 || bn == 64 || bn == 128, "bn must be 16/32/64/128");
  const int64_t M = x.size(0);
  TORCH_CHECK(M % bn == 0 && tile_expert.numel() >= M / bn, "rows must be a multiple of bn, one expert per tile");
  TORCH_CHECK((x.stride(0) * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) == 0,
              "x rows must be 16-byte aligned");
  if (M == 0) return;
  const c10::cuda::CUDAGuard g(x.device());
  sq::W4A16Params p{};
  p.wq = ptr<uint32_t>(wq);
  p.sz = p.wq;
  p.y = ptr<__nv_bfloat16>(y);
  p.ws = ptr<float>(ws);
  p.counters = ptr<int>(counters);
  p.status = ptr<int>(status);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldy = (int)y.stride(0);
  p.kb_total = (int)((K + 63) / 64);
  p.splits = 1;
  p.kb_per_split = p.kb_total;
  p.gpk = group >= 64 ? 1 : (int)(64 / group);
  p.epilogue = (int)epilogue;
  p.tile_expert = ptr<int>(tile_expert);
  p.num_tiles = ptr<int>(num_tiles);
  p.expert_stride = (long long)wq.stride(0) * wq.element_size();
  TORCH_CHECK(p.expert_stride % 16 == 0, "expert stride must be 16-byte aligned");
  p.xg = gemm_xg(K, p, (int)bn);
  const CUtensorMap xmap = make_x_map(x, (int)M, (int)K, (int)bn, p.xg);
  CUDA_OK(sq::w4a16_gemm_launch(xmap, p, (int)bn, 1, cur_stream()));
}

void moe_route(torch::Tensor logits, int64_t K, bool renorm, torch::Tensor topk_ids, torch::Tensor topk_w) {
  CHECK_CUDA(logits);
  CHECK_DT(logits, torch::kBFloat16);
  CHECK_DT(topk_ids, torch::kInt32);
  CHECK_DT(topk_w, torch::kFloat32);
  TORCH_CHECK(logits.stride(1) == 1, "logits must have unit column stride");
  const c10::cuda::CUDAGuard g(logits.device());
  CUDA_OK(sq::moe_route_launch(ptr<__nv_bfloat16>(logits), (int)logits.stride(0), (int)logits.size(0),
                               (int)logits.size(1), (int)K, renorm, ptr<int>(topk_ids), ptr<float>(topk_w),
                               cur_stream()));
}

void moe_align(torch::Tensor ids, int64_t E, int64_t bn, torch::Tensor sorted_slot, torch::Tensor slot_pos,
               torch::Tensor tile_expert, torch::Tensor num_tiles, c10::optional<torch::Tensor> counts,
               c10::optional<torch::Tensor> wait_flags, int64_t wait_expect, c10::optional<torch::Tensor> status) {
  CHECK_CUDA(ids);
  CHECK_DT(ids, torch::kInt32);
  CHECK_CONTIG(ids);
  const int64_t TK = ids.numel();
  TORCH_CHECK(sorted_slot.numel() >= TK + E * (bn - 1), "sorted_slot too small for the padded layout");
  TORCH_CHECK(tile_expert.numel() * bn >= sorted_slot.numel(), "tile_expert too small");
  const c10::cuda::CUDAGuard g(ids.device());
  TORCH_CHECK(!wait_flags || (status && wait_flags->is_cuda() && wait_flags->scalar_type() == torch::kInt32),
              "wait_flags needs an int32 device tensor and a status word");
  CUDA_OK(sq::moe_align_launch(ptr<int>(ids), (int)TK, (int)E, (int)bn, (int)tile_expert.numel(),
                               ptr<int>(sorted_slot), ptr<int>(slot_pos), ptr<int>(tile_expert), ptr<int>(num_tiles),
                               optr<int>(counts), cur_stream(), optr<int>(wait_flags),
                               wait_flags ? (int)wait_flags->numel() : 0, (int)wait_expect, optr<int>(status)));
}

void moe_gather(torch::Tensor x, torch::Tensor sorted_slot, torch::Tensor num_tiles, int64_t bn, int64_t K,
                torch::Tensor xs) {
  CHECK_CUDA(x);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(xs, torch::kBFloat16);
  TORCH_CHECK(x.stride(1) == 1 && xs.stride(1) == 1 && x.size(1) == xs.size(1), "bad gather shapes");
  const c10::cuda::CUDAGuard g(x.device());
  CUDA_OK(sq::moe_gather_launch(ptr<__nv_bfloat16>(x), (int)x.stride(0), ptr<int>(sorted_slot), ptr<int>(num_tiles),
                                (int)std::min<int64_t>(xs.size(0), sorted_slot.numel()), (int)bn, (int)K,
                                (int)x.size(1), ptr<__nv_bfloat16>(xs), (int)xs.stride(0), cur_stream()));
}

void moe_combine(torch::Tensor ys, torch::Tensor slot_pos, torch::Tensor topk_w, int64_t K, torch::Tensor h) {
  CHECK_CUDA(ys);
  CHECK_DT(ys, torch::kBFloat16);
  CHECK_DT(h, torch::kBFloat16);
  TORCH_CHECK(ys.stride(1) == 1 && h.stride(1) == 1 && ys.size(1) == h.size(1), "bad combine shapes");
  const c10::cuda::CUDAGuard g(h.device());
  CUDA_OK(sq::moe_combine_launch(ptr<__nv_bfloat16>(ys), (int)ys.stride(0), ptr<int>(slot_pos), ptr<float>(topk_w),
                                 (int)h.size(0), (int)K, (int)h.size(1), ptr<__nv_bfloat16>(h), (int)h.stride(0),
                                 cur_stream()));
}

// ------------------------------------------------------------------ speculative decoding
void tree_verify(torch::Tensor logits, c10::optional<torch::Tensor> draft_logits, torch::Tensor meta,
                 torch::Tensor temperature, torch::Tensor step, int64_t seed, torch::Tensor scratch, torch::Tensor out) {
  CHECK_CUDA(logits);
  CHECK_DT(logits, torch::kBFloat16);
  CHECK_DT(meta, torch::kInt32);
  CHECK_DT(out, torch::kInt32);
  CHECK_DT(scratch, torch::kFloat32);
  TORCH_CHECK(logits.stride(1) == 1, "logits must have unit column stride");
  const int64_t G = meta.size(0);
  TORCH_CHECK(meta.size(1) == sq::kTreeMetaInts && out.size(1) == 2 + sq::kMaxTreeNodes, "bad tree meta/out shape");
  TORCH_CHECK(scratch.numel() >= G * logits.size(1), "scratch too small");
  const c10::cuda::CUDAGuard g(logits.device());
  sq::TreeVerifyParams p{};
  p.logits = ptr<__nv_bfloat16>(logits);
  p.ld = (int)logits.stride(0);
  p.V = (int)logits.size(1);
  if (draft_logits.has_value() && draft_logits->defined()) {
    CHECK_DT((*draft_logits), torch::kBFloat16);
    TORCH_CHECK(draft_logits->size(1) == logits.size(1), "draft vocabulary differs from the target's");
    p.draft_logits = ptr<__nv_bfloat16>(*draft_logits);
    p.ld_draft = (int)draft_logits->stride(0);
  }
  p.meta = ptr<int>(meta);
  p.temperature = ptr<float>(temperature);
  p.step = ptr<int>(step);
  p.seed = (unsigned long long)seed;
  p.scratch = ptr<float>(scratch);
  p.out = ptr<int>(out);
  CUDA_OK(sq::tree_verify_launch(p, (int)G, cur_stream()));
}

void kv_compact(torch::Tensor layer_ptrs, torch::Tensor src, torch::Tensor dst, int64_t Hkv, int64_t page_size,
                int64_t kc_bytes, int64_t vc_bytes, int64_t ks_n, int64_t vs_n) {
  CHECK_CUDA(layer_ptrs);
  TORCH_CHECK(layer_ptrs.scalar_type() == torch::kInt64 && layer_ptrs.size(1) == 4, "layer_ptrs must be [L, 4] int64");
  const c10::cuda::CUDAGuard g(layer_ptrs.device());
  sq::KvCompactParams p{};
  p.layers = reinterpret_cast<const sq::KvLayerPtrs*>(layer_ptrs.data_ptr());
  p.src = ptr<int>(src);
  p.dst = ptr<int>(dst);
  p.n_pairs = (int)src.numel();
  p.Hkv = (int)Hkv;
  p.page_size = (int)page_size;
  p.kc_bytes = (int)kc_bytes;
  p.vc_bytes = (int)vc_bytes;
  p.ks_n = (int)ks_n;
  p.vs_n = (int)vs_n;
  CUDA_OK(sq::kv_compact_launch(p, (int)layer_ptrs.size(0), cur_stream()));
}

// ------------------------------------------------------------------ tensor parallel (NVLink peer memory)
// Device memory shared across processes with CUDA IPC: one cudaMalloc per buffer, its
// handle exchanged through torch.distributed, opened by every peer.
std::vector<torch::Tensor> ipc_alloc(int64_t bytes) {
  void* p = nullptr;
  CUDA_OK(cudaMalloc(&p, (size_t)bytes));
  CUDA_OK(cudaMemset(p, 0, (size_t)bytes));
  cudaIpcMemHandle_t h;
  CUDA_OK(cudaIpcGetMemHandle(&h, p));
  auto ht = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  std::memcpy(ht.data_ptr(), &h, sizeof(h));
  auto pt = torch::tensor({(int64_t)reinterpret_cast<uintptr_t>(p)}, torch::kInt64);
  return {pt, ht};
}

int64_t ipc_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "bad IPC handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* p = nullptr;
  CUDA_OK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)reinterpret_cast<uintptr_t>(p);
}

void ipc_close(int64_t ptr) { CUDA_OK(cudaIpcCloseMemHandle(reinterpret_cast<void*>((uintptr_t)ptr))); }
void ipc_free(int64_t ptr) { CUDA_OK(cudaFree(reinterpret_cast<void*>((uintptr_t)ptr))); }

torch::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> sizes, torch::ScalarType dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, (int)device);
  return torch::from_blob(reinterpret_cast<void*>((uintptr_t)ptr), sizes, opts);
}

// INT4 GEMM whose output tiles are pushed to every rank (fused all-reduce, producer side).
// Returns the launch plan {bn, nt, splits, grid_x, grid_y} for the matching tp_reduce.
std::vector<int64_t> w4a16_gemm_push(torch::Tensor x, torch::Tensor wq, int64_t N, int64_t K, int64_t group,
                                     int64_t ldy, torch::Tensor push_dst, torch::Tensor push_flags,
                                     int64_t push_stride, int64_t flag_stride, torch::Tensor seq, int64_t tp,
                                     torch::Tensor ws, torch::Tensor counters, torch::Tensor status) {
  CHECK_CUDA(x);
  CHECK_DT(x, torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(1) == K, "x must be [M, K]");
  TORCH_CHECK(push_dst.scalar_type() == torch::kInt64 && push_dst.numel() == tp, "push_dst: [tp] int64 pointers");
  TORCH_CHECK(push_flags.scalar_type() == torch::kInt64 && push_flags.numel() == tp, "push_flags: [tp] pointers");
  const int64_t M = x.size(0);
  const c10::cuda::CUDAGuard g(x.device());
  auto plan = gemm_plan(M, N, K, group, sq::WF_INT4);
  const int bn = (int)plan[0], nt = (int)plan[1];
  sq::W4A16Params p{};
  p.wq = ptr<uint32_t>(wq);
  p.sz = p.wq;
  p.y = nullptr;
  p.ws = ptr<float>(ws);
  p.counters = ptr<int>(counters);
  p.status = ptr<int>(status);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldy = (int)ldy;
  p.kb_total = (int)((K + 63) / 64);
  p.splits = (int)plan[2];
  p.kb_per_split = (int)plan[3];
  p.gpk = group >= 64 ? 1 : (int)(64 / group);
  p.epilogue = sq::EPI_PLAIN;
  p.push_dst = reinterpret_cast<__nv_bfloat16* const*>(push_dst.data_ptr());
  p.push_flags = reinterpret_cast<int* const*>(push_flags.data_ptr());
  p.push_stride = push_stride;
  p.flag_stride = (int)flag_stride;
  p.seq = ptr<int>(seq);
  p.tp = (int)tp;
  const int64_t gx = (N + 128 * nt - 1) / (128 * nt), gy = (M + bn - 1) / bn;
  if (M > 0) {
    p.xg = gemm_xg(K, p, bn);
    const CUtensorMap xmap = make_x_map(x, (int)M, (int)K, bn, p.xg);
    CUDA_OK(sq::w4a16_gemm_launch(xmap, p, bn, nt, cur_stream()));
  }
  return {bn, nt, plan[2], gx, gy};
}

// Row-parallel GEMM with reduce-scatter routing: the bf16 partial of token row m goes only to
// its owner rank (m / rows_per_rank) at push_dst[owner] + (m % rows_per_rank) * ldy, and every
// CTA counts one arrival at push_flags[r] + parity * flag_stride on every rank. Returns
// {total CTAs of the launch} (the owners' expected count).
int64_t w4a16_gemm_rs(torch::Tensor x, torch::Tensor wq, int64_t N, int64_t K, int64_t group, int64_t ldy,
                      torch::Tensor push_dst, torch::Tensor push_flags, int64_t flag_stride, torch::Tensor seq,
                      int64_t tp, int64_t rows_per_rank, torch::Tensor ws, torch::Tensor counters,
                      torch::Tensor status) {
  CHECK_CUDA(x);
  CHECK_DT(x, torch::kBFloat16);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(1) == K, "x must be [M, K]");
  TORCH_CHECK(push_dst.scalar_type() == torch::kInt64 && push_dst.numel() == tp, "push_dst: [tp] int64 pointers");
  TORCH_CHECK(push_flags.scalar_type() == torch::kInt64 && push_flags.numel() == tp, "push_flags: [tp] pointers");
  const int64_t M = x.size(0);
  TORCH_CHECK(rows_per_rank > 0 && rows_per_rank * tp >= M, "rows_per_rank * tp must cover every row");
  const c10::cuda::CUDAGuard g(x.device());
  auto plan = gemm_plan(M, N, K, group, sq::WF_INT4);
  const int bn = (int)plan[0], nt = (int)plan[1];
  sq::W4A16Params p{};
  p.wq = ptr<uint32_t>(wq);
  p.sz = p.wq;
  p.ws = ptr<float>(ws);
  p.counters = ptr<int>(counters);
  p.status = ptr<int>(status);
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.ldy = (int)ldy;
  p.kb_total = (int)((K + 63) / 64);
  p.splits = (int)plan[2];
  p.kb_per_split = (int)plan[3];
  p.gpk = group >= 64 ? 1 : (int)(64 / group);
  p.epilogue = sq::EPI_PLAIN;
  p.push_dst = reinterpret_cast<__nv_bfloat16* const*>(push_dst.data_ptr());
  p.push_flags = reinterpret_cast<int* const*>(push_flags.data_ptr());
  p.push_stride = 0;  // one data buffer (the owners finish reading before any peer can push again)
  p.flag_stride = (int)flag_stride;
  p.seq = ptr<int>(seq);
  p.tp = (int)tp;
  p.push_rows = (int)rows_per_rank;
  const int64_t gx = (N + 128 * nt - 1) / (128 * nt), gy = (M + bn - 1) / bn;
  if (M > 0) {
    p.xg = gemm_xg(K, p, bn);
    const CUtensorMap xmap = make_x_map(x, (int)M, (int)K, bn, p.xg);
    CUDA_OK(sq::w4a16_gemm_launch(xmap, p, bn, nt, cur_stream()));
  }
  return gx * gy * plan[2];
}

// One-shot all-reduce: out (+)= sum over ranks of src, through double-buffered peer slots.
void tp_oneshot(torch::Tensor src, torch::Tensor part_ptrs, int64_t par_stride, torch::Tensor flag_ptrs,
                torch::Tensor out, bool residual_in_out, int64_t rank, int64_t tp, torch::Tensor seq, torch::Tensor done,
                torch::Tensor status) {
  CHECK_CUDA(src);
  CHECK_DT(src, torch::kBFloat16);
  CHECK_DT(out, torch::kBFloat16);
  TORCH_CHECK(src.dim() == 2 && out.dim() == 2 && src.size(0) == out.size(0) && src.size(1) == out.size(1) &&
                  src.stride(1) == 1 && out.stride(1) == 1,
              "src / out: [M, N] with unit column stride");
  TORCH_CHECK(part_ptrs.numel() == tp && flag_ptrs.numel() == tp && part_ptrs.is_cuda() && flag_ptrs.is_cuda(),
              "one device pointer per rank");
  const c10::cuda::CUDAGuard g(src.device());
  sq::TpOneshotParams p{};
  p.src = ptr<__nv_bfloat16>(src);
  p.ld_src = (int)src.stride(0);
  p.part = reinterpret_cast<__nv_bfloat16* const*>(part_ptrs.data_ptr());
  p.par_stride = par_stride;
  p.flags = reinterpret_cast<int* const*>(flag_ptrs.data_ptr());
  p.out = ptr<__nv_bfloat16>(out);
  p.ld_out = (int)out.stride(0);
  p.residual_in_out = residual_in_out ? 1 : 0;
  p.M = (int)src.size(0);
  p.N = (int)src.size(1);
  p.rank = (int)rank;
  p.tp = (int)tp;
  p.seq = ptr<int>(seq);
  p.done = ptr<int>(done);
  p.status = ptr<int>(status);
  CUDA_OK(sq::tp_oneshot_launch(p, cur_stream()));
}

void tp_rs_norm_ag(torch::Tensor recv, int64_t src_stride, int64_t ld_recv, torch::Tensor rs_flags, int64_t rs_expect,
                   torch::Tensor h, torch::Tensor w, double eps, torch::Tensor ag_dst, int64_t ld_ag,
                   torch::Tensor ag_flags, int64_t rank, int64_t tp, int64_t rows_per_rank, int64_t T,
                   torch::Tensor seq, torch::Tensor done, torch::Tensor status, bool local_only) {
  CHECK_CUDA(h);
  CHECK_DT(h, torch::kBFloat16);
  CHECK_DT(w, torch::kBFloat16);
  TORCH_CHECK(ag_dst.scalar_type() == torch::kInt64 && ag_dst.numel() == tp, "ag_dst: [tp] int64 pointers");
  TORCH_CHECK(ag_flags.scalar_type() == torch::kInt64 && ag_flags.numel() == tp, "ag_flags: [tp] pointers");
  TORCH_CHECK(h.dim() == 2 && h.stride(1) == 1 && h.size(0) >= T && w.numel() == h.size(1), "h [>= T, N], w [N]");
  const c10::cuda::CUDAGuard g(h.device());
  sq::TpRsNormParams p{};
  p.recv = ptr<__nv_bfloat16>(recv);
  p.src_stride = src_stride;
  p.ld_recv = (int)ld_recv;
  p.rs_flags = ptr<int>(rs_flags);
  p.rs_expect = (int)rs_expect;
  p.h = ptr<__nv_bfloat16>(h);
  p.ldh = (int)h.stride(0);
  p.w = ptr<__nv_bfloat16>(w);
  p.eps = (float)eps;
  p.ag_dst = reinterpret_cast<__nv_bfloat16* const*>(ag_dst.data_ptr());
  p.ld_ag = (int)ld_ag;
  p.ag_flags = reinterpret_cast<int* const*>(ag_flags.data_ptr());
  p.rank = (int)rank;
  p.tp = (int)tp;
  p.rows_per_rank = (int)rows_per_rank;
  p.T = (int)T;
  p.N = (int)h.size(1);
  p.seq = ptr<int>(seq);
  p.done = ptr<int>(done);
  p.status = ptr<int>(status);
  p.local_only = local_only ? 1 : 0;
  CUDA_OK(sq::tp_rs_norm_ag_launch(p, cur_stream()));
}

// Expert-parallel dispatch of this rank's owned rows (see ep_a2a.cu). Pointer arrays are
// [tp] int64 device tensors of every rank's buffers.
void ep_dispatch(torch::Tensor x, c10::optional<torch::Tensor> logits, bool renorm, torch::Tensor ids,
                 torch::Tensor w, int64_t own, int64_t R, int64_t K, int64_t E_local, int64_t rank, int64_t tp,
                 torch::Tensor recv_x, torch::Tensor recv_ids, torch::Tensor recv_w, torch::Tensor flags) {
  CHECK_CUDA(x);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(ids, torch::kInt32);
  CHECK_DT(w, torch::kFloat32);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(0) >= own, "x: [>= own, H]");
  TORCH_CHECK(ids.is_contiguous() && w.is_contiguous() && ids.numel() >= own * K && w.numel() >= own * K,
              "ids / w: contiguous [own, K]");
  TORCH_CHECK(own <= R, "own rows exceed the slots per source");
  for (const auto* t : {&recv_x, &recv_ids, &recv_w, &flags})
    TORCH_CHECK(t->scalar_type() == torch::kInt64 && t->numel() == tp && t->is_cuda(), "pointer arrays: [tp] int64");
  const c10::cuda::CUDAGuard g(x.device());
  sq::EpDispatchParams p{};
  p.x = ptr<__nv_bfloat16>(x);
  p.ldx = (int)x.stride(0);
  p.ids = ptr<int>(ids);
  p.w = ptr<float>(w);
  if (logits) {  // route in the dispatch kernel
    CHECK_DT((*logits), torch::kBFloat16);
    TORCH_CHECK(logits->dim() == 2 && logits->stride(1) == 1 && logits->size(0) >= own, "logits: [>= own, E]");
    p.logits = ptr<__nv_bfloat16>(*logits);
    p.ld_logits = (int)logits->stride(0);
    p.E = (int)logits->size(1);
    p.renorm = renorm ? 1 : 0;
  }
  p.recv_x = reinterpret_cast<__nv_bfloat16* const*>(recv_x.data_ptr());
  p.recv_ids = reinterpret_cast<int* const*>(recv_ids.data_ptr());
  p.recv_w = reinterpret_cast<float* const*>(recv_w.data_ptr());
  p.flags = reinterpret_cast<int* const*>(flags.data_ptr());
  p.own = (int)own;
  p.R = (int)R;
  p.H = (int)x.size(1);
  p.K = (int)K;
  p.E_local = (int)E_local;
  p.rank = (int)rank;
  p.tp = (int)tp;
  CUDA_OK(sq::ep_dispatch_launch(p, cur_stream()));
}

void ep_combine(torch::Tensor ys, torch::Tensor slot_pos, torch::Tensor w, int64_t R, int64_t K, int64_t tp,
                int64_t T, torch::Tensor dst, int64_t ld_dst, torch::Tensor flags, int64_t flag_stride,
                torch::Tensor seq) {
  CHECK_CUDA(ys);
  CHECK_DT(ys, torch::kBFloat16);
  CHECK_DT(slot_pos, torch::kInt32);
  CHECK_DT(w, torch::kFloat32);
  TORCH_CHECK(ys.dim() == 2 && ys.stride(1) == 1, "ys: [P, H]");
  TORCH_CHECK(slot_pos.numel() >= tp * R * K && w.numel() >= tp * R * K, "slot_pos / w: [tp R K]");
  TORCH_CHECK(dst.scalar_type() == torch::kInt64 && dst.numel() == tp && flags.scalar_type() == torch::kInt64 &&
                  flags.numel() == tp,
              "dst / flags: [tp] int64 pointers");
  const c10::cuda::CUDAGuard g(ys.device());
  sq::EpCombineParams p{};
  p.ys = ptr<__nv_bfloat16>(ys);
  p.ldys = (int)ys.stride(0);
  p.slot_pos = ptr<int>(slot_pos);
  p.w = ptr<float>(w);
  p.dst = reinterpret_cast<__nv_bfloat16* const*>(dst.data_ptr());
  p.ld_dst = (int)ld_dst;
  p.flags = reinterpret_cast<int* const*>(flags.data_ptr());
  p.flag_stride = (int)flag_stride;
  p.seq = ptr<int>(seq);
  p.R = (int)R;
  p.H = (int)ys.size(1);
  p.K = (int)K;
  p.tp = (int)tp;
  p.T = (int)T;
  CUDA_OK(sq::ep_combine_launch(p, cur_stream()));
}

void tp_ag_wait(torch::Tensor ag_flags, int64_t expect, int64_t tp, torch::Tensor status) {
  CHECK_CUDA(ag_flags);
  const c10::cuda::CUDAGuard g(ag_flags.device());
  CUDA_OK(sq::tp_ag_wait_launch(ptr<int>(ag_flags), (int)expect, (int)tp, ptr<int>(status), cur_stream()));
}

void tp_push(torch::Tensor src, torch::Tensor push_dst, int64_t parity_stride, int64_t ld_dst,
             torch::Tensor push_flags, int64_t flag_stride, int64_t tile_m, int64_t grid_x, int64_t grid_y, int64_t tp,
             torch::Tensor seq) {
  CHECK_CUDA(src);
  CHECK_DT(src, torch::kBFloat16);
  TORCH_CHECK(src.stride(1) == 1, "src must have unit column stride");
  const c10::cuda::CUDAGuard g(src.device());
  sq::TpPushParams p{};
  p.src = ptr<__nv_bfloat16>(src);
  p.ld_src = (int)src.stride(0);
  p.dst = reinterpret_cast<__nv_bfloat16* const*>(push_dst.data_ptr());
  p.parity_stride = parity_stride;
  p.ld_dst = (int)ld_dst;
  p.flags = reinterpret_cast<int* const*>(push_flags.data_ptr());
  p.flag_stride = (int)flag_stride;
  p.M = (int)src.size(0);
  p.N = (int)src.size(1);
  p.tile_m = (int)tile_m;
  p.tp = (int)tp;
  p.seq = ptr<int>(seq);
  CUDA_OK(sq::tp_push_launch(p, (int)grid_x, (int)grid_y, cur_stream()));
}

void tp_reduce(torch::Tensor recv, int64_t recv_stride, int64_t src_stride, int64_t ld, torch::Tensor flags,
               int64_t flag_stride, int64_t flag_src_stride, int64_t expect, torch::Tensor out, bool residual,
               int64_t M, int64_t N, int64_t tile_m, int64_t tile_n, int64_t grid_x, int64_t grid_y, int64_t tp,
               torch::Tensor seq, torch::Tensor done, torch::Tensor status) {
  CHECK_CUDA(out);
  CHECK_DT(out, torch::kBFloat16);
  const c10::cuda::CUDAGuard g(out.device());
  sq::TpReduceParams p{};
  p.recv = ptr<__nv_bfloat16>(recv);
  p.recv_stride = recv_stride;
  p.src_stride = src_stride;
  p.ld = (int)ld;
  p.flags = ptr<int>(flags);
  p.flag_stride = (int)flag_stride;
  p.flag_src_stride = (int)flag_src_stride;
  p.expect = (int)expect;
  p.out = ptr<__nv_bfloat16>(out);
  p.ld_out = (int)out.stride(0);
  p.residual_in_out = residual ? 1 : 0;
  p.M = (int)M;
  p.N = (int)N;
  p.tile_m = (int)tile_m;
  p.tile_n = (int)tile_n;
  p.tp = (int)tp;
  p.seq = ptr<int>(seq);
  p.done = ptr<int>(done);
  p.status = ptr<int>(status);
  if (M == 0) return;
  CUDA_OK(sq::tp_reduce_launch(p, (int)grid_x, (int)grid_y, cur_stream()));
}

void tp_gather(torch::Tensor src, torch::Tensor dst_ptrs, int64_t ld_dst, int64_t row0, int64_t col0,
               torch::Tensor flag_ptrs,
               torch::Tensor local_flags, int64_t flag_stride, int64_t blocks, int64_t rank, int64_t tp,
               torch::Tensor seq, torch::Tensor status) {
  CHECK_CUDA(src);
  CHECK_DT(src, torch::kBFloat16);
  const c10::cuda::CUDAGuard g(src.device());
  sq::TpGatherParams p{};
  p.src = ptr<__nv_bfloat16>(src);
  p.ld_src = (int)src.stride(0);
  p.dst = reinterpret_cast<__nv_bfloat16* const*>(dst_ptrs.data_ptr());
  p.ld_dst = (int)ld_dst;
  p.row0 = (int)row0;
  p.col0 = (int)col0;
  p.rows = (int)src.size(0);
  p.cols = (int)src.size(1);
  p.flags = reinterpret_cast<int* const*>(flag_ptrs.data_ptr());
  p.local_flags = ptr<int>(local_flags);
  p.flag_stride = (int)flag_stride;
  p.expect = (int)blocks;
  p.rank = (int)rank;
  p.tp = (int)tp;
  p.seq = ptr<int>(seq);
  p.status = ptr<int>(status);
  CUDA_OK(sq::tp_gather_launch(p, cur_stream()));
}

// ------------------------------------------------------------------ norm / rope / attention
void rmsnorm(torch::Tensor x, torch::Tensor w, torch::Tensor y, c10::optional<torch::Tensor> row_idx, double eps) {
  CHECK_CUDA(x);
  CHECK_DT(x, torch::kBFloat16);
  CHECK_DT(w, torch::kBFloat16);
  const int64_t H = x.size(-1);
  TORCH_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  const int64_t rows = row_idx.has_value() ? row_idx->numel() : x.size(0);
  const c10::cuda::CUDAGuard g(x.device());
  CUDA_OK(sq::rmsnorm_launch(ptr<__nv_bfloat16>(x), ptr<__nv_bfloat16>(w), ptr<__nv_bfloat16>(y),
                             optr<int>(row_idx), (int)rows, (int)H, (int)x.stride(0), (int)y.stride(0), (float)eps,
                             cur_stream()));
}

void rope_kv_write(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_sin, torch::Tensor q_out,
                   torch::Tensor slot_mapping, torch::Tensor k_codes, torch::Tensor k_scales, torch::Tensor v_codes,
                   torch::Tensor v_scales, int64_t Hq, int64_t Hkv, int64_t D, int64_t page_size, int64_t group,
                   int64_t fmt_k, int64_t fmt_v, c10::optional<torch::Tensor> q_norm,
                   c10::optional<torch::Tensor> k_norm, double norm_eps, c10::optional<torch::Tensor> status,
                   c10::optional<torch::Tensor> had_k, c10::optional<torch::Tensor> had_v) {
  CHECK_CUDA(qkv);
  for (const auto* h : {&had_k, &had_v})
    if (h->has_value())
      TORCH_CHECK((*h)->scalar_type() == torch::kFloat32 && (*h)->numel() == D && (*h)->is_cuda(),
                  "Hadamard signs: float32 [head_dim] on the device");
  CHECK_DT(qkv, torch::kBFloat16);
  CHECK_DT(positions, torch::kInt32);
  CHECK_DT(slot_mapping, torch::kInt32);
  TORCH_CHECK(group >= 32 && D % group == 0, "KV group must be >= 32 and divide head_dim");
  const c10::cuda::CUDAGuard g(qkv.device());
  sq::RopeKvParams p{};
  p.qkv = ptr<__nv_bfloat16>(qkv);
  p.ld_qkv = (int)qkv.stride(0);
  p.positions = ptr<int>(positions);
  p.cos_sin = ptr<float>(cos_sin);
  p.q_out = ptr<__nv_bfloat16>(q_out);
  p.slot_mapping = ptr<int>(slot_mapping);
  p.k_codes = ptr<uint8_t>(k_codes);
  p.k_scales = reinterpret_cast<__half*>(k_scales.data_ptr());
  p.v_codes = ptr<uint8_t>(v_codes);
  p.v_scales = reinterpret_cast<__half*>(v_scales.data_ptr());
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.D = (int)D;
  p.page_size = (int)page_size;
  p.group = (int)group;
  p.fmt_k = (int)fmt_k;
  p.fmt_v = (int)fmt_v;
  p.q_norm = optr<__nv_bfloat16>(q_norm);
  p.k_norm = optr<__nv_bfloat16>(k_norm);
  p.norm_eps = (float)norm_eps;
  p.num_pages = k_codes.dim() == 4 ? (int)k_codes.size(0) : 0;
  p.status = optr<int>(status);
  p.had_k = optr<float>(had_k);
  p.had_v = optr<float>(had_v);
  CUDA_OK(sq::rope_kv_write_launch(p, (int)qkv.size(0), cur_stream()));
}

sq::AttnParams attn_common(torch::Tensor q, torch::Tensor k_codes, torch::Tensor k_scales, torch::Tensor v_codes,
                           torch::Tensor v_scales, torch::Tensor block_tables, torch::Tensor out, int64_t Hq,
                           int64_t Hkv, int64_t D, int64_t page_size, int64_t group, int64_t fmt_k, int64_t fmt_v,
                           double sm_scale) {
  CHECK_CUDA(q);
  CHECK_DT(q, torch::kBFloat16);
  CHECK_DT(out, torch::kBFloat16);
  CHECK_DT(block_tables, torch::kInt32);
  TORCH_CHECK(page_size % 16 == 0, "page size must be a multiple of 16");
  TORCH_CHECK(Hq % Hkv == 0 && Hq / Hkv <= 16, "GQA group must be <= 16");
  sq::AttnParams p{};
  p.q = ptr<__nv_bfloat16>(q);
  p.ld_q = (int)q.stride(0);
  p.k_codes = ptr<uint8_t>(k_codes);
  p.k_scales = reinterpret_cast<const __half*>(k_scales.data_ptr());
  p.v_codes = ptr<uint8_t>(v_codes);
  p.v_scales = reinterpret_cast<const __half*>(v_scales.data_ptr());
  p.block_tables = ptr<int>(block_tables);
  p.bt_stride = (int)block_tables.stride(0);
  p.out = ptr<__nv_bfloat16>(out);
  p.ld_out = (int)out.stride(0);
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.D = (int)D;
  p.page_size = (int)page_size;
  p.group = (int)group;
  p.fmt_k = (int)fmt_k;
  p.fmt_v = (int)fmt_v;
  p.sm_scale = (float)sm_scale;
  p.num_pages = k_codes.dim() == 4 ? (int)k_codes.size(0) : 0;  // [pages, Hkv, page_size, bytes]
  return p;
}

void paged_decode_attention(torch::Tensor q, torch::Tensor k_codes, torch::Tensor k_scales, torch::Tensor v_codes,
                            torch::Tensor v_scales, torch::Tensor block_tables, torch::Tensor seq_lens,
                            torch::Tensor out, torch::Tensor o_part, torch::Tensor lse_part, int64_t Hq, int64_t Hkv,
                            int64_t D, int64_t page_size, int64_t group, int64_t fmt_k, int64_t fmt_v,
                            double sm_scale, int64_t splits, int64_t tiles_per_split,
                            c10::optional<torch::Tensor> status) {
  const c10::cuda::CUDAGuard g(q.device());
  auto p = attn_common(q, k_codes, k_scales, v_codes, v_scales, block_tables, out, Hq, Hkv, D, page_size, group,
                       fmt_k, fmt_v, sm_scale);
  p.status = optr<int>(status);
  CHECK_DT(seq_lens, torch::kInt32);
  p.seq_lens = ptr<int>(seq_lens);
  p.B = (int)seq_lens.size(0);
  p.splits = (int)splits;
  p.tiles_per_split = (int)tiles_per_split;
  if (splits > 1) {
    TORCH_CHECK(o_part.numel() >= p.B * Hq * splits * D && lse_part.numel() >= p.B * Hq * splits,
                "decode split workspace too small");
  }
  p.o_part = ptr<float>(o_part);
  p.lse_part = ptr<float>(lse_part);
  CUDA_OK(sq::paged_decode_attn_launch(p, cur_stream()));
}

// Attention mass per KV page (H2O-style scores), accumulated into mass[num_pages] (float32).
void page_mass(torch::Tensor q, torch::Tensor k_codes, torch::Tensor k_scales, torch::Tensor block_tables,
               torch::Tensor seq_lens, torch::Tensor mass, int64_t Hq, int64_t Hkv, int64_t D, int64_t page_size,
               int64_t group, int64_t fmt_k, double sm_scale, c10::optional<torch::Tensor> status) {
  CHECK_CUDA(q);
  CHECK_DT(q, torch::kBFloat16);
  CHECK_DT(block_tables, torch::kInt32);
  CHECK_DT(seq_lens, torch::kInt32);
  CHECK_DT(mass, torch::kFloat32);
  TORCH_CHECK(q.dim() == 2 && q.stride(1) == 1, "q: [B, Hq * D] with unit column stride");
  TORCH_CHECK(k_codes.dim() == 4 && mass.numel() >= k_codes.size(0), "mass: one float per page");
  TORCH_CHECK(block_tables.dim() == 2 && block_tables.stride(1) == 1 && block_tables.size(0) >= seq_lens.size(0),
              "block_tables: [>= B, pages]");
  const c10::cuda::CUDAGuard g(q.device());
  sq::PageMassParams p{};
  p.q = ptr<__nv_bfloat16>(q);
  p.ld_q = (int)q.stride(0);
  p.k_codes = ptr<uint8_t>(k_codes);
  p.k_scales = reinterpret_cast<const __half*>(k_scales.data_ptr());
  p.block_tables = ptr<int>(block_tables);
  p.bt_stride = (int)block_tables.stride(0);
  p.seq_lens = ptr<int>(seq_lens);
  p.mass = ptr<float>(mass);
  p.B = (int)seq_lens.size(0);
  p.Hq = (int)Hq;
  p.Hkv = (int)Hkv;
  p.D = (int)D;
  p.page_size = (int)page_size;
  p.group = (int)group;
  p.fmt_k = (int)fmt_k;
  p.num_pages = (int)k_codes.size(0);
  p.sm_scale = (float)sm_scale;
  p.status = optr<int>(status);
  CUDA_OK(sq::page_mass_launch(p, cur_stream()));
}

void paged_prefill_attention(torch::Tensor q, torch::Tensor k_codes, torch::Tensor k_scales, torch::Tensor v_codes,
                             torch::Tensor v_scales, torch::Tensor block_tables, torch::Tensor tile_seq,
                             torch::Tensor tile_q0, torch::Tensor q_start, torch::Tensor q_len, torch::Tensor ctx_len,
                             int64_t n_tiles, torch::Tensor out, int64_t Hq, int64_t Hkv, int64_t D,
                             int64_t page_size, int64_t group, int64_t fmt_k, int64_t fmt_v, double sm_scale,
                             c10::optional<torch::Tensor> tree_mask, c10::optional<torch::Tensor> status,
                             c10::optional<torch::Tensor> trace) {
  const c10::cuda::CUDAGuard g(q.device());
  auto p = attn_common(q, k_codes, k_scales, v_codes, v_scales, block_tables, out, Hq, Hkv, D, page_size, group,
                       fmt_k, fmt_v, sm_scale);
  p.tree_mask = optr<int>(tree_mask);
  p.status = optr<int>(status);
  p.tile_seq = ptr<int>(tile_seq);
  p.tile_q0 = ptr<int>(tile_q0);
  p.q_start = ptr<int>(q_start);
  p.q_len = ptr<int>(q_len);
  p.ctx_len = ptr<int>(ctx_len);
  p.n_tiles = (int)n_tiles;
  static const bool tc_off = [] {
    const char* e = std::getenv("SQ_PREFILL_ATTN_LEGACY");
    return e != nullptr && e[0] == '1';
  }();
  if (!tc_off && status.has_value() && sq::prefill_tc_supported(p)) {
    const int hs = sq::prefill_tc_head_slots((int)(Hq / Hkv));
    CUtensorMap m;
    cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Hq, (cuuint64_t)q.size(0)};
    cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)q.stride(0) * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)hs, (cuuint32_t)(128 / hs)};
    cuuint32_t estr[3] = {1, 1, 1};
    TORCH_CHECK(reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 && q.stride(1) == 1, "q rows must be aligned");
    CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, q.data_ptr(), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(r == CUDA_SUCCESS, std::string("cuTensorMapEncodeTiled (q) failed (") + std::to_string((int)r) + ")");
    CUDA_OK(sq::paged_prefill_attn_tc_launch(m, p, ptr<int>(*status), optr<unsigned long long>(trace),
                                             cur_stream()));
    return;
  }
  CUDA_OK(sq::paged_prefill_attn_launch(p, cur_stream()));
}

void sample(torch::Tensor logits, c10::optional<torch::Tensor> temperature, c10::optional<torch::Tensor> top_p,
            c10::optional<torch::Tensor> top_k, c10::optional<torch::Tensor> min_p,
            c10::optional<torch::Tensor> rep_penalty, c10::optional<torch::Tensor> hist,
            c10::optional<torch::Tensor> allow_mask, int64_t seed, c10::optional<torch::Tensor> step,
            torch::Tensor out_tokens, c10::optional<torch::Tensor> out_logprob, torch::Tensor work) {
  CHECK_CUDA(logits);
  CHECK_DT(logits, torch::kBFloat16);
  CHECK_DT(work, torch::kFloat32);
  const c10::cuda::CUDAGuard g(logits.device());
  sq::SamplerParams p{};
  p.logits = ptr<__nv_bfloat16>(logits);
  p.ld = (int)logits.stride(0);
  p.V = (int)logits.size(1);
  p.B = (int)logits.size(0);
  TORCH_CHECK(work.numel() >= (int64_t)p.B * p.V, "sampler workspace too small");
  p.temperature = optr<float>(temperature);
  p.top_p = optr<float>(top_p);
  p.top_k = optr<int>(top_k);
  p.min_p = optr<float>(min_p);
  p.rep_penalty = optr<float>(rep_penalty);
  p.hist = optr<int>(hist);
  p.hist_stride = hist.has_value() ? (int)hist->size(1) : 0;
  p.allow_mask = optr<uint32_t>(allow_mask);
  p.seed = (uint64_t)seed;
  p.step = optr<int>(step);
  p.out_tokens = ptr<int>(out_tokens);
  p.out_logprob = optr<float>(out_logprob);
  CUDA_OK(sq::sampler_launch(p, ptr<float>(work), cur_stream()));
}

// GPU weight quantizers with the CPU library's output layouts (cpu_ref.cpp): returns
// [codes, scales] (+ offsets for INT2). x: [rows, cols] float32 or bf16 on the GPU.
std::vector<torch::Tensor> quantize_codec_cuda(torch::Tensor x, int64_t codec, int64_t group, double fixed_scale) {
  CHECK_CUDA(x);
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous(), "x must be a contiguous 2-D tensor");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 || x.scalar_type() == torch::kBFloat16, "x: float32 or bf16");
  TORCH_CHECK(codec >= 0 && codec <= 6, "codec: 0 int8, 1 int4 sym, 2 nf4, 3 int3, 4 int2, 5 fp8 e4m3, 6 fp8 e5m2");
  const int64_t N = x.size(0), D = x.size(1);
  const int64_t g = ((codec == 0 || codec >= 5) && group <= 0) ? D : group;
  TORCH_CHECK(g > 0 && D % g == 0, "group must divide columns");
  TORCH_CHECK(codec == 0 || codec >= 5 || g % (codec == 3 ? 8 : codec == 4 ? 4 : 2) == 0,
              "group too small for the codec's packing");
  const c10::cuda::CUDAGuard guard(x.device());
  auto u8 = x.options().dtype(torch::kUInt8);
  torch::Tensor codes;
  int64_t ld;
  if (codec == 0) {
    codes = torch::empty({N, D}, x.options().dtype(torch::kInt8));
    ld = D;
  } else if (codec >= 5) {
    codes = torch::empty({N, D}, u8);
    ld = D;
  } else if (codec == 3) {
    ld = (D + 7) / 8 * 3;
    codes = torch::zeros({N, ld}, u8);
  } else {
    ld = codec == 4 ? D / 4 : D / 2;
    codes = torch::empty({N, ld}, u8);
  }
  auto scales = torch::empty({N, D / g}, x.options().dtype(torch::kFloat32));
  auto offsets = torch::empty({codec == 4 ? N : 0, D / g}, x.options().dtype(torch::kFloat32));
  CUDA_OK(sq::quantize_codec_launch(x.data_ptr(), x.scalar_type() == torch::kBFloat16, (int)codec,
                                    reinterpret_cast<uint8_t*>(codes.data_ptr()), (int)ld, ptr<float>(scales),
                                    codec == 4 ? ptr<float>(offsets) : nullptr, (int)N, (int)D, (int)g,
                                    (float)fixed_scale, cur_stream()));
  if (codec == 4) return {codes, scales, offsets};
  return {codes, scales};
}

std::vector<torch::Tensor> hqq_cuda(torch::Tensor x, int64_t group, int64_t levels, double lam, int64_t iters) {
  CHECK_CUDA(x);
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous(), "x must be a contiguous 2-D tensor");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 || x.scalar_type() == torch::kBFloat16, "x: float32 or bf16");
  const int64_t N = x.size(0), D = x.size(1);
  TORCH_CHECK(group > 0 && group <= 512 && D % group == 0, "group must divide columns and be <= 512");
  TORCH_CHECK(levels >= 2 && levels <= 256, "levels must be in [2, 256]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto codes = torch::empty({N, D}, x.options().dtype(torch::kUInt8));
  auto scales = torch::empty({N, D / group}, x.options().dtype(torch::kFloat32));
  auto zeros = torch::empty({N, D / group}, x.options().dtype(torch::kFloat32));
  CUDA_OK(sq::hqq_launch(x.data_ptr(), x.scalar_type() == torch::kBFloat16,
                         reinterpret_cast<uint8_t*>(codes.data_ptr()), ptr<float>(scales), ptr<float>(zeros), (int)N,
                         (int)D, (int)group, (int)levels, (float)lam, (int)iters, cur_stream()));
  return {codes, scales, zeros};
}

void channel_abs_mean_cuda(torch::Tensor x, torch::Tensor acc) {
  CHECK_CUDA(x);
  CHECK_CUDA(acc);
  TORCH_CHECK(x.dim() == 2 && x.is_contiguous(), "x must be a contiguous 2-D tensor");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 || x.scalar_type() == torch::kBFloat16, "x: float32 or bf16");
  TORCH_CHECK(acc.scalar_type() == torch::kFloat64 && acc.numel() == x.size(1) && acc.is_contiguous(),
              "acc: float64 with one entry per column");
  const c10::cuda::CUDAGuard guard(x.device());
  CUDA_OK(sq::channel_abs_mean_launch(x.data_ptr(), x.scalar_type() == torch::kBFloat16, acc.data_ptr<double>(),
                                      (int)x.size(0), (int)x.size(1), cur_stream()));
}

std::vector<torch::Tensor> quantize_int4_asym_cuda(torch::Tensor x, int64_t group, int64_t n_clip) {
  CHECK_CUDA(x);
  CHECK_CONTIG(x);
  TORCH_CHECK(x.dim() == 2, "x must be 2-D");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 || x.scalar_type() == torch::kBFloat16, "x must be f32 or bf16");
  const int64_t rows = x.size(0), cols = x.size(1);
  TORCH_CHECK(cols % group == 0 && group % 2 == 0, "group must divide columns and be even");
  const c10::cuda::CUDAGuard g(x.device());
  auto packed = torch::empty({rows, cols / 2}, x.options().dtype(torch::kUInt8));
  auto scales = torch::empty({rows, cols / group}, x.options().dtype(torch::kFloat32));
  auto offsets = torch::empty({rows, cols / group}, x.options().dtype(torch::kFloat32));
  CUDA_OK(sq::quantize_int4_asym_launch(x.data_ptr(), x.scalar_type() == torch::kBFloat16, ptr<uint8_t>(packed),
                                        ptr<float>(scales), ptr<float>(offsets), (int)rows, (int)cols, (int)group,
                                        (int)n_clip, cur_stream()));
  return {packed, scales, offsets};
}

}  // namespace

namespace {

void check_kmeans_inputs(const torch::Tensor& x, const torch::Tensor& c) {
  CHECK_CUDA(x);
  CHECK_CUDA(c);
  TORCH_CHECK(x.dim() == 2 && c.dim() == 2 && x.size(1) == c.size(1), "x [n, d] and centroids [k, d]");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && c.scalar_type() == torch::kFloat32, "float32 inputs");
  TORCH_CHECK(x.is_contiguous() && c.is_contiguous(), "contiguous inputs");
  const int64_t d = x.size(1);
  TORCH_CHECK(d == 1 || d == 2 || d == 4 || d == 8 || d == 16 || d == 32 || d == 64,
              "vector width must be 1, 2, 4, 8, 16, 32 or 64 (zero-pad others)");
  TORCH_CHECK(c.size(0) >= 1, "at least one centroid");
}

}  // namespace

std::vector<torch::Tensor> kmeans_assign_cuda(torch::Tensor x, torch::Tensor c) {
  check_kmeans_inputs(x, c);
  const c10::cuda::CUDAGuard guard(x.device());
  auto assign = torch::empty({x.size(0)}, x.options().dtype(torch::kInt32));
  auto dist = torch::empty({x.size(0)}, x.options());
  CUDA_OK(sq::kmeans_assign_launch(ptr<float>(x), (int)x.size(0), (int)x.size(1), ptr<float>(c), (int)c.size(0),
                                   ptr<int>(assign), ptr<float>(dist), nullptr, cur_stream()));
  return {assign, dist};
}

// Lloyd iterations from the given centroids (updated in place); stops early when no assignment
// changes. Returns (assignments, iterations run).
std::vector<torch::Tensor> kmeans_fit_cuda(torch::Tensor x, torch::Tensor c, int64_t iters) {
  check_kmeans_inputs(x, c);
  const c10::cuda::CUDAGuard guard(x.device());
  const int n = (int)x.size(0), d = (int)x.size(1), k = (int)c.size(0);
  auto assign = torch::full({n}, -1, x.options().dtype(torch::kInt32));
  auto sums = torch::empty({k, d}, x.options());
  auto counts = torch::empty({k}, x.options().dtype(torch::kInt32));
  auto changed = torch::zeros({1}, x.options().dtype(torch::kInt32));
  auto s = cur_stream();
  CUDA_OK(sq::kmeans_assign_launch(ptr<float>(x), n, d, ptr<float>(c), k, ptr<int>(assign), nullptr, nullptr, s));
  int64_t it = 0;
  for (; it < iters; ++it) {
    CUDA_OK(sq::kmeans_update_launch(ptr<float>(x), n, d, ptr<int>(assign), ptr<float>(c), k, ptr<float>(sums),
                                     ptr<int>(counts), s));
    changed.zero_();
    CUDA_OK(sq::kmeans_assign_launch(ptr<float>(x), n, d, ptr<float>(c), k, ptr<int>(assign), nullptr,
                                     ptr<int>(changed), s));
    if (changed.item<int>() == 0) {
      ++it;
      break;
    }
  }
  return {assign, torch::full({1}, it, torch::kInt64)};
}

torch::Tensor pq_adc_cuda(torch::Tensor codes, torch::Tensor lut) {
  CHECK_CUDA(codes);
  CHECK_CUDA(lut);
  TORCH_CHECK(codes.scalar_type() == torch::kUInt8 && codes.dim() == 2 && codes.is_contiguous(), "codes: uint8 [n, m]");
  TORCH_CHECK(lut.scalar_type() == torch::kFloat32 && lut.dim() == 2 && lut.is_contiguous(), "lut: float32 [m, k]");
  TORCH_CHECK(lut.size(0) == codes.size(1) && lut.size(1) <= 256, "lut [m, k <= 256] matching the codes' m");
  TORCH_CHECK(lut.numel() <= 12288, "lut too large for shared memory (m * k <= 12288)");
  const c10::cuda::CUDAGuard guard(codes.device());
  auto out = torch::empty({codes.size(0)}, lut.options());
  CUDA_OK(sq::pq_adc_launch(reinterpret_cast<const uint8_t*>(codes.data_ptr()), (int)codes.size(0),
                            (int)codes.size(1), ptr<float>(lut), (int)lut.size(1), ptr<float>(out), cur_stream()));
  return out;
}

torch::Tensor hadamard_rows_cuda(torch::Tensor x, torch::Tensor signs, int64_t block, c10::optional<torch::Tensor> out) {
  CHECK_CUDA(x);
  CHECK_CUDA(signs);
  TORCH_CHECK(x.dim() == 2 && x.scalar_type() == torch::kBFloat16 && x.stride(1) == 1, "x: bf16 [M, K], unit column stride");
  TORCH_CHECK(signs.scalar_type() == torch::kFloat32 && signs.is_contiguous() && signs.numel() == x.size(1),
              "signs: float32 [K]");
  TORCH_CHECK(block >= 2 && block <= 4096 && (block & (block - 1)) == 0 && x.size(1) % block == 0,
              "block must be a power of two in [2, 4096] dividing K");
  const c10::cuda::CUDAGuard guard(x.device());
  torch::Tensor y = out.has_value() ? *out : torch::empty({x.size(0), x.size(1)}, x.options());
  TORCH_CHECK(y.scalar_type() == torch::kBFloat16 && y.dim() == 2 && y.size(0) >= x.size(0) && y.size(1) == x.size(1) &&
              y.stride(1) == 1, "out: bf16 [>= M, K]");
  CUDA_OK(sq::hadamard_rows_launch(ptr<__nv_bfloat16>(x), (int)x.stride(0), ptr<__nv_bfloat16>(y), (int)y.stride(0),
                                   ptr<float>(signs), (int)x.size(0), (int)x.size(1), (int)block, cur_stream()));
  return y;
}

namespace sqhost {
void register_host(pybind11::module& m);  // host_utils.cpp
}
namespace sqgram {
void register_grammar(pybind11::module& m);  // grammar.cpp
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "squish_b200 native kernels (sm_100a CUDA + C++ CPU reference)";
  m.def("repack_int4", &repack_int4);
  m.def("gemm_plan", &gemm_plan, py::arg("M"), py::arg("N"), py::arg("K"), py::arg("group") = 64,
        py::arg("wfmt") = 0);
  m.def("w4a16_gemm", &w4a16_gemm, py::arg("x"), py::arg("wq"), py::arg("sz"), py::arg("N"), py::arg("K"),
        py::arg("group"), py::arg("y"), py::arg("bias"), py::arg("residual"), py::arg("epilogue"), py::arg("ws"),
        py::arg("counters"), py::arg("status"), py::arg("trace"), py::arg("wfmt"), py::arg("codebook"),
        py::arg("ag_flags") = py::none(), py::arg("ag_done") = py::none(), py::arg("ag_expect") = 0,
        py::arg("ag_tp") = 0);
  m.def("w4a16_gemm_rs", &w4a16_gemm_rs);
  m.def("tp_rs_norm_ag", &tp_rs_norm_ag);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_combine", &ep_combine);
  m.def("tp_oneshot", &tp_oneshot);
  m.def("tp_ag_wait", &tp_ag_wait);
  m.def("dequant_weight", &dequant_weight);
  m.def("bf16_gemm", &bf16_gemm);
  m.def("w4a16_grouped_gemm", &w4a16_grouped_gemm);
  m.def("moe_route", &moe_route);
  m.def("tree_verify", &tree_verify);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("ipc_free", &ipc_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("w4a16_gemm_push", &w4a16_gemm_push);
  m.def("tp_reduce", &tp_reduce);
  m.def("tp_push", &tp_push);
  m.def("tp_gather", &tp_gather);
  m.def("kv_compact", &kv_compact);
  m.def("moe_align", &moe_align, py::arg("ids"), py::arg("E"), py::arg("bn"), py::arg("sorted_slot"),
        py::arg("slot_pos"), py::arg("tile_expert"), py::arg("num_tiles"), py::arg("counts") = py::none(),
        py::arg("wait_flags") = py::none(), py::arg("wait_expect") = 0, py::arg("status") = py::none());
  m.def("moe_gather", &moe_gather);
  m.def("moe_combine", &moe_combine);
  m.def("rmsnorm", &rmsnorm);
  m.def("rope_kv_write", &rope_kv_write);
  m.def("page_mass", &page_mass);
  m.def("paged_decode_attention", &paged_decode_attention);
  m.def("paged_prefill_attention", &paged_prefill_attention);
  m.def("sample", &sample);
  m.def("quantize_int4_asym", &quantize_int4_asym_cuda);
  m.def("quantize_codec", &quantize_codec_cuda, py::arg("x"), py::arg("codec"), py::arg("group"),
        py::arg("fixed_scale") = 0.0);
  m.def("hqq", &hqq_cuda);
  m.def("channel_abs_mean", &channel_abs_mean_cuda);
  m.def("kmeans_assign", &kmeans_assign_cuda);
  m.def("kmeans_fit", &kmeans_fit_cuda);
  m.def("pq_adc", &pq_adc_cuda);
  m.def("hadamard_rows", &hadamard_rows_cuda, py::arg("x"), py::arg("signs"), py::arg("block"),
        py::arg("out") = py::none());
  sqcpu::register_cpu(m);
  sqhost::register_host(m);
  sqgram::register_grammar(m);
}
