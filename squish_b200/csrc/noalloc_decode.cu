// noalloc_decode.cu — allocation-free variant of the paged decode attention launch.
//
// For callers that cannot allocate device memory (see noalloc_decode.h): the kernel is the
// same split-K flash-decoding kernel as paged_decode_attn_launch (attention.cu), but its
// per-split partials (output rows and log-sum-exp values) go to a fixed file-scope device
// array rather than a caller-supplied workspace. Nothing here calls cudaMalloc, cudaFree
// or any allocating library routine.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "kernels.h"
#include "noalloc_decode.h"

namespace {

constexpr int kMaxDevices = 64;

// The scratch every call shares: [partials | lse]. In host code `g_decode_scratch` names a
// host-side stand-in, not device memory; host code only uses the address returned by
// cudaGetSymbolAddress for the current device.
static __device__ __align__(256) float g_decode_scratch[SQ_NOALLOC_MAX_PARTIAL_FLOATS + SQ_NOALLOC_MAX_LSE];

std::atomic<float*> g_scratch_ptr[kMaxDevices] = {};
std::mutex g_mu;

// Device address of the scratch array on the current device (set-up on first use). After
// the first call on a device the cached address is read without taking the lock.
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  float* cached = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (cached == nullptr) {
    std::lock_guard<std::mutex> lock(g_mu);
    cached = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (cached == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_decode_scratch);
      if (e != cudaSuccess) return e;
      cached = static_cast<float*>(p);
      g_scratch_ptr[dev].store(cached, std::memory_order_release);
    }
  }
  *out = cached;
  return cudaSuccess;
}

bool valid_kv_formats(int fk, int fv) {
  // the (key, value) page format pairs the decode kernel is built for
  return (fk == fv && fk >= 0 && fk <= 3) || (fk == 4 && fv == 5);
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int sq_paged_decode_attention_noalloc(
    const void* q, int ld_q, const void* k_codes, const void* k_scales, const void* v_codes, const void* v_scales,
    const int* block_tables, int bt_stride, const int* seq_lens, int B, void* out, int ld_out, int Hq, int Hkv, int D,
    int page_size, int group, int fmt_k, int fmt_v, float sm_scale, int splits, int tiles_per_split, void* stream) {
  // The decode kernel assumes all of these; a caller handing raw pointers gets no other check.
  if (B < 0 || Hq <= 0 || Hkv <= 0 || splits < 1 || tiles_per_split < 1) return SQ_NOALLOC_BAD_ARGUMENT;
  if (D != 32 && D != 64 && D != 128) return SQ_NOALLOC_BAD_ARGUMENT;
  if (Hq % Hkv != 0 || Hq / Hkv > 16) return SQ_NOALLOC_BAD_ARGUMENT;
  if (page_size <= 0 || page_size % 16 != 0) return SQ_NOALLOC_BAD_ARGUMENT;
  if (!valid_kv_formats(fmt_k, fmt_v)) return SQ_NOALLOC_BAD_ARGUMENT;
  if (fmt_k != 0 && (group < 32 || D % group != 0)) return SQ_NOALLOC_BAD_ARGUMENT;
  if (ld_q < Hq * D || ld_out < Hq * D || bt_stride < 1) return SQ_NOALLOC_BAD_ARGUMENT;
  const long long partial = (long long)B * Hq * splits * D;
  const long long lse = (long long)B * Hq * splits;
  if (partial > SQ_NOALLOC_MAX_PARTIAL_FLOATS || lse > SQ_NOALLOC_MAX_LSE) return SQ_NOALLOC_TOO_LARGE;
  float* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess) return (int)e;
  sq::AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ld_q = ld_q;
  p.k_codes = static_cast<const uint8_t*>(k_codes);
  p.k_scales = static_cast<const __half*>(k_scales);
  p.v_codes = static_cast<const uint8_t*>(v_codes);
  p.v_scales = static_cast<const __half*>(v_scales);
  p.block_tables = block_tables;
  p.bt_stride = bt_stride;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ld_out = ld_out;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.D = D;
  p.page_size = page_size;
  p.group = group;
  p.fmt_k = fmt_k;
  p.fmt_v = fmt_v;
  p.sm_scale = sm_scale;
  p.seq_lens = seq_lens;
  p.B = B;
  p.splits = splits;
  p.tiles_per_split = tiles_per_split;
  p.o_part = scratch;
  p.lse_part = scratch + SQ_NOALLOC_MAX_PARTIAL_FLOATS;
  return (int)sq::paged_decode_attn_launch(p, static_cast<cudaStream_t>(stream));
}

extern "C" __attribute__((visibility("default"))) const char* sq_noalloc_error_string(int code) {
  if (code == 0) return "ok";
  if (code == SQ_NOALLOC_TOO_LARGE)
    return "request too large for the fixed scratch: B*Hq*splits*D must be <= 1048576 and B*Hq*splits <= 32768";
  if (code == SQ_NOALLOC_BAD_ARGUMENT)
    return "invalid argument: needs Hkv > 0, Hq % Hkv == 0, Hq / Hkv <= 16, D in {32, 64, 128}, page_size a "
           "positive multiple of 16, splits >= 1, tiles_per_split >= 1, a supported KV format pair, a KV group "
           ">= 32 dividing D, and row strides of at least Hq * D";
  return cudaGetErrorString(static_cast<cudaError_t>(code));
}
