// noalloc_decode.h — an allocation-free C entry point for paged decode attention.
//
// This entry point has no counterpart in the reference framework; it exists for callers
// of this library that cannot allocate device memory themselves: code that runs inside
// another runtime's memory budget with no allocator handle (a plug-in loaded by a host
// application that owns every cudaMalloc, a foreign-language binding that only passes
// pointers, or a host path that must not call into an allocator at all). They pass
// inputs and outputs; the split-K partials the kernel needs live in a fixed,
// file-scope device array instead of a caller-provided workspace.
//
// Declaration (exported with C linkage from the squish_b200._C shared library):
//
//   int sq_paged_decode_attention_noalloc(
//       const void* q, int ld_q,                      // bf16 [B, ld_q], Hq*D values per row
//       const void* k_codes, const void* k_scales,    // KV page pools of one layer
//       const void* v_codes, const void* v_scales,
//       const int* block_tables, int bt_stride,       // int32 [B, bt_stride]
//       const int* seq_lens, int B,                   // int32 [B], KV length incl. the new token
//       void* out, int ld_out,                        // bf16 [B, ld_out]
//       int Hq, int Hkv, int D, int page_size, int group, int fmt_k, int fmt_v,
//       float sm_scale, int splits, int tiles_per_split, void* stream);
//
// Returns 0 on success; SQ_NOALLOC_TOO_LARGE if B*Hq*splits*D exceeds
// SQ_NOALLOC_MAX_PARTIAL_FLOATS or B*Hq*splits exceeds SQ_NOALLOC_MAX_LSE;
// SQ_NOALLOC_BAD_ARGUMENT if the shape is one the kernel does not handle (Hkv <= 0,
// Hq not a multiple of Hkv, more than 16 query heads per KV head, D not 32/64/128,
// page_size not a positive multiple of 16, splits or tiles_per_split below 1, a KV
// format pair other than bf16/int8/int4/int2 for both or k8 keys with v4 values, a KV
// group below 32 or not dividing D, or a q/out row stride below Hq*D); otherwise a CUDA
// error code. Nothing is launched when a check fails. sq_noalloc_error_string() turns a
// return code into a message.
//
// Scratch: one static device array of SQ_NOALLOC_MAX_PARTIAL_FLOATS + SQ_NOALLOC_MAX_LSE
// floats (4.125 MiB), present on every GPU that loads the library until the process exits.
// All calls share it: calls that overlap on the GPU (different streams, or different
// host threads on one stream without ordering) race on it. Every partial a call reads is
// written earlier in the same call, so no part of it has to start at zero.
//
// Set-up: the first call on each device (with that device current) looks up the array's
// device address with cudaGetSymbolAddress and caches it; make that first call before
// any stream capture on the device. The cached address belongs to the device's current
// context: after cudaDeviceReset on a device the cache is stale, so a process that resets
// a device must not call this entry point on it again.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

#define SQ_NOALLOC_MAX_PARTIAL_FLOATS (1 << 20)
#define SQ_NOALLOC_MAX_LSE (1 << 15)
#define SQ_NOALLOC_TOO_LARGE (-1)
#define SQ_NOALLOC_BAD_ARGUMENT (-2)

int sq_paged_decode_attention_noalloc(const void* q, int ld_q, const void* k_codes, const void* k_scales,
                                      const void* v_codes, const void* v_scales, const int* block_tables,
                                      int bt_stride, const int* seq_lens, int B, void* out, int ld_out, int Hq,
                                      int Hkv, int D, int page_size, int group, int fmt_k, int fmt_v, float sm_scale,
                                      int splits, int tiles_per_split, void* stream);

const char* sq_noalloc_error_string(int code);

#ifdef __cplusplus
}
#endif
