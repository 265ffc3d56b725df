// Scratch-free C entry point of the paged-KV decode attention.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that cannot allocate GPU memory while they run: a
// host program that plans all of its device memory at start-up and forbids
// allocation afterwards, or a plugin loaded into another runtime that must not
// touch that runtime's allocator (or call cudaMalloc behind its back).  The
// ordinary entry point (`paged_decode_attn` in the Python extension) takes
// its split-K scratch (partial outputs and log-sum-exps) from PyTorch's
// allocator; this one never allocates.  Its scratch is one file-scope device
// array of LRL_DECODE_NOALLOC_SCRATCH_BYTES (8 MiB) that every GPU which loads
// the library keeps until the process exits.
//
// Contract:
// * The caller passes device pointers to all inputs and to the output, and
//   the stream to launch on.  No cudaMalloc, cudaFree or allocating library
//   routine is called.
// * The first call on a device looks the scratch array's device address up
//   (cudaGetSymbolAddress) with that device current and caches it; make that
//   first call before any stream capture begins.
// * All calls share the one array, which keeps the last call's contents.
//   Every scratch entry a call reads was written earlier in the same call, so
//   nothing needs clearing between calls.  Calls whose work overlaps on the
//   GPU (several streams, or several host threads) race on the array: order
//   them on one stream.
// * A shape whose split-K scratch would exceed the array is rejected with
//   cudaErrorInvalidValue; lrl_decode_noalloc_last_error() says why.
//
// Layouts are those of the Python entry point: q and out [B, Hq, 128] bf16;
// k_cache/v_cache [num_blocks, block_size, Hk, 128] bf16 (kv_fp8 = 0) or
// fp8 E4M3 (kv_fp8 = 1); block_table [B, max_blocks] int32; seq_lens [B]
// int32.  Returns a cudaError_t value (0 on success).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#define LRL_DECODE_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)

#ifdef __cplusplus
extern "C" {
#endif

int lrl_paged_decode_attn_noalloc(const void* q, const void* k_cache, const void* v_cache, const int* block_table,
                                  const int* seq_lens, void* out, int batch, int num_q_heads, int num_kv_heads,
                                  int block_size, int max_blocks, int kv_fp8, float scale, float k_scale,
                                  float v_scale, int max_len_hint, cudaStream_t stream);

const char* lrl_decode_noalloc_last_error(void);

size_t lrl_decode_noalloc_scratch_bytes(void);

#ifdef __cplusplus
}
#endif
