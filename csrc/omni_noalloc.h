// Allocation-free entry point of the paged decode attention.
//
// This entry point has no counterpart in the reference (sgl-project/sglang-omni
// has no C ABI and no kernels of its own).  It exists for callers that cannot
// call cudaMalloc: code running while a CUDA stream is being captured into a
// graph by another library, host runtimes that hand this library only the
// input and output buffers and forbid it to allocate, and embedders whose
// memory is owned by a custom allocator.  Such callers still pass every input
// and output; the split-KV scratch comes from a static device array inside
// this library instead of a caller-provided workspace.
//
// int omni_attention_decode_noalloc(q, q_stride, k_cache, v_cache, block_table,
//     bt_stride, kv_lens, batch, num_heads, num_kv_heads, head_dim, scale,
//     keys_per_split, max_splits, num_pages, out, out_stride, stream)
//
//   Same math, arguments and layouts as the torch entry `attention_decode`
//   (KV cache [num_pages, num_kv_heads, 64, head_dim] bf16, one query token per
//   request, out [batch, num_heads * head_dim] bf16 rows of out_stride).
//   num_pages is the page count of the cache: block-table entries outside
//   [0, num_pages) read page 0 instead of memory past the cache, and a request
//   reads at most bt_stride * 64 keys whatever its kv_lens entry says.  A
//   request with kv_lens <= 0 gets a zero output row.
//   Returns 0 on success, a cudaError_t value on a CUDA error,
//   OMNI_NOALLOC_ERR_INVALID (with a message on stderr) for arguments the
//   kernel cannot take (num_heads or num_kv_heads <= 0 or not dividing, more
//   than 16 query heads per KV head, head_dim other than 64 / 128,
//   keys_per_split not a positive multiple of 64, max_splits or num_pages < 1,
//   a negative block-table stride, row strides shorter than a row, or a null
//   pointer with batch > 0), or OMNI_NOALLOC_ERR_TOO_LARGE when
//   batch * num_heads * max_splits * head_dim exceeds
//   OMNI_NOALLOC_DECODE_PART_FLOATS or batch * num_heads * max_splits exceeds
//   OMNI_NOALLOC_DECODE_LSE_FLOATS.  Both checks run before anything is
//   launched.
//
//   It calls no cudaMalloc, cudaFree or allocating library routine.  The first
//   call on each device resolves the scratch array's device address
//   (cudaGetSymbolAddress, with that device current); make that first call
//   before any stream capture.  A lookup that fails is not remembered: the next
//   call tries again.  All calls share the one array and it keeps the
//   previous call's contents; this kernel writes every scratch element it later
//   reads, so nothing needs clearing between calls.  Calls whose executions
//   overlap on the GPU (different streams, or concurrent graph replays) race on
//   the array: serialise them.
#pragma once

#define OMNI_NOALLOC_DECODE_PART_FLOATS (4LL * 1024 * 1024)  // 16 MiB of fp32 partial outputs
#define OMNI_NOALLOC_DECODE_LSE_FLOATS (64LL * 1024)         // 256 KiB of fp32 log-sum-exps
#define OMNI_NOALLOC_ERR_TOO_LARGE (-1)
#define OMNI_NOALLOC_ERR_INVALID (-2)

#ifdef __cplusplus
extern "C" {
#endif
int omni_attention_decode_noalloc(const void* q, long long q_stride, const void* k_cache, const void* v_cache,
                                  const int* block_table, int bt_stride, const int* kv_lens, int batch,
                                  int num_heads, int num_kv_heads, int head_dim, float scale, int keys_per_split,
                                  int max_splits, int num_pages, void* out, long long out_stride, void* stream);
#ifdef __cplusplus
}
#endif
