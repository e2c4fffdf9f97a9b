// C interface of the allocation-free paged decode attention (libaf3 extension library,
// defined in decode_attention_noalloc.cu).
//
// This interface has no counterpart in the reference.  It exists for callers that cannot
// allocate device memory while they decode: a C or C++ host without PyTorch (no caching
// allocator, and cudaMalloc/cudaFree can synchronise the device mid-loop), a server that gave
// all free device memory to its KV pages at start-up, or code running inside an allocator's
// own out-of-memory handling.  The call launches two kernels on the caller's stream; its
// split-KV partials live in one static 16 MiB device array per device instead of per-call
// buffers.  Calls on one device share that array, so calls whose kernels can overlap on the
// device race; issue them on one stream.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes.
#define AF3_NOALLOC_OK 0
#define AF3_NOALLOC_INVALID_ARGUMENT 1  // bad size, pointer, alignment or stride
#define AF3_NOALLOC_TOO_LARGE 2         // needs more than af3_decode_attention_noalloc_scratch_bytes()
#define AF3_NOALLOC_CUDA_ERROR 3        // a CUDA runtime call or launch failed

// Bytes of device scratch one call may use (16 MiB).  A call needs
// batch * num_q_heads * ceil(max_seq_len / (16 * page_size)) * 264 bytes.
size_t af3_decode_attention_noalloc_scratch_bytes(void);

// Message of the last failed call on this host thread ("" after a success).
const char* af3_decode_attention_noalloc_last_error(void);

// Looks up the scratch array of the CURRENT device (optional: the first decode call on a
// device does the same).  Make this call, or the first decode call, on every device before
// any stream capture starts.  Returns an AF3_NOALLOC_* code.
int af3_decode_attention_noalloc_init(void);

// Decode attention of one new query token per request over a paged bf16 KV cache, with
// learned per-head sinks and an optional sliding window (same results as the library's
// torch entry point).  Shapes, in elements:
//   q           bf16, request b's Hq x 64 query at q + b * ld_q; 16-byte aligned, ld_q a
//               multiple of 8 and >= num_q_heads * 64
//   k_pages,    bf16 [num_pages, page_size, num_kv_heads, 64]; 16-byte aligned
//   v_pages
//   page_table  int32 [batch, max_pages]; seq_lens int32 [batch] (context incl. new token)
//   sinks       fp32 [num_q_heads]
//   out         bf16, request b's Hq x 64 output at out + b * ld_out; ld_out >= Hq * 64
//   lse         optional fp32 [batch, num_q_heads] natural-log normaliser, may be NULL
//   window      sliding window in tokens (0 = full); scale = softmax scale
//   max_seq_len upper bound of seq_lens; num_q_heads / num_kv_heads in {1, 2, 4, 8, 16}
// Every pointer is a device pointer of the current device.  Returns an AF3_NOALLOC_* code;
// on failure nothing was launched and af3_decode_attention_noalloc_last_error() says why.
int af3_decode_attention_noalloc(const void* q, long long ld_q, const void* k_pages,
                                 const void* v_pages, const int* page_table, int max_pages,
                                 const int* seq_lens, const float* sinks, void* out,
                                 long long ld_out, float* lse, int batch, int num_q_heads,
                                 int num_kv_heads, int page_size, int window, float scale,
                                 int max_seq_len, cudaStream_t stream);

#ifdef __cplusplus
}  // extern "C"
#endif
