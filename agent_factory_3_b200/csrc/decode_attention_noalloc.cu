// Allocation-free C entry point of the paged decode attention.
//
// This entry point has no counterpart in the reference.  The reference leaves decode
// attention to its serving engine; here the same split-KV kernels as the torch entry point
// `decode_attention` are launched, but the split partials (per request, head and KV chunk: a
// 64-float partial output plus its running max and sum) live in one fixed-size static device
// array instead of tensors allocated per call.
//
// Who needs it: callers that must not allocate device memory while they decode.
//   * A C or C++ host without PyTorch.  It has no caching allocator to borrow from, so every
//     temporary would be a cudaMalloc/cudaFree, and those can synchronise the whole device in
//     the middle of a decode loop that otherwise only enqueues work.
//   * A server that hands all free device memory to its KV pages at start-up.  Any later
//     allocation can fail under load, so the decode step must not make one.
//   * Code that runs inside an allocator's own callbacks or out-of-memory handling, where
//     allocating again would re-enter the allocator.
// The entry point calls no cudaMalloc/cudaFree, no allocating library function and nothing
// of torch; it only launches the two kernels on the caller's stream.
//
// Scratch limit: kScratchBytes (16 MiB) per device.  A call needs
//     batch * num_q_heads * chunks * 66 * 4 bytes,  chunks = ceil(max_seq_len / (16 * page_size)),
// e.g. 64 requests x 64 heads x 15 chunks (15360 tokens at page size 64) fits.  Larger calls
// are rejected with AF3_NOALLOC_TOO_LARGE before anything is launched; split the batch.
//
// Set-up: the first call on a device (or an explicit af3_decode_attention_noalloc_init() with
// that device current) looks up the scratch array's device address with cudaGetSymbolAddress
// and caches it for that device.  That lookup can load this module onto the device, so make
// the first call (or the init call) on each device before any stream capture begins.
//
// Nothing in the scratch has to start at zero: every launch writes each partial slot it will
// read (chunks past a request's length write an empty partial), so no clearing is needed.
//
// Concurrency: all calls on one device share the one scratch array.  Two calls whose kernels
// can overlap on the device (different streams without ordering between them, or several
// host threads on separate streams) race on it and give wrong results.  Serialise the calls
// of a device, e.g. issue them all on one stream.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "decode_attention_kernels.cuh"
#include "decode_attention_noalloc.h"

namespace {
constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr size_t kScratchFloats = kScratchBytes / sizeof(float);
}  // namespace

// The scratch itself: one per device, part of this module's device image.  Host code must
// not pass this name to a kernel: on the host it is a stand-in, not the device address.
static __device__ __align__(256) float g_decode_scratch[kScratchFloats];

namespace {

constexpr int kMaxDevices = 64;
constexpr int kFloatsPerPartial = af3::dec::kD + 2;  // partial output + (max, sum)

std::atomic<float*> g_scratch_ptr[kMaxDevices] = {};
std::mutex g_setup_mutex;
thread_local char g_last_error[256] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

// Address of the current device's scratch, looked up once per device.
int scratch_for_current_device(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return fail(AF3_NOALLOC_CUDA_ERROR, "cudaGetDevice failed: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(AF3_NOALLOC_INVALID_ARGUMENT, "device %d outside the supported 0..%d", dev,
                kMaxDevices - 1);
  float* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (p == nullptr) {
      void* sym = nullptr;
      e = cudaGetSymbolAddress(&sym, g_decode_scratch);
      if (e != cudaSuccess || sym == nullptr)
        return fail(AF3_NOALLOC_CUDA_ERROR, "cudaGetSymbolAddress of the decode scratch failed: %s",
                    cudaGetErrorString(e));
      p = static_cast<float*>(sym);
      g_scratch_ptr[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return AF3_NOALLOC_OK;
}

}  // namespace

extern "C" {

// Bytes of device scratch available to one call.
__attribute__((visibility("default"))) size_t af3_decode_attention_noalloc_scratch_bytes() {
  return kScratchBytes;
}

// Message of the last failed call on this host thread ("" after a successful call).
__attribute__((visibility("default"))) const char* af3_decode_attention_noalloc_last_error() {
  return g_last_error;
}

// Looks up the scratch of the CURRENT device.  Optional: the first decode call on a device
// does the same.  Call it before any stream capture.  Returns 0 or an error code.
__attribute__((visibility("default"))) int af3_decode_attention_noalloc_init() {
  float* p = nullptr;
  const int rc = scratch_for_current_device(&p);
  if (rc == AF3_NOALLOC_OK) g_last_error[0] = '\0';
  return rc;
}

// Paged decode attention of one new query token per request, same semantics as the torch
// entry point decode_attention:
//   q          bf16, request b's heads at q + b * ld_q (Hq x 64 contiguous)
//   k_pages    bf16 [num_pages, page_size, Hkv, 64], v_pages likewise
//   page_table int32 [batch, max_pages]; seq_lens int32 [batch] (context incl. the new token)
//   sinks      fp32 [Hq]; out bf16, request b at out + b * ld_out (Hq x 64)
//   lse        optional fp32 [batch, Hq] (natural log), may be null
//   window     sliding window in tokens (0 = full), scale = softmax scale
//   max_seq_len  upper bound of seq_lens (sets the number of KV chunks)
// All pointers are device pointers of the current device; the kernels run on `stream`.
// Returns 0 on success; otherwise an error code (1 invalid argument, 2 needs more scratch
// than kScratchBytes, 3 CUDA error) and af3_decode_attention_noalloc_last_error() says why.
__attribute__((visibility("default"))) int af3_decode_attention_noalloc(
    const void* q, long long ld_q, const void* k_pages, const void* v_pages,
    const int* page_table, int max_pages, const int* seq_lens, const float* sinks, void* out,
    long long ld_out, float* lse, int batch, int num_q_heads, int num_kv_heads, int page_size,
    int window, float scale, int max_seq_len, cudaStream_t stream) {
  using namespace af3::dec;
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || page_size <= 0 || max_pages <= 0 ||
      max_seq_len < 0 || window < 0)
    return fail(AF3_NOALLOC_INVALID_ARGUMENT,
                "bad sizes: heads, page_size and max_pages must be positive, batch, window and "
                "max_seq_len non-negative");
  if (num_q_heads % num_kv_heads != 0)
    return fail(AF3_NOALLOC_INVALID_ARGUMENT, "num_q_heads %d is not a multiple of num_kv_heads %d",
                num_q_heads, num_kv_heads);
  const int G = num_q_heads / num_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16)
    return fail(AF3_NOALLOC_INVALID_ARGUMENT, "GQA group %d unsupported (1, 2, 4, 8 or 16)", G);
  if ((long long)max_seq_len > (long long)max_pages * page_size)
    return fail(AF3_NOALLOC_INVALID_ARGUMENT, "max_seq_len %d exceeds the page table's %lld tokens",
                max_seq_len, (long long)max_pages * page_size);
  if (batch > 0 && (!q || !k_pages || !v_pages || !page_table || !seq_lens || !sinks || !out))
    return fail(AF3_NOALLOC_INVALID_ARGUMENT, "null device pointer");
  // The kernels read q and the K/V page rows with 16-byte vector loads and write out per
  // bf16 element; a misaligned operand would fault on the device, so refuse it here.
  const long long row_elems = (long long)num_q_heads * kD;
  auto misaligned = [](const void* ptr, uintptr_t a) {
    return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) != 0;
  };
  if (batch > 0) {
    if (misaligned(q, 16) || misaligned(k_pages, 16) || misaligned(v_pages, 16))
      return fail(AF3_NOALLOC_INVALID_ARGUMENT, "q, k_pages and v_pages must be 16-byte aligned");
    if (ld_q % 8 != 0 || ld_q < row_elems)
      return fail(AF3_NOALLOC_INVALID_ARGUMENT,
                  "ld_q %lld must be a multiple of 8 and at least num_q_heads * 64 = %lld", ld_q,
                  row_elems);
    if (ld_out < row_elems)
      return fail(AF3_NOALLOC_INVALID_ARGUMENT, "ld_out %lld is below num_q_heads * 64 = %lld",
                  ld_out, row_elems);
    if (misaligned(out, 2) || misaligned(page_table, 4) || misaligned(seq_lens, 4) ||
        misaligned(sinks, 4) || (lse && misaligned(lse, 4)))
      return fail(AF3_NOALLOC_INVALID_ARGUMENT,
                  "out must be 2-byte aligned; page_table, seq_lens, sinks and lse 4-byte aligned");
  }
  const long long chunk_tokens = (long long)kChunkPages * page_size;
  const long long chunks = max_seq_len > 0 ? (max_seq_len + chunk_tokens - 1) / chunk_tokens : 1;
  const long long need = (long long)batch * num_q_heads * chunks * kFloatsPerPartial;
  if (need > (long long)kScratchFloats)
    return fail(AF3_NOALLOC_TOO_LARGE,
                "decode call needs %lld bytes of scratch but the static scratch holds %lld bytes; "
                "split the batch", need * (long long)sizeof(float), (long long)kScratchBytes);
  float* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != AF3_NOALLOC_OK) return rc;
  g_last_error[0] = '\0';
  if (batch == 0) return AF3_NOALLOC_OK;

  Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ld_q = ld_q;
  p.kp = static_cast<const __nv_bfloat16*>(k_pages);
  p.vp = static_cast<const __nv_bfloat16*>(v_pages);
  p.page_table = page_table;
  p.max_pages = max_pages;
  p.seq_lens = seq_lens;
  p.part_o = scratch;                                               // [B, Hq, chunks, 64]
  p.part_ml = scratch + (size_t)batch * num_q_heads * chunks * kD;  // [B, Hq, chunks, 2]
  p.page_size = page_size;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.window = window;
  p.chunks = (int)chunks;
  p.scale_log2 = scale * 1.4426950408889634f;
  const dim3 grid((unsigned)chunks, (unsigned)num_kv_heads, (unsigned)batch);
  switch (G) {
    case 1: decode_attn_kernel<1><<<grid, kWarps * 32, 0, stream>>>(p); break;
    case 2: decode_attn_kernel<2><<<grid, kWarps * 32, 0, stream>>>(p); break;
    case 4: decode_attn_kernel<4><<<grid, kWarps * 32, 0, stream>>>(p); break;
    case 8: decode_attn_mma_kernel<<<grid, kWarps * 32, 0, stream>>>(p); break;   // tensor cores
    default: decode_attn_kernel<16><<<grid, kWarps * 32, 0, stream>>>(p); break;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(AF3_NOALLOC_CUDA_ERROR, "decode kernel launch failed: %s", cudaGetErrorString(e));
  decode_combine_kernel<<<dim3((unsigned)num_q_heads, (unsigned)batch), kD, 0, stream>>>(
      p.part_o, p.part_ml, sinks, static_cast<__nv_bfloat16*>(out), ld_out, num_q_heads,
      (int)chunks, lse);
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(AF3_NOALLOC_CUDA_ERROR, "combine kernel launch failed: %s", cudaGetErrorString(e));
  return AF3_NOALLOC_OK;
}

}  // extern "C"
