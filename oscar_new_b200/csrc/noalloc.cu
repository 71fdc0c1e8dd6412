// Decode-step entry point that performs no device allocation of any kind.
//
// Who needs it: callers that cannot call cudaMalloc at decode time.  A serving engine
// that has already handed all free device memory to its KV-cache pool cannot get a new
// buffer without breaking its memory plan, and a host reaching this library through a
// plain C FFI may have no device allocator at all.  Such callers still provide every
// input and the output buffer, but not the split-KV scratch that
// oscar_decode_attention needs.
//
// How: the scratch lives in file-scope __device__ arrays of a fixed size, loaded with
// the library on every GPU that loads it and held until the process exits.  Host code
// cannot use those array names as device addresses, so the first call on each device
// asks the runtime for their addresses (cudaGetSymbolAddress, with that device current)
// and caches them; that first call should be made before any stream capture starts, and
// a first call made while its stream is capturing is refused (OSCAR_ERR_INVALID) rather
// than risk invalidating the capture.  The cached addresses belong to the device's
// primary context, the one the CUDA runtime uses: after cudaDeviceReset, or when the
// caller drives the device through another context, they are not valid for it.
// Every call on a device shares the same arrays and leaves its partials behind: calls
// whose GPU work overlaps (two streams, two threads) race on them.  Nothing has to be
// zeroed between calls, because each decode step writes every partial row it reads.
#include <mutex>

#include "common.cuh"

namespace oscar {

// Capacity: rows = tokens * query_heads * (splits + 1) split partials of 256 fp32.
constexpr int64_t kNoAllocMaxRows = 32768;                      // 32 MiB of partials
static __device__ __align__(256) float g_noalloc_partials[kNoAllocMaxRows * kDim];
static __device__ __align__(256) float g_noalloc_lse[kNoAllocMaxRows];

constexpr int kMaxDevices = 64;
static float *g_partials_addr[kMaxDevices];
static float *g_lse_addr[kMaxDevices];
static std::mutex g_setup_mutex;

static int noalloc_scratch(float **partials, float **lse, cudaStream_t stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return OSCAR_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_partials_addr[dev]) {
    // the address lookup is a runtime call that must not land inside a stream capture
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
      cudaGetLastError();
      return OSCAR_ERR_LAUNCH;
    }
    if (cap != cudaStreamCaptureStatusNone) return OSCAR_ERR_INVALID;
    void *p = nullptr, *l = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_partials) != cudaSuccess ||
        cudaGetSymbolAddress(&l, g_noalloc_lse) != cudaSuccess) {
      cudaGetLastError();
      return OSCAR_ERR_LAUNCH;
    }
    g_partials_addr[dev] = static_cast<float *>(p);
    g_lse_addr[dev] = static_cast<float *>(l);
  }
  *partials = g_partials_addr[dev];
  *lse = g_lse_addr[dev];
  return OSCAR_OK;
}

}  // namespace oscar

using namespace oscar;

extern "C" int64_t oscar_decode_attention_noalloc_max_rows(void) { return kNoAllocMaxRows; }

extern "C" int oscar_decode_attention_noalloc(const void *qrot, const void *query, int64_t qs0, int64_t qs1,
                                              const void *key, int64_t ks0, int64_t ks1, const void *value,
                                              int64_t vs0, int64_t vs1, const uint8_t *history, void *window,
                                              const int32_t *qstarts, const int32_t *seq_lens,
                                              const int32_t *table, const int32_t *counts, const int32_t *tasks,
                                              const int32_t *task_count, int32_t num_tasks, int64_t n,
                                              const void *rv, void *output, oscar_geometry geo, float scale,
                                              int32_t splits, int32_t window_programs, int32_t *status,
                                              void *stream) {
  // bound every factor before multiplying, so the row count cannot overflow
  if (n < 0 || splits <= 0 || splits > 64 || geo.kv_heads <= 0 || geo.group <= 0) return OSCAR_ERR_INVALID;
  if (n > kNoAllocMaxRows || geo.kv_heads > kNoAllocMaxRows || geo.group > kNoAllocMaxRows) return OSCAR_ERR_INVALID;
  const int64_t per_token = (int64_t)geo.kv_heads * geo.group * (splits + 1);  // < 2^15 * 2^15 * 65
  if (per_token > kNoAllocMaxRows || n > kNoAllocMaxRows / per_token) return OSCAR_ERR_INVALID;  // beyond the scratch
  if (n == 0) return OSCAR_OK;
  float *partials = nullptr, *lse = nullptr;
  const int rc = noalloc_scratch(&partials, &lse, (cudaStream_t)stream);
  if (rc != OSCAR_OK) return rc;
  return oscar_decode_attention(qrot, query, qs0, qs1, key, ks0, ks1, value, vs0, vs1, history, window, qstarts,
                                seq_lens, table, counts, tasks, task_count, num_tasks, n, rv, partials, lse, output,
                                geo, scale, splits, window_programs, status, stream);
}
