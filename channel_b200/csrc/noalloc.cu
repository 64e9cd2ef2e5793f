// noalloc.cu -- ch_gemv_q4_noalloc: the Q4 decode matvec for callers that may
// not allocate device memory.
//
// The ordinary entry point (ch_gemv_q4) keeps its stream-K scratch -- one
// partial-sum slot per warp and one arrival counter per 16-row tile -- in a
// ch_ctx, which allocates it on first use.  Some callers cannot allow that: a
// host runtime whose own pool allocator already holds the device's memory
// (a cudaMalloc beside it fails or breaks the pool's accounting), a serving
// loop that bans cudaFree in steady state because it synchronizes the whole
// device, and bindings (JNI, cgo, N-API) that hand over buffers owned by
// another runtime and expect the callee to take nothing more.  For them this
// file keeps that scratch in one static device array, reserved when the CUDA
// module is loaded and held by every GPU that loads the library until the
// process exits.
//
// Limits (the array is sized for them; larger calls are rejected with
// CH_EINVAL): rows <= 32768, cols <= 16384, and a grid of at most 148 CTAs
// (one per SM of a B200).
#include <mutex>
#include <string>

#include "../../include/channel_cuda.h"
#include "common.cuh"
#include "kernels.cuh"

namespace ch {
int set_last_error(int code, const std::string &msg);
}
using namespace ch;

namespace {
constexpr uint32_t kMaxRows = 32768;
constexpr uint32_t kMaxCols = 16384;
constexpr int kMaxGrid = 148;
constexpr int kMaxDevices = 64;
constexpr size_t kPartialWords = 148 * 16 * 2 * 16;  // gemv_partial_floats(kMaxGrid)
constexpr size_t kCounterWords = kMaxRows / 16;      // one per 16-row tile
constexpr size_t kScratchWords = kPartialWords + kCounterWords + 64;  // + status word, padded

// [partials | counters | status].  A host-side name for a device object: its
// device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) uint32_t g_gemv_scratch[kScratchWords];

std::mutex g_mu;
uint32_t *g_scratch_dev[kMaxDevices] = {};

// Device address of g_gemv_scratch on the current device; resolved on the
// first call per device (that call also loads this library's CUDA module on
// the device if nothing has loaded it yet).
int scratch_on_current_device(uint32_t **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_last_error(CH_ECUDA, std::string("gemv_q4_noalloc: cudaGetDevice: ") +
                                                            cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_last_error(CH_EINVAL, "gemv_q4_noalloc: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_dev[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_gemv_scratch);
    if (e != cudaSuccess || !p)
      return set_last_error(CH_ECUDA, std::string("gemv_q4_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_scratch_dev[dev] = static_cast<uint32_t *>(p);
  }
  *out = g_scratch_dev[dev];
  return CH_OK;
}
}  // namespace

extern "C" int ch_gemv_q4_noalloc(const void *tiles, uint32_t rows, uint32_t cols, const float *x, float *y,
                                  uint32_t *status, void *stream) {
  if (!tiles || !x || !y) return set_last_error(CH_EINVAL, "gemv_q4_noalloc: NULL argument");
  if (rows == 0 || rows % 16 || cols == 0 || cols % 64)
    return set_last_error(CH_EINVAL, "gemv_q4_noalloc: rows % 16 == 0 and cols % 64 == 0 required");
  if (rows > kMaxRows || cols > kMaxCols)
    return set_last_error(CH_EINVAL, "gemv_q4_noalloc: " + std::to_string(rows) + " x " + std::to_string(cols) +
                                         " exceeds the static scratch (rows <= 32768, cols <= 16384)");
  uint32_t *scratch = nullptr;
  int rc = scratch_on_current_device(&scratch);
  if (rc != CH_OK) return rc;
  const int grid = num_sms() < kMaxGrid ? num_sms() : kMaxGrid;
  static_assert(kPartialWords >= (size_t)kMaxGrid * 16 * 2 * 16, "partial slots");
  if (gemv_partial_floats(grid) > kPartialWords) return set_last_error(CH_EINVAL, "gemv_q4_noalloc: grid");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t *counters = scratch + kPartialWords;
  uint32_t *own_status = counters + kCounterWords;
  // The counters must be zero when the kernel starts.  A completed launch
  // leaves them zero, but one that gave up on a stalled copy may not; so clear
  // this call's range (and the spare status word) on the stream first.
  cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)(rows / 16) * sizeof(uint32_t), s);
  if (e == cudaSuccess && !status) e = cudaMemsetAsync(own_status, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return set_last_error(CH_ECUDA, std::string("gemv_q4_noalloc: ") + cudaGetErrorString(e));
  GemvArgs a;
  GemvPlan p;
  p.fmt = FMT_Q4;
  p.epi = EPI_STORE;
  p.grid = grid;
  a.tiles = static_cast<const uint8_t *>(tiles);
  a.row_tiles = rows / 16;
  a.k_tiles = cols / 64;
  a.K = cols;
  a.x = x;
  a.y = y;
  a.partial = reinterpret_cast<float *>(scratch);
  a.counters = counters;
  a.err = status ? status : own_status;
  e = launch_gemv(p, a, s, false);
  if (e != cudaSuccess) return set_last_error(CH_ECUDA, std::string("gemv_q4_noalloc: ") + cudaGetErrorString(e));
  return CH_OK;
}
