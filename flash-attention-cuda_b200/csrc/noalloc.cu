// fa_decode_noalloc: the decode step for callers that cannot allocate GPU
// memory.
//
// fa_decode needs scratch memory (log-sum-exp partials of sequences that
// several CTAs share, and one arrival counter per (batch, head)), which its
// callers normally provide. Some callers cannot: code running inside a
// framework that forbids cudaMalloc after start-up (a serving engine whose
// memory pool is fixed at launch), plugins that only receive pointers to
// their inputs and outputs, or hosts with no allocator hooked up to the
// CUDA context. For them this entry point keeps its scratch in a fixed
// file-scope device array, so the library itself allocates nothing at any
// time. The array is part of the library image: every GPU that loads the
// library holds it (about 2.5 MB) until the process exits.
//
// Host code cannot pass the array's name to a kernel: on the host that name
// is only a stand-in symbol, not a device address. The device address is
// looked up once per device with cudaGetSymbolAddress, with that device
// current, on the first call made on the device.

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "fa_b200.h"
#include "fa_kernels.h"

namespace fa {
namespace noalloc {

// Largest batch * heads one call may use, and the largest grid the automatic
// schedule may launch (2 CTAs per SM; a B200 has 148 SMs).
constexpr int kMaxSegments = FA_NOALLOC_MAX_BH;
constexpr int kMaxGrid = 1024;
constexpr size_t kCounterBytes = static_cast<size_t>(kMaxSegments) * 4;
constexpr size_t kPartialBytes = static_cast<size_t>(kMaxSegments + kMaxGrid) *
                                 kPartialFloats * sizeof(float);
constexpr size_t kScratchBytes = kCounterBytes + kPartialBytes;
static_assert(kCounterBytes % 256 == 0, "partials must stay 256-byte aligned");

// [counters: kMaxSegments uint32][partials: (kMaxSegments + kMaxGrid) x 68 f32]
static __device__ __align__(256) uint8_t g_scratch[kScratchBytes];

struct DeviceScratch {
  bool ready = false;
  cudaError_t status = cudaSuccess;
  uint8_t *ptr = nullptr;
};

std::mutex g_mutex;
DeviceScratch g_scratch_of[kMaxDevices];

// Device address of g_scratch on the current device (set-up on first use).
int scratch_address(int dev, uint8_t **out) {
  if (dev < 0 || dev >= kMaxDevices) return FA_EDEVICE;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceScratch &d = g_scratch_of[dev];
  if (!d.ready) {
    // A failed look-up is not cached: the next call on this device tries
    // again instead of failing for the rest of the process.
    void *p = nullptr;
    d.status = cudaGetSymbolAddress(&p, g_scratch);
    if (d.status != cudaSuccess || p == nullptr) {
      cudaGetLastError();  // clear the runtime's last-error record
      return FA_ECUDA;
    }
    d.ptr = static_cast<uint8_t *>(p);
    d.ready = true;
  }
  *out = d.ptr;
  return FA_OK;
}

}  // namespace noalloc
}  // namespace fa

extern "C" int fa_decode_noalloc(const void *q, const void *k_cache,
                                 const void *v_cache, const int32_t *seq_lens,
                                 void *o, int B, int H, int S_max, float scale,
                                 void *stream) {
  using namespace fa;
  if (B <= 0 || H <= 0) return FA_EINVAL;
  if (static_cast<long long>(B) * H > noalloc::kMaxSegments)
    return FA_ENOSPACE;  // beyond the fixed scratch array
  // The checks run_decode makes, made here too so a rejected call writes
  // nothing to the shared array (the counter clear below comes first).
  if (!decode_shape_ok(B, H, S_max, scale)) return FA_EINVAL;
  if (!q || !k_cache || !v_cache || !seq_lens || !o) return FA_EINVAL;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) ||
      !aligned16(o) || (reinterpret_cast<uintptr_t>(seq_lens) & 3u))
    return FA_EALIGN;
  int dev = 0;
  int rc = ensure_device(&dev);
  if (rc != FA_OK) return rc;
  const int grid = decode_grid(g_devices[dev].sms, B, H, S_max, 0);
  if (grid > noalloc::kMaxGrid) return FA_ENOSPACE;
  uint8_t *scratch = nullptr;
  rc = noalloc::scratch_address(dev, &scratch);
  if (rc != FA_OK) return rc;
  // The counters must start at zero. A completed call leaves them at zero,
  // but one that was abandoned (device error) may not, so clear the ones
  // this call uses; the memset is ordered on the caller's stream.
  uint32_t *counters = reinterpret_cast<uint32_t *>(scratch);
  const size_t n_seg = static_cast<size_t>(B) * H;
  if (cudaMemsetAsync(counters, 0, n_seg * 4,
                      static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return FA_ECUDA;
  return run_decode(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, S_max,
                    scale, 0, scratch + noalloc::kCounterBytes,
                    noalloc::kPartialBytes, counters, n_seg, stream);
}
