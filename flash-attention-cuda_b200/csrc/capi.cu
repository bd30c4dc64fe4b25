// C ABI (include/fa_b200.h): argument checks, TMA descriptor construction,
// per-device one-time set-up and kernel launches. No allocation happens here;
// callers own every buffer.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "fa_b200.h"
#include "fa_kernels.h"
#include "fa_sm100.cuh"

namespace fa {

namespace {

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  int status = FA_OK;
  int sms = 0;
};

std::mutex g_mutex;
DeviceState g_devices[kMaxDevices];

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t,
                                  void *, const cuuint64_t *, const cuuint64_t *,
                                  const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

bool aligned16(const void *p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// One-time set-up of the current device: checks it is an sm_100 part, raises
// the kernels' dynamic shared-memory limits and resolves the driver's tensor
// map encoder.
int ensure_device(int *device_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ECUDA;
  if (dev < 0 || dev >= kMaxDevices) return FA_EDEVICE;
  if (device_out) *device_out = dev;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState &st = g_devices[dev];
  if (st.ready) return st.status;
  st.ready = true;
  int major = 0, minor = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) !=
          cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
          cudaSuccess) {
    st.status = FA_ECUDA;
    return st.status;
  }
  if (major != 10 || minor != 0) {
    st.status = FA_EDEVICE;
    return st.status;
  }
  st.sms = sms;
  // Every kernel instantiation: its dynamic shared memory limit, and the
  // whole unified L1/shared array configured as shared memory.
  for (int dt = FA_DTYPE_F16; dt <= FA_DTYPE_BF16; ++dt) {
    const void *big_smem[] = {prefill_kernel_ptr(dt), decode_kernel_ptr(dt),
                              decode_d128_kernel_ptr(dt),
                              prefill_d128_kernel_ptr(dt),
                              decode_gqa_kernel_ptr(64, dt),
                              decode_gqa_kernel_ptr(128, dt),
                              prefill_solo_kernel_ptr(dt),
                              prefill_d128_solo_kernel_ptr(dt),
                              prefill_split_kernel_ptr(dt),
                              prefill_d128_wide_kernel_ptr(dt)};
    const int bytes[] = {prefill_smem_bytes(), decode_smem_bytes(),
                         decode_d128_smem_bytes(), prefill_d128_smem_bytes(),
                         decode_gqa_smem_bytes(64), decode_gqa_smem_bytes(128),
                         prefill_solo_smem_bytes(), prefill_d128_solo_smem_bytes(),
                         prefill_split_smem_bytes(),
                         prefill_d128_wide_smem_bytes()};
    static_assert(sizeof(big_smem) / sizeof(big_smem[0]) ==
                      sizeof(bytes) / sizeof(bytes[0]),
                  "one shared-memory size per kernel");
    for (size_t i = 0; i < sizeof(bytes) / sizeof(bytes[0]); ++i) {
      if (cudaFuncSetAttribute(big_smem[i],
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               bytes[i]) != cudaSuccess ||
          cudaFuncSetAttribute(big_smem[i],
                               cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared) != cudaSuccess) {
        st.status = FA_ECUDA;
        return st.status;
      }
    }
  }
  if (!g_encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault,
                                &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr) {
      st.status = FA_EDEVICE;
      return st.status;
    }
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  st.status = FA_OK;
  return st.status;
}

// (B*H, N, 64) fp16 view of a (B, H, N, 64) tensor, 128-row x 64-column
// boxes written with the 128-byte swizzle; rows past N read as zero.
// Boxes are always 64 columns (128 bytes, the swizzle span); a 128-wide
// head is loaded as two boxes at columns 0 and 64.
int make_bhnd_map(CUtensorMap *map, const void *base, int BH, int N, int D,
                  int box_rows, int dtype = FA_DTYPE_F16) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D),
                        static_cast<cuuint64_t>(N),
                        static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                           static_cast<cuuint64_t>(N) * D * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map,
                        dtype == FA_DTYPE_BF16
                            ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        3,
                        const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FA_OK : FA_EINVAL;
}

int decode_grid(int sms, int B, int H, int S_max, int split_size) {
  const long long cap_rows = static_cast<long long>(B) * H * S_max;
  if (split_size > 0) {
    const long long g = (cap_rows + split_size - 1) / split_size;
    return static_cast<int>(g < 1 ? 1 : g);
  }
  const long long by_rows =
      (cap_rows + decode_min_rows_per_cta() - 1) / decode_min_rows_per_cta();
  long long g = static_cast<long long>(sms) * decode_ctas_per_sm();
  if (by_rows < g) g = by_rows;
  return static_cast<int>(g < 1 ? 1 : g);
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

size_t workspace_bytes_for(int B, int H, int grid) {
  return (static_cast<size_t>(B) * H + grid) * kPartialFloats * sizeof(float);
}

// Grouped-query decode: segments are (b, K/V head, chunk of up to
// decode_gqa_max_heads() query heads); partial slots hold one 68-float
// record per query head of a segment.
struct GqaPlan {
  int n_seg_per_b;   // segments per batch entry
  int heads_per_seg; // query heads per segment (at most 16)
};

GqaPlan gqa_plan(int H, int H_kv) {
  const int group = H / H_kv;
  const int mh = decode_gqa_max_heads();
  GqaPlan p;
  const int n_hc = (group + mh - 1) / mh;
  p.n_seg_per_b = H_kv * n_hc;
  p.heads_per_seg = group < mh ? group : mh;
  return p;
}

// Grouped decode grid: at least kGqaMinRowsPerCta cache rows per CTA, at
// most one CTA per SM, and at most as many CTAs per segment as one round
// of the final merge gathers (measured, B1 H14 H_kv 2 d64: 74 CTAs per
// segment took two gather rounds and 36.9 us at S 131072, 64 took 28.7;
// S 16384 with 1024-row pieces 20.5 us against 26.8 with 128-row pieces).
constexpr long long kGqaMinRowsPerCta = 1024;

int decode_gqa_grid(int sms, int B, const GqaPlan &p, int S_max,
                    int split_size, int head_dim) {
  const long long segs = static_cast<long long>(B) * p.n_seg_per_b;
  const long long cap_rows = segs * S_max;
  long long g;
  if (split_size > 0) {
    g = (cap_rows + split_size - 1) / split_size;
  } else {
    g = (cap_rows + kGqaMinRowsPerCta - 1) / kGqaMinRowsPerCta;
    if (g > sms) g = sms;  // one CTA per SM
    const long long by_merge =
        segs * decode_gqa_merge_batch(head_dim, p.heads_per_seg);
    if (g > by_merge) g = by_merge;
  }
  return static_cast<int>(g < 1 ? 1 : g);
}

size_t gqa_workspace_bytes_for(int B, const GqaPlan &p, int grid,
                               int head_dim = FA_HEAD_DIM) {
  return (static_cast<size_t>(B) * p.n_seg_per_b + grid) * p.heads_per_seg *
         (4 + head_dim) * sizeof(float);
}

bool decode_shape_ok(int B, int H, int S_max, float scale) {
  if (B <= 0 || H <= 0 || S_max <= 0 || !isfinite(scale)) return false;
  const long long rows = static_cast<long long>(B) * H * S_max;
  return rows < (1ll << 40) && static_cast<long long>(B) * H < (1ll << 30);
}

int run_decode_gqa(const void *q, const void *k_cache, const void *v_cache,
                   const int32_t *seq_lens, void *o, float *partial_out, int B,
                   int H, int H_kv, int S_max, float scale, int split_size,
                   void *workspace, size_t workspace_bytes, uint32_t *counters,
                   size_t counter_count, void *stream,
                   const void *k_new = nullptr, const void *v_new = nullptr,
                   float *const *x_peers = nullptr, int x_rank = 0,
                   int x_world = 1, uint32_t x_epoch = 0,
                   int head_dim = FA_HEAD_DIM, int dtype = FA_DTYPE_F16) {
  if (head_dim != FA_HEAD_DIM && (head_dim != 128 || H_kv == H || x_peers ||
                                  partial_out || split_size > 0))
    return FA_EINVAL;
  if (!decode_shape_ok(B, H, S_max, scale)) return FA_EINVAL;
  if (H_kv <= 0 || H % H_kv != 0) return FA_EINVAL;
  if (split_size > 0 && split_size % 4 != 0) return FA_EINVAL;
  if (!q || !k_cache || !v_cache || !seq_lens || (!o && !partial_out) ||
      !workspace || !counters)
    return FA_EINVAL;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) ||
      (o && !aligned16(o)) || (partial_out && !aligned16(partial_out)) ||
      !aligned16(workspace) || (reinterpret_cast<uintptr_t>(seq_lens) & 3u) ||
      (reinterpret_cast<uintptr_t>(counters) & 3u))
    return FA_EALIGN;
  int dev = 0;
  int rc = ensure_device(&dev);
  if (rc != FA_OK) return rc;
  const bool grouped = H_kv < H;
  const GqaPlan plan = gqa_plan(H, H_kv);
  const int grid =
      grouped ? decode_gqa_grid(g_devices[dev].sms, B, plan, S_max, split_size,
                                head_dim)
              : decode_grid(g_devices[dev].sms, B, H, S_max, split_size);
  const size_t need = grouped ? gqa_workspace_bytes_for(B, plan, grid, head_dim)
                              : workspace_bytes_for(B, H, grid);
  if (workspace_bytes < need || counter_count < static_cast<size_t>(B) * H)
    return FA_ENOSPACE;
  if ((k_new == nullptr) != (v_new == nullptr)) return FA_EINVAL;
  if (k_new && (!aligned16(k_new) || !aligned16(v_new))) return FA_EALIGN;
  if (x_peers && (H_kv != H || partial_out || k_new || x_world < 1 ||
                  x_world > 32 || x_rank < 0 || x_rank >= x_world))
    return FA_EINVAL;
  DecodeArgs a{};
  a.dtype = dtype;
  a.x_peers = x_peers;
  a.x_rank = x_rank;
  a.x_world = x_world;
  a.x_epoch = x_epoch;
  a.k_new = static_cast<const __half *>(k_new);
  a.v_new = static_cast<const __half *>(v_new);
  a.k_cache_w = k_new ? static_cast<__half *>(const_cast<void *>(k_cache)) : nullptr;
  a.v_cache_w = k_new ? static_cast<__half *>(const_cast<void *>(v_cache)) : nullptr;
  a.q = static_cast<const __half *>(q);
  a.k = static_cast<const __half *>(k_cache);
  a.v = static_cast<const __half *>(v_cache);
  a.seq_lens = seq_lens;
  a.out = static_cast<__half *>(o);
  a.partial_out = partial_out;
  a.ws_counters = counters;
  a.ws_partials = static_cast<float *>(workspace);
  a.B = B;
  a.H = H;
  a.S_max = S_max;
  a.H_kv = H_kv;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.rows_per_cta = split_size > 0 ? split_size : 0;
  a.grid = grid;
  if (grouped) {
    CUtensorMap tk, tv;
    const int rows = decode_gqa_box_rows(head_dim);
    if (make_bhnd_map(&tk, k_cache, B * H_kv, S_max, head_dim, rows, dtype) !=
            FA_OK ||
        make_bhnd_map(&tv, v_cache, B * H_kv, S_max, head_dim, rows, dtype) !=
            FA_OK)
      return FA_EINVAL;
    return launch_decode_gqa_kernel(a, tk, tv, head_dim,
                                    static_cast<cudaStream_t>(stream)) ==
                   cudaSuccess
               ? FA_OK
               : FA_ECUDA;
  }
  return launch_decode_kernel(a, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? FA_OK
             : FA_ECUDA;
}

int run_decode(const void *q, const void *k_cache, const void *v_cache,
               const int32_t *seq_lens, void *o, float *partial_out, int B,
               int H, int S_max, float scale, int split_size, void *workspace,
               size_t workspace_bytes, uint32_t *counters,
               size_t counter_count, void *stream) {
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, partial_out, B, H, H,
                        S_max, scale, split_size, workspace, workspace_bytes,
                        counters, counter_count, stream);
}

// Prefill for head_dim 64 or 128, fp16 or bf16: argument checks, tensor
// maps and the launch.
int run_prefill(const void *q, const void *k, const void *v, void *o, int B,
                int H, int H_kv, int N, int head_dim, int dtype, int causal,
                float scale, void *stream, long long plan_bh = 0) {
  if (head_dim != FA_HEAD_DIM && head_dim != 128) return FA_EINVAL;
  if (B <= 0 || H <= 0 || N <= 0 || !isfinite(scale)) return FA_EINVAL;
  if (H_kv <= 0 || H % H_kv != 0) return FA_EINVAL;
  if (static_cast<long long>(B) * H >= (1ll << 31) / head_dim ||
      static_cast<long long>(N) >= (1ll << 31))
    return FA_EINVAL;
  if (!q || !k || !v || !o) return FA_EINVAL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return FA_EALIGN;
  int dev = 0;
  int rc = ensure_device(&dev);
  if (rc != FA_OK) return rc;
  CUtensorMap tq, tk, tv;
  const int kv_rows = head_dim == FA_HEAD_DIM ? 128 : 64;
  if (make_bhnd_map(&tq, q, B * H, N, head_dim, 128, dtype) != FA_OK ||
      make_bhnd_map(&tk, k, B * H_kv, N, head_dim, kv_rows, dtype) != FA_OK ||
      make_bhnd_map(&tv, v, B * H_kv, N, head_dim, kv_rows, dtype) != FA_OK)
    return FA_EINVAL;
  const cudaError_t err =
      head_dim == FA_HEAD_DIM
          ? launch_prefill_kernel(tq, tk, tv, static_cast<__half *>(o), B, H,
                                  N, causal != 0, scale, H_kv,
                                  g_devices[dev].sms, dtype,
                                  static_cast<cudaStream_t>(stream), plan_bh)
          : launch_prefill_d128_kernel(tq, tk, tv, static_cast<__half *>(o), B,
                                       H, N, causal != 0, scale, H_kv,
                                       g_devices[dev].sms, dtype,
                                       static_cast<cudaStream_t>(stream));
  return err == cudaSuccess ? FA_OK : FA_ECUDA;
}

}  // namespace

int prefill_chunk_ex(const void *q, const void *k, const void *v, void *o,
                     int B, int H, int H_kv, int N, int head_dim, int dtype,
                     int causal, float scale, void *stream, long long plan_bh) {
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_EINVAL;
  return run_prefill(q, k, v, o, B, H, H_kv, N, head_dim, dtype, causal,
                     scale, stream, plan_bh);
}

}  // namespace fa

using namespace fa;

extern "C" {

int fa_prefill(const void *q, const void *k, const void *v, void *o, int B,
               int H, int N, int causal, float scale, void *stream) {
  return fa_prefill_gqa(q, k, v, o, B, H, H, N, causal, scale, stream);
}

int fa_prefill_hd(const void *q, const void *k, const void *v, void *o, int B,
                  int H, int H_kv, int N, int head_dim, int causal,
                  float scale, void *stream) {
  return run_prefill(q, k, v, o, B, H, H_kv, N, head_dim, FA_DTYPE_F16,
                     causal, scale, stream);
}

int fa_prefill_gqa(const void *q, const void *k, const void *v, void *o, int B,
                   int H, int H_kv, int N, int causal, float scale,
                   void *stream) {
  return run_prefill(q, k, v, o, B, H, H_kv, N, FA_HEAD_DIM, FA_DTYPE_F16,
                     causal, scale, stream);
}

int fa_prefill_ex(const void *q, const void *k, const void *v, void *o, int B,
                  int H, int H_kv, int N, int head_dim, int dtype, int causal,
                  float scale, void *stream) {
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_EINVAL;
  return run_prefill(q, k, v, o, B, H, H_kv, N, head_dim, dtype, causal,
                     scale, stream);
}

int fa_prefill_form(long long bh, int n, int causal, int sms, int *ctas) {
  if (bh <= 0 || n <= 0 || sms <= 0) return -1;
  return prefill_form_of(bh, n, causal != 0, sms, 0, ctas);
}

size_t fa_decode_workspace_bytes(int B, int H, int S_max, int split_size,
                                 int device) {
  if (B <= 0 || H <= 0 || S_max <= 0) return 0;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) !=
      cudaSuccess)
    return 0;
  return workspace_bytes_for(B, H, decode_grid(sms, B, H, S_max, split_size));
}

size_t fa_exchange_bytes(int B, int H, int world) {
  return fa_exchange_bytes_hd(B, H, world, FA_HEAD_DIM);
}

size_t fa_exchange_bytes_hd(int B, int H, int world, int head_dim) {
  if (B <= 0 || H <= 0 || world <= 0 || world > 32) return 0;
  if (head_dim != FA_HEAD_DIM && head_dim != 128) return 0;
  const size_t bh = static_cast<size_t>(B) * H;
  // two banks of partials (alternate epochs) + one counter per segment
  return align_up(2 * bh * world * (4 + head_dim) * sizeof(float) +
                      bh * sizeof(uint32_t),
                  256);
}

int fa_exchange_alloc(size_t bytes, void **buffer, void *ipc_handle) {
  if (!buffer || !ipc_handle || bytes == 0) return FA_EINVAL;
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return FA_ECUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return FA_ECUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *buffer = p;
  return FA_OK;
}

int fa_exchange_open(const void *ipc_handle, void **peer_buffer) {
  if (!ipc_handle || !peer_buffer) return FA_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(peer_buffer, h, cudaIpcMemLazyEnablePeerAccess) ==
                 cudaSuccess
             ? FA_OK
             : FA_ECUDA;
}

int fa_exchange_close(void *peer_buffer) {
  return cudaIpcCloseMemHandle(peer_buffer) == cudaSuccess ? FA_OK : FA_ECUDA;
}

int fa_exchange_free(void *buffer) {
  return cudaFree(buffer) == cudaSuccess ? FA_OK : FA_ECUDA;
}

int fa_decode_exchange(const void *q, const void *k_cache, const void *v_cache,
                       const int32_t *seq_lens, void *o, int B, int H,
                       int S_max, float scale, void *workspace,
                       size_t workspace_bytes, uint32_t *counters,
                       size_t counter_count, float *const *peer_buffers,
                       int rank, int world, uint32_t epoch, void *stream) {
  if (!o || !peer_buffers || epoch == 0) return FA_EINVAL;
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, H,
                        S_max, scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream, nullptr, nullptr, peer_buffers,
                        rank, world, epoch);
}


size_t fa_decode_hd_workspace_bytes(int B, int H, int S_max, int head_dim,
                                    int split_size, int device) {
  if (head_dim == FA_HEAD_DIM)
    return fa_decode_workspace_bytes(B, H, S_max, split_size, device);
  if (head_dim != 128 || B <= 0 || H <= 0 || S_max <= 0) return 0;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) !=
      cudaSuccess)
    return 0;
  const int grid = decode_grid(sms, B, H, S_max, split_size);
  return (static_cast<size_t>(B) * H + grid) * decode_d128_partial_floats() *
         sizeof(float);
}

namespace fa {
namespace {
// head_dim 128, one K/V head per query head (optionally with the append).
int run_decode_d128(const void *q, const void *k_cache, const void *v_cache,
                    const int32_t *seq_lens, void *o, int B, int H, int S_max,
                    float scale, int split_size, void *workspace,
                    size_t workspace_bytes, uint32_t *counters,
                    size_t counter_count, void *stream, const void *k_new,
                    const void *v_new, int dtype = FA_DTYPE_F16,
                    float *const *x_peers = nullptr, int x_rank = 0,
                    int x_world = 1, uint32_t x_epoch = 0) {
  if (!decode_shape_ok(B, H, S_max, scale)) return FA_EINVAL;
  if (split_size > 0 && split_size % 4 != 0) return FA_EINVAL;
  if (!q || !k_cache || !v_cache || !seq_lens || !o || !workspace || !counters)
    return FA_EINVAL;
  if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) ||
      !aligned16(o) || !aligned16(workspace) ||
      (reinterpret_cast<uintptr_t>(seq_lens) & 3u) ||
      (reinterpret_cast<uintptr_t>(counters) & 3u))
    return FA_EALIGN;
  int dev = 0;
  int rc = ensure_device(&dev);
  if (rc != FA_OK) return rc;
  const int grid = decode_grid(g_devices[dev].sms, B, H, S_max, split_size);
  if (workspace_bytes < (static_cast<size_t>(B) * H + grid) *
                            decode_d128_partial_floats() * sizeof(float) ||
      counter_count < static_cast<size_t>(B) * H)
    return FA_ENOSPACE;
  if ((k_new == nullptr) != (v_new == nullptr)) return FA_EINVAL;
  if (k_new && (!aligned16(k_new) || !aligned16(v_new))) return FA_EALIGN;
  if (x_peers && (k_new || x_world < 1 || x_world > 32 || x_rank < 0 ||
                  x_rank >= x_world))
    return FA_EINVAL;
  DecodeArgs a{};
  a.dtype = dtype;
  a.x_peers = x_peers;
  a.x_rank = x_rank;
  a.x_world = x_world;
  a.x_epoch = x_epoch;
  a.k_new = static_cast<const __half *>(k_new);
  a.v_new = static_cast<const __half *>(v_new);
  a.k_cache_w = k_new ? static_cast<__half *>(const_cast<void *>(k_cache)) : nullptr;
  a.v_cache_w = k_new ? static_cast<__half *>(const_cast<void *>(v_cache)) : nullptr;
  a.q = static_cast<const __half *>(q);
  a.k = static_cast<const __half *>(k_cache);
  a.v = static_cast<const __half *>(v_cache);
  a.seq_lens = seq_lens;
  a.out = static_cast<__half *>(o);
  a.partial_out = nullptr;
  a.ws_counters = counters;
  a.ws_partials = static_cast<float *>(workspace);
  a.B = B;
  a.H = H;
  a.S_max = S_max;
  a.H_kv = H;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.rows_per_cta = split_size > 0 ? split_size : 0;
  a.grid = grid;
  return launch_decode_d128_kernel(a, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? FA_OK
             : FA_ECUDA;
}
}  // namespace
}  // namespace fa

int fa_decode_exchange_ex(const void *q, const void *k_cache,
                          const void *v_cache, const int32_t *seq_lens,
                          void *o, int B, int H, int S_max, int head_dim,
                          int dtype, float scale, void *workspace,
                          size_t workspace_bytes, uint32_t *counters,
                          size_t counter_count, float *const *peer_buffers,
                          int rank, int world, uint32_t epoch, void *stream) {
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_EINVAL;
  if (!o || !peer_buffers || epoch == 0) return FA_EINVAL;
  if (head_dim != FA_HEAD_DIM && head_dim != 128) return FA_EINVAL;
  if (head_dim == 128)
    return run_decode_d128(q, k_cache, v_cache, seq_lens, o, B, H, S_max,
                           scale, 0, workspace, workspace_bytes, counters,
                           counter_count, stream, nullptr, nullptr, dtype,
                           peer_buffers, rank, world, epoch);
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, H,
                        S_max, scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream, nullptr, nullptr, peer_buffers,
                        rank, world, epoch, FA_HEAD_DIM, dtype);
}

int fa_decode_hd(const void *q, const void *k_cache, const void *v_cache,
                 const int32_t *seq_lens, void *o, int B, int H, int S_max,
                 int head_dim, float scale, int split_size, void *workspace,
                 size_t workspace_bytes, uint32_t *counters,
                 size_t counter_count, void *stream) {
  if (head_dim == FA_HEAD_DIM)
    return fa_decode(q, k_cache, v_cache, seq_lens, o, B, H, S_max, scale,
                     split_size, workspace, workspace_bytes, counters,
                     counter_count, stream);
  if (head_dim != 128) return FA_EINVAL;
  return run_decode_d128(q, k_cache, v_cache, seq_lens, o, B, H, S_max, scale,
                         split_size, workspace, workspace_bytes, counters,
                         counter_count, stream, nullptr, nullptr);
}

int fa_decode_append_hd(const void *q, const void *k_new, const void *v_new,
                        void *k_cache, void *v_cache, const int32_t *seq_lens,
                        void *o, int B, int H, int H_kv, int S_max,
                        int head_dim, float scale, void *workspace,
                        size_t workspace_bytes, uint32_t *counters,
                        size_t counter_count, void *stream) {
  if (!o || !k_new || !v_new) return FA_EINVAL;
  if (head_dim == FA_HEAD_DIM)
    return fa_decode_append(q, k_new, v_new, k_cache, v_cache, seq_lens, o, B,
                            H, H_kv, S_max, scale, workspace, workspace_bytes,
                            counters, counter_count, stream);
  if (head_dim != 128) return FA_EINVAL;
  if (H_kv == H)
    return run_decode_d128(q, k_cache, v_cache, seq_lens, o, B, H, S_max,
                           scale, 0, workspace, workspace_bytes, counters,
                           counter_count, stream, k_new, v_new);
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, H_kv,
                        S_max, scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream, k_new, v_new, nullptr, 0, 1, 0,
                        128);
}

int fa_decode_append_ex(const void *q, const void *k_new, const void *v_new,
                        void *k_cache, void *v_cache, const int32_t *seq_lens,
                        void *o, int B, int H, int H_kv, int S_max,
                        int head_dim, int dtype, float scale, void *workspace,
                        size_t workspace_bytes, uint32_t *counters,
                        size_t counter_count, void *stream) {
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_EINVAL;
  if (!o || !k_new || !v_new) return FA_EINVAL;
  if (head_dim != FA_HEAD_DIM && head_dim != 128) return FA_EINVAL;
  if (head_dim == 128 && H_kv == H)
    return run_decode_d128(q, k_cache, v_cache, seq_lens, o, B, H, S_max,
                           scale, 0, workspace, workspace_bytes, counters,
                           counter_count, stream, k_new, v_new, dtype);
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, H_kv,
                        S_max, scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream, k_new, v_new, nullptr, 0, 1, 0,
                        head_dim, dtype);
}

size_t fa_decode_gqa_hd_workspace_bytes(int B, int H, int H_kv, int S_max,
                                        int head_dim, int device) {
  if (head_dim == FA_HEAD_DIM)
    return fa_decode_gqa_workspace_bytes(B, H, H_kv, S_max, device);
  if (head_dim != 128 || B <= 0 || H <= 0 || S_max <= 0 || H_kv <= 0 ||
      H % H_kv != 0)
    return 0;
  if (H_kv == H) return fa_decode_hd_workspace_bytes(B, H, S_max, 128, 0, device);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) !=
      cudaSuccess)
    return 0;
  const GqaPlan p = gqa_plan(H, H_kv);
  return gqa_workspace_bytes_for(B, p, decode_gqa_grid(sms, B, p, S_max, 0, 128),
                                 128);
}

int fa_decode_gqa_hd(const void *q, const void *k_cache, const void *v_cache,
                     const int32_t *seq_lens, void *o, int B, int H, int H_kv,
                     int S_max, int head_dim, float scale, void *workspace,
                     size_t workspace_bytes, uint32_t *counters,
                     size_t counter_count, void *stream) {
  if (head_dim == 128 && H_kv == H)
    return fa_decode_hd(q, k_cache, v_cache, seq_lens, o, B, H, S_max, 128,
                        scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream);
  if (!o) return FA_EINVAL;
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, H_kv,
                        S_max, scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream, nullptr, nullptr, nullptr, 0, 1,
                        0, head_dim);
}

size_t fa_decode_ex_workspace_bytes(int B, int H, int H_kv, int S_max,
                                    int head_dim, int device) {
  return fa_decode_gqa_hd_workspace_bytes(B, H, H_kv, S_max, head_dim, device);
}

int fa_decode_ex(const void *q, const void *k_cache, const void *v_cache,
                 const int32_t *seq_lens, void *o, int B, int H, int H_kv,
                 int S_max, int head_dim, int dtype, float scale,
                 void *workspace, size_t workspace_bytes, uint32_t *counters,
                 size_t counter_count, void *stream) {
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_EINVAL;
  if (!o || (head_dim != FA_HEAD_DIM && head_dim != 128)) return FA_EINVAL;
  if (head_dim == 128 && H_kv == H)
    return run_decode_d128(q, k_cache, v_cache, seq_lens, o, B, H, S_max,
                           scale, 0, workspace, workspace_bytes, counters,
                           counter_count, stream, nullptr, nullptr, dtype);
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, H_kv,
                        S_max, scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream, nullptr, nullptr, nullptr, 0, 1,
                        0, head_dim, dtype);
}

size_t fa_decode_gqa_workspace_bytes(int B, int H, int H_kv, int S_max,
                                     int device) {
  if (B <= 0 || H <= 0 || S_max <= 0 || H_kv <= 0 || H % H_kv != 0) return 0;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) !=
      cudaSuccess)
    return 0;
  if (H_kv == H)
    return workspace_bytes_for(B, H, decode_grid(sms, B, H, S_max, 0));
  const GqaPlan p = gqa_plan(H, H_kv);
  return gqa_workspace_bytes_for(
      B, p, decode_gqa_grid(sms, B, p, S_max, 0, FA_HEAD_DIM));
}

int fa_decode(const void *q, const void *k_cache, const void *v_cache,
              const int32_t *seq_lens, void *o, int B, int H, int S_max,
              float scale, int split_size, void *workspace,
              size_t workspace_bytes, uint32_t *counters,
              size_t counter_count, void *stream) {
  if (!o) return FA_EINVAL;
  return run_decode(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, S_max,
                    scale, split_size, workspace, workspace_bytes, counters,
                    counter_count, stream);
}

int fa_decode_gqa(const void *q, const void *k_cache, const void *v_cache,
                  const int32_t *seq_lens, void *o, int B, int H, int H_kv,
                  int S_max, float scale, void *workspace,
                  size_t workspace_bytes, uint32_t *counters,
                  size_t counter_count, void *stream) {
  if (!o) return FA_EINVAL;
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, H_kv,
                        S_max, scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream);
}

int fa_decode_append(const void *q, const void *k_new, const void *v_new,
                     void *k_cache, void *v_cache, const int32_t *seq_lens,
                     void *o, int B, int H, int H_kv, int S_max, float scale,
                     void *workspace, size_t workspace_bytes,
                     uint32_t *counters, size_t counter_count, void *stream) {
  if (!o || !k_new || !v_new) return FA_EINVAL;
  return run_decode_gqa(q, k_cache, v_cache, seq_lens, o, nullptr, B, H, H_kv,
                        S_max, scale, 0, workspace, workspace_bytes, counters,
                        counter_count, stream, k_new, v_new);
}

int fa_decode_partial(const void *q, const void *k_cache, const void *v_cache,
                      const int32_t *seq_lens, float *partial_out, int B,
                      int H, int S_max, float scale, void *workspace,
                      size_t workspace_bytes, uint32_t *counters,
                      size_t counter_count, void *stream) {
  if (!partial_out) return FA_EINVAL;
  return run_decode(q, k_cache, v_cache, seq_lens, nullptr, partial_out, B, H,
                    S_max, scale, 0, workspace, workspace_bytes, counters,
                    counter_count, stream);
}

int fa_merge_partials(const float *partials, int G, void *o, int B, int H,
                      void *stream) {
  if (!partials || !o || G <= 0 || B <= 0 || H <= 0) return FA_EINVAL;
  if (static_cast<long long>(B) * H >= (1ll << 31)) return FA_EINVAL;
  if (!aligned16(partials) || !aligned16(o)) return FA_EALIGN;
  int rc = ensure_device(nullptr);
  if (rc != FA_OK) return rc;
  return launch_merge_kernel(partials, G, static_cast<__half *>(o), B, H,
                             static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? FA_OK
             : FA_ECUDA;
}

int fa_legacy_attention_f32(const float *q, const float *k, const float *v,
                            float *o, int N, void *stream) {
  if (!q || !k || !v || !o || N <= 0) return FA_EINVAL;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return FA_EALIGN;
  int rc = ensure_device(nullptr);
  if (rc != FA_OK) return rc;
  return launch_legacy_kernel(q, k, v, o, N, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? FA_OK
             : FA_ECUDA;
}

int fa_choose_decode_split(int max_seq, int batch, int heads, int min_blocks) {
  const long long per_split = static_cast<long long>(batch) * heads;
  for (int split = 1024; split > 128; split >>= 1) {
    const long long splits = (static_cast<long long>(max_seq) + split - 1) / split;
    if (per_split * splits >= min_blocks) return split;
  }
  return 128;
}

int fa_occupancy(fa_occupancy_entry *out, int max_entries, int *count) {
  int dev = 0;
  int rc = ensure_device(&dev);
  if (rc != FA_OK) return rc;
  int max_threads = 0;
  if (cudaDeviceGetAttribute(&max_threads,
                             cudaDevAttrMaxThreadsPerMultiProcessor,
                             dev) != cudaSuccess)
    return FA_ECUDA;
  struct K {
    const char *name;
    const void *fn;
    int threads;
    int dyn_smem;
  } kernels[] = {
      {"prefill_kernel", prefill_kernel_ptr(), prefill_threads(),
       prefill_smem_bytes()},
      {"prefill_solo_kernel", prefill_solo_kernel_ptr(),
       prefill_solo_threads(), prefill_solo_smem_bytes()},
      {"prefill_split_kernel", prefill_split_kernel_ptr(), prefill_threads(),
       prefill_split_smem_bytes()},
      {"decode_kernel", decode_kernel_ptr(), decode_threads(),
       decode_smem_bytes()},
      {"merge_kernel", merge_kernel_ptr(), merge_threads(), 0},
  };
  const int n = static_cast<int>(sizeof(kernels) / sizeof(kernels[0]));
  if (count) *count = n;
  for (int i = 0; i < n && i < max_entries; ++i) {
    cudaFuncAttributes attr;
    if (cudaFuncGetAttributes(&attr, kernels[i].fn) != cudaSuccess)
      return FA_ECUDA;
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &blocks, kernels[i].fn, kernels[i].threads,
            kernels[i].dyn_smem) != cudaSuccess)
      return FA_ECUDA;
    fa_occupancy_entry &e = out[i];
    memset(&e, 0, sizeof(e));
    strncpy(e.name, kernels[i].name, sizeof(e.name) - 1);
    e.threads_per_block = kernels[i].threads;
    e.registers_per_thread = attr.numRegs;
    e.shared_bytes_per_block =
        static_cast<int>(attr.sharedSizeBytes) + kernels[i].dyn_smem;
    e.max_active_blocks_per_sm = blocks;
    e.theoretical_occupancy =
        static_cast<double>(blocks) * kernels[i].threads / max_threads;
  }
  return FA_OK;
}

int fa_take_device_error(unsigned int *bits) {
  if (!bits) return FA_EINVAL;
  if (cudaDeviceSynchronize() != cudaSuccess) return FA_ECUDA;
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_fa_error_word, sizeof(v)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_fa_error_word, &zero, sizeof(zero)) != cudaSuccess)
    return FA_ECUDA;
  *bits = v;
  return FA_OK;
}

int fa_set_wait_limit_ns(unsigned long long ns) {
  if (ns < 1000ull || ns > 60000000000ull) return FA_EINVAL;
  int dev = 0;
  const int rc = ensure_device(&dev);
  if (rc != FA_OK) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyToSymbol(g_fa_wait_limit_ns, &ns, sizeof(ns)) != cudaSuccess)
    return FA_ECUDA;
  return FA_OK;
}

const char *fa_status_string(int status) {
  switch (status) {
    case FA_OK: return "ok";
    case FA_EINVAL: return "invalid argument";
    case FA_EALIGN: return "pointer not 16-byte aligned";
    case FA_ECUDA: return "CUDA runtime error";
    case FA_ENOSPACE: return "workspace too small";
    case FA_EDEVICE: return "device is not sm_100 or driver entry point missing";
    default: return "unknown status";
  }
}

#ifdef FA_TRACE
// Copies the pipeline trace stamps (profiling builds only).
int fa_trace_read(unsigned long long *dst, size_t n) {
  if (n > sizeof(g_fa_trace) / sizeof(g_fa_trace[0])) return FA_EINVAL;
  cudaDeviceSynchronize();
  return cudaMemcpyFromSymbol(dst, g_fa_trace, n * sizeof(*dst)) == cudaSuccess
             ? FA_OK
             : FA_ECUDA;
}
#endif


int fa_num_sms(void) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) !=
      cudaSuccess)
    return 0;
  return sms;
}

}  // extern "C"
