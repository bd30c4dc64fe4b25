// Prefill from host memory (fa_prefill_host): the inputs are streamed to the
// device in chunks while earlier chunks compute and later results stream
// back, so the PCIe copies in both directions and the kernels overlap
// instead of running back to back.
//
// A unit is one (batch, K/V head) group: its H / H_kv query heads plus the
// K/V head they read, contiguous in every (B, heads, N, D) array. Chunks of
// whole units go through a ring of device staging slots:
//
//   copy-in stream   H2D q,k,v of chunk i into slot i % R      -> in_done[r]
//   caller's stream  wait in_done[r] (and out_done[r] of chunk i - R),
//                    prefill of chunk i                         -> computed[r]
//   copy-out stream  wait computed[r], D2H o of chunk i         -> out_done[r]
//
// and before chunk i + R overwrites slot r the copy-in stream waits for
// computed[r] of chunk i. The caller's stream finally waits for the last
// D2H, so everything stays ordered on the stream the caller passed.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <mutex>

#include "fa_b200.h"
#include "fa_kernels.h"

namespace fa {
namespace {

// Measured on a B200 over PCIe 5 x16 (config 3, 88 MB in, 29 MB out): the
// uploads run at ~55 GB/s alone and ~49 GB/s while downloads and kernels
// overlap them; the ring depth does not matter (3 and 8 slots equal) and
// four chunks with the last one split in two (a shorter tail of kernel +
// download after the final upload) beat eight or sixteen: 1.99 ms vs
// 2.11 / 2.03 ms, serial copy-compute-copy 2.31 ms.
constexpr int kRing = 3;              // staging slots in flight
constexpr int kTargetChunks = 4;      // chunks per call when units allow
constexpr size_t kMinChunkIn = 2u << 20;   // q+k+v bytes per chunk, at least
constexpr size_t kMaxChunkIn = 64u << 20;  // ... and at most (one unit min)
constexpr int kMaxStageDevices = 64;

struct HostPlan {
  int units = 0;           // B * H_kv
  int unit_heads = 0;      // H / H_kv query heads per unit
  size_t unit_q = 0;       // bytes of q (and o) per unit
  size_t unit_kv = 0;      // bytes of k (and of v) per unit
  int chunk_units = 0;     // units per chunk (the last ones may hold fewer)
  int chunks = 0;
  int split_from = 0;      // chunks [0, split_from) hold chunk_units each;
                           // the rest split what remains in two
  int slots = 0;           // ring depth actually used
  size_t slot_bytes = 0;   // q + k + v + o of one full chunk, 256-aligned
  size_t workspace = 0;
};

size_t round256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// First unit and unit count of chunk c.
void chunk_range(const HostPlan &p, int c, int *u0, int *nu) {
  if (c < p.split_from) {
    *u0 = c * p.chunk_units;
    *nu = p.units - *u0 < p.chunk_units ? p.units - *u0 : p.chunk_units;
    return;
  }
  const int base = p.split_from * p.chunk_units;
  const int rest = p.units - base;
  const int first = (rest + 1) / 2;
  *u0 = c == p.split_from ? base : base + first;
  *nu = c == p.split_from ? first : rest - first;
}

int make_plan(int B, int H, int H_kv, int N, int head_dim, HostPlan *p) {
  if (B <= 0 || H <= 0 || N <= 0 || H_kv <= 0 || H % H_kv != 0)
    return FA_EINVAL;
  if (head_dim != 64 && head_dim != 128) return FA_EINVAL;
  if (static_cast<long long>(B) * H >= (1ll << 31) / 128) return FA_EINVAL;
  p->units = B * H_kv;
  p->unit_heads = H / H_kv;
  const size_t row = static_cast<size_t>(head_dim) * 2;
  p->unit_q = static_cast<size_t>(p->unit_heads) * N * row;
  p->unit_kv = static_cast<size_t>(N) * row;
  const size_t unit_in = p->unit_q + 2 * p->unit_kv;
  int cu = (p->units + kTargetChunks - 1) / kTargetChunks;
  const int max_units = static_cast<int>(kMaxChunkIn / unit_in);
  const int min_units =
      static_cast<int>((kMinChunkIn + unit_in - 1) / unit_in);
  if (cu > max_units) cu = max_units;
  if (cu < min_units) cu = min_units;
  if (cu < 1) cu = 1;
  if (cu > p->units) cu = p->units;
  p->chunk_units = cu;
  p->chunks = (p->units + cu - 1) / cu;
  p->split_from = p->chunks;
  const int last = p->units - (p->chunks - 1) * cu;
  if (last >= 2) {  // split the last chunk in two
    p->split_from = p->chunks - 1;
    p->chunks += 1;
  }
  p->slots = p->chunks < kRing ? p->chunks : kRing;
  p->slot_bytes = round256(cu * p->unit_q) * 2 + round256(cu * p->unit_kv) * 2;
  p->workspace = p->slot_bytes * p->slots;
  return FA_OK;
}

// Copy streams and events of one device, created on first use and kept for
// the life of the process (they are reused by every call on that device).
struct StageState {
  bool ready = false;
  cudaStream_t copy_in = nullptr;
  cudaStream_t copy_out = nullptr;
  cudaEvent_t start = nullptr;
  cudaEvent_t in_done[kRing] = {};
  cudaEvent_t computed[kRing] = {};
  cudaEvent_t out_done[kRing] = {};
  std::mutex mutex;  // one enqueue sequence at a time per device
};

std::mutex g_stage_mutex;
StageState g_stage[kMaxStageDevices];

int stage_state(int dev, StageState **out) {
  if (dev < 0 || dev >= kMaxStageDevices) return FA_EDEVICE;
  std::lock_guard<std::mutex> lock(g_stage_mutex);
  StageState &s = g_stage[dev];
  if (!s.ready) {
    const unsigned ev_flags = cudaEventDisableTiming;
    bool ok = cudaStreamCreateWithFlags(&s.copy_in, cudaStreamNonBlocking) ==
                  cudaSuccess &&
              cudaStreamCreateWithFlags(&s.copy_out, cudaStreamNonBlocking) ==
                  cudaSuccess &&
              cudaEventCreateWithFlags(&s.start, ev_flags) == cudaSuccess;
    for (int r = 0; ok && r < kRing; ++r)
      ok = cudaEventCreateWithFlags(&s.in_done[r], ev_flags) == cudaSuccess &&
           cudaEventCreateWithFlags(&s.computed[r], ev_flags) == cudaSuccess &&
           cudaEventCreateWithFlags(&s.out_done[r], ev_flags) == cudaSuccess;
    if (!ok) return FA_ECUDA;
    s.ready = true;
  }
  *out = &s;
  return FA_OK;
}

}  // namespace
}  // namespace fa

using namespace fa;

extern "C" {

int fa_prefill_host_plan(int B, int H, int H_kv, int N, int head_dim,
                         int *chunks, size_t *workspace_bytes) {
  HostPlan p;
  const int rc = make_plan(B, H, H_kv, N, head_dim, &p);
  if (rc != FA_OK) return rc;
  if (chunks) *chunks = p.chunks;
  if (workspace_bytes) *workspace_bytes = p.workspace;
  return FA_OK;
}

int fa_prefill_host(const void *q, const void *k, const void *v, void *o,
                    int B, int H, int H_kv, int N, int head_dim, int causal,
                    float scale, void *workspace, size_t workspace_bytes,
                    void *stream) {
  return fa_prefill_host_ex(q, k, v, o, B, H, H_kv, N, head_dim, FA_DTYPE_F16,
                            causal, scale, workspace, workspace_bytes, stream);
}

int fa_prefill_host_ex(const void *q, const void *k, const void *v, void *o,
                       int B, int H, int H_kv, int N, int head_dim, int dtype,
                       int causal, float scale, void *workspace,
                       size_t workspace_bytes, void *stream) {
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_EINVAL;
  HostPlan p;
  int rc = make_plan(B, H, H_kv, N, head_dim, &p);
  if (rc != FA_OK) return rc;
  if (!isfinite(scale)) return FA_EINVAL;
  if (!q || !k || !v || !o || !workspace) return FA_EINVAL;
  if (workspace_bytes < p.workspace) return FA_ENOSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return FA_EALIGN;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ECUDA;
  StageState *st = nullptr;
  rc = stage_state(dev, &st);
  if (rc != FA_OK) return rc;
  std::lock_guard<std::mutex> lock(st->mutex);

  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const char *hq = static_cast<const char *>(q);
  const char *hk = static_cast<const char *>(k);
  const char *hv = static_cast<const char *>(v);
  char *ho = static_cast<char *>(o);
  char *ws = static_cast<char *>(workspace);
  const size_t q_cap = round256(p.chunk_units * p.unit_q);
  const size_t kv_cap = round256(p.chunk_units * p.unit_kv);

  // Inputs and outputs may still be written / read by earlier work on the
  // caller's stream: both copy streams start after it.
  if (cudaEventRecord(st->start, cs) != cudaSuccess ||
      cudaStreamWaitEvent(st->copy_in, st->start, 0) != cudaSuccess ||
      cudaStreamWaitEvent(st->copy_out, st->start, 0) != cudaSuccess)
    return FA_ECUDA;

  rc = FA_OK;
  for (int c = 0; c < p.chunks && rc == FA_OK; ++c) {
    const int r = c % p.slots;
    int u0 = 0, nu = 0;
    chunk_range(p, c, &u0, &nu);
    char *sq = ws + r * p.slot_bytes;
    char *sk = sq + q_cap;
    char *sv = sk + kv_cap;
    char *so = sv + kv_cap;
    const size_t qb = nu * p.unit_q, kvb = nu * p.unit_kv;
    const size_t qoff = u0 * p.unit_q, kvoff = u0 * p.unit_kv;
    if ((c >= p.slots &&
         cudaStreamWaitEvent(st->copy_in, st->computed[r], 0) != cudaSuccess) ||
        cudaMemcpyAsync(sq, hq + qoff, qb, cudaMemcpyHostToDevice,
                        st->copy_in) != cudaSuccess ||
        cudaMemcpyAsync(sk, hk + kvoff, kvb, cudaMemcpyHostToDevice,
                        st->copy_in) != cudaSuccess ||
        cudaMemcpyAsync(sv, hv + kvoff, kvb, cudaMemcpyHostToDevice,
                        st->copy_in) != cudaSuccess ||
        cudaEventRecord(st->in_done[r], st->copy_in) != cudaSuccess ||
        cudaStreamWaitEvent(cs, st->in_done[r], 0) != cudaSuccess ||
        (c >= p.slots &&
         cudaStreamWaitEvent(cs, st->out_done[r], 0) != cudaSuccess)) {
      rc = FA_ECUDA;
      break;
    }
    rc = prefill_chunk_ex(sq, sk, sv, so, nu, p.unit_heads, 1, N, head_dim,
                          dtype, causal, scale, stream,
                          static_cast<long long>(B) * H);
    if (rc != FA_OK) break;
    if (cudaEventRecord(st->computed[r], cs) != cudaSuccess ||
        cudaStreamWaitEvent(st->copy_out, st->computed[r], 0) != cudaSuccess ||
        cudaMemcpyAsync(ho + qoff, so, qb, cudaMemcpyDeviceToHost,
                        st->copy_out) != cudaSuccess ||
        cudaEventRecord(st->out_done[r], st->copy_out) != cudaSuccess)
      rc = FA_ECUDA;
  }
  // The caller's stream waits for everything enqueued on both copy streams
  // (after an error midway too), so the workspace and the host buffers are
  // free once that stream reaches this point.
  if (cudaEventRecord(st->in_done[0], st->copy_in) != cudaSuccess ||
      cudaEventRecord(st->out_done[0], st->copy_out) != cudaSuccess ||
      cudaStreamWaitEvent(cs, st->in_done[0], 0) != cudaSuccess ||
      cudaStreamWaitEvent(cs, st->out_done[0], 0) != cudaSuccess)
    return FA_ECUDA;
  return rc;
}

}  // extern "C"
