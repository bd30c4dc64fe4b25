// Decode (single query row per sequence) attention against a KV cache, B200.
//
// Behaviour follows the reference's split-K decode (csrc/decode.cu:50-175):
// out[b,h] = softmax(scale * q[b,h] . K[b,h,:len_b]^T) V[b,h,:len_b] with
// len_b = min(seq_lens[b], S_max); a sequence with no rows gets 0; partial
// results are combined with the log-sum-exp rule, skipping empty partials.
//
// The schedule is different. The reference launches ceil(S_max/split) CTAs
// per (b, h), sized by cache capacity, and merges in a second kernel. Here
// the valid rows of all (b, h) segments are laid end to end
// (segment g = b*H + h holds len_b rows) and a persistent grid cuts that flat
// row range into equal pieces, so every CTA streams the same number of bytes
// whatever the length distribution. A CTA's range can cover the tail of one
// segment, several whole segments and the head of another. Each
// (segment, CTA) overlap produces one (m, l, acc[64]) partial; a segment
// covered by one CTA is finished in place, otherwise the partials go to
// workspace slot (g + cta) — unique because the overlaps form a monotone
// staircase — and the last CTA to arrive on the segment's counter (an
// atomicInc that wraps back to 0, so the counters are clean for the next
// call) merges them in a fixed order. One launch, no second pass.
//
// CTA = 9 warps. Warp 8 plans and streams: it walks the segment pieces and
// issues cp.async.bulk copies of up to 128 K rows and 128 V rows (16 KiB each,
// contiguous in the cache) into a 3-stage shared-memory ring, with a stage
// header describing the rows. Warps 0-7 consume: each takes 16 rows of a
// stage, 8 lanes per row (16 bytes, 8 head dims per lane), 4 rows per warp
// instruction, 3-step shuffle dot products, block-wise online softmax in the
// exp2 domain.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "fa_kernels.h"
#include "fa_sm100.cuh"

namespace fa {
namespace decode {

constexpr int kConsumerWarps = 8;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kMergerWarp = kConsumerWarps + 1;
constexpr int kThreads = (kConsumerWarps + 2) * 32;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kStageRows = 128;
constexpr int kStages = 3;
constexpr int kRowsPerWarp = kStageRows / kConsumerWarps;  // 16
constexpr int kRowIters = kRowsPerWarp / 4;  // a warp covers 4 rows at once
static_assert(kRowsPerWarp % 4 == 0, "rows per warp must be a multiple of 4");
constexpr int kMinRowsPerCta = 128;
constexpr int kCtasPerSm = 2;
constexpr uint32_t kStageBytes = kStageRows * kRowBytes;  // 16 KiB

struct StageHeader {
  int g;      // segment (b * H + h)
  int n;      // rows in this stage (0 for the end marker)
  int flags;  // kLast | kWhole | kDone
  int c0;     // first CTA covering the segment
  int c1;     // last CTA covering the segment
  int r0;     // segment row of the stage's first row
  int pad[2];
};
constexpr int kLast = 1;   // last stage of this CTA's piece of the segment
constexpr int kWhole = 2;  // the segment lies entirely inside this CTA
constexpr int kDone = 4;   // no more stages

constexpr uint32_t kKOff = 0;
constexpr uint32_t kVOff = kStages * kStageBytes;
constexpr uint32_t kHdrOff = 2 * kStages * kStageBytes;
constexpr uint32_t kRedOff = kHdrOff + kStages * sizeof(StageHeader);
// Hand-off buffers from the consumer warps to the merger warp, double
// buffered: per buffer one (m, l, acc) per consumer warp plus a header.
constexpr int kRedBufs = 2;
constexpr uint32_t kRedBufBytes = kConsumerWarps * kPartialFloats * 4 + 32;
constexpr uint32_t kRedBytes = kRedBufs * kRedBufBytes;
constexpr uint32_t kBarOff = kRedOff + kRedBytes;
// full[kStages], empty[kStages], red_full[kRedBufs], red_empty[kRedBufs]
constexpr uint32_t kSmemBytes = kBarOff + (2 * kStages + 2 * kRedBufs) * 8;

constexpr float kNegBig = -1e30f;  // finite "no max yet", as the reference

__device__ __forceinline__ int clamp_len(int len, int s_max) {
  return len < 0 ? 0 : (len > s_max ? s_max : len);
}

// Rows sequence b attends. With a fused append the new token's row
// (index max(len, 0)) is added while it still fits in the cache.
__device__ __forceinline__ int seq_rows(const DecodeArgs &a, int b) {
  const int len = a.seq_lens[b];
  if (!a.k_new) return clamp_len(len, a.S_max);
  return clamp_len((len < 0 ? 0 : len) + 1, a.S_max);
}

// Row of sequence b that holds the appended token, or -1 (no append, or the
// cache is full and the token is not stored).
__device__ __forceinline__ int appended_row(const DecodeArgs &a, int b) {
  if (!a.k_new) return -1;
  const int len = a.seq_lens[b] < 0 ? 0 : a.seq_lens[b];
  return len < a.S_max ? len : -1;
}

// The appended token's 16-byte chunk held by this lane (lanes 0-7: K,
// 8-15: V; other lanes get zeros), loaded when a segment starts so the load
// overlaps the query load.
template <int D = kHeadDim>
__device__ __forceinline__ uint4 load_new_row(const DecodeArgs &a, int g_kv) {
  constexpr int kChunks = D / 8;  // 16-byte chunks per row
  const int lane = threadIdx.x & 31;
  if (lane >= 2 * kChunks) return make_uint4(0, 0, 0, 0);
  const __half *src =
      (lane >= kChunks ? a.v_new : a.k_new) + static_cast<size_t>(g_kv) * D;
  return reinterpret_cast<const uint4 *>(src)[lane % kChunks];
}

// Fused append, run by the warp that owns stage row `local` of plane g_kv:
// the new K/V row (val from load_new_row) replaces the stale cache row in
// shared memory and, when `store` is set, is written to the cache. Swizzled
// stages hold 64-dim blocks of kRows x 128 B with 16-byte chunk c of a row
// at chunk c ^ (row & 7); plain stages hold rows of 2 D bytes.
template <bool kSwizzled, int D = kHeadDim, int kRows = kStageRows>
__device__ __forceinline__ void patch_new_row(const DecodeArgs &a, int g_kv,
                                              int row_in_plane, int local,
                                              uint8_t *k_stage,
                                              uint8_t *v_stage, bool store,
                                              uint4 val) {
  constexpr int kChunks = D / 8;
  const int lane = threadIdx.x & 31;
  if (lane < 2 * kChunks) {
    const int c = lane % kChunks;
    const bool is_v = lane >= kChunks;
    const int off =
        kSwizzled ? (c >> 3) * kRows * 128 + local * 128 +
                        (((c & 7) ^ (local & 7)) << 4)
                  : local * 2 * D + c * 16;
    uint8_t *stage = is_v ? v_stage : k_stage;
    *reinterpret_cast<uint4 *>(stage + off) = val;
    if (store) {
      __half *dst = (is_v ? a.v_cache_w : a.k_cache_w) +
                    (static_cast<size_t>(g_kv) * a.S_max + row_in_plane) * D;
      reinterpret_cast<uint4 *>(dst)[c] = val;
    }
  }
  // the stage is refilled by the async proxy once it is released
  fence_proxy_async_smem();
  __syncwarp();
}

__device__ __forceinline__ long long warp_sum_ll(long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Writes the result of a sequence with no valid rows: 0 (reference
// decode.cu:164-172), or an empty partial (l = 0) in partial mode.
__device__ void write_empty_sequence(const DecodeArgs &a, int b) {
  for (int h = 0; h < a.H; ++h) {
    const size_t g = static_cast<size_t>(b) * a.H + h;
    if (a.partial_out) {
      float *p = a.partial_out + g * kPartialFloats;
      p[0] = kNegBig;
      for (int i = 1; i < kPartialFloats; ++i) p[i] = 0.f;
    } else {
      uint4 *o = reinterpret_cast<uint4 *>(a.out + g * kHeadDim);
      for (int i = 0; i < kHeadDim / 8; ++i) o[i] = make_uint4(0, 0, 0, 0);
    }
  }
}

// ---- cross-GPU exchange of finished segments (sequence-sharded decode) ----
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];"
               : "=r"(v)
               : "l"(p)
               : "memory");
  return v;
}

// Exchange buffer of rank r for head_dim D: two banks of (x_world, B*H,
// 4 + D) fp32 partials, then B*H uint32 arrival counters. Epoch e writes
// bank e & 1. A rank can start epoch e + 1 (and store into the other bank)
// while a peer still reads bank e & 1 of epoch e; it cannot reach epoch
// e + 2 before every peer has finished epoch e, because finishing e + 1
// needs every peer's e + 1 partials, which a peer sends only after its
// epoch-e launch has completed on its stream.
template <int D>
__device__ __forceinline__ float *x_bank(const DecodeArgs &a, int r) {
  return a.x_peers[r] + static_cast<size_t>(a.x_epoch & 1u) * a.x_world *
                            a.B * a.H * (4 + D);
}

template <int D>
__device__ __forceinline__ uint32_t *x_counters(const DecodeArgs &a, int r) {
  return reinterpret_cast<uint32_t *>(
      a.x_peers[r] + 2 * static_cast<size_t>(a.x_world) * a.B * a.H * (4 + D));
}

// Whole warp: stores this rank's (m, l, acc) of segment g into slot
// [x_rank][g] of this epoch's bank in every rank's buffer (peer memory over NVLink, plain
// stores), then raises each rank's counter of g. Lane l holds dims
// l + 32 i.
template <int D>
__device__ void x_send(const DecodeArgs &a, size_t g, float M, float L,
                       const float (&A)[D / 32], int lane) {
  const size_t BH = static_cast<size_t>(a.B) * a.H;
  for (int r = 0; r < a.x_world; ++r) {
    float *dst = x_bank<D>(a, r) + (static_cast<size_t>(a.x_rank) * BH + g) * (4 + D);
#pragma unroll
    for (int i = 0; i < D / 32; ++i) dst[4 + 32 * i + lane] = A[i];
    if (lane == 0) {
      dst[0] = M;
      dst[1] = L;
    }
  }
  __threadfence_system();
  __syncwarp();
  if (lane < a.x_world) atomicAdd_system(x_counters<D>(a, lane) + g, 1u);
  __syncwarp();
}

// Whole warp: waits (bounded) until all x_world partials of segment g are
// in this rank's buffer, merges them (log-sum-exp, empty partials skipped,
// rank order) and writes the output row.
template <int D>
__device__ void x_finish(const DecodeArgs &a, size_t g, int lane) {
  const size_t BH = static_cast<size_t>(a.B) * a.H;
  const uint32_t *ctr = x_counters<D>(a, a.x_rank) + g;
  const uint32_t target = a.x_epoch * static_cast<uint32_t>(a.x_world);
  int ok = 1;
  if (lane == 0) {
    unsigned long long t0 = 0;
    const unsigned long long limit = wait_limit_ns();
    while (static_cast<int>(ld_acquire_sys(ctr) - target) < 0) {
      const unsigned long long now = global_timer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > limit || device_failed()) {
        // out of time, or another wait already ran out: give up at once
        record_error(FA_ERR_TIMEOUT);
        ok = 0;
        break;
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) return;
  (void)ld_acquire_sys(ctr);  // order this lane's reads after the arrivals
  const float *base = x_bank<D>(a, a.x_rank);
  float M = kNegBig;
  for (int r = 0; r < a.x_world; ++r) {
    const float *p = base + (static_cast<size_t>(r) * BH + g) * (4 + D);
    if (__ldcg(p + 1) > 0.f) M = fmaxf(M, __ldcg(p));
  }
  float L = 0.f;
  float acc[D / 32];
#pragma unroll
  for (int i = 0; i < D / 32; ++i) acc[i] = 0.f;
  for (int r = 0; r < a.x_world; ++r) {
    const float *p = base + (static_cast<size_t>(r) * BH + g) * (4 + D);
    const float l = __ldcg(p + 1);
    if (l <= 0.f) continue;
    const float f = fast_exp2(__ldcg(p) - M);
    L = fmaf(l, f, L);
#pragma unroll
    for (int i = 0; i < D / 32; ++i)
      acc[i] = fmaf(__ldcg(p + 4 + 32 * i + lane), f, acc[i]);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int i = 0; i < D / 32; ++i)
    a.out[g * D + 32 * i + lane] = store_elem(acc[i] * inv, a.dtype);
}

// Segments this CTA has sent to every rank and still has to merge: the
// merger warp sends a finished segment at once but waits for the other
// ranks' partials of it only after the CTA's last piece, so a slower peer
// does not hold up this CTA's own stream (the hand-off buffers stay free).
constexpr int kMaxDeferred = 64;
struct XDeferred {
  int n;
  int g[kMaxDeferred];
};
__device__ __forceinline__ XDeferred &x_deferred() {
  __shared__ XDeferred d;
  return d;
}

// Whole warp: x_send, then either defer the merge (room in the list) or
// do it now.
template <int D>
__device__ __forceinline__ void x_send_deferred(const DecodeArgs &a, size_t g,
                                                float M, float L,
                                                const float (&A)[D / 32],
                                                int lane) {
  x_send<D>(a, g, M, L, A, lane);
  XDeferred &d = x_deferred();
  const int n = d.n;
  if (n < kMaxDeferred) {
    __syncwarp();
    if (lane == 0) {
      d.g[n] = static_cast<int>(g);
      d.n = n + 1;
    }
    __syncwarp();
  } else {
    x_finish<D>(a, g, lane);
  }
}

// Whole warp: the deferred merges, in the order the segments were sent.
template <int D>
__device__ __forceinline__ void x_finish_deferred(const DecodeArgs &a,
                                                  int lane) {
  XDeferred &d = x_deferred();
  __syncwarp();
  for (int i = 0; i < d.n; ++i) x_finish<D>(a, static_cast<size_t>(d.g[i]), lane);
}

// Writes a finished (m, l, acc) for segment g: the fp16 output, or the
// partial in partial mode, or (sharded) sends it to every rank and writes
// the merge of all ranks. Lane l holds dims l and l + 32.
__device__ __forceinline__ void finish_segment(const DecodeArgs &a, size_t g,
                                               float M, float L, float A0,
                                               float A1, int lane) {
  if (a.x_peers) {
    const float A[2] = {A0, A1};
    x_send_deferred<kHeadDim>(a, g, M, L, A, lane);
    return;
  }
  if (a.partial_out) {
    float *p = a.partial_out + g * kPartialFloats;
    p[4 + lane] = A0;
    p[4 + 32 + lane] = A1;
    if (lane == 0) {
      p[0] = M;
      p[1] = L;
      p[2] = 0.f;
      p[3] = 0.f;
    }
  } else {
    const float inv = L > 0.f ? 1.f / L : 0.f;
    a.out[g * kHeadDim + lane] = store_elem(A0 * inv, a.dtype);
    a.out[g * kHeadDim + 32 + lane] = store_elem(A1 * inv, a.dtype);
  }
}

// Merger warp: combines the consumer warps' partials of each finished piece,
// writes whole segments directly, and for segments split across CTAs
// publishes this CTA's partial; the last CTA to arrive on the segment's
// counter merges all of them (partials are read in parallel, merged in CTA
// order, so the result is deterministic).
__device__ void merger(const DecodeArgs &a, uint8_t *red_base,
                       uint64_t *red_full, uint64_t *red_empty) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) x_deferred().n = 0;
  __syncwarp();
  for (int piece = 0;; ++piece) {
    const int buf = piece & 1;
    if (!mbar_wait(&red_full[buf], (piece >> 1) & 1)) return;
    const float *red = reinterpret_cast<const float *>(red_base + buf * kRedBufBytes);
    const int *hdr_in = reinterpret_cast<const int *>(red + kConsumerWarps * kPartialFloats);
    const int flags = hdr_in[1];
    if (flags & kDone) {
      if (a.x_peers) x_finish_deferred<kHeadDim>(a, lane);
      return;
    }
    const size_t g = static_cast<size_t>(hdr_in[0]);
    const int c0 = hdr_in[2];
    const int c1 = hdr_in[3];
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red[w * kPartialFloats]);
    float L = 0.f, A0 = 0.f, A1 = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float fw = fast_exp2(red[w * kPartialFloats] - M);
      L = fmaf(red[w * kPartialFloats + 1], fw, L);
      A0 = fmaf(red[w * kPartialFloats + 4 + lane], fw, A0);
      A1 = fmaf(red[w * kPartialFloats + 4 + 32 + lane], fw, A1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&red_empty[buf]);  // buffer consumed

    if (flags & kWhole) {
      finish_segment(a, g, M, L, A0, A1, lane);
      continue;
    }
    float *ws = a.ws_partials + (g + blockIdx.x) * static_cast<size_t>(kPartialFloats);
    ws[4 + lane] = A0;
    ws[4 + 32 + lane] = A1;
    if (lane == 0) {
      ws[0] = M;
      ws[1] = L;
    }
    __threadfence();
    __syncwarp();
    unsigned last = 0;
    if (lane == 0) {
      const unsigned n_parts = static_cast<unsigned>(c1 - c0);
      last = atomicInc(&a.ws_counters[g], n_parts) == n_parts;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    if (lane == 0) FA_TRACE_CTA(5);
    __threadfence();
    // every partial of the segment is in place: merge them
    // (m, l) of up to 32 partials per lane round; with at most 32 partials
    // (the usual case) the first round's values are kept for the weights.
    float M2 = kNegBig, m_keep = kNegBig, l_keep = 0.f;
    for (int c = c0 + lane; c <= c1; c += 32) {
      const float *pp = a.ws_partials + (g + c) * static_cast<size_t>(kPartialFloats);
      const float lc = __ldcg(pp + 1);
      const float mc = __ldcg(pp);
      if (c < c0 + 32) {
        m_keep = mc;
        l_keep = lc;
      }
      if (lc > 0.f) M2 = fmaxf(M2, mc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      M2 = fmaxf(M2, __shfl_xor_sync(0xffffffffu, M2, o));
    // Weights one partial per lane, then the head dims in batches of 16
    // partials whose loads are all in flight together (the merge is on the
    // kernel's tail: a load round trip per partial would cost microseconds).
    float L2 = 0.f, B0 = 0.f, B1 = 0.f;
    for (int cb = c0; cb <= c1; cb += 32) {
      const int nb = c1 - cb + 1 < 32 ? c1 - cb + 1 : 32;
      float fc = 0.f;
      if (lane < nb) {
        float lc = l_keep, mc = m_keep;
        if (cb != c0) {
          const float *pp = a.ws_partials +
                            (g + cb + lane) * static_cast<size_t>(kPartialFloats);
          lc = __ldcg(pp + 1);
          mc = __ldcg(pp);
        }
        if (lc > 0.f) fc = fast_exp2(mc - M2);
        L2 = fmaf(lc, fc, L2);
      }
      for (int i0 = 0; i0 < nb; i0 += 16) {
        float x0[16], x1[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          x0[i] = 0.f;
          x1[i] = 0.f;
          if (i0 + i < nb) {
            const float *pp = a.ws_partials +
                              (g + cb + i0 + i) * static_cast<size_t>(kPartialFloats);
            x0[i] = __ldcg(pp + 4 + lane);
            x1[i] = __ldcg(pp + 4 + 32 + lane);
          }
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float f = __shfl_sync(0xffffffffu, fc, (i0 + i) & 31);
          B0 = fmaf(x0[i], f, B0);
          B1 = fmaf(x1[i], f, B1);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L2 += __shfl_xor_sync(0xffffffffu, L2, o);
    finish_segment(a, g, M2, L2, B0, B1, lane);
  }
}

// Producer warp of both decode kernels: plans this CTA's share of the flat
// row range (segments of nseg per batch entry laid end to end, len_b rows
// each) and streams it through the stage ring. Segment s of batch entry b
// reads cache plane b * H_kv + s / seg_per_plane. kTiled: 128-row TMA boxes
// with the 128-byte swizzle (for ldmatrix consumers); otherwise contiguous
// bulk copies of exactly the rows of the stage.
// kD: head dim of the cache rows; kRowsPerStage x 2 kD bytes = one stage.
template <bool kTiled, int kNumStages, int kD = kHeadDim,
          int kRowsPerStage = kStageRows>
// (every stage is kStageBytes: kRowsPerStage * 2 * kD == kStageBytes)
__device__ void produce(const DecodeArgs &a, int nseg, int seg_per_plane,
                        uint8_t *smem, uint32_t k_off, uint32_t v_off,
                        uint64_t *full, uint64_t *empty, StageHeader *hdr,
                        const CUtensorMap *tm_k, const CUtensorMap *tm_v) {
  const int lane = threadIdx.x & 31;
  // A kernel that gave up on a bounded wait earlier (device error word)
  // leaves this CTA with nothing to stream: the end marker goes out at once
  // and every role exits through its normal path. The word is read here,
  // beside the first sequence lengths, so the two global round trips
  // overlap instead of one gating the CTA's start.
  const bool failed = device_failed();
    // ------------------------------------------------------------ planning
    long long sum_len = 0;
    int max_len = 0;
    for (int chunk = 0; chunk < a.B; chunk += 32) {
      const int b = chunk + lane;
      const int len = b < a.B ? seq_rows(a, b) : 1;
      if (b < a.B) sum_len += len;
      if (b < a.B) max_len = max(max_len, len);
      // sequences without rows (other widths: written by the caller)
      unsigned todo = __ballot_sync(
          0xffffffffu, b < a.B && len == 0 &&
                           (b % static_cast<int>(gridDim.x)) ==
                               static_cast<int>(blockIdx.x));
      while (todo && !failed && (kD == kHeadDim || a.x_peers)) {
        const int i = __ffs(todo) - 1;
        todo &= todo - 1;
        if (a.x_peers) {
          // an empty partial for every rank now; merged after streaming
          const float zero[kD / 32] = {};
          for (int h = 0; h < a.H; ++h)
            x_send<kD>(a, static_cast<size_t>(chunk + i) * a.H + h, kNegBig,
                       0.f, zero, lane);
        } else if (lane == 0) {
          write_empty_sequence(a, chunk + i);
        }
      }
    }
    const long long total = warp_sum_ll(sum_len) * nseg;
    long long per = a.rows_per_cta;
    if (per <= 0) {
      per = (total + gridDim.x - 1) / gridDim.x;
      if (per < kMinRowsPerCta) per = kMinRowsPerCta;
      // Short sequences (at most two stages each): one CTA streams a whole
      // segment rather than splitting it and merging partials across CTAs
      // (B1 H12 S256: 14.4 -> 12.3 us on the B200).
#pragma unroll 1
      for (int o = 16; o > 0; o >>= 1)
        max_len = max(max_len, __shfl_xor_sync(0xffffffffu, max_len, o));
      if (max_len <= 2 * kRowsPerStage && per < max_len)
        per = (max_len + 3) & ~3;
    }
    const long long start = static_cast<long long>(blockIdx.x) * per;
    const long long end = start + per < total ? start + per : total;

    // Locate the batch entry holding flat row `start`: warp-wide inclusive
    // scan of H * len_b, 32 entries at a time.
    int b_start = 0;
    long long base_b = 0;
    if (start < end) {
      long long base = 0;
      for (int chunk = 0; chunk < a.B; chunk += 32) {
        const int b = chunk + lane;
        const long long rows =
            b < a.B ? static_cast<long long>(seq_rows(a, b)) * nseg
                    : 0;
        long long incl = rows;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const long long t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        const unsigned hit =
            __ballot_sync(0xffffffffu, b < a.B && base + incl > start);
        if (hit) {
          const int first = __ffs(hit) - 1;
          const long long incl_first = __shfl_sync(0xffffffffu, incl, first);
          const long long rows_first = __shfl_sync(0xffffffffu, rows, first);
          b_start = chunk + first;
          base_b = base + incl_first - rows_first;
          break;
        }
        base += __shfl_sync(0xffffffffu, incl, 31);
      }
    }

    // ------------------------------------------------------------ streaming
    if (lane == 0) {
      if (kNumStages == kStages) FA_TRACE_CTA(2);
      const uint64_t policy = l2_policy_evict_first();
      int it = 0;
      bool ok = true;
      long long cur = start;
      int b = b_start;
      while (ok && !failed && cur < end && b < a.B) {
        const int len = seq_rows(a, b);
        if (len == 0) {
          ++b;
          continue;
        }
        const long long off = cur - base_b;
        const int h = static_cast<int>(off / len);
        const int r = static_cast<int>(off - static_cast<long long>(h) * len);
        const long long seg_start = base_b + static_cast<long long>(h) * len;
        const long long seg_end = seg_start + len;
        const long long piece_end = end < seg_end ? end : seg_end;
        const int c0 = static_cast<int>(seg_start / per);
        const int c1 = static_cast<int>((seg_end - 1) / per);
        const int g = b * nseg + h;
        // cache plane (K/V head) of this segment
        const int g_kv = b * a.H_kv + h / seg_per_plane;
        const size_t row0 = static_cast<size_t>(g_kv) * a.S_max + r;
        for (long long r0 = cur; r0 < piece_end; r0 += kRowsPerStage) {
          const int n = static_cast<int>(
              piece_end - r0 < kRowsPerStage ? piece_end - r0 : kRowsPerStage);
          const int slot = it % kNumStages;
          const int use = it / kNumStages;
          if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1)) {
            ok = false;
            break;
          }
          StageHeader &hd = hdr[slot];
          hd.g = g;
          hd.n = n;
          hd.flags = (r0 + n == piece_end ? kLast : 0) | (c0 == c1 ? kWhole : 0);
          hd.c0 = c0;
          hd.c1 = c1;
          hd.r0 = r + static_cast<int>(r0 - cur);
          if (kTiled) {
            // whole boxes of kRowsPerStage rows, 128-byte swizzled, one box
            // per 64 head dims (blocks of kRowsPerStage x 128 B); rows past
            // the piece are loaded but masked by the consumers
            const int row_in_plane = r + static_cast<int>(r0 - cur);
            mbar_arrive_expect_tx(&full[slot], 2 * kStageBytes);
#pragma unroll
            for (int hb = 0; hb < kD / 64; ++hb) {
              tma_load_3d(smem + k_off + slot * kStageBytes + hb * kRowsPerStage * 128,
                          tm_k, &full[slot], 64 * hb, row_in_plane, g_kv);
              tma_load_3d(smem + v_off + slot * kStageBytes + hb * kRowsPerStage * 128,
                          tm_v, &full[slot], 64 * hb, row_in_plane, g_kv);
            }
          } else {
            const size_t elem = (row0 + static_cast<size_t>(r0 - cur)) * kD;
            const uint32_t bytes = static_cast<uint32_t>(n) * 2 * kD;
            mbar_arrive_expect_tx(&full[slot], 2 * bytes);
            bulk_load(smem + k_off + slot * kStageBytes, a.k + elem, bytes,
                      &full[slot], policy);
            bulk_load(smem + v_off + slot * kStageBytes, a.v + elem, bytes,
                      &full[slot], policy);
          }
          ++it;
        }
        cur = piece_end;
        if (cur == base_b + static_cast<long long>(nseg) * len) {
          base_b += static_cast<long long>(nseg) * len;
          ++b;
        }
      }
      // End marker.
      const int slot = it % kNumStages;
      const int use = it / kNumStages;
      if (ok && (use == 0 || mbar_wait(&empty[slot], (use - 1) & 1))) {
        hdr[slot].n = 0;
        hdr[slot].flags = kDone;
        mbar_arrive(&full[slot]);
      } else {
        // Consumers stopped early: let our copies land before the CTA exits.
        for (int j = (it > kNumStages ? it - kNumStages : 0); j < it; ++j)
          mbar_wait(&full[j % kNumStages], (j / kNumStages) & 1);
      }
    }
    // Sharded: the rows of this CTA's empty sequences come from other
    // ranks; merge them now that this CTA's own stream is issued.
    if (a.x_peers && !failed) {
      __syncwarp();
      for (int chunk = 0; chunk < a.B; chunk += 32) {
        const int b = chunk + lane;
        unsigned todo = __ballot_sync(
            0xffffffffu, b < a.B && seq_rows(a, b) == 0 &&
                             (b % static_cast<int>(gridDim.x)) ==
                                 static_cast<int>(blockIdx.x));
        while (todo) {
          const int i = __ffs(todo) - 1;
          todo &= todo - 1;
          for (int h = 0; h < a.H; ++h)
            x_finish<kD>(a, static_cast<size_t>(chunk + i) * a.H + h, lane);
        }
      }
    }
}

template <typename Dt>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    decode_kernel(const DecodeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *empty = full + kStages;
  StageHeader *hdr = reinterpret_cast<StageHeader *>(smem + kHdrOff);
  uint64_t *red_full = empty + kStages;
  uint64_t *red_empty = red_full + kRedBufs;
  if (threadIdx.x == 0) FA_TRACE_CTA(0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    for (int r = 0; r < kRedBufs; ++r) {
      mbar_init(&red_full[r], kConsumerWarps);
      mbar_init(&red_empty[r], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) FA_TRACE_CTA(1);

  if (warp == kProducerWarp) {
    produce<false, kStages>(a, a.H, a.H / a.H_kv, smem, kKOff, kVOff, full,
                            empty, hdr, nullptr, nullptr);
    return;
  }

  if (warp == kMergerWarp) {
    merger(a, smem + kRedOff, red_full, red_empty);
    if (lane == 0) FA_TRACE_CTA(7);
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int grp = lane >> 3;  // which of the warp's 4 rows per instruction
  const int sub = lane & 7;   // head dims [8*sub, 8*sub + 8)
  float qf[8];
  int cur_g = -1;
  int app_row = -1;  // segment row of the appended token, -1 for none
  uint4 app_val = make_uint4(0, 0, 0, 0);
  float m_run = kNegBig, l_run = 0.f;
  int piece = 0;  // pieces handed to the merger warp so far
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;

  for (int it = 0;; ++it) {
    const int slot = it % kStages;
    if (!mbar_wait(&full[slot], (it / kStages) & 1)) break;
    if (it == 0 && threadIdx.x == 0) FA_TRACE_CTA(3);
    const StageHeader hd = hdr[slot];
    if (hd.flags & kDone) {
      if (threadIdx.x == 0) FA_TRACE_CTA(4);
      // tell the merger warp there is nothing more (same hand-off protocol)
      const int buf = piece & 1;
      if (piece >= kRedBufs &&
          !mbar_wait(&red_empty[buf], ((piece >> 1) - 1) & 1))
        break;
      if (warp == 0 && lane == 0) {
        int *hdr_out = reinterpret_cast<int *>(smem + kRedOff + buf * kRedBufBytes +
                                               kConsumerWarps * kPartialFloats * 4);
        hdr_out[1] = kDone;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[buf]);
      break;
    }
    if (hd.g != cur_g) {
      cur_g = hd.g;
      if (a.k_new) {
        const int b = cur_g / a.H;
        app_row = appended_row(a, b);
        if (app_row >= 0)
          app_val = load_new_row(a, b * a.H_kv + (cur_g - b * a.H) / (a.H / a.H_kv));
      }
      const uint4 qv = *reinterpret_cast<const uint4 *>(
          a.q + static_cast<size_t>(cur_g) * kHeadDim + sub * 8);
      const uint32_t *qh = reinterpret_cast<const uint32_t *>(&qv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Dt::unpack2(qh[e]);
        qf[2 * e] = f.x * a.scale_log2;
        qf[2 * e + 1] = f.y * a.scale_log2;
      }
    }

    if (app_row >= 0) {
      const int local = app_row - hd.r0;
      if (local >= 0 && local < hd.n && warp == local / kRowsPerWarp) {
        const int b = hd.g / a.H;
        const int h = hd.g - b * a.H;
        const int group = a.H / a.H_kv;
        patch_new_row<false>(a, b * a.H_kv + h / group, app_row, local,
                             smem + kKOff + slot * kStageBytes,
                             smem + kVOff + slot * kStageBytes, h % group == 0,
                             app_val);
      }
    }
    const uint32_t kb = smem_u32(smem + kKOff + slot * kStageBytes);
    const uint32_t vb = smem_u32(smem + kVOff + slot * kStageBytes);
    const int row_base = warp * kRowsPerWarp + grp;
    if (warp * kRowsPerWarp < hd.n) {  // warp-uniform: shuffles below
      float sc[kRowIters];
#pragma unroll
      for (int i = 0; i < kRowIters; ++i) {
        const int row = row_base + 4 * i;
        float d = 0.f;
        if (row < hd.n) {
          const uint4 kv = ld_shared_v4(kb + row * kRowBytes + sub * 16);
          const uint32_t *kh = reinterpret_cast<const uint32_t *>(&kv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Dt::unpack2(kh[e]);
            d = fmaf(qf[2 * e], f.x, d);
            d = fmaf(qf[2 * e + 1], f.y, d);
          }
        }
        sc[i] = d;
      }
#pragma unroll
      for (int i = 0; i < kRowIters; ++i) {
        sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], 1);
        sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], 2);
        sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], 4);
        if (row_base + 4 * i >= hd.n) sc[i] = -INFINITY;
      }
      float mx = sc[0];
#pragma unroll
      for (int i = 1; i < kRowIters; ++i) mx = fmaxf(mx, sc[i]);
      const float m_new = fmaxf(m_run, mx);
      const float corr = fast_exp2(m_run - m_new);
      m_run = m_new;
      float p[kRowIters];
      float psum = 0.f;
#pragma unroll
      for (int i = 0; i < kRowIters; ++i) {
        p[i] = fast_exp2(sc[i] - m_new);
        psum += p[i];
      }
      l_run = fmaf(l_run, corr, psum);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] *= corr;
#pragma unroll
      for (int i = 0; i < kRowIters; ++i) {
        const int row = row_base + 4 * i;
        if (row < hd.n) {
          const uint4 vv = ld_shared_v4(vb + row * kRowBytes + sub * 16);
          const uint32_t *vh = reinterpret_cast<const uint32_t *>(&vv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = Dt::unpack2(vh[e]);
            acc[2 * e] = fmaf(p[i], f.x, acc[2 * e]);
            acc[2 * e + 1] = fmaf(p[i], f.y, acc[2 * e + 1]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);

    if (!(hd.flags & kLast)) continue;

    // ---- this CTA's piece of segment hd.g is complete: reduce the warp's 4
    // row groups to one (m, l, acc[64]) and hand it to the merger warp, which
    // combines the 8 warps and finishes the segment while the consumers go
    // on streaming the next piece.
    float m_w = fmaxf(m_run, __shfl_xor_sync(0xffffffffu, m_run, 8));
    m_w = fmaxf(m_w, __shfl_xor_sync(0xffffffffu, m_w, 16));
    const float f = fast_exp2(m_run - m_w);
    float l_w = l_run * f;
    l_w += __shfl_xor_sync(0xffffffffu, l_w, 8);
    l_w += __shfl_xor_sync(0xffffffffu, l_w, 16);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float v = acc[e] * f;
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      acc[e] = v;
    }
    const int buf = piece & 1;
    if (piece >= kRedBufs &&
        !mbar_wait(&red_empty[buf], ((piece >> 1) - 1) & 1))
      break;
    float *red = reinterpret_cast<float *>(smem + kRedOff + buf * kRedBufBytes);
    float *my = red + warp * kPartialFloats;
    if (lane < 8) {
#pragma unroll
      for (int e = 0; e < 8; ++e) my[4 + lane * 8 + e] = acc[e];
      if (lane == 0) {
        my[0] = m_w;
        my[1] = l_w;
      }
    }
    if (warp == 0 && lane == 0) {
      int *hdr_out = reinterpret_cast<int *>(red + kConsumerWarps * kPartialFloats);
      hdr_out[0] = hd.g;
      hdr_out[1] = hd.flags;
      hdr_out[2] = hd.c0;
      hdr_out[3] = hd.c1;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&red_full[buf]);
    ++piece;
    m_run = kNegBig;
    l_run = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  }
}

// Log-sum-exp merge of G partial sets (G, B*H, 68) -> fp16 (B*H, 64).
__global__ void __launch_bounds__(kHeadDim)
    merge_kernel(const float *__restrict__ partials, int G, int BH,
                 __half *__restrict__ out) {
  const size_t g = blockIdx.x;
  const int d = threadIdx.x;
  float M = kNegBig;
  for (int r = 0; r < G; ++r) {
    const float *p = partials + (static_cast<size_t>(r) * BH + g) * kPartialFloats;
    if (p[1] > 0.f) M = fmaxf(M, p[0]);
  }
  float L = 0.f, A = 0.f;
  for (int r = 0; r < G; ++r) {
    const float *p = partials + (static_cast<size_t>(r) * BH + g) * kPartialFloats;
    if (p[1] <= 0.f) continue;
    const float f = fast_exp2(p[0] - M);
    L = fmaf(p[1], f, L);
    A = fmaf(p[4 + d], f, A);
  }
  out[g * kHeadDim + d] = __float2half_rn(L > 0.f ? A / L : 0.f);
}


}  // namespace decode

const void *decode_kernel_ptr(int dtype) {
  return dtype == FA_DTYPE_BF16
             ? reinterpret_cast<const void *>(decode::decode_kernel<BF16>)
             : reinterpret_cast<const void *>(decode::decode_kernel<F16>);
}
int decode_threads() { return decode::kThreads; }
int decode_smem_bytes() { return static_cast<int>(decode::kSmemBytes); }
int decode_ctas_per_sm() { return decode::kCtasPerSm; }
int decode_min_rows_per_cta() { return decode::kMinRowsPerCta; }

cudaError_t launch_decode_kernel(const DecodeArgs &args, cudaStream_t stream) {
  auto kernel = args.dtype == FA_DTYPE_BF16 ? decode::decode_kernel<BF16>
                                            : decode::decode_kernel<F16>;
  kernel<<<args.grid, decode::kThreads, decode::kSmemBytes, stream>>>(args);
  return cudaGetLastError();
}

const void *merge_kernel_ptr() {
  return reinterpret_cast<const void *>(decode::merge_kernel);
}
int merge_threads() { return kHeadDim; }

cudaError_t launch_merge_kernel(const float *partials, int G, __half *out,
                                int B, int H, cudaStream_t stream) {
  decode::merge_kernel<<<B * H, kHeadDim, 0, stream>>>(partials, G, B * H, out);
  return cudaGetLastError();
}

}  // namespace fa
