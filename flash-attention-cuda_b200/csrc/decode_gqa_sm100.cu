// Grouped-query decode on B200: every K/V row is read once for all the query
// heads that share its K/V head, for head_dim 64 and 128.
//
// Semantics as the per-head decode (reference csrc/decode.cu:50-175 with the
// K/V head of query head h being h / (H / H_kv)); the reference has no
// kernel-side GQA and names it as future work.
//
// A segment is (b, K/V head, chunk of up to 16 of its query heads). The
// producer (produce<true>, shared with the per-head kernel) streams
// length-balanced pieces of the flat row range as TMA boxes of the K and V
// planes with the 128-byte swizzle: 128 rows per stage at head_dim 64, 64
// rows (two 64-column blocks) at 128. Consumer warp w takes keys
// [16w, 16w + 16) of a stage and works on the tensor cores with warp-level
// MMAs (m16n8k16, fp16 in, fp32 accumulate): S (16 heads x 16 keys) = Q K^T
// with the group's queries as the M dimension, an online softmax per head
// row, then O (16 heads x D) += P V with P taken straight from the S
// registers. K is read with ldmatrix, V with its transposed form, both
// conflict-free on the swizzled rows. At the end of a piece the warps'
// per-head partials go to the merger warp; a segment split over several
// CTAs is merged by its last arrival with the whole CTA after streaming,
// the partials gathered into shared memory with bulk copies.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "fa_kernels.h"
#include "fa_sm100.cuh"

namespace fa {
namespace decode {

constexpr int kGqaMaxHeads = 16;  // query heads per segment (MMA M)
constexpr int kGqaMaxPending = 4;

template <int D>
struct GqaCfg {
  static constexpr int kPF = 4 + D;                    // partial floats
  static constexpr int kRows = D == 64 ? 128 : 64;     // rows per stage
  static constexpr int kStages = 4;
  static constexpr int kWarps = kRows / 16;            // consumers, 16 keys each
  static constexpr int kThreads = (kWarps + 2) * 32;
  static constexpr uint32_t kBlock = kRows * 128;      // one 64-dim block
  static constexpr uint32_t kKOff = 0;
  static constexpr uint32_t kVOff = kStages * kStageBytes;
  static constexpr uint32_t kHdrOff = 2 * kStages * kStageBytes;
  static constexpr uint32_t kRedOff = kHdrOff + kStages * sizeof(StageHeader);
  static constexpr uint32_t kRedWarpFloats = kGqaMaxHeads * kPF;
  static constexpr uint32_t kRedBufBytes = kWarps * kRedWarpFloats * 4 + 32;
  static constexpr uint32_t kBarOff = kRedOff + kRedBufs * kRedBufBytes;
  // bars: full[], empty[], red_full[], red_empty[], gather
  static constexpr uint32_t kPendOff =
      kBarOff + (2 * kStages + 2 * kRedBufs + 1) * 8;
  static constexpr uint32_t kSmemBytes = kPendOff + 64;
  // outputs (head, float4 of dims) a merging thread owns at most
  static constexpr int kOwn = (kGqaMaxHeads * D / 4 + kThreads - 1) / kThreads;
  static_assert(kRows * 2 * D == static_cast<int>(kStageBytes),
                "stages keep their size");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

struct GqaSegment {
  int b, h0, hv;  // batch entry, first query head, query heads in the chunk
};

__device__ __forceinline__ GqaSegment gqa_segment(int g, int nseg, int n_hc,
                                                  int group) {
  GqaSegment sg;
  sg.b = g / nseg;
  const int s = g - sg.b * nseg;
  const int kvh = s / n_hc;
  const int hc = s - kvh * n_hc;
  sg.h0 = kvh * group + hc * kGqaMaxHeads;
  const int left = group - hc * kGqaMaxHeads;
  sg.hv = left < kGqaMaxHeads ? left : kGqaMaxHeads;
  return sg;
}

// Segments whose cross-CTA merge this CTA owns, merged by the whole CTA once
// streaming is over.
struct GqaPending {
  int count;
  int g[kGqaMaxPending], c0[kGqaMaxPending], c1[kGqaMaxPending];
};
static_assert(sizeof(GqaPending) <= 64, "pending list slot");

// Writes one finished query head: fp16 output row, or the partial in
// partial mode. Lane l holds dims l + 32 i.
template <int D>
__device__ __forceinline__ void gqa_finish_head(const DecodeArgs &a, size_t gq,
                                                float M, float L,
                                                const float (&A)[D / 32],
                                                int lane) {
  if (a.partial_out) {
    float *p = a.partial_out + gq * GqaCfg<D>::kPF;
#pragma unroll
    for (int i = 0; i < D / 32; ++i) p[4 + 32 * i + lane] = A[i];
    if (lane == 0) {
      p[0] = M;
      p[1] = L;
      p[2] = 0.f;
      p[3] = 0.f;
    }
  } else {
    const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
    for (int i = 0; i < D / 32; ++i)
      a.out[gq * D + 32 * i + lane] = store_elem(A[i] * inv, a.dtype);
  }
}

// Merger warp: per query head of the finished piece, combines the consumer
// warps' partials; whole segments are written out, split ones published to
// workspace slot (g + cta) * hs + head (hs = query heads per segment) and
// queued for the cooperative merge when this CTA arrives last.
template <int D>
__device__ void merger_gqa(const DecodeArgs &a, int nseg, int n_hc, int group,
                           uint8_t *red_base, uint64_t *red_full,
                           uint64_t *red_empty, GqaPending *pend) {
  using C = GqaCfg<D>;
  const int lane = threadIdx.x & 31;
  const int hs = group < kGqaMaxHeads ? group : kGqaMaxHeads;
  for (int piece = 0;; ++piece) {
    const int buf = piece & 1;
    if (!mbar_wait(&red_full[buf], (piece >> 1) & 1)) return;
    const float *red =
        reinterpret_cast<const float *>(red_base + buf * C::kRedBufBytes);
    const int *hdr_in =
        reinterpret_cast<const int *>(red + C::kWarps * C::kRedWarpFloats);
    const int flags = hdr_in[1];
    if (flags & kDone) return;
    const int g = hdr_in[0];
    const int c0 = hdr_in[2];
    const int c1 = hdr_in[3];
    const GqaSegment sg = gqa_segment(g, nseg, n_hc, group);
    for (int i = 0; i < sg.hv; ++i) {
      float M = kNegBig;
#pragma unroll
      for (int w = 0; w < C::kWarps; ++w)
        M = fmaxf(M, red[w * C::kRedWarpFloats + i * C::kPF]);
      float L = 0.f, A[D / 32];
#pragma unroll
      for (int k = 0; k < D / 32; ++k) A[k] = 0.f;
#pragma unroll
      for (int w = 0; w < C::kWarps; ++w) {
        const float *pw = red + w * C::kRedWarpFloats + i * C::kPF;
        const float fw = fast_exp2(pw[0] - M);
        L = fmaf(pw[1], fw, L);
#pragma unroll
        for (int k = 0; k < D / 32; ++k)
          A[k] = fmaf(pw[4 + 32 * k + lane], fw, A[k]);
      }
      const size_t gq = static_cast<size_t>(sg.b) * a.H + sg.h0 + i;
      if (flags & kWhole) {
        gqa_finish_head<D>(a, gq, M, L, A, lane);
      } else {
        float *ws = a.ws_partials +
                    ((static_cast<size_t>(g) + blockIdx.x) * hs + i) * C::kPF;
#pragma unroll
        for (int k = 0; k < D / 32; ++k) ws[4 + 32 * k + lane] = A[k];
        if (lane == 0) {
          ws[0] = M;
          ws[1] = L;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&red_empty[buf]);  // buffer consumed
    if (flags & kWhole) continue;

    __threadfence();
    __syncwarp();
    unsigned last = 0;
    if (lane == 0) {
      const unsigned n_parts = static_cast<unsigned>(c1 - c0);
      last = atomicInc(&a.ws_counters[g], n_parts) == n_parts;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) continue;
    __threadfence();
    if (pend->count < kGqaMaxPending) {
      if (lane == 0) {
        const int k = pend->count;
        pend->g[k] = g;
        pend->c0[k] = c0;
        pend->c1[k] = c1;
        pend->count = k + 1;
      }
      __syncwarp();
      continue;
    }
    // more last arrivals than the list holds (rare): merge here, one warp
    for (int i = 0; i < sg.hv; ++i) {
      float M2 = kNegBig;
      for (int c = c0 + lane; c <= c1; c += 32) {
        const float *pp =
            a.ws_partials + ((static_cast<size_t>(g) + c) * hs + i) * C::kPF;
        if (__ldcg(pp + 1) > 0.f) M2 = fmaxf(M2, __ldcg(pp));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        M2 = fmaxf(M2, __shfl_xor_sync(0xffffffffu, M2, o));
      float L2 = 0.f, B[D / 32];
#pragma unroll
      for (int k = 0; k < D / 32; ++k) B[k] = 0.f;
      for (int c = c0; c <= c1; ++c) {
        const float *pp =
            a.ws_partials + ((static_cast<size_t>(g) + c) * hs + i) * C::kPF;
        const float lc = __ldcg(pp + 1);
        const float fc = lc > 0.f ? fast_exp2(__ldcg(pp) - M2) : 0.f;
        L2 = fmaf(lc, fc, L2);
#pragma unroll
        for (int k = 0; k < D / 32; ++k)
          B[k] = fmaf(__ldcg(pp + 4 + 32 * k + lane), fc, B[k]);
      }
      gqa_finish_head<D>(a, static_cast<size_t>(sg.b) * a.H + sg.h0 + i, M2,
                         L2, B, lane);
    }
  }
}

// Cooperative last-arrival merge of segment g over CTAs c0..c1 by all the
// threads of the CTA (every thread calls it). The partials are gathered into
// shared memory with bulk async copies (one copy of hv records per CTA, as
// many CTAs per round as `gather_bytes` holds), so each round costs one L2
// round trip, then combined there: per head a running (M, L), and each
// thread owns up to kOwn float4s of the heads' outputs.
template <int D>
__device__ void coop_merge(const DecodeArgs &a, int g, int c0, int c1,
                           const GqaSegment &sg, int hs, uint8_t *gather,
                           uint32_t gather_bytes, float *stats,
                           uint64_t *gbar, uint32_t &gphase) {
  using C = GqaCfg<D>;
  constexpr int kQ = D / 4;  // float4s per head
  const int tid = static_cast<int>(threadIdx.x);
  const int nthreads = static_cast<int>(blockDim.x);
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = nthreads >> 5;
  const int nc = c1 - c0 + 1;
  const uint32_t rec_bytes = static_cast<uint32_t>(sg.hv) * C::kPF * 4;
  const int per_round = static_cast<int>(gather_bytes / rec_bytes);
  const float *recs = reinterpret_cast<const float *>(gather);
  const int outs = sg.hv * kQ;
  float4 acc[C::kOwn];
#pragma unroll
  for (int k = 0; k < C::kOwn; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  // stats: per head M, L (running) and the previous M of the round
  for (int i = tid; i < sg.hv; i += nthreads) {
    stats[3 * i] = kNegBig;
    stats[3 * i + 1] = 0.f;
  }
  for (int cb = 0; cb < nc; cb += per_round) {
    const int n = nc - cb < per_round ? nc - cb : per_round;
    if (warp == 0) {
      // generic-proxy writes of the partials (other CTAs, ordered by the
      // counter) and earlier shared-memory use come before the async copies
      asm volatile("fence.proxy.async.global;" ::: "memory");
      fence_proxy_async_smem();
      if (lane == 0) mbar_arrive_expect_tx(gbar, rec_bytes * n);
      __syncwarp();
      for (int c = lane; c < n; c += 32) {
        const float *src = a.ws_partials +
                           (static_cast<size_t>(g) + c0 + cb + c) * hs * C::kPF;
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
            "[%0], [%1], %2, [%3];" ::"r"(smem_u32(gather + c * rec_bytes)),
            "l"(src), "r"(rec_bytes), "r"(smem_u32(gbar))
            : "memory");
      }
    }
    const bool ok = mbar_wait(gbar, gphase);
    gphase ^= 1u;
    if (!__syncthreads_and(ok)) break;  // uniform: every thread leaves
    for (int i = warp; i < sg.hv; i += nwarps) {
      float mx = kNegBig;
      for (int c = lane; c < n; c += 32) {
        const float *r = recs + (c * sg.hv + i) * C::kPF;
        if (r[1] > 0.f) mx = fmaxf(mx, r[0]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = stats[3 * i];
      const float m_new = fmaxf(m_old, mx);
      float l = 0.f;
      for (int c = lane; c < n; c += 32) {
        const float *r = recs + (c * sg.hv + i) * C::kPF;
        if (r[1] > 0.f) l = fmaf(r[1], fast_exp2(r[0] - m_new), l);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      __syncwarp();
      if (lane == 0) {
        stats[3 * i + 1] = fmaf(stats[3 * i + 1], fast_exp2(m_old - m_new), l);
        stats[3 * i] = m_new;
        stats[3 * i + 2] = m_old;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < C::kOwn; ++k) {
      const int o = tid + k * nthreads;
      if (o >= outs) continue;
      const int i = o / kQ, dq = o % kQ;
      const float m_new = stats[3 * i];
      const float f = fast_exp2(stats[3 * i + 2] - m_new);
      float4 v = acc[k];
      v.x *= f;
      v.y *= f;
      v.z *= f;
      v.w *= f;
      for (int c = 0; c < n; ++c) {
        const float *r = recs + (c * sg.hv + i) * C::kPF;
        const float w = r[1] > 0.f ? fast_exp2(r[0] - m_new) : 0.f;
        const float4 x = *reinterpret_cast<const float4 *>(r + 4 + 4 * dq);
        v.x = fmaf(w, x.x, v.x);
        v.y = fmaf(w, x.y, v.y);
        v.z = fmaf(w, x.z, v.z);
        v.w = fmaf(w, x.w, v.w);
      }
      acc[k] = v;
    }
    __syncthreads();  // the buffer is free for the next round
  }
#pragma unroll
  for (int k = 0; k < C::kOwn; ++k) {
    const int o = tid + k * nthreads;
    if (o >= outs) continue;
    const int i = o / kQ, dq = o % kQ;
    const size_t gq = static_cast<size_t>(sg.b) * a.H + sg.h0 + i;
    const float M = stats[3 * i], L = stats[3 * i + 1];
    if (a.partial_out) {
      float *p = a.partial_out + gq * C::kPF;
      *reinterpret_cast<float4 *>(p + 4 + 4 * dq) = acc[k];
      if (dq == 0) {
        p[0] = M;
        p[1] = L;
        p[2] = 0.f;
        p[3] = 0.f;
      }
    } else {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      const bool bf = a.dtype == FA_DTYPE_BF16;
      uint2 v;
      v.x = bf ? BF16::pack2(acc[k].x * inv, acc[k].y * inv)
               : F16::pack2(acc[k].x * inv, acc[k].y * inv);
      v.y = bf ? BF16::pack2(acc[k].z * inv, acc[k].w * inv)
               : F16::pack2(acc[k].z * inv, acc[k].w * inv);
      *reinterpret_cast<uint2 *>(a.out + gq * D + 4 * dq) = v;
    }
  }
  __syncthreads();
}

// Consumer warps of the grouped kernel.
template <int D, typename Dt>
__device__ __forceinline__ void gqa_consume(
    const DecodeArgs &a, int nseg, int n_hc, int group, uint8_t *smem,
    uint64_t *full, uint64_t *empty, uint64_t *red_full, uint64_t *red_empty,
    const StageHeader *hdr) {
  using C = GqaCfg<D>;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int quad = lane >> 2;  // MMA row (query head) quad and quad + 8
  const int qid = lane & 3;    // MMA column pair
  const int key0 = warp * 16;  // this warp's keys within a stage
  uint32_t qa[D / 16][4];      // Q as the A operand, head dims 16kk..16kk+16
  float o[D / 8][4];           // O: dims 8dt + 2qid (+1), rows quad / quad+8
  float m_r[2], l_r[2];
  int cur_g = -1;
  int app_row = -1;  // segment row of the appended token, -1 for none
  uint4 app_val = make_uint4(0, 0, 0, 0);
  int piece = 0;
  auto reset = [&]() {
    m_r[0] = m_r[1] = kNegBig;
    l_r[0] = l_r[1] = 0.f;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[dt][e] = 0.f;
  };
  reset();

  for (int it = 0;; ++it) {
    const int slot = it % C::kStages;
    if (!mbar_wait(&full[slot], (it / C::kStages) & 1)) break;
    const StageHeader hd = hdr[slot];
    if (hd.flags & kDone) {
      const int buf = piece & 1;
      if (piece >= kRedBufs &&
          !mbar_wait(&red_empty[buf], ((piece >> 1) - 1) & 1))
        break;
      if (warp == 0 && lane == 0) {
        int *hdr_out = reinterpret_cast<int *>(
            smem + C::kRedOff + buf * C::kRedBufBytes +
            C::kWarps * C::kRedWarpFloats * 4);
        hdr_out[1] = kDone;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[buf]);
      break;
    }
    if (hd.g != cur_g) {
      cur_g = hd.g;
      const GqaSegment sg = gqa_segment(cur_g, nseg, n_hc, group);
      app_row = a.k_new ? appended_row(a, sg.b) : -1;
      if (app_row >= 0)
        app_val = load_new_row<D>(a, sg.b * a.H_kv + (cur_g - sg.b * nseg) / n_hc);
      const uint32_t *q0 =
          quad < sg.hv
              ? reinterpret_cast<const uint32_t *>(
                    a.q + (static_cast<size_t>(sg.b) * a.H + sg.h0 + quad) * D)
              : nullptr;
      const uint32_t *q1 =
          quad + 8 < sg.hv
              ? reinterpret_cast<const uint32_t *>(
                    a.q + (static_cast<size_t>(sg.b) * a.H + sg.h0 + quad + 8) * D)
              : nullptr;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        qa[kk][0] = q0 ? q0[8 * kk + qid] : 0u;
        qa[kk][1] = q1 ? q1[8 * kk + qid] : 0u;
        qa[kk][2] = q0 ? q0[8 * kk + 4 + qid] : 0u;
        qa[kk][3] = q1 ? q1[8 * kk + 4 + qid] : 0u;
      }
    }

    if (app_row >= 0) {
      const int local = app_row - hd.r0;
      if (local >= key0 && local < key0 + 16 && local < hd.n) {
        const int b = hd.g / nseg;
        const int s_in_b = hd.g - b * nseg;
        patch_new_row<true, D, C::kRows>(a, b * a.H_kv + s_in_b / n_hc, app_row, local,
                            smem + C::kKOff + slot * kStageBytes,
                            smem + C::kVOff + slot * kStageBytes,
                            s_in_b % n_hc == 0, app_val);
      }
    }
    if (key0 < hd.n) {  // warp-uniform
      const uint32_t kb = smem_u32(smem + C::kKOff + slot * kStageBytes);
      const uint32_t vb = smem_u32(smem + C::kVOff + slot * kStageBytes);
      // S = Q K^T for keys key0 + 8j + [0, 8): two k-steps (32 head dims,
      // four 16-byte chunks of a 64-dim block) per ldmatrix
      float sc[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[j][e] = 0.f;
        const int row = key0 + 8 * j + (lane & 7);
#pragma unroll
        for (int pp = 0; pp < D / 32; ++pp) {
          const int blk = pp >> 1;
          const int chunk = 4 * (pp & 1) + (lane >> 3);
          uint32_t kf[4];
          ldsm_x4(kb + blk * C::kBlock + row * 128 +
                      ((chunk ^ (row & 7)) << 4),
                  kf);
          Dt::mma16816(sc[j], qa[2 * pp], kf[0], kf[1]);
          Dt::mma16816(sc[j], qa[2 * pp + 1], kf[2], kf[3]);
        }
      }
      // online softmax per head row (rows quad and quad + 8)
      const int n_here = hd.n - key0;
      float x[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = 8 * j + 2 * qid + (e & 1);
          x[j][e] = key < n_here ? sc[j][e] * a.scale_log2 : -INFINITY;
        }
      float mx0 = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
      float mx1 = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m_r[0], mx0);
      const float mn1 = fmaxf(m_r[1], mx1);
      const float corr0 = fast_exp2(m_r[0] - mn0);
      const float corr1 = fast_exp2(m_r[1] - mn1);
      m_r[0] = mn0;
      m_r[1] = mn1;
      float p[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        p[j][0] = fast_exp2(x[j][0] - mn0);
        p[j][1] = fast_exp2(x[j][1] - mn0);
        p[j][2] = fast_exp2(x[j][2] - mn1);
        p[j][3] = fast_exp2(x[j][3] - mn1);
      }
      l_r[0] = fmaf(l_r[0], corr0, (p[0][0] + p[0][1]) + (p[1][0] + p[1][1]));
      l_r[1] = fmaf(l_r[1], corr1, (p[0][2] + p[0][3]) + (p[1][2] + p[1][3]));
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[dt][0] *= corr0;
        o[dt][1] *= corr0;
        o[dt][2] *= corr1;
        o[dt][3] *= corr1;
      }
      // P as the A operand: k index = key within the 16 (C -> A layout)
      const uint32_t pa[4] = {Dt::pack2(p[0][0], p[0][1]),
                              Dt::pack2(p[0][2], p[0][3]),
                              Dt::pack2(p[1][0], p[1][1]),
                              Dt::pack2(p[1][2], p[1][3])};
      // O += P V over dims 8dt..8dt+8, V read transposed; chunk c of the
      // row (8 dims) lives in block c / 8
      const int vrow = key0 + 8 * ((lane >> 3) & 1) + (lane & 7);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int chunk = 2 * dp + (lane >> 4);
        uint32_t vf[4];
        ldsm_x4_trans(vb + (chunk >> 3) * C::kBlock + vrow * 128 +
                          (((chunk & 7) ^ (vrow & 7)) << 4),
                      vf);
        Dt::mma16816(o[2 * dp], pa, vf[0], vf[1]);
        Dt::mma16816(o[2 * dp + 1], pa, vf[2], vf[3]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);

    if (!(hd.flags & kLast)) continue;

    // ---- piece complete: per head row (m, l, O) of this warp to the merger
    float l0 = l_r[0], l1 = l_r[1];
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const int buf = piece & 1;
    if (piece >= kRedBufs &&
        !mbar_wait(&red_empty[buf], ((piece >> 1) - 1) & 1))
      break;
    float *red =
        reinterpret_cast<float *>(smem + C::kRedOff + buf * C::kRedBufBytes);
    float *r0p = red + warp * C::kRedWarpFloats + quad * C::kPF;
    float *r1p = r0p + 8 * C::kPF;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      *reinterpret_cast<float2 *>(r0p + 4 + 8 * dt + 2 * qid) =
          make_float2(o[dt][0], o[dt][1]);
      *reinterpret_cast<float2 *>(r1p + 4 + 8 * dt + 2 * qid) =
          make_float2(o[dt][2], o[dt][3]);
    }
    if (qid == 0) {
      r0p[0] = m_r[0];
      r0p[1] = l0;
      r1p[0] = m_r[1];
      r1p[1] = l1;
    }
    if (warp == 0 && lane == 0) {
      int *hdr_out =
          reinterpret_cast<int *>(red + C::kWarps * C::kRedWarpFloats);
      hdr_out[0] = hd.g;
      hdr_out[1] = hd.flags;
      hdr_out[2] = hd.c0;
      hdr_out[3] = hd.c1;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&red_full[buf]);
    ++piece;
    reset();
  }
}

template <int D, typename Dt>
__global__ void __launch_bounds__(GqaCfg<D>::kThreads, 1)
    decode_gqa_kernel(const DecodeArgs a,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v) {
  using C = GqaCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::kBarOff);
  uint64_t *empty = full + C::kStages;
  uint64_t *red_full = empty + C::kStages;
  uint64_t *red_empty = red_full + kRedBufs;
  StageHeader *hdr = reinterpret_cast<StageHeader *>(smem + C::kHdrOff);
  // (the device error word is read by the producer: produce())
  if (smem_u32(smem) & 1023u) {  // the swizzled stages need 1 KiB alignment
    if (threadIdx.x == 0) record_error(FA_ERR_SMEM_ALIGN);
    return;
  }
  const int group = a.H / a.H_kv;
  const int n_hc = (group + kGqaMaxHeads - 1) / kGqaMaxHeads;
  const int nseg = a.H_kv * n_hc;

  GqaPending *pend = reinterpret_cast<GqaPending *>(smem + C::kPendOff);
  if (threadIdx.x == 0) {
    pend->count = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::kWarps);
    }
    for (int r = 0; r < kRedBufs; ++r) {
      mbar_init(&red_full[r], C::kWarps);
      mbar_init(&red_empty[r], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == C::kWarps) {
    if (lane == 0) {
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      if (D != kHeadDim) {
        // the shared planner writes 64-wide empty rows only
        for (int b = 0; b < a.B; ++b) {
          if (seq_rows(a, b) != 0 ||
              (b % static_cast<int>(gridDim.x)) != static_cast<int>(blockIdx.x))
            continue;
          for (int h = 0; h < a.H; ++h) {
            __half *o = a.out + (static_cast<size_t>(b) * a.H + h) * D;
            for (int i = 0; i < D; ++i) o[i] = __float2half_rn(0.f);
          }
        }
      }
    }
    __syncwarp();
    produce<true, C::kStages, D, C::kRows>(a, nseg, n_hc, smem, C::kKOff,
                                           C::kVOff, full, empty, hdr, &tm_k,
                                           &tm_v);
  } else if (warp == C::kWarps + 1) {
    merger_gqa<D>(a, nseg, n_hc, group, smem + C::kRedOff, red_full,
                  red_empty, pend);
  } else {
    gqa_consume<D, Dt>(a, nseg, n_hc, group, smem, full, empty, red_full,
                   red_empty, hdr);
  }
  // Streaming is over for every warp (the stage and hand-off buffers are
  // free): the whole CTA merges the segments it arrived on last.
  __syncthreads();
  const int hs = group < kGqaMaxHeads ? group : kGqaMaxHeads;
  // everything below the barriers is free now: gather area + stats
  float *stats =
      reinterpret_cast<float *>(smem + C::kBarOff) - 3 * kGqaMaxHeads;
  uint8_t *gather = smem;
  const uint32_t gather_bytes = C::kBarOff - 3 * kGqaMaxHeads * 4;
  uint64_t *gbar = red_empty + kRedBufs;
  if (threadIdx.x == 0) {
    mbar_init(gbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  uint32_t gphase = 0;
  for (int k = 0; k < pend->count; ++k) {
    const GqaSegment sg = gqa_segment(pend->g[k], nseg, n_hc, group);
    coop_merge<D>(a, pend->g[k], pend->c0[k], pend->c1[k], sg, hs, gather,
                  gather_bytes, stats, gbar, gphase);
  }
}

}  // namespace decode

const void *decode_gqa_kernel_ptr(int head_dim, int dtype) {
  const bool bf = dtype == FA_DTYPE_BF16;
  if (head_dim == 128)
    return bf ? reinterpret_cast<const void *>(
                    decode::decode_gqa_kernel<128, BF16>)
              : reinterpret_cast<const void *>(
                    decode::decode_gqa_kernel<128, F16>);
  return bf ? reinterpret_cast<const void *>(decode::decode_gqa_kernel<64, BF16>)
            : reinterpret_cast<const void *>(decode::decode_gqa_kernel<64, F16>);
}
int decode_gqa_smem_bytes(int head_dim) {
  return static_cast<int>(head_dim == 128 ? decode::GqaCfg<128>::kSmemBytes
                                          : decode::GqaCfg<64>::kSmemBytes);
}
int decode_gqa_max_heads() { return decode::kGqaMaxHeads; }
int decode_gqa_merge_batch(int head_dim, int heads_per_seg) {
  // partial records of one segment that one gather round of the final merge
  // holds (coop_merge: the stage buffers less the per-head statistics)
  const uint32_t bar_off = head_dim == 128 ? decode::GqaCfg<128>::kBarOff
                                           : decode::GqaCfg<64>::kBarOff;
  const uint32_t pf = head_dim == 128 ? decode::GqaCfg<128>::kPF
                                      : decode::GqaCfg<64>::kPF;
  const uint32_t gather = bar_off - 3 * decode::kGqaMaxHeads * 4;
  const uint32_t rec = static_cast<uint32_t>(heads_per_seg) * pf * 4;
  return rec > 0 ? static_cast<int>(gather / rec) : 1;
}
int decode_gqa_box_rows(int head_dim) {
  return head_dim == 128 ? decode::GqaCfg<128>::kRows
                         : decode::GqaCfg<64>::kRows;
}

cudaError_t launch_decode_gqa_kernel(const DecodeArgs &args,
                                     const CUtensorMap &tm_k,
                                     const CUtensorMap &tm_v, int head_dim,
                                     cudaStream_t stream) {
  const bool bf = args.dtype == FA_DTYPE_BF16;
  if (head_dim == 128) {
    using C = decode::GqaCfg<128>;
    auto kernel = bf ? decode::decode_gqa_kernel<128, BF16>
                     : decode::decode_gqa_kernel<128, F16>;
    kernel<<<args.grid, C::kThreads, C::kSmemBytes, stream>>>(args, tm_k, tm_v);
  } else {
    using C = decode::GqaCfg<64>;
    auto kernel = bf ? decode::decode_gqa_kernel<64, BF16>
                     : decode::decode_gqa_kernel<64, F16>;
    kernel<<<args.grid, C::kThreads, C::kSmemBytes, stream>>>(args, tm_k, tm_v);
  }
  return cudaGetLastError();
}

}  // namespace fa
