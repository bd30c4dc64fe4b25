// Decode attention for head_dim 128 on B200: the per-head split-K kernel of
// decode_sm100.cu re-sized for 256-byte cache rows (same semantics:
// reference csrc/decode.cu:50-175 restated for d = 128, which the reference
// names as its next size).
//
// Same machine as the 64 kernel: the valid rows of all (b, h) segments are
// laid end to end and cut into equal pieces by a persistent grid; warp 8
// plans and streams (produce<>), warps 0-7 consume, warp 9 finishes pieces
// and merges segments split across CTAs (slot g + cta, last arrival on the
// segment's counter merges). Stages stay 16 KiB, now 64 rows; each row is
// read by 16 lanes (16 bytes, 8 head dims per lane), a warp covers 2 rows
// per instruction and 8 rows of a stage. Partials are (m, l, pad, pad,
// acc[128]) = 132 floats.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "fa_kernels.h"
#include "fa_sm100.cuh"

namespace fa {
namespace decode128 {

using decode::StageHeader;
using decode::kLast;
using decode::kWhole;
using decode::kDone;
using decode::kNegBig;

constexpr int kD = 128;
constexpr int kRowB = 2 * kD;
constexpr int kPF = 4 + kD;  // partial floats
constexpr int kConsumerWarps = 8;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kMergerWarp = kConsumerWarps + 1;
constexpr int kThreads = (kConsumerWarps + 2) * 32;
constexpr int kStageRows = 64;
constexpr int kStages = 3;
constexpr int kLanesPerRow = kD / 8;                     // 16
constexpr int kRowsPerInstr = 32 / kLanesPerRow;         // 2
constexpr int kRowsPerWarp = kStageRows / kConsumerWarps;  // 8
constexpr int kRowIters = kRowsPerWarp / kRowsPerInstr;  // 4
constexpr int kCtasPerSm = 2;
constexpr uint32_t kStageBytes = kStageRows * kRowB;  // 16 KiB
static_assert(kStageBytes == decode::kStageBytes, "stages keep their size");

constexpr uint32_t kKOff = 0;
constexpr uint32_t kVOff = kStages * kStageBytes;
constexpr uint32_t kHdrOff = 2 * kStages * kStageBytes;
constexpr uint32_t kRedOff = kHdrOff + kStages * sizeof(StageHeader);
constexpr int kRedBufs = 2;
constexpr uint32_t kRedBufBytes = kConsumerWarps * kPF * 4 + 32;
constexpr uint32_t kBarOff = kRedOff + kRedBufs * kRedBufBytes;
constexpr uint32_t kSmemBytes = kBarOff + (2 * kStages + 2 * kRedBufs) * 8;

__device__ void write_empty_sequence(const DecodeArgs &a, int b) {
  for (int h = 0; h < a.H; ++h) {
    const size_t g = static_cast<size_t>(b) * a.H + h;
    if (a.partial_out) {
      float *p = a.partial_out + g * kPF;
      p[0] = kNegBig;
      for (int i = 1; i < kPF; ++i) p[i] = 0.f;
    } else {
      uint4 *o = reinterpret_cast<uint4 *>(a.out + g * kD);
      for (int i = 0; i < kD / 8; ++i) o[i] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Lane l holds dims l, l + 32, l + 64, l + 96.
__device__ __forceinline__ void finish_segment(const DecodeArgs &a, size_t g,
                                               float M, float L,
                                               const float (&A)[4], int lane) {
  if (a.x_peers) {  // sequence-sharded: send to every rank, merge all
    decode::x_send_deferred<kD>(a, g, M, L, A, lane);
    return;
  }
  if (a.partial_out) {
    float *p = a.partial_out + g * kPF;
#pragma unroll
    for (int i = 0; i < 4; ++i) p[4 + 32 * i + lane] = A[i];
    if (lane == 0) {
      p[0] = M;
      p[1] = L;
      p[2] = 0.f;
      p[3] = 0.f;
    }
  } else {
    const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      a.out[g * kD + 32 * i + lane] = store_elem(A[i] * inv, a.dtype);
  }
}

__device__ void merger(const DecodeArgs &a, uint8_t *red_base,
                       uint64_t *red_full, uint64_t *red_empty) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) decode::x_deferred().n = 0;
  __syncwarp();
  for (int piece = 0;; ++piece) {
    const int buf = piece & 1;
    if (!mbar_wait(&red_full[buf], (piece >> 1) & 1)) return;
    const float *red = reinterpret_cast<const float *>(red_base + buf * kRedBufBytes);
    const int *hdr_in = reinterpret_cast<const int *>(red + kConsumerWarps * kPF);
    const int flags = hdr_in[1];
    if (flags & kDone) {
      if (a.x_peers) decode::x_finish_deferred<kD>(a, lane);
      return;
    }
    const size_t g = static_cast<size_t>(hdr_in[0]);
    const int c0 = hdr_in[2];
    const int c1 = hdr_in[3];
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red[w * kPF]);
    float L = 0.f, A[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float fw = fast_exp2(red[w * kPF] - M);
      L = fmaf(red[w * kPF + 1], fw, L);
#pragma unroll
      for (int i = 0; i < 4; ++i)
        A[i] = fmaf(red[w * kPF + 4 + 32 * i + lane], fw, A[i]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&red_empty[buf]);

    if (flags & kWhole) {
      finish_segment(a, g, M, L, A, lane);
      continue;
    }
    float *ws = a.ws_partials + (g + blockIdx.x) * static_cast<size_t>(kPF);
#pragma unroll
    for (int i = 0; i < 4; ++i) ws[4 + 32 * i + lane] = A[i];
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
    __threadfence();
    float M2 = kNegBig;
    for (int c = c0 + lane; c <= c1; c += 32) {
      const float *pp = a.ws_partials + (g + c) * static_cast<size_t>(kPF);
      if (__ldcg(pp + 1) > 0.f) M2 = fmaxf(M2, __ldcg(pp));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      M2 = fmaxf(M2, __shfl_xor_sync(0xffffffffu, M2, o));
    float L2 = 0.f, B[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int c = c0; c <= c1; ++c) {
      const float *pp = a.ws_partials + (g + c) * static_cast<size_t>(kPF);
      const float lc = __ldcg(pp + 1);
      const float mc = __ldcg(pp);
      float x[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = __ldcg(pp + 4 + 32 * i + lane);
      const float fc = lc > 0.f ? fast_exp2(mc - M2) : 0.f;
      L2 = fmaf(lc, fc, L2);
#pragma unroll
      for (int i = 0; i < 4; ++i) B[i] = fmaf(x[i], fc, B[i]);
    }
    finish_segment(a, g, M2, L2, B, lane);
  }
}

template <typename Dt>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    decode_d128_kernel(const DecodeArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint64_t *empty = full + kStages;
  StageHeader *hdr = reinterpret_cast<StageHeader *>(smem + kHdrOff);
  uint64_t *red_full = empty + kStages;
  uint64_t *red_empty = red_full + kRedBufs;
  // (the device error word is read by the producer: decode::produce())

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

  if (warp == kProducerWarp) {
    // empty sequences are written here: the shared planner writes 64-wide
    // rows, so it only sees their lengths
    for (int b = lane; b < a.B; b += 32) {
      const int len = decode::seq_rows(a, b);
      if (len == 0 && !a.x_peers &&  // sharded: exchanged in produce()
          (b % static_cast<int>(gridDim.x)) == static_cast<int>(blockIdx.x))
        write_empty_sequence(a, b);
    }
    decode::produce<false, kStages, kD, kStageRows>(
        a, a.H, a.H / a.H_kv, smem, kKOff, kVOff, full, empty, hdr, nullptr,
        nullptr);
    return;
  }
  if (warp == kMergerWarp) {
    merger(a, smem + kRedOff, red_full, red_empty);
    return;
  }

  // ---------------------------------------------------------------- consumers
  const int grp = lane / kLanesPerRow;  // which of the warp's 2 rows
  const int sub = lane % kLanesPerRow;  // head dims [8*sub, 8*sub + 8)
  float qf[8];
  int cur_g = -1;
  int app_row = -1;  // segment row of the appended token, -1 for none
  uint4 app_val = make_uint4(0, 0, 0, 0);
  float m_run = kNegBig, l_run = 0.f;
  int piece = 0;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;

  for (int it = 0;; ++it) {
    const int slot = it % kStages;
    if (!mbar_wait(&full[slot], (it / kStages) & 1)) break;
    const StageHeader hd = hdr[slot];
    if (hd.flags & kDone) {
      const int buf = piece & 1;
      if (piece >= kRedBufs &&
          !mbar_wait(&red_empty[buf], ((piece >> 1) - 1) & 1))
        break;
      if (warp == 0 && lane == 0) {
        int *hdr_out = reinterpret_cast<int *>(smem + kRedOff + buf * kRedBufBytes +
                                               kConsumerWarps * kPF * 4);
        hdr_out[1] = kDone;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&red_full[buf]);
      break;
    }
    if (hd.g != cur_g) {
      cur_g = hd.g;
      if (a.k_new) {
        app_row = decode::appended_row(a, cur_g / a.H);
        if (app_row >= 0) app_val = decode::load_new_row<kD>(a, cur_g);
      }
      const uint4 qv = *reinterpret_cast<const uint4 *>(
          a.q + static_cast<size_t>(cur_g) * kD + sub * 8);
      const uint32_t *qh = reinterpret_cast<const uint32_t *>(&qv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = Dt::unpack2(qh[e]);
        qf[2 * e] = f.x * a.scale_log2;
        qf[2 * e + 1] = f.y * a.scale_log2;
      }
    }

    if (app_row >= 0) {  // fused append: the owner warp patches and stores
      const int local = app_row - hd.r0;
      if (local >= 0 && local < hd.n && warp == local / kRowsPerWarp)
        decode::patch_new_row<false, kD, kStageRows>(
            a, hd.g, app_row, local, smem + kKOff + slot * kStageBytes,
            smem + kVOff + slot * kStageBytes, true, app_val);
    }
    const uint32_t kb = smem_u32(smem + kKOff + slot * kStageBytes);
    const uint32_t vb = smem_u32(smem + kVOff + slot * kStageBytes);
    const int row_base = warp * kRowsPerWarp + grp;
    if (warp * kRowsPerWarp < hd.n) {  // warp-uniform: shuffles below
      float sc[kRowIters];
#pragma unroll
      for (int i = 0; i < kRowIters; ++i) {
        const int row = row_base + kRowsPerInstr * i;
        float d = 0.f;
        if (row < hd.n) {
          const uint4 kv = ld_shared_v4(kb + row * kRowB + sub * 16);
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
#pragma unroll
        for (int o = 1; o < kLanesPerRow; o <<= 1)
          sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], o);
        if (row_base + kRowsPerInstr * i >= hd.n) sc[i] = -INFINITY;
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
        const int row = row_base + kRowsPerInstr * i;
        if (row < hd.n) {
          const uint4 vv = ld_shared_v4(vb + row * kRowB + sub * 16);
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

    // ---- piece complete: combine the warp's 2 row groups, hand to merger
    float m_w = fmaxf(m_run, __shfl_xor_sync(0xffffffffu, m_run, 16));
    const float f = fast_exp2(m_run - m_w);
    float l_w = l_run * f;
    l_w += __shfl_xor_sync(0xffffffffu, l_w, 16);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float v = acc[e] * f;
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      acc[e] = v;
    }
    const int buf = piece & 1;
    if (piece >= kRedBufs &&
        !mbar_wait(&red_empty[buf], ((piece >> 1) - 1) & 1))
      break;
    float *red = reinterpret_cast<float *>(smem + kRedOff + buf * kRedBufBytes);
    float *my = red + warp * kPF;
    if (lane < kLanesPerRow) {
#pragma unroll
      for (int e = 0; e < 8; ++e) my[4 + lane * 8 + e] = acc[e];
      if (lane == 0) {
        my[0] = m_w;
        my[1] = l_w;
      }
    }
    if (warp == 0 && lane == 0) {
      int *hdr_out = reinterpret_cast<int *>(red + kConsumerWarps * kPF);
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

}  // namespace decode128

const void *decode_d128_kernel_ptr(int dtype) {
  return dtype == FA_DTYPE_BF16
             ? reinterpret_cast<const void *>(decode128::decode_d128_kernel<BF16>)
             : reinterpret_cast<const void *>(decode128::decode_d128_kernel<F16>);
}
int decode_d128_smem_bytes() {
  return static_cast<int>(decode128::kSmemBytes);
}
int decode_d128_partial_floats() { return decode128::kPF; }

cudaError_t launch_decode_d128_kernel(const DecodeArgs &args,
                                      cudaStream_t stream) {
  auto kernel = args.dtype == FA_DTYPE_BF16
                    ? decode128::decode_d128_kernel<BF16>
                    : decode128::decode_d128_kernel<F16>;
  kernel<<<args.grid, decode128::kThreads, decode128::kSmemBytes, stream>>>(
      args);
  return cudaGetLastError();
}

}  // namespace fa
