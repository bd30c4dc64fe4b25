// Prefill (full-sequence) attention forward for B200, head_dim 64, fp16 in,
// fp32 accumulate, fp16 out.
//
// Behaviour follows the reference's prefill_kernel (csrc/prefill.cu:164-343):
// O = softmax(scale * Q K^T, causal mask k <= q) V per (batch, head), with
// fully-masked causal key tiles skipped. The implementation is a different
// machine: QK^T and PV run on the 5th-generation tensor cores (tcgen05.mma,
// fp32 accumulators in tensor memory), Q/K/V tiles arrive by TMA into a
// two-stage mbarrier ring, and the online softmax runs in registers of four
// dedicated warps that read S straight out of tensor memory.
//
// CTA = 6 warps, one 128-row query tile of one (batch, head):
//   warps 0-3  softmax: thread t owns query row t (= TMEM lane t). Reads S,
//              applies mask / running max / exp2 / row sum, writes P (fp16)
//              into shared memory, rescales O in TMEM when the max moved.
//   warp 4     TMA producer: Q once, then K_j, V_j per 128-key tile.
//   warp 5     MMA issuer (one thread): S_j = Q K_j^T, O += P_j V_j.
// Two CTAs share an SM (112 KiB shared memory and 256 TMEM columns each), so
// one CTA's softmax overlaps the other's tensor-core work; inside a CTA, S_{j+1}
// is computed while the softmax warps exponentiate S_j.
//
// Shared memory (1 KiB aligned, every tile in the 128-byte-swizzled layout
// the TMA writes and the MMA descriptors describe):
//   Q  [128 rows x 128 B]            16 KiB
//   K  2 stages x [128 keys x 128 B] 32 KiB
//   V  2 stages x [128 keys x 128 B] 32 KiB
//   P  2 halves x [128 rows x 64 keys x 2 B] 32 KiB  (keys 0-63, 64-127)
//   mbarriers, TMEM base address, abort flag
// Tensor memory: S at columns [0,128), O at columns [128,192).

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "fa_sm100.cuh"
#include "fa_kernels.h"

namespace fa {
namespace prefill {

constexpr int kBlockM = 128;  // query rows per CTA
constexpr int kBlockN = 128;  // keys per KV tile
constexpr int kStages = 2;
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr uint32_t kTileBytes = kBlockN * kRowBytes;  // 16 KiB

constexpr uint32_t kQOff = 0;
constexpr uint32_t kKOff = kQOff + kTileBytes;
constexpr uint32_t kVOff = kKOff + kStages * kTileBytes;
constexpr uint32_t kPOff = kVOff + kStages * kTileBytes;
constexpr uint32_t kBarOff = kPOff + 2 * kTileBytes;
// barrier slots
constexpr int kBarQFull = 0;
constexpr int kBarKFull = 1;                     // + stage
constexpr int kBarVFull = kBarKFull + kStages;   // + stage
constexpr int kBarKVEmpty = kBarVFull + kStages; // + stage
constexpr int kBarSFull = kBarKVEmpty + kStages;
constexpr int kBarSFree = kBarSFull + 1;
constexpr int kBarPFull = kBarSFree + 1;
constexpr int kBarODone = kBarPFull + 1;
constexpr int kBarDrain = kBarODone + 1;
constexpr int kNumBars = kBarDrain + 1;
constexpr uint32_t kTmemSlotOff = kBarOff + kNumBars * 8;
constexpr uint32_t kAbortOff = kTmemSlotOff + 4;
constexpr uint32_t kSmemBytes = kAbortOff + 4 + 8;

constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kTmemS = 0;
constexpr uint32_t kTmemO = 128;

constexpr uint32_t kIdescS = idesc_f16_f32(kBlockM, kBlockN, false);
constexpr uint32_t kIdescPV = idesc_f16_f32(kBlockM, kHeadDim, true);

// The max is only moved (and O rescaled) when a row's running max grows by
// more than this many powers of two; until then exponents are taken against
// the stale max, which bounds P by 2^8 and keeps l and O consistent because
// both use the same reference point.
constexpr float kRescaleThreshold = 8.0f;

__global__ void __launch_bounds__(kThreads, 2)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                   const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v,
                   __half *__restrict__ out, int N, int BH, int causal,
                   float scale_log2) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (device_failed()) return;
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) record_error(FA_ERR_SMEM_ALIGN);
    return;
  }

  // Heaviest causal tiles first: blockIdx.x walks query tiles from the last
  // (most keys) to the first, heads fastest.
  const int n_qt = (N + kBlockM - 1) / kBlockM;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x / BH);
  const int bh = static_cast<int>(blockIdx.x % BH);
  const int n_kv = causal ? (qt + 1) : (N + kBlockN - 1) / kBlockN;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kBarOff);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kTmemSlotOff);
  volatile uint32_t *abort_flag =
      reinterpret_cast<volatile uint32_t *>(smem + kAbortOff);

  if (threadIdx.x == 0) {
    mbar_init(&bars[kBarQFull], 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kBarKFull + s], 1);
      mbar_init(&bars[kBarVFull + s], 1);
      mbar_init(&bars[kBarKVEmpty + s], 1);
    }
    mbar_init(&bars[kBarSFull], 1);
    mbar_init(&bars[kBarSFree], kSoftmaxThreads);
    mbar_init(&bars[kBarPFull], kSoftmaxThreads);
    mbar_init(&bars[kBarODone], 1);
    mbar_init(&bars[kBarDrain], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const uint32_t sbase = smem_u32(smem);

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA
    if (lane == 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
      prefetch_tensormap(&tm_v);
      mbar_arrive_expect_tx(&bars[kBarQFull], kTileBytes);
      tma_load_3d(smem + kQOff, &tm_q, &bars[kBarQFull], 0, qt * kBlockM, bh);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        if (*abort_flag) break;
        const int s = j & 1;
        if (j >= kStages) {
          if (!mbar_wait(&bars[kBarKVEmpty + s], ((j >> 1) - 1) & 1)) {
            *abort_flag = 1;
            break;
          }
        }
        mbar_arrive_expect_tx(&bars[kBarKFull + s], kTileBytes);
        tma_load_3d(smem + kKOff + s * kTileBytes, &tm_k, &bars[kBarKFull + s],
                    0, j * kBlockN, bh);
        mbar_arrive_expect_tx(&bars[kBarVFull + s], kTileBytes);
        tma_load_3d(smem + kVOff + s * kTileBytes, &tm_v, &bars[kBarVFull + s],
                    0, j * kBlockN, bh);
        issued = j + 1;
      }
      // Make sure no copy of ours is still landing in shared memory when the
      // CTA exits (only matters when another role gave up early).
      if (*abort_flag) {
        mbar_wait(&bars[kBarQFull], 0);
        for (int j = (issued > kStages ? issued - kStages : 0); j < issued;
             ++j) {
          mbar_wait(&bars[kBarKFull + (j & 1)], (j >> 1) & 1);
          mbar_wait(&bars[kBarVFull + (j & 1)], (j >> 1) & 1);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t q_addr = sbase + kQOff;
      const uint32_t p_addr = sbase + kPOff;
      const uint32_t tS = tmem_base + kTmemS;
      const uint32_t tO = tmem_base + kTmemO;
      auto issue_s = [&](int j) {
        const uint32_t k_addr = sbase + kKOff + (j & 1) * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {
          mma_f16_ss(tS, sw128_desc(q_addr + 32 * kk),
                     sw128_desc(k_addr + 32 * kk), kIdescS, kk > 0);
        }
      };
      bool ok = mbar_wait(&bars[kBarQFull], 0) &&
                mbar_wait(&bars[kBarKFull + 0], 0);
      if (ok) {
        tc_fence_after();
        issue_s(0);
        mma_commit(&bars[kBarSFull]);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (*abort_flag) {
          ok = false;
          break;
        }
        if (j + 1 < n_kv) {
          const int s1 = (j + 1) & 1;
          if (!mbar_wait(&bars[kBarKFull + s1], ((j + 1) >> 1) & 1) ||
              !mbar_wait(&bars[kBarSFree], j & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(j + 1);
          mma_commit(&bars[kBarSFull]);
        }
        const int s = j & 1;
        if (!mbar_wait(&bars[kBarPFull], j & 1) ||
            !mbar_wait(&bars[kBarVFull + s], (j >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t v_addr = sbase + kVOff + s * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < kBlockN / 16; ++kk) {
          const uint32_t a = p_addr + (kk >> 2) * kTileBytes + 32 * (kk & 3);
          mma_f16_ss(tO, sw128_desc(a), sw128_desc(v_addr + 2048 * kk),
                     kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bars[kBarODone]);
        mma_commit(&bars[kBarKVEmpty + s]);
      }
      if (!ok) *abort_flag = 1;
      // Every MMA issued above has retired once this commit lands; TMEM is
      // not released before that.
      mma_commit(&bars[kBarDrain]);
      mbar_wait(&bars[kBarDrain], 0);
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------- softmax
    const int row = threadIdx.x;  // 0..127 == TMEM lane
    const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem_base + lane_addr + kTmemS;
    const uint32_t tO = tmem_base + lane_addr + kTmemO;
    const uint32_t p_row = sbase + kPOff + row * kRowBytes;
    const int swz = row & 7;
    float m_use = -INFINITY;  // running max, in log2 units of scale * q.k
    float l_sum = 0.f;
    bool ok = true;

    for (int j = 0; j < n_kv; ++j) {
      if (*abort_flag || !mbar_wait(&bars[kBarSFull], j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[4][32];
      tmem_ld32(tS + 0, sr[0]);
      tmem_ld32(tS + 32, sr[1]);
      tmem_ld32(tS + 64, sr[2]);
      tmem_ld32(tS + 96, sr[3]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars[kBarSFree]);

      float s[128];
#pragma unroll
      for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(sr[c >> 5][c & 31]);

      // Scale handling: for scale > 0 the exponent is folded into one FMA per
      // element below; a zero or negative scale is applied up front so the
      // max is taken over the scaled logits (rare, off the fast path).
      float sl = scale_log2;
      if (scale_log2 <= 0.f) {
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] *= scale_log2;
        sl = 1.f;
      }
      const int kbase = j * kBlockN;
      const bool diag = causal && (j == qt);
      if (diag || kbase + kBlockN > N) {
        int lim = N - kbase;
        if (diag) lim = min(lim, row + 1);
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = (c < lim) ? s[c] : -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int c = 1; c < 128; ++c) mx = fmaxf(mx, s[c]);
      const float m_tile = mx * sl;
      float corr = 1.f;
      const bool rescale = m_tile > m_use + kRescaleThreshold;
      if (rescale) {
        corr = fast_exp2(m_use - m_tile);  // 0 on the first tile
        m_use = m_tile;
      }
      l_sum *= corr;
      const float neg_m = -m_use;

      uint32_t pk[64];
      float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
      for (int c = 0; c < 128; c += 2) {
        const float p0 = fast_exp2(fmaf(s[c], sl, neg_m));
        const float p1 = fast_exp2(fmaf(s[c + 1], sl, neg_m));
        rs0 += p0;
        rs1 += p1;
        pk[c >> 1] = pack_half2(p0, p1);
      }
      l_sum += rs0 + rs1;

      if (j > 0) {
        // PV_{j-1} must have retired: it still reads the P buffer and it
        // writes the O columns a rescale would touch.
        if (!mbar_wait(&bars[kBarODone], (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint32_t o[32];
            tmem_ld32(tO + 32 * h, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c)
              o[c] = __float_as_uint(__uint_as_float(o[c]) * corr);
            tmem_st32(tO + 32 * h, o);
          }
          tmem_wait_st();
        }
      }
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) {
        const uint32_t addr = p_row + (cc >> 3) * kTileBytes +
                              (static_cast<uint32_t>((cc & 7) ^ swz) << 4);
        st_shared_v4(addr, pk[4 * cc], pk[4 * cc + 1], pk[4 * cc + 2],
                     pk[4 * cc + 3]);
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars[kBarPFull]);
    }

    if (ok && mbar_wait(&bars[kBarODone], (n_kv - 1) & 1)) {
      tc_fence_after();
      uint32_t o[2][32];
      tmem_ld32(tO, o[0]);
      tmem_ld32(tO + 32, o[1]);
      tmem_wait_ld();
      const int q_row = qt * kBlockM + row;
      if (q_row < N) {
        const float inv_l = (l_sum > 0.f) ? 1.f / l_sum : 0.f;
        uint4 *dst = reinterpret_cast<uint4 *>(
            out + (static_cast<size_t>(bh) * N + q_row) * kHeadDim);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 v;
          const uint32_t *src = &o[c >> 2][(c & 3) * 8];
          v.x = pack_half2(__uint_as_float(src[0]) * inv_l,
                           __uint_as_float(src[1]) * inv_l);
          v.y = pack_half2(__uint_as_float(src[2]) * inv_l,
                           __uint_as_float(src[3]) * inv_l);
          v.z = pack_half2(__uint_as_float(src[4]) * inv_l,
                           __uint_as_float(src[5]) * inv_l);
          v.w = pack_half2(__uint_as_float(src[6]) * inv_l,
                           __uint_as_float(src[7]) * inv_l);
          dst[c] = v;
        }
      }
    } else {
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace prefill

const void *prefill_kernel_ptr() {
  return reinterpret_cast<const void *>(prefill::prefill_kernel);
}
int prefill_threads() { return prefill::kThreads; }
int prefill_smem_bytes() { return static_cast<int>(prefill::kSmemBytes); }

cudaError_t launch_prefill_kernel(const CUtensorMap &tm_q,
                                  const CUtensorMap &tm_k,
                                  const CUtensorMap &tm_v, __half *out, int B,
                                  int H, int N, bool causal, float scale,
                                  cudaStream_t stream) {
  static_assert(prefill::kBlockM == prefill::kBlockN,
                "causal tile skipping assumes square tiles");
  const int BH = B * H;
  const int n_qt = (N + prefill::kBlockM - 1) / prefill::kBlockM;
  const unsigned grid = static_cast<unsigned>(n_qt) * static_cast<unsigned>(BH);
  const float scale_log2 = scale * 1.4426950408889634f;
  prefill::prefill_kernel<<<grid, prefill::kThreads, prefill::kSmemBytes,
                            stream>>>(tm_q, tm_k, tm_v, out, N, BH,
                                      causal ? 1 : 0, scale_log2);
  return cudaGetLastError();
}

}  // namespace fa
