// Prefill attention forward for head_dim 128 on B200: fp16 in, fp32
// accumulate, fp16 out. Same semantics as the head_dim-64 kernel
// (prefill_sm100.cu; reference csrc/prefill.cu:164-343 for the math, the
// reference itself is specialised to 64 and names 128 as its next size).
//
// With 128-wide rows the PV accumulator needs 128 tensor-memory columns per
// query tile, so the key tiles are 64 wide: per query tile S (64 columns),
// O (128) and P (32) fit twice in the 512 columns, and the two 128-row
// query tiles of a (batch, head) ping-pong as in the 64 kernel. Per 64-key
// step the tensor core does twice the work of the 64 kernel per
// exponential, so this kernel leans towards the tensor-core bound.
//
// CTA = 12 warps (384 threads):
//   warps 0-3 / 4-7  softmax of query tile 0 / 1 (thread = row = TMEM lane)
//   warp 8     TMA producer: Q tiles once, then K_j, V_j per 64-key tile
//   warp 9     MMA issuer (one elected thread); owns the TMEM allocation
//   warps 10-11 idle (they give their registers to the softmax warps)
//
// Shared memory (1 KiB aligned). Every row is 256 bytes, stored as two
// 128-byte-swizzled halves (head dims 0-63 and 64-127) in separate blocks,
// the layout TMA writes with one 64-column box per half:
//   Q0, Q1  2 x [128 rows x 128 B] each            64 KiB
//   K       3 slots x 2 x [64 keys x 128 B]         48 KiB
//   V       3 slots x 2 x [64 keys x 128 B]         48 KiB
// Tensor memory (512 columns x 128 lanes, fp32 words):
//   S_t [64t, 64t+64)   O_t [128+128t, 256+128t)   P_t [384+32t, 416+32t)

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "fa_kernels.h"
#include "fa_sm100.cuh"

namespace fa {
namespace prefill128 {

constexpr int kD = 128;
constexpr int kHalfBytes = 128;  // one swizzled half-row (64 dims)
constexpr int kBlockM = 128;     // query rows per tile
constexpr int kBlockN = 64;      // keys per K/V tile
constexpr int kTilesPerCta = 2;
// K/V ring slots of the paired form: two key tiles stream ahead of the
// one in use.
constexpr int kRingSlots = 3;
constexpr int kSoftmaxThreads = 128;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 384;
constexpr int kCtrlRegs = 24;
constexpr int kSoftmaxRegs = 240;
static_assert(128 * kCtrlRegs + 256 * kSoftmaxRegs <= kThreads * 168,
              "register split exceeds the launch allocation");
constexpr uint32_t kQHalf = kBlockM * kHalfBytes;   // 16 KiB
constexpr uint32_t kQTile = 2 * kQHalf;             // 32 KiB
constexpr uint32_t kKVHalf = kBlockN * kHalfBytes;  // 8 KiB
constexpr uint32_t kKVTile = 2 * kKVHalf;           // 16 KiB

constexpr uint32_t kQOff = 0;
constexpr uint32_t kKOff = kQOff + kTilesPerCta * kQTile;
constexpr uint32_t kVOff = kKOff + kRingSlots * kKVTile;
constexpr uint32_t kBarOff = kVOff + kRingSlots * kKVTile;
constexpr int kBarQFull = 0;
constexpr int kBarKFull = kBarQFull + 1;          // + stage: K and V tile
constexpr int kBarKVEmpty = kBarKFull + kRingSlots;  // + stage
constexpr int kBarSFull = kBarKVEmpty + kRingSlots;  // + tile
constexpr int kBarSFree = kBarSFull + kTilesPerCta;
constexpr int kBarPFull = kBarSFree + kTilesPerCta;
constexpr int kBarODone = kBarPFull + kTilesPerCta;
constexpr int kBarDrain = kBarODone + kTilesPerCta;
constexpr int kNumBars = kBarDrain + 1;
constexpr uint32_t kTmemSlotOff = kBarOff + kNumBars * 8;
constexpr uint32_t kAbortOff = kTmemSlotOff + 4;
constexpr uint32_t kSmemBytes = kAbortOff + 4 + 8;
static_assert(kSmemBytes <= 227 * 1024,
              "above the sm_100 per-CTA shared memory limit");

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // + 64 * tile
constexpr uint32_t kTmemO = 128;  // + 128 * tile
constexpr uint32_t kTmemP = 384;  // + 32 * tile

// Two CTA forms, as in the head_dim-64 kernel. Paired (kSolo false): the
// layout above, one CTA per SM. Solo: one query tile per CTA and two CTAs
// per SM: 256 threads (softmax warps 0-3, producer 4, MMA 5, donors 6-7),
// tensor memory S [0,64) O [64,192) P [192,224) of a 256-column
// allocation, and Q (32 KiB) plus a 2-slot K/V ring (64 KiB) of shared
// memory.
template <bool kSolo>
struct Form {
  static constexpr int kThreads = kSolo ? 256 : 384;
  static constexpr int kCtasPerSm = kSolo ? 2 : 1;
  static constexpr int kCtrlWarp0 = kSolo ? 4 : 8;
  static constexpr int kProducerWarp = kCtrlWarp0;
  static constexpr int kMmaWarp = kCtrlWarp0 + 1;
  static constexpr int kSoftmaxRegs = kSolo ? 232 : 240;
  static constexpr int kQTiles = kSolo ? 1 : 2;
  static constexpr int kSlots = kSolo ? 2 : kRingSlots;
  static constexpr uint32_t kKOff = kQOff + kQTiles * kQTile;
  static constexpr uint32_t kVOff = kKOff + kSlots * kKVTile;
  static constexpr uint32_t kBarOff = kVOff + kSlots * kKVTile;
  static constexpr uint32_t kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr uint32_t kAbortOff = kTmemSlotOff + 4;
  static constexpr uint32_t kSmemBytes = kAbortOff + 4 + 8;
  static constexpr uint32_t kTmemCols = kSolo ? 256 : 512;
  static constexpr uint32_t kTmemO = kSolo ? 64 : 128;   // + 128 * tile
  static constexpr uint32_t kTmemP = kSolo ? 192 : 384;  // + 32 * tile
  static_assert(128 * kCtrlRegs + 128 * kQTiles * kSoftmaxRegs <=
                    kThreads * (65536 / (kThreads * kCtasPerSm)),
                "register split exceeds the launch allocation");
  static_assert(kCtasPerSm * (kSmemBytes + 1024) <= 228 * 1024,
                "shared memory of the resident CTAs exceeds the SM's");
};

template <typename Dt>
constexpr uint32_t kIdescS = idesc_f16_f32(kBlockM, kBlockN, false, Dt::kFmt);
template <typename Dt>
constexpr uint32_t kIdescPV = idesc_f16_f32(kBlockM, kD, true, Dt::kFmt);
constexpr float kRescaleThreshold = 8.0f;
// K/V bytes of one block of heads in the launch order (measured on C3-shape
// and N 2048-8192 grids: 32 MiB best or tied; 56 MiB lost 20 % on C3).
constexpr long long kHeadBlockL2Bytes = 32ll << 20;
// Bit i set: column pair i of every 8 takes its exponentials from the MUFU
// unit, the others from the polynomial on the FMA pipe (the same balance as
// the head_dim-64 kernel).
constexpr unsigned kMufuMask8 = 0x3B;

// S = Q K^T for one 128x64 tile: 8 MMAs of K=16; steps 0-3 read the first
// 64-dim half of Q and K, steps 4-7 the second half (a separate block).
template <typename Dt>
__device__ __forceinline__ void issue_s_tile(uint32_t d, uint64_t q_desc,
                                             uint64_t k_desc) {
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
    const uint64_t off_q = (kk >> 2) * (kQHalf >> 4) + 2 * (kk & 3);
    const uint64_t off_k = (kk >> 2) * (kKVHalf >> 4) + 2 * (kk & 3);
    mma_f16_ss(d, q_desc + off_q, k_desc + off_k, kIdescS<Dt>, kk > 0 ? 1u : 0u);
  }
}

// O (+)= P V for one tile: 4 MMAs of K=16 keys, N=128 head dims. V is the
// MN-major B operand whose two 64-dim halves are kKVHalf bytes apart (the
// descriptor's leading byte offset); each step advances 16 rows.
template <typename Dt>
__device__ __forceinline__ void issue_pv_tile(uint32_t d, uint32_t p_tmem,
                                              uint64_t v_desc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < kBlockN / 16; ++kk)
    mma_f16_ts(d, p_tmem + 8 * kk, v_desc + 128 * kk, kIdescPV<Dt>,
               (accumulate || kk > 0) ? 1u : 0u);
}

// Shared-memory descriptor of a 128-byte-swizzled operand whose blocks of
// 64 elements along M/N are `lbo` bytes apart.
__device__ __forceinline__ uint64_t sw128_desc_lbo(uint32_t smem_addr,
                                                   uint32_t lbo) {
  return (sw128_desc(smem_addr) & ~(static_cast<uint64_t>(0x3FFFu) << 16)) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16);
}

struct TileInfo {
  int qt;    // query tile index along the sequence
  int n_kv;  // 64-key tiles this query tile attends (0: tile past the end)
};

__device__ __forceinline__ TileInfo tile_info(int pair, int t, int N,
                                              int causal, int zigzag) {
  TileInfo ti;
  const int n_qt = (N + kBlockM - 1) / kBlockM;
  // zig-zag: tile p with tile n_qt - 1 - p, so every causal pair attends
  // the same number of keys (one-wave grids)
  ti.qt = zigzag ? (t == 0 ? pair : n_qt - 1 - pair) : kTilesPerCta * pair + t;
  if (ti.qt >= n_qt || (t == 1 && zigzag && ti.qt == pair)) {
    ti.n_kv = 0;
  } else {
    const int keys = causal ? min((ti.qt + 1) * kBlockM, N) : N;
    ti.n_kv = (keys + kBlockN - 1) / kBlockN;
  }
  return ti;
}

template <typename Dt, bool kSolo = false>
__global__ void __launch_bounds__(Form<kSolo>::kThreads, Form<kSolo>::kCtasPerSm)
    prefill_d128_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        __half *__restrict__ out, int N, int BH, int causal,
                        float scale_log2, int H, int group,
                        int head_block) {
  using F = Form<kSolo>;
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int kStages = F::kSlots;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // bit 0: causal; bit 1: zig-zag query-tile pairing
  const int zigzag = causal >> 1;
  causal &= 1;
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) record_error(FA_ERR_SMEM_ALIGN);
    return;
  }

  // Heaviest causal pairs first, heads fastest, within blocks of
  // head_block heads (0: one block of all heads) whose K/V fit in L2, so a
  // head's tiles run close together and its K/V is read from HBM once.
  const int n_qt = (N + kBlockM - 1) / kBlockM;
  const int n_pairs = (n_qt + kTilesPerCta - 1) / kTilesPerCta;
  const int n_units = kSolo ? n_qt : n_pairs;  // per head
  const int hb = head_block > 0 ? head_block : BH;
  const int blk = static_cast<int>(blockIdx.x) / (hb * n_units);
  const int r = static_cast<int>(blockIdx.x) % (hb * n_units);
  const int h0 = blk * hb;
  const int h_here = min(hb, BH - h0);
  const int h_div = h_here > 0 ? h_here : 1;
  const int unit = n_units - 1 - r / h_div;  // heaviest first
  const int pair = unit;
  const int bh = h0 + r % h_div;
  if (h_here <= 0 || bh >= BH) return;  // only if the grid outran the work
  const int kv_bh = (bh / H) * (H / group) + (bh % H) / group;
  TileInfo t0 = tile_info(pair, 0, N, causal, zigzag);
  TileInfo t1 = tile_info(pair, 1, N, causal, zigzag);
  if (kSolo) {
    // one query tile per CTA, heaviest first, heads fastest
    t0.qt = unit;
    t0.n_kv = ((causal ? min((t0.qt + 1) * kBlockM, N) : N) + kBlockN - 1) /
              kBlockN;
    t1.qt = t0.qt;
    t1.n_kv = 0;
  }
  const int n_kv = t0.n_kv > t1.n_kv ? t0.n_kv : t1.n_kv;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + F::kBarOff);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + F::kTmemSlotOff);
  volatile uint32_t *abort_flag =
      reinterpret_cast<volatile uint32_t *>(smem + F::kAbortOff);

  // Ring positions (tile 1's skipped when the CTA has one head); a
  // position's stage is p % kStages.
  const int n_pos = n_kv;
  auto load_pos = [&](int p) {
    const int j = p;
    const int kvh = kv_bh;
    const int s = p % kStages;
    mbar_arrive_expect_tx(&bars[kBarKFull + s], 2 * kKVTile);
    for (int h = 0; h < 2; ++h) {
      tma_load_3d(smem + F::kKOff + s * kKVTile + h * kKVHalf, &tm_k,
                  &bars[kBarKFull + s], 64 * h, j * kBlockN, kvh);
      tma_load_3d(smem + F::kVOff + s * kKVTile + h * kKVHalf, &tm_v,
                  &bars[kBarKFull + s], 64 * h, j * kBlockN, kvh);
    }
  };

  // The producer lane sets up the barriers and issues the Q tiles and the
  // first kStages K/V tiles before the CTA-wide barrier (their latency
  // overlaps the TMEM allocation), then turns the device error word into
  // the abort flag.
  int preissued = 0;
  if (warp == F::kProducerWarp && lane == 0) {
    mbar_init(&bars[kBarQFull], 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kBarKFull + s], 1);
      mbar_init(&bars[kBarKVEmpty + s], 1);
    }
    for (int t = 0; t < kTilesPerCta; ++t) {
      mbar_init(&bars[kBarSFull + t], 1);
      mbar_init(&bars[kBarSFree + t], kSoftmaxThreads);
      mbar_init(&bars[kBarPFull + t], kSoftmaxThreads);
      mbar_init(&bars[kBarODone + t], 1);
    }
    mbar_init(&bars[kBarDrain], 1);
    fence_barrier_init();
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    const bool two = t1.n_kv > 0;
    mbar_arrive_expect_tx(&bars[kBarQFull], (two ? 2 : 1) * kQTile);
    for (int t = 0; t < (two ? 2 : 1); ++t) {
      const int row0 = (t == 0 ? t0.qt : t1.qt) * kBlockM;
      for (int h = 0; h < 2; ++h)
        tma_load_3d(smem + kQOff + t * kQTile + h * kQHalf, &tm_q,
                    &bars[kBarQFull], 64 * h, row0, bh);
    }
    for (; preissued < n_pos && preissued < kStages; ++preissued)
      load_pos(preissued);
    *abort_flag = device_failed() ? 1u : 0u;
  }
  if (warp == F::kMmaWarp) {
    tmem_alloc(tmem_slot, F::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t sbase = smem_u32(smem);

  if (warp >= F::kCtrlWarp0) {
    setmaxnreg_dec<kCtrlRegs>();
    if (warp == F::kProducerWarp) {
      // ---------------------------------------------------------------- TMA
      if (lane == 0) {
        int issued = preissued;
        for (int p = preissued; p < n_pos; ++p) {
          if (*abort_flag) break;
          const int s = p % kStages;
          const int use = p / kStages;
          if (use > 0 &&
              !mbar_wait(&bars[kBarKVEmpty + s], (use - 1) & 1)) {
            *abort_flag = 1;
            break;
          }
          load_pos(p);
          issued = p + 1;
        }
        if (*abort_flag) {
          mbar_wait(&bars[kBarQFull], 0);
          for (int p = (issued > kStages ? issued - kStages : 0); p < issued;
               ++p)
            mbar_wait(&bars[kBarKFull + p % kStages], (p / kStages) & 1);
        }
      }
    } else if (warp == F::kMmaWarp) {
      // ---------------------------------------------------------------- MMA
      const bool leader = elect_one();
      const uint32_t tmem = __shfl_sync(0xffffffffu, tmem_base, 0);
      const int n_t[2] = {t0.n_kv, t1.n_kv};
      const uint64_t desc0 = sw128_desc(sbase);
      const uint64_t vdesc0 = sw128_desc_lbo(sbase, kKVHalf);
      bool ok = mbar_wait(&bars[kBarQFull], 0) &&
                mbar_wait(&bars[kBarKFull + 0], 0);
      if (ok) {
        tc_fence_after();
        if (leader) {
          for (int t = 0; t < kTilesPerCta; ++t) {
            if (n_t[t] == 0) continue;
            issue_s_tile<Dt>(tmem + kTmemS + 64 * t,
                         desc0 + ((kQOff + t * kQTile) >> 4),
                         desc0 + (F::kKOff >> 4));
            mma_commit(&bars[kBarSFull + t]);
          }
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (*abort_flag) {
          ok = false;
          break;
        }
#pragma unroll
        for (int t = 0; t < kTilesPerCta; ++t) {
          const int nt = n_t[t];
          if (!ok || j >= nt) continue;
          const int s = j % kStages;  // K_j, V_j
          const int p1 = j + 1;
          const int s1 = p1 % kStages;         // K_{j+1}
          if (j + 1 < nt) {
            // K/V tile j+1 is waited on once per round (by the first tile
            // that uses it)
            const bool need_kv = (t == 0) || (n_t[0] <= j + 1);
            if ((need_kv &&
                 !mbar_wait(&bars[kBarKFull + s1], (p1 / kStages) & 1)) ||
                !mbar_wait(&bars[kBarSFree + t], j & 1)) {
              ok = false;
              continue;
            }
            tc_fence_after();
            if (leader) {
              issue_s_tile<Dt>(tmem + kTmemS + 64 * t,
                           desc0 + ((kQOff + t * kQTile) >> 4),
                           desc0 + ((F::kKOff + s1 * kKVTile) >> 4));
              mma_commit(&bars[kBarSFull + t]);
            }
            __syncwarp();
          }
          if (!mbar_wait(&bars[kBarPFull + t], j & 1)) {
            ok = false;
            continue;
          }
          tc_fence_after();
          if (leader) {
            issue_pv_tile<Dt>(tmem + F::kTmemO + 128 * t, tmem + F::kTmemP + 32 * t,
                          vdesc0 + ((F::kVOff + s * kKVTile) >> 4), j > 0);
            mma_commit(&bars[kBarODone + t]);
          }
          __syncwarp();
        }
        if (!ok) break;
        // release round j's ring stage
        if (leader) {
          mma_commit(&bars[kBarKVEmpty + j % kStages]);
        }
        __syncwarp();
      }
      if (!ok && leader) *abort_flag = 1;
      if (leader) mma_commit(&bars[kBarDrain]);
      __syncwarp();
      mbar_wait(&bars[kBarDrain], 0);
    }
  } else {
    setmaxnreg_inc<F::kSoftmaxRegs>();
    // -------------------------------------------------------------- softmax
    const int t = warp >> 2;
    const int row = threadIdx.x & 127;
    const TileInfo ti = t == 0 ? t0 : t1;
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem_base + lane_addr + kTmemS + 64 * t;
    const uint32_t tO = tmem_base + lane_addr + F::kTmemO + 128 * t;
    const uint32_t tP = tmem_base + lane_addr + F::kTmemP + 32 * t;
    uint64_t *s_full = &bars[kBarSFull + t];
    uint64_t *s_free = &bars[kBarSFree + t];
    uint64_t *p_full = &bars[kBarPFull + t];
    uint64_t *o_done = &bars[kBarODone + t];
    const int q_row = ti.qt * kBlockM + row;
    float m_use = -INFINITY;
    float l_sum = 0.f;
    bool ok = true;

    for (int j = 0; j < ti.n_kv; ++j) {
      if (*abort_flag || !mbar_wait(s_full, j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(tS + 0, sr[0]);
      tmem_ld32(tS + 32, sr[1]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(s_free);

      float s[kBlockN];
#pragma unroll
      for (int c = 0; c < kBlockN; ++c) s[c] = __uint_as_float(sr[c >> 5][c & 31]);
      float sl = scale_log2;
      if (scale_log2 <= 0.f) {
#pragma unroll
        for (int c = 0; c < kBlockN; ++c) s[c] *= scale_log2;
        sl = 1.f;
      }
      const int kbase = j * kBlockN;
      const bool diag = causal && (kbase + kBlockN > ti.qt * kBlockM);
      if (diag || kbase + kBlockN > N) {
        int lim = N - kbase;
        if (diag) lim = min(lim, q_row + 1 - kbase);
#pragma unroll
        for (int c = 0; c < kBlockN; ++c) s[c] = (c < lim) ? s[c] : -INFINITY;
      }
      float mxp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxp[i] = s[i];
#pragma unroll
      for (int c = 8; c + 16 <= kBlockN; c += 16) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          mxp[i] = fmax3(mxp[i], s[c + i], s[c + 8 + i]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) mxp[i] = fmaxf(mxp[i], s[kBlockN - 8 + i]);
      const float mx = fmax3(fmax3(mxp[0], mxp[1], mxp[2]),
                             fmax3(mxp[3], mxp[4], mxp[5]),
                             fmaxf(mxp[6], mxp[7]));
      const float m_tile = mx * sl;
      float corr = 1.f;
      const bool rescale = m_tile > m_use + kRescaleThreshold;
      if (rescale) {
        corr = fast_exp2(m_use - m_tile);
        m_use = m_tile;
      }
      l_sum *= corr;
      const float neg_m = -m_use;
      const float2 sl2 = make_float2(sl, sl);
      const float2 nm2 = make_float2(neg_m, neg_m);
      // polynomial argument in clamped affine form (exp2_poly2_affine)
      const float xa = sl * (1.f / kExp2Span);
      const float xb = (neg_m - kExp2Lo) * (1.f / kExp2Span);
      float2 rs[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) rs[i] = make_float2(0.f, 0.f);
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < kBlockN; c += 2) {
        float2 p;
        if (!((kMufuMask8 >> ((c >> 1) & 7)) & 1)) {
          p = exp2_poly2_affine(
              make_float2(fma_sat(s[c], xa, xb), fma_sat(s[c + 1], xa, xb)));
        } else {
          const float2 x = ffma2(make_float2(s[c], s[c + 1]), sl2, nm2);
          p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        }
        rs[(c >> 1) & 3] = fadd2(rs[(c >> 1) & 3], p);
        pk[c >> 1] = Dt::pack2(p.x, p.y);
      }
      const float2 rsum = fadd2(fadd2(rs[0], rs[1]), fadd2(rs[2], rs[3]));
      l_sum += rsum.x + rsum.y;

      if (j > 0) {
        if (!mbar_wait(o_done, (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int h = 0; h < kD / 32; ++h) {
            uint32_t o[32];
            tmem_ld32(tO + 32 * h, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c)
              o[c] = __float_as_uint(__uint_as_float(o[c]) * corr);
            tmem_st32(tO + 32 * h, o);
          }
        }
      }
      tmem_st32(tP, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);
    }

    if (ti.n_kv > 0) {
      if (ok && mbar_wait(o_done, (ti.n_kv - 1) & 1)) {
        tc_fence_after();
        const float inv_l = (l_sum > 0.f) ? 1.f / l_sum : 0.f;
        uint4 *dst = reinterpret_cast<uint4 *>(
            out + (static_cast<size_t>(bh) * N + q_row) * kD);
#pragma unroll
        for (int h = 0; h < kD / 32; ++h) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * h, o);
          tmem_wait_ld();
          if (q_row < N) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t *src = &o[c * 8];
              uint4 v;
              v.x = Dt::pack2(__uint_as_float(src[0]) * inv_l,
                               __uint_as_float(src[1]) * inv_l);
              v.y = Dt::pack2(__uint_as_float(src[2]) * inv_l,
                               __uint_as_float(src[3]) * inv_l);
              v.z = Dt::pack2(__uint_as_float(src[4]) * inv_l,
                               __uint_as_float(src[5]) * inv_l);
              v.w = Dt::pack2(__uint_as_float(src[6]) * inv_l,
                               __uint_as_float(src[7]) * inv_l);
              dst[4 * h + c] = v;
            }
          }
        }
      } else {
        *abort_flag = 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == F::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, F::kTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Wide form: 128-key tiles, P written over S.
//
// The form above keeps P in its own tensor-memory columns, which at head
// dim 128 leaves room only for 64-key S tiles: each QK^T is an N=64 MMA
// (shared-memory bound on the B200) and every 128 keys cost two rounds of
// barriers, loads and waits. Here S_t takes 128 columns, O_t 128, and P_t
// is stored as fp16 pairs over the first 64 columns of S_t once the softmax
// warps hold S_t in registers:
//   S0 / P0 [0,128)  S1 / P1 [128,256)  O0 [256,384)  O1 [384,512)
// Since S_t(j+1) overwrites P_t(j), the MMA warp issues it only once
// PV_t(j) has completed (its commit barrier); the other query tile's
// softmax runs meanwhile, so the two tiles alternate between the softmax
// warps and the tensor core. Shared memory: Q0, Q1 (2 x 32 KiB) and a
// 2-slot ring of 128-key K and V tiles (4 x 32 KiB), each row as two
// 128-byte-swizzled 64-dim halves (16 KiB blocks); the K/V boxes are the
// 64-row boxes of the form above, two per half.
// ---------------------------------------------------------------------------
namespace wide {
constexpr int kBlockN = 128;
constexpr int kSlots = 2;
constexpr uint32_t kKVHalf = kBlockN * kHalfBytes;  // 16 KiB
constexpr uint32_t kKVTile = 2 * kKVHalf;           // 32 KiB
constexpr uint32_t kQOff = 0;
constexpr uint32_t kKOff = kQOff + kTilesPerCta * kQTile;
constexpr uint32_t kVOff = kKOff + kSlots * kKVTile;
constexpr uint32_t kBarOff = kVOff + kSlots * kKVTile;
constexpr int kBarQFull = 0;
constexpr int kBarKFull = kBarQFull + 1;          // + stage: K and V tile
constexpr int kBarKVEmpty = kBarKFull + kSlots;   // + stage
constexpr int kBarSFull = kBarKVEmpty + kSlots;   // + tile
constexpr int kBarPFull = kBarSFull + kTilesPerCta;
constexpr int kBarODone = kBarPFull + kTilesPerCta;
constexpr int kBarDrain = kBarODone + kTilesPerCta;
constexpr int kNumBars = kBarDrain + 1;
constexpr uint32_t kTmemSlotOff = kBarOff + kNumBars * 8;
constexpr uint32_t kAbortOff = kTmemSlotOff + 4;
constexpr uint32_t kSmemBytes = kAbortOff + 4 + 8;
static_assert(kSmemBytes + 1024 <= 228 * 1024,
              "above the sm_100 per-CTA shared memory limit");
constexpr uint32_t kTmemS = 0;    // + 128 * tile (P_t over its first 64)
constexpr uint32_t kTmemO = 256;  // + 128 * tile

template <typename Dt>
constexpr uint32_t kIdescS = idesc_f16_f32(kBlockM, kBlockN, false, Dt::kFmt);

// S = Q K^T for one 128x128 tile: 8 MMAs of K=16, steps 0-3 on the first
// 64-dim half of Q and K, steps 4-7 on the second.
template <typename Dt>
__device__ __forceinline__ void issue_s_tile(uint32_t d, uint64_t q_desc,
                                             uint64_t k_desc) {
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
    const uint64_t off_q = (kk >> 2) * (kQHalf >> 4) + 2 * (kk & 3);
    const uint64_t off_k = (kk >> 2) * (kKVHalf >> 4) + 2 * (kk & 3);
    mma_f16_ss(d, q_desc + off_q, k_desc + off_k, kIdescS<Dt>, kk > 0 ? 1u : 0u);
  }
}

// O (+)= P V for one tile: 8 MMAs of K=16 keys, N=128 head dims; V's two
// 64-dim halves are kKVHalf bytes apart (the descriptor's leading byte
// offset) and each step advances 16 rows (2048 bytes).
template <typename Dt>
__device__ __forceinline__ void issue_pv_tile(uint32_t d, uint32_t p_tmem,
                                              uint64_t v_desc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < kBlockN / 16; ++kk)
    mma_f16_ts(d, p_tmem + 8 * kk, v_desc + 128 * kk, kIdescPV<Dt>,
               (accumulate || kk > 0) ? 1u : 0u);
}

__device__ __forceinline__ TileInfo tile_info(int pair, int t, int N,
                                              int causal, int zigzag) {
  TileInfo ti;
  const int n_qt = (N + kBlockM - 1) / kBlockM;
  ti.qt = zigzag ? (t == 0 ? pair : n_qt - 1 - pair) : kTilesPerCta * pair + t;
  if (ti.qt >= n_qt || (t == 1 && zigzag && ti.qt == pair)) {
    ti.n_kv = 0;
  } else {
    ti.n_kv = causal ? ti.qt + 1 : (N + kBlockN - 1) / kBlockN;
  }
  return ti;
}
}  // namespace wide

template <typename Dt>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_d128_wide_kernel(const __grid_constant__ CUtensorMap tm_q,
                             const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v,
                             __half *__restrict__ out, int N, int BH,
                             int causal, float scale_log2, int H, int group,
                             int head_block) {
  static_assert(kBlockM == wide::kBlockN, "causal tile skipping assumes square tiles");
  extern __shared__ __align__(1024) uint8_t smem[];
  constexpr int kStages = wide::kSlots;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // bit 0: causal; bit 1: zig-zag query-tile pairing
  const int zigzag = causal >> 1;
  causal &= 1;
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) record_error(FA_ERR_SMEM_ALIGN);
    return;
  }

  // Heaviest pairs first, heads fastest, within blocks of head_block heads
  // (0: all heads) whose K/V fit in L2.
  const int n_qt = (N + kBlockM - 1) / kBlockM;
  const int n_pairs = (n_qt + kTilesPerCta - 1) / kTilesPerCta;
  const int hb = head_block > 0 ? head_block : BH;
  const int blk = static_cast<int>(blockIdx.x) / (hb * n_pairs);
  const int r = static_cast<int>(blockIdx.x) % (hb * n_pairs);
  const int h0 = blk * hb;
  const int h_here = min(hb, BH - h0);
  const int h_div = h_here > 0 ? h_here : 1;
  const int pair = n_pairs - 1 - r / h_div;
  const int bh = h0 + r % h_div;
  if (h_here <= 0 || bh >= BH) return;
  const int kv_bh = (bh / H) * (H / group) + (bh % H) / group;
  const TileInfo t0 = wide::tile_info(pair, 0, N, causal, zigzag);
  const TileInfo t1 = wide::tile_info(pair, 1, N, causal, zigzag);
  const int n_kv = t0.n_kv > t1.n_kv ? t0.n_kv : t1.n_kv;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + wide::kBarOff);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + wide::kTmemSlotOff);
  volatile uint32_t *abort_flag =
      reinterpret_cast<volatile uint32_t *>(smem + wide::kAbortOff);

  // Key tile p goes to ring stage p % kStages: per 64-dim half, two boxes
  // of 64 rows for K and two for V.
  auto load_pos = [&](int p) {
    const int s = p % kStages;
    mbar_arrive_expect_tx(&bars[wide::kBarKFull + s], 2 * wide::kKVTile);
    for (int h = 0; h < 2; ++h) {
      for (int rb = 0; rb < 2; ++rb) {
        const uint32_t off = s * wide::kKVTile + h * wide::kKVHalf + rb * (wide::kKVHalf / 2);
        tma_load_3d(smem + wide::kKOff + off, &tm_k, &bars[wide::kBarKFull + s], 64 * h,
                    p * wide::kBlockN + 64 * rb, kv_bh);
        tma_load_3d(smem + wide::kVOff + off, &tm_v, &bars[wide::kBarKFull + s], 64 * h,
                    p * wide::kBlockN + 64 * rb, kv_bh);
      }
    }
  };

  int preissued = 0;
  if (warp == kProducerWarp && lane == 0) {
    mbar_init(&bars[wide::kBarQFull], 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[wide::kBarKFull + s], 1);
      mbar_init(&bars[wide::kBarKVEmpty + s], 1);
    }
    for (int t = 0; t < kTilesPerCta; ++t) {
      mbar_init(&bars[wide::kBarSFull + t], 1);
      mbar_init(&bars[wide::kBarPFull + t], kSoftmaxThreads);
      mbar_init(&bars[wide::kBarODone + t], 1);
    }
    mbar_init(&bars[wide::kBarDrain], 1);
    fence_barrier_init();
    prefetch_tensormap(&tm_q);
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    const bool two = t1.n_kv > 0;
    mbar_arrive_expect_tx(&bars[wide::kBarQFull], (two ? 2 : 1) * kQTile);
    for (int t = 0; t < (two ? 2 : 1); ++t) {
      const int row0 = (t == 0 ? t0.qt : t1.qt) * kBlockM;
      for (int h = 0; h < 2; ++h)
        tma_load_3d(smem + wide::kQOff + t * kQTile + h * kQHalf, &tm_q,
                    &bars[wide::kBarQFull], 64 * h, row0, bh);
    }
    for (; preissued < n_kv && preissued < kStages; ++preissued)
      load_pos(preissued);
    *abort_flag = device_failed() ? 1u : 0u;
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

  if (warp >= 8) {
    setmaxnreg_dec<kCtrlRegs>();
    if (warp == kProducerWarp) {
      // ---------------------------------------------------------------- TMA
      if (lane == 0) {
        int issued = preissued;
        for (int p = preissued; p < n_kv; ++p) {
          if (*abort_flag) break;
          const int s = p % kStages;
          const int use = p / kStages;
          if (use > 0 && !mbar_wait(&bars[wide::kBarKVEmpty + s], (use - 1) & 1)) {
            *abort_flag = 1;
            break;
          }
          load_pos(p);
          issued = p + 1;
        }
        // no copy of ours may still be landing when the CTA exits
        if (*abort_flag) {
          mbar_wait(&bars[wide::kBarQFull], 0);
          for (int p = (issued > kStages ? issued - kStages : 0); p < issued; ++p)
            mbar_wait(&bars[wide::kBarKFull + p % kStages], (p / kStages) & 1);
        }
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------------------- MMA
      const bool leader = elect_one();
      const uint32_t tmem = __shfl_sync(0xffffffffu, tmem_base, 0);
      const int n_t[2] = {t0.n_kv, t1.n_kv};
      const uint64_t desc0 = sw128_desc(sbase);
      const uint64_t vdesc0 = sw128_desc_lbo(sbase, wide::kKVHalf);
      bool ok = mbar_wait(&bars[wide::kBarQFull], 0) &&
                mbar_wait(&bars[wide::kBarKFull + 0], 0);
      if (ok) {
        tc_fence_after();
        if (leader) {
          for (int t = 0; t < kTilesPerCta; ++t) {
            if (n_t[t] == 0) continue;
            wide::issue_s_tile<Dt>(tmem + wide::kTmemS + 128 * t,
                                   desc0 + ((wide::kQOff + t * kQTile) >> 4),
                                   desc0 + (wide::kKOff >> 4));
            mma_commit(&bars[wide::kBarSFull + t]);
          }
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (*abort_flag) {
          ok = false;
          break;
        }
        const int s = j % kStages;  // K_j, V_j
#pragma unroll
        for (int t = 0; t < kTilesPerCta; ++t) {
          const int nt = n_t[t];
          if (!ok || j >= nt) continue;
          if (!mbar_wait(&bars[wide::kBarPFull + t], j & 1)) {
            ok = false;
            continue;
          }
          tc_fence_after();
          if (leader) {
            wide::issue_pv_tile<Dt>(tmem + wide::kTmemO + 128 * t,
                                    tmem + wide::kTmemS + 128 * t,
                                    vdesc0 + ((wide::kVOff + s * wide::kKVTile) >> 4), j > 0);
            mma_commit(&bars[wide::kBarODone + t]);
            // the round's last PV releases its ring stage
            if (t == 1 || n_t[1] <= j) mma_commit(&bars[wide::kBarKVEmpty + s]);
          }
          __syncwarp();
          if (j + 1 < nt) {
            // S_t(j+1) overwrites P_t(j): wait for PV_t(j) to complete.
            // K/V tile j+1 is waited on by its first user.
            const int p1 = j + 1;
            const bool need_kv = (t == 0) || (n_t[0] <= j + 1);
            if ((need_kv &&
                 !mbar_wait(&bars[wide::kBarKFull + p1 % kStages], (p1 / kStages) & 1)) ||
                !mbar_wait(&bars[wide::kBarODone + t], j & 1)) {
              ok = false;
              continue;
            }
            tc_fence_after();
            if (leader) {
              wide::issue_s_tile<Dt>(tmem + wide::kTmemS + 128 * t,
                                     desc0 + ((wide::kQOff + t * kQTile) >> 4),
                                     desc0 + ((wide::kKOff + (p1 % kStages) * wide::kKVTile) >> 4));
              mma_commit(&bars[wide::kBarSFull + t]);
            }
            __syncwarp();
          }
        }
      }
      if (!ok && leader) *abort_flag = 1;
      if (leader) mma_commit(&bars[wide::kBarDrain]);
      __syncwarp();
      mbar_wait(&bars[wide::kBarDrain], 0);
    }
  } else {
    setmaxnreg_inc<kSoftmaxRegs>();
    // -------------------------------------------------------------- softmax
    const int t = warp >> 2;
    const int row = threadIdx.x & 127;
    const TileInfo ti = t == 0 ? t0 : t1;
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem_base + lane_addr + wide::kTmemS + 128 * t;
    const uint32_t tO = tmem_base + lane_addr + wide::kTmemO + 128 * t;
    uint64_t *s_full = &bars[wide::kBarSFull + t];
    uint64_t *p_full = &bars[wide::kBarPFull + t];
    uint64_t *o_done = &bars[wide::kBarODone + t];
    const int q_row = ti.qt * kBlockM + row;
    float m_use = -INFINITY;
    float l_sum = 0.f;
    bool ok = true;

    for (int j = 0; j < ti.n_kv; ++j) {
      if (*abort_flag || !mbar_wait(s_full, j & 1)) {
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

      float s[128];
#pragma unroll
      for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(sr[c >> 5][c & 31]);
      float sl = scale_log2;
      if (scale_log2 <= 0.f) {
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] *= scale_log2;
        sl = 1.f;
      }
      const int kbase = j * wide::kBlockN;
      const bool diag = causal && (j == ti.qt);
      if (diag || kbase + wide::kBlockN > N) {
        int lim = N - kbase;
        if (diag) lim = min(lim, row + 1);
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = (c < lim) ? s[c] : -INFINITY;
      }
      float corr = 1.f;
      bool rescale = false;
      const float m_tile = row_max_128(s) * sl;
      if (m_tile > m_use + prefill128::kRescaleThreshold) {
        corr = fast_exp2(m_use - m_tile);  // 0 on the first tile
        m_use = m_tile;
        rescale = true;
      }
      uint32_t pk[2][32];
      const float rowsum = exp_row<Dt>(s, sl, m_use, pk);
      l_sum = fmaf(l_sum, corr, rowsum);
      // PV_t(j-1) has completed: S_t(j) was issued after it.
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int h = 0; h < kD / 32; ++h) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * h, o);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c)
            o[c] = __float_as_uint(__uint_as_float(o[c]) * corr);
          tmem_st32(tO + 32 * h, o);
        }
      }
      tmem_st32(tS, pk[0]);  // P_t over the first 64 columns of S_t
      tmem_st32(tS + 32, pk[1]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);
    }

    if (ti.n_kv > 0) {
      if (ok && mbar_wait(o_done, (ti.n_kv - 1) & 1)) {
        tc_fence_after();
        const float inv_l = (l_sum > 0.f) ? 1.f / l_sum : 0.f;
        uint4 *dst = reinterpret_cast<uint4 *>(
            out + (static_cast<size_t>(bh) * N + q_row) * kD);
#pragma unroll
        for (int h = 0; h < kD / 32; ++h) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * h, o);
          tmem_wait_ld();
          if (q_row < N) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const uint32_t *src = &o[c * 8];
              uint4 v;
              v.x = Dt::pack2(__uint_as_float(src[0]) * inv_l,
                               __uint_as_float(src[1]) * inv_l);
              v.y = Dt::pack2(__uint_as_float(src[2]) * inv_l,
                               __uint_as_float(src[3]) * inv_l);
              v.z = Dt::pack2(__uint_as_float(src[4]) * inv_l,
                               __uint_as_float(src[5]) * inv_l);
              v.w = Dt::pack2(__uint_as_float(src[6]) * inv_l,
                               __uint_as_float(src[7]) * inv_l);
              dst[4 * h + c] = v;
            }
          }
        }
      } else {
        *abort_flag = 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace prefill128

const void *prefill_d128_kernel_ptr(int dtype) {
  using prefill128::prefill_d128_kernel;
  return dtype == FA_DTYPE_BF16
             ? reinterpret_cast<const void *>(prefill_d128_kernel<BF16>)
             : reinterpret_cast<const void *>(prefill_d128_kernel<F16>);
}
const void *prefill_d128_solo_kernel_ptr(int dtype) {
  return dtype == FA_DTYPE_BF16
             ? reinterpret_cast<const void *>(
                   prefill128::prefill_d128_kernel<BF16, true>)
             : reinterpret_cast<const void *>(
                   prefill128::prefill_d128_kernel<F16, true>);
}
int prefill_d128_solo_smem_bytes() {
  return static_cast<int>(prefill128::Form<true>::kSmemBytes);
}
int prefill_d128_smem_bytes() {
  return static_cast<int>(prefill128::kSmemBytes);
}
const void *prefill_d128_wide_kernel_ptr(int dtype) {
  using prefill128::prefill_d128_wide_kernel;
  return dtype == FA_DTYPE_BF16
             ? reinterpret_cast<const void *>(prefill_d128_wide_kernel<BF16>)
             : reinterpret_cast<const void *>(prefill_d128_wide_kernel<F16>);
}
int prefill_d128_wide_smem_bytes() {
  return static_cast<int>(prefill128::wide::kSmemBytes);
}

cudaError_t launch_prefill_d128_kernel(const CUtensorMap &tm_q,
                                       const CUtensorMap &tm_k,
                                       const CUtensorMap &tm_v, __half *out,
                                       int B, int H, int N, bool causal,
                                       float scale, int H_kv, int sms,
                                       int dtype, cudaStream_t stream) {
  const int BH = B * H;
  const int n_qt = (N + prefill128::kBlockM - 1) / prefill128::kBlockM;
  const int n_pairs =
      (n_qt + prefill128::kTilesPerCta - 1) / prefill128::kTilesPerCta;
  const unsigned grid =
      static_cast<unsigned>(n_pairs) * static_cast<unsigned>(BH);
  const float scale_log2 = scale * 1.4426950408889634f;
  // One wave of CTAs: zig-zag pairs of equal causal work, so the kernel
  // does not wait on the heaviest pair. Several waves: heaviest first.
  const int zigzag = causal && grid <= static_cast<unsigned>(sms) ? 2 : 0;
  // Solo form for short sequences (measured, TFLOP/s, solo vs paired:
  // B64 H32 N128 causal 145 vs 123, B16 H12 N384 causal 253 vs 208, B8 H32
  // N640 causal 392 vs 369; from four tiles on its 2-slot K/V ring loses:
  // B16 H32 N512 causal 343 vs 385, config 3's shape 806 vs 954).
  const bool solo = (n_qt <= 3 || n_qt == 5) &&
                    (n_qt == 1 || grid > static_cast<unsigned>(sms));
  if (solo) {
    auto kernel = dtype == FA_DTYPE_BF16
                      ? prefill128::prefill_d128_kernel<BF16, true>
                      : prefill128::prefill_d128_kernel<F16, true>;
    kernel<<<static_cast<unsigned>(n_qt) * BH, prefill128::Form<true>::kThreads,
             prefill128::Form<true>::kSmemBytes, stream>>>(
        tm_q, tm_k, tm_v, out, N, BH, causal ? 1 : 0, scale_log2, H,
        H / H_kv, 0);
    return cudaGetLastError();
  }
  // Wide form (128-key tiles, P over S) for every multi-tile grid:
  // measured against the 64-key paired form (µs, L2 flushed): config 3's
  // shape causal 216 vs 238, full 434 vs 484, B1 H8 N8192 causal 118 vs
  // 135, B8 H12 N2048 causal 119 vs 127, B1 H14 N4096 causal 66 vs 74.
  // FA_PREFILL_D128_FORM=paired selects the 64-key form (measurement only).
  static const char *force = getenv("FA_PREFILL_D128_FORM");
  const bool wide = !(force && !strcmp(force, "paired"));
  auto kernel = dtype == FA_DTYPE_BF16 ? prefill128::prefill_d128_kernel<BF16>
                                       : prefill128::prefill_d128_kernel<F16>;
  // Blocks of heads whose K/V (both tensors, all N rows) fit in about
  // kHeadBlockL2Bytes of L2, equal in size, for multi-wave grids.
  int head_block = 0;
  if (!zigzag) {
    // K and V bytes per query head (grouped heads share theirs)
    const long long per_head = std::max(
        1LL, static_cast<long long>(N) * 2 * prefill128::kD * 2 * H_kv / H);
    const long long budget = prefill128::kHeadBlockL2Bytes;
    const int fit = static_cast<int>(std::max(1LL, budget / per_head));
    if (fit < BH) {
      const int blocks = (BH + fit - 1) / fit;
      head_block = (BH + blocks - 1) / blocks;
    }
  }
  if (wide) {
    auto wkernel = dtype == FA_DTYPE_BF16
                       ? prefill128::prefill_d128_wide_kernel<BF16>
                       : prefill128::prefill_d128_wide_kernel<F16>;
    wkernel<<<grid, prefill128::kThreads, prefill128::wide::kSmemBytes,
              stream>>>(tm_q, tm_k, tm_v, out, N, BH,
                        (causal ? 1 : 0) | zigzag, scale_log2, H, H / H_kv,
                        head_block);
    return cudaGetLastError();
  }
  kernel<<<grid, prefill128::kThreads, prefill128::kSmemBytes, stream>>>(
      tm_q, tm_k, tm_v, out, N, BH, (causal ? 1 : 0) | zigzag, scale_log2, H,
      H / H_kv, head_block);
  return cudaGetLastError();
}

}  // namespace fa
