// Prefill (full-sequence) attention forward for B200, head_dim 64, fp16 in,
// fp32 accumulate, fp16 out.
//
// Behaviour follows the reference's prefill_kernel (csrc/prefill.cu:164-343):
// O = softmax(scale * Q K^T, causal mask k <= q) V per (batch, head), with
// fully-masked causal key tiles skipped. The implementation is a different
// machine: QK^T and PV run on the 5th-generation tensor cores (tcgen05.mma,
// fp32 accumulators in tensor memory), Q/K/V tiles arrive by TMA into an
// mbarrier ring, and the online softmax runs in registers of dedicated warps
// that read S straight out of tensor memory and write P back into it.
//
// Two CTA forms share one kernel template.
//
// Paired form (one CTA per SM): the CTA owns two 128-row query tiles of one
// (batch, head) and ping-pongs them. While one softmax warpgroup
// exponentiates its S tile, the tensor core computes the other tile's S or
// PV; both tiles share every K/V tile loaded. 12 warps (384 threads):
//   warps 0-3  softmax of query tile 0 (thread = row = TMEM lane)
//   warps 4-7  softmax of query tile 1
//   warp 8     TMA producer: Q tiles once, then K_j, V_j per 128-key tile
//   warp 9     MMA issuer (one thread); owns the TMEM allocation
//   warps 10-11 only donate registers
// Shared memory: Q0, Q1 (32 KiB), K and V rings of 3 x 16 KiB, mbarriers.
// Tensor memory (512 columns x 128 lanes, fp32 words):
//   S0 [0,128)  S1 [128,256)  O0 [256,320)  O1 [320,384)
//   P0 [384,448)  P1 [448,512)   (P = fp16 pairs, the A operand of PV)
//
// Solo form (two CTAs per SM): one query tile per CTA, 8 warps (softmax
// 0-3, producer 4, MMA 5, donors 6-7), Q (16 KiB) and the two 3-slot rings
// in 112 KiB of shared memory, S [0,128) O [128,192) P [192,256) in 256
// tensor-memory columns. Two resident CTAs take the place of the two tiles
// of the paired form, and one CTA's start-up (its first tiles from HBM) and
// epilogue overlap the other's key steps.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <functional>
#include <map>
#include <queue>
#include <vector>

#include "fa_kernels.h"
#include "fa_sm100.cuh"

namespace fa {
namespace prefill {

constexpr int kBlockM = 128;  // query rows per tile
constexpr int kBlockN = 128;  // keys per KV tile
constexpr int kTilesPerCta = 2;
// K/V ring slots in shared memory: two key tiles stream ahead of the one in
// use.
constexpr int kRingSlots = 3;
// Ring slots of the key-split form, which consumes two key tiles per round.
constexpr int kSplitRingSlots = 5;
constexpr int kMaxRingSlots = kSplitRingSlots;
// Longest sequence, in query tiles, that runs in the solo form (measured:
// N 4096 solo 743 vs paired 724 TFLOP/s, N 8192 798 vs 809, N 16384 738 vs
// 746).
constexpr int kSoloMaxTiles = 48;
// K/V bytes of one block of heads in the launch order (the same budget as
// the head_dim-128 kernel; B8 H12 N4096 full +5 %, C3 unchanged).
constexpr long long kHeadBlockL2Bytes = 32ll << 20;
constexpr int kSoftmaxThreads = 128;  // per query tile
constexpr int kCtrlRegs = 24;
constexpr uint32_t kTileBytes = kBlockN * kRowBytes;  // 16 KiB

constexpr uint32_t kQOff = 0;
// barrier slots
constexpr int kBarQFull = 0;
constexpr int kBarKFull = kBarQFull + 1;          // + stage: K and V tile
constexpr int kBarKVEmpty = kBarKFull + kMaxRingSlots;  // + stage
constexpr int kBarSFull = kBarKVEmpty + kMaxRingSlots;  // + tile
constexpr int kBarSFree = kBarSFull + kTilesPerCta;
constexpr int kBarPFull = kBarSFree + kTilesPerCta;
constexpr int kBarODone = kBarPFull + kTilesPerCta;
constexpr int kBarDrain = kBarODone + kTilesPerCta;
constexpr int kNumBars = kBarDrain + 1;
constexpr uint32_t kTmemS = 0;    // + 128 * tile

// Threads, roles, shared-memory offsets and tensor-memory columns of the
// paired (kSolo false), solo and key-split forms described at the top of
// this file. The key-split form has the paired form's warps and tensor
// memory but one Q tile, a deeper ring and the merge rows (m, l of the
// second warpgroup) in shared memory.
template <bool kSolo, bool kSplit = false>
struct Form {
  static_assert(!(kSolo && kSplit), "one form at a time");
  static constexpr int kThreads = kSolo ? 256 : 384;
  static constexpr int kCtasPerSm = kSolo ? 2 : 1;
  static constexpr int kCtrlWarp0 = kSolo ? 4 : 8;  // first control warp
  static constexpr int kProducerWarp = kCtrlWarp0;
  static constexpr int kMmaWarp = kCtrlWarp0 + 1;
  static constexpr int kSoftmaxRegs = kSolo ? 232 : 240;
  static constexpr int kQTiles = (kSolo || kSplit) ? 1 : 2;
  static constexpr int kSlots = kSplit ? kSplitRingSlots : kRingSlots;
  static constexpr uint32_t kKOff = kQOff + kQTiles * kTileBytes;
  static constexpr uint32_t kVOff = kKOff + kSlots * kTileBytes;
  static constexpr uint32_t kBarOff = kVOff + kSlots * kTileBytes;
  static constexpr uint32_t kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr uint32_t kAbortOff = kTmemSlotOff + 4;
  static constexpr uint32_t kMergeOff = kAbortOff + 12;  // 16-byte aligned
  static constexpr uint32_t kSmemBytes = kMergeOff + (kSplit ? 2 * 128 * 4 : 0);
  static constexpr uint32_t kTmemCols = kSolo ? 256 : 512;
  static constexpr uint32_t kTmemO = kSolo ? 128 : 256;  // + 64 * tile
  static constexpr uint32_t kTmemP = kSolo ? 192 : 384;  // + 64 * tile
  static_assert(kMergeOff % 16 == 0, "merge rows misaligned");
  static constexpr int kSoftmaxGroups = kSolo ? 1 : 2;
  static_assert(128 * kCtrlRegs + 128 * kSoftmaxGroups * kSoftmaxRegs <=
                    kThreads * (65536 / (kThreads * kCtasPerSm)),
                "register split exceeds the launch allocation");
  static_assert(kCtasPerSm * (kSmemBytes + 1024) <= 228 * 1024,
                "shared memory of the resident CTAs exceeds the SM's");
};

template <typename Dt>
constexpr uint32_t kIdescS = idesc_f16_f32(kBlockM, kBlockN, false, Dt::kFmt);
template <typename Dt>
constexpr uint32_t kIdescPV = idesc_f16_f32(kBlockM, kHeadDim, true, Dt::kFmt);

// The max is only moved (and O rescaled) when a row's running max grows by
// more than this many powers of two; until then exponents are taken against
// the stale max, which bounds P by 2^8 and keeps l and O consistent because
// both use the same reference point.
constexpr float kRescaleThreshold = 8.0f;

// S = Q K^T for one 128x128 tile: 4 MMAs of K=16 (32 bytes further along
// the swizzled 128-byte rows each).
template <typename Dt>
__device__ __forceinline__ void issue_s_tile(uint32_t d, uint64_t q_desc,
                                             uint64_t k_desc) {
#pragma unroll
  for (int kk = 0; kk < kHeadDim / 16; ++kk)
    mma_f16_ss(d, q_desc + 2 * kk, k_desc + 2 * kk, kIdescS<Dt>, kk > 0 ? 1u : 0u);
}

// O (+)= P V for one tile: 8 MMAs of K=16 keys. P is read from tensor memory
// (8 columns = 16 fp16 per step); V steps by 16 rows = 2048 bytes.
template <typename Dt>
__device__ __forceinline__ void issue_pv_tile(uint32_t d, uint32_t p_tmem,
                                              uint64_t v_desc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < kBlockN / 16; ++kk)
    mma_f16_ts(d, p_tmem + 8 * kk, v_desc + 128 * kk, kIdescPV<Dt>,
               (accumulate || kk > 0) ? 1u : 0u);
}

struct TileInfo {
  int qt;    // query tile index along the sequence
  int n_kv;  // key tiles this query tile attends (0: tile past the end)
};

__device__ __forceinline__ TileInfo tile_info(int pair, int t, int N,
                                              int causal, int zigzag) {
  TileInfo ti;
  const int n_qt = (N + kBlockM - 1) / kBlockM;
  // zig-zag: tile p with tile n_qt - 1 - p, so every causal pair attends
  // the same number of keys (one-wave grids)
  ti.qt = zigzag ? (t == 0 ? pair : n_qt - 1 - pair) : 2 * pair + t;
  if (ti.qt >= n_qt || (t == 1 && zigzag && ti.qt == pair)) {
    ti.n_kv = 0;
  } else {
    ti.n_kv = causal ? ti.qt + 1 : (N + kBlockN - 1) / kBlockN;
  }
  return ti;
}

template <typename Dt, bool kSolo = false, bool kSplit = false>
__global__ void __launch_bounds__(Form<kSolo, kSplit>::kThreads,
                                  Form<kSolo, kSplit>::kCtasPerSm)
    prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                   const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v,
                   __half *__restrict__ out, int N, int BH, int causal,
                   float scale_log2, int H, int group, int head_block) {
  using F = Form<kSolo, kSplit>;
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

  // Heaviest first: blockIdx.x walks query tiles (solo) or query-tile pairs
  // from the last (most keys) to the first, heads fastest.
  // Within blocks of head_block heads (0: all heads) whose K/V fit in L2,
  // so a head's tiles run close together and its K/V is read once.
  const int n_qt = (N + kBlockM - 1) / kBlockM;
  const int n_pairs = (n_qt + 1) / 2;
  const int n_units = (kSolo || kSplit) ? n_qt : n_pairs;  // per head
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
  // K/V head of the query head: `group` query heads share one K/V head
  // (group == 1 without grouped-query attention).
  const int kv_bh = (bh / H) * (H / group) + (bh % H) / group;
  TileInfo t0, t1;
  // Key-split form: one query tile whose key tiles alternate between the two
  // softmax warpgroups (even key tiles to t0, odd to t1); TileInfo.n_kv then
  // counts rounds of that warpgroup.
  int n_keys = 0;
  if (kSplit) {
    t0.qt = unit;
    t1.qt = unit;
    n_keys = causal ? unit + 1 : n_qt;
    t0.n_kv = (n_keys + 1) / 2;
    t1.n_kv = n_keys / 2;
  } else if (kSolo) {
    t0.qt = unit;
    t0.n_kv = causal ? t0.qt + 1 : n_qt;
    t1.qt = t0.qt;
    t1.n_kv = 0;
  } else {
    t0 = tile_info(pair, 0, N, causal, zigzag);
    t1 = tile_info(pair, 1, N, causal, zigzag);
  }
  const int n_kv = t0.n_kv > t1.n_kv ? t0.n_kv : t1.n_kv;

  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + F::kBarOff);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + F::kTmemSlotOff);
  volatile uint32_t *abort_flag =
      reinterpret_cast<volatile uint32_t *>(smem + F::kAbortOff);

  // Key tile j goes to ring stage j % kStages.
  const int n_pos = kSplit ? n_keys : n_kv;
  auto load_pos = [&](int p) {
    const int s = p % kStages;
    mbar_arrive_expect_tx(&bars[kBarKFull + s], 2 * kTileBytes);
    tma_load_3d(smem + F::kKOff + s * kTileBytes, &tm_k, &bars[kBarKFull + s], 0,
                p * kBlockN, kv_bh);
    tma_load_3d(smem + F::kVOff + s * kTileBytes, &tm_v, &bars[kBarKFull + s], 0,
                p * kBlockN, kv_bh);
  };

  // The producer lane sets up the barriers and issues the Q tiles and the
  // first kStages K/V tiles before the CTA-wide barrier, so their latency
  // overlaps the TMEM allocation; the device error word (a global read) is
  // checked after that and turns into the abort flag.
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
    const bool two = !kSplit && t1.n_kv > 0;
    mbar_arrive_expect_tx(&bars[kBarQFull], (two ? 2 : 1) * kTileBytes);
    tma_load_3d(smem + kQOff, &tm_q, &bars[kBarQFull], 0, t0.qt * kBlockM, bh);
    if (two)
      tma_load_3d(smem + kQOff + kTileBytes, &tm_q, &bars[kBarQFull], 0,
                  t1.qt * kBlockM, bh);
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

  // Register split: the control warpgroup (producer, MMA, two idle warps)
  // gives registers to the two softmax warpgroups, which hold a full S row.
  // 128 * kCtrlRegs + 128 * tiles * kSoftmaxRegs fits the launch budget
  // (checked in Form).
  // Each role's code sits inside the branch that sized its registers, so
  // the compiler allocates each region for its own budget.
  if (warp >= F::kCtrlWarp0) {
    setmaxnreg_dec<kCtrlRegs>();
  if (warp == F::kProducerWarp) {
    // ------------------------------------------------------------------ TMA
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
      // No copy of ours may still be landing when the CTA exits (matters
      // only when another role gave up early).
      if (*abort_flag) {
        mbar_wait(&bars[kBarQFull], 0);
        for (int p = (issued > kStages ? issued - kStages : 0); p < issued;
             ++p) {
          mbar_wait(&bars[kBarKFull + p % kStages], (p / kStages) & 1);
        }
      }
    }
  } else if (warp == F::kMmaWarp) {
    // ------------------------------------------------------------------ MMA
    // The whole warp runs the control flow, so every operand below is
    // warp-uniform; one elected lane issues the tcgen05 instructions.
    // Descriptors are formed once and advanced by adding byte offsets >> 4.
    const bool leader = elect_one();
    const uint32_t tmem = __shfl_sync(0xffffffffu, tmem_base, 0);
    const int n0 = t0.n_kv;
    const int n1 = t1.n_kv;
    const uint64_t desc0 = sw128_desc(sbase);
    // Q tile of warpgroup t and the key position (ring order) of its round j.
    auto q_off = [](int t) -> uint32_t {
      return kSplit ? kQOff : kQOff + t * kTileBytes;
    };
    auto kpos = [](int j, int t) { return kSplit ? 2 * j + t : j; };
    bool ok = mbar_wait(&bars[kBarQFull], 0) &&
              mbar_wait(&bars[kBarKFull + 0], 0) &&
              (!kSplit || n1 == 0 || mbar_wait(&bars[kBarKFull + 1], 0));
    if (ok) {
      tc_fence_after();
      if (leader) {
        if (n0 > 0) {
          issue_s_tile<Dt>(tmem + kTmemS, desc0 + (q_off(0) >> 4),
                           desc0 + (F::kKOff >> 4));
          mma_commit(&bars[kBarSFull + 0]);
        }
        if (n1 > 0) {
          issue_s_tile<Dt>(tmem + kTmemS + 128, desc0 + (q_off(1) >> 4),
                           desc0 + ((F::kKOff + kpos(0, 1) * kTileBytes) >> 4));
          mma_commit(&bars[kBarSFull + 1]);
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
        const int nt = t ? n1 : n0;
        if (!ok || j >= nt) continue;
        const int s = kpos(j, t) % kStages;         // K_j, V_j
        const int p1 = kpos(j + 1, t);
        const int s1 = p1 % kStages;                // K_{j+1}
        if (j + 1 < nt) {
          // K/V tile j+1 is waited on once per round (by the first tile
          // that uses it); V_j was waited on with K_j the round before.
          // In the key-split form each key tile has one user.
          const bool need_kv = kSplit || (t == 0) || (n0 <= j + 1);
          if ((need_kv &&
               !mbar_wait(&bars[kBarKFull + s1], (p1 / kStages) & 1)) ||
              !mbar_wait(&bars[kBarSFree + t], j & 1)) {
            ok = false;
            continue;
          }
          FA_TRACE_EVENT(2048 + j * 16 + t * 8 + 3);
          tc_fence_after();
          if (leader) {
            issue_s_tile<Dt>(tmem + kTmemS + 128 * t, desc0 + (q_off(t) >> 4),
                             desc0 + ((F::kKOff + s1 * kTileBytes) >> 4));
            mma_commit(&bars[kBarSFull + t]);
          }
          __syncwarp();
          FA_TRACE_EVENT(2048 + j * 16 + t * 8 + 1);
        }
        if (!mbar_wait(&bars[kBarPFull + t], j & 1)) {
          ok = false;
          continue;
        }
        FA_TRACE_EVENT(2048 + j * 16 + t * 8 + 4);
        tc_fence_after();
        if (leader) {
          issue_pv_tile<Dt>(tmem + F::kTmemO + 64 * t, tmem + F::kTmemP + 64 * t,
                        desc0 + ((F::kVOff + s * kTileBytes) >> 4), j > 0);
          mma_commit(&bars[kBarODone + t]);
          // key-split form: this key tile's ring stage is free once its PV
          // retires
          if (kSplit) mma_commit(&bars[kBarKVEmpty + s]);
        }
        __syncwarp();
        FA_TRACE_EVENT(2048 + j * 16 + t * 8 + 2);
      }
      if (!ok) break;
      // release round j's ring stage
      if (!kSplit && leader) {
        mma_commit(&bars[kBarKVEmpty + j % kStages]);
      }
      __syncwarp();
    }
    if (!ok && leader) *abort_flag = 1;
    // Every MMA issued above has retired once this commit lands; TMEM is
    // not released before that.
    if (leader) mma_commit(&bars[kBarDrain]);
    __syncwarp();
    mbar_wait(&bars[kBarDrain], 0);
  }
  } else {
    setmaxnreg_inc<F::kSoftmaxRegs>();
    // -------------------------------------------------------------- softmax
    const int t = warp >> 2;            // query tile of this warpgroup
    const int row = threadIdx.x & 127;  // row in the tile == TMEM lane
    const TileInfo ti = t == 0 ? t0 : t1;
    const uint32_t lane_addr = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem_base + lane_addr + kTmemS + 128 * t;
    const uint32_t tO = tmem_base + lane_addr + F::kTmemO + 64 * t;
    const uint32_t tP = tmem_base + lane_addr + F::kTmemP + 64 * t;
    uint64_t *s_full = &bars[kBarSFull + t];
    uint64_t *s_free = &bars[kBarSFree + t];
    uint64_t *p_full = &bars[kBarPFull + t];
    uint64_t *o_done = &bars[kBarODone + t];
    float m_use = -INFINITY;  // running max, in log2 units of scale * q.k
    float l_sum = 0.f;
    bool ok = true;

    for (int j = 0; j < ti.n_kv; ++j) {
      if (row == 0) FA_TRACE_EVENT(t * 1024 + j * 8 + 0);
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
      tc_fence_before();
      mbar_arrive(s_free);
      if (row == 0) FA_TRACE_EVENT(t * 1024 + j * 8 + 1);

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
      uint32_t pk[2][32];  // P row as fp16 pairs, TMEM columns [0,32), [32,64)
      const int kt = kSplit ? 2 * j + t : j;  // key tile of this round
      const int kbase = kt * kBlockN;
      const bool diag = causal && (kt == ti.qt);
      if (diag || kbase + kBlockN > N) {
        int lim = N - kbase;
        if (diag) lim = min(lim, row + 1);
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = (c < lim) ? s[c] : -INFINITY;
      }
      // Row max of the tile; the reference max m_use moves only when it
      // grows by more than kRescaleThreshold (then l and O are rescaled).
      float corr = 1.f;
      bool rescale = false;
      const float m_tile = row_max_128(s) * sl;
      if (m_tile > m_use + kRescaleThreshold) {
        corr = fast_exp2(m_use - m_tile);  // 0 on the first tile
        m_use = m_tile;
        rescale = true;
      }
      const float rowsum = exp_row<Dt>(s, sl, m_use, pk);
      l_sum = fmaf(l_sum, corr, rowsum);

      if (j > 0) {
        // PV_{j-1} must have retired: it reads the P columns about to be
        // overwritten and writes the O columns a rescale would touch.
        if (row == 0) FA_TRACE_EVENT(t * 1024 + j * 8 + 2);
        if (!mbar_wait(o_done, (j - 1) & 1)) {
          ok = false;
          break;
        }
        if (row == 0) FA_TRACE_EVENT(t * 1024 + j * 8 + 3);
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
        }
      }
      tmem_st32(tP, pk[0]);
      tmem_st32(tP + 32, pk[1]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);
      if (row == 0) FA_TRACE_EVENT(t * 1024 + j * 8 + 4);
    }

    // Row q_row of the output: O (fp32 words, 64 columns) times w.
    auto store_row = [&](const uint32_t (&o)[2][32], float w) {
      const int q_row = ti.qt * kBlockM + row;
      if (q_row >= N) return;
      uint4 *dst = reinterpret_cast<uint4 *>(
          out + (static_cast<size_t>(bh) * N + q_row) * kHeadDim);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 v;
        const uint32_t *src = &o[c >> 2][(c & 3) * 8];
        v.x = Dt::pack2(__uint_as_float(src[0]) * w, __uint_as_float(src[1]) * w);
        v.y = Dt::pack2(__uint_as_float(src[2]) * w, __uint_as_float(src[3]) * w);
        v.z = Dt::pack2(__uint_as_float(src[4]) * w, __uint_as_float(src[5]) * w);
        v.w = Dt::pack2(__uint_as_float(src[6]) * w, __uint_as_float(src[7]) * w);
        dst[c] = v;
      }
    };

    if (kSplit) {
      // Merge of the two warpgroups' partial rows (same query row, disjoint
      // key tiles). Warpgroup 1 leaves its (m, l) in shared memory and
      // arrives; warpgroup 0 waits, reads them and warpgroup 1's O from
      // tensor memory (warps w and w + 4 reach the same lanes), rescales
      // both to the larger max and writes the row. Both warpgroups always
      // reach the barrier, also after giving up.
      float *merge_m = reinterpret_cast<float *>(smem + F::kMergeOff);
      float *merge_l = merge_m + 128;
      const bool done =
          ok && (ti.n_kv == 0 || mbar_wait(o_done, (ti.n_kv - 1) & 1));
      if (!done) *abort_flag = 1;
      if (t == 1) {
        merge_m[row] = ti.n_kv > 0 ? m_use : -INFINITY;
        merge_l[row] = ti.n_kv > 0 ? l_sum : 0.f;
        tc_fence_before();
        named_bar_arrive(1, 2 * kSoftmaxThreads);
      } else {
        named_bar_sync(1, 2 * kSoftmaxThreads);
        tc_fence_after();
        if (!*abort_flag) {
          const float m1 = merge_m[row];
          const float l1 = merge_l[row];
          const float m = fmaxf(m_use, m1);
          const float c0 = fast_exp2(m_use - m);
          const float c1 = l1 > 0.f ? fast_exp2(m1 - m) : 0.f;
          const float l = l_sum * c0 + l1 * c1;
          const float inv_l = l > 0.f ? 1.f / l : 0.f;
          uint32_t o[2][32];
          tmem_ld32(tO, o[0]);
          tmem_ld32(tO + 32, o[1]);
          tmem_wait_ld();
          if (t1.n_kv > 0) {  // CTA-uniform: warpgroup 1 had key tiles
            const uint32_t tO1 = tO + 64;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint32_t o1[32];
              tmem_ld32(tO1 + 32 * h, o1);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 32; ++c) {
                const float a = __uint_as_float(o[h][c]) * c0;
                const float b = l1 > 0.f ? __uint_as_float(o1[c]) * c1 : 0.f;
                o[h][c] = __float_as_uint(a + b);
              }
            }
            store_row(o, inv_l);
          } else {
            store_row(o, c0 * inv_l);
          }
        }
      }
    } else if (ti.n_kv > 0) {
      if (ok && mbar_wait(o_done, (ti.n_kv - 1) & 1)) {
        tc_fence_after();
        uint32_t o[2][32];
        tmem_ld32(tO, o[0]);
        tmem_ld32(tO + 32, o[1]);
        tmem_wait_ld();
        store_row(o, (l_sum > 0.f) ? 1.f / l_sum : 0.f);
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

}  // namespace prefill

namespace prefill {

// Kernel-time estimates of the causal forms, in microseconds, from list
// scheduling of the grid in launch order (each CTA to the slot that frees
// first) with per-CTA costs fitted to B200 measurements of the three forms
// (20 causal shapes, N 512-32768, 2-96 heads; the estimate picks the faster
// form on 19 of them, and the one miss costs 1.5 %):
//   paired / key-split CTA: 4.0 + 1.35 per round in which both warpgroups
//     compute + 1.0 per round in which one does; one CTA per SM;
//   solo CTA: 3.0 + 1.2 per key step, two CTAs per SM, and no shorter than
//     3.0 + 0.8 per step of the longest tile (a CTA alone on an SM).
double list_schedule(const std::vector<double> &costs, int slots) {
  std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
  for (int i = 0; i < slots; ++i) free_at.push(0.0);
  double end = 0.0;
  for (double c : costs) {
    const double t = free_at.top() + c;
    free_at.pop();
    free_at.push(t);
    end = std::max(end, t);
  }
  return end;
}

bool key_split_pays(int n_qt, long long bh, int sms) {
  // Beyond about four tiles per SM the forms differ only by per-CTA costs,
  // which the key split doubles; 1 tile cannot be split.
  if (n_qt < 2 || n_qt * bh > 4LL * sms || sms <= 0) return false;
  struct Memo {
    int n_qt;
    long long bh;
    int sms;
    bool pays;
  };
  static thread_local Memo memo[8] = {};
  static thread_local int memo_next = 0;
  for (const Memo &m : memo)
    if (m.n_qt == n_qt && m.bh == bh && m.sms == sms) return m.pays;

  constexpr double kCta = 4.0, kDouble = 1.35, kSingle = 1.0;
  constexpr double kSoloCta = 3.0, kSoloStep = 1.2, kSoloAlone = 0.8;
  std::vector<double> costs;
  costs.reserve(static_cast<size_t>(n_qt * bh));
  for (int n = n_qt; n >= 1; --n)  // heaviest query tile first
    for (long long h = 0; h < bh; ++h)
      costs.push_back(kCta + kDouble * ((n + 1) / 2));
  const double t_split = list_schedule(costs, sms);

  const int n_pairs = (n_qt + 1) / 2;
  const bool solo = n_qt <= kSoloMaxTiles && n_pairs * bh > sms;
  double t_default;
  costs.clear();
  if (solo) {
    for (int n = n_qt; n >= 1; --n)
      for (long long h = 0; h < bh; ++h) costs.push_back(kSoloCta + kSoloStep * n);
    t_default = std::max(kSoloCta + kSoloAlone * n_qt,
                         list_schedule(costs, 2 * sms));
  } else {
    // paired: zig-zag pairs (p, n_qt - 1 - p) in one wave, else (2p, 2p+1)
    // heaviest first; a pair's rounds are those of its longer tile
    const bool zigzag = n_pairs * bh <= sms;
    for (int p = n_pairs - 1; p >= 0; --p) {
      int hi, lo;
      if (zigzag) {
        hi = n_qt - p;
        lo = (p == n_qt - 1 - p) ? 0 : p + 1;
      } else {
        hi = std::min(2 * p + 2, n_qt);
        lo = 2 * p + 1 < n_qt ? 2 * p + 1 : 0;
      }
      if (lo > hi) std::swap(lo, hi);
      for (long long h = 0; h < bh; ++h)
        costs.push_back(kCta + kDouble * lo + kSingle * (hi - lo));
    }
    std::sort(costs.begin(), costs.end(), std::greater<double>());
    t_default = list_schedule(costs, sms);
  }
  const bool pays = t_split < t_default;
  memo[memo_next] = {n_qt, bh, sms, pays};
  memo_next = (memo_next + 1) % 8;
  return pays;
}

}  // namespace prefill

int prefill_form_of(long long BH, int N, bool causal, int sms,
                    long long plan_bh, int *ctas) {
  const int n_qt = (N + prefill::kBlockM - 1) / prefill::kBlockM;
  const long long n_pairs = (n_qt + 1) / 2;
  // Solo form (one query tile per CTA, two CTAs per SM) unless the paired
  // grid fits one wave, where zig-zag pairs give every SM equal work, or
  // the sequence is long enough that the pairs' shared K/V loads win.
  int form = n_qt <= prefill::kSoloMaxTiles && (n_qt == 1 || n_pairs * BH > sms)
                 ? FA_PREFILL_FORM_SOLO
                 : FA_PREFILL_FORM_PAIRED;
  // Key-split form (one query tile per CTA, its key tiles alternating
  // between two softmax warpgroups) where the list-scheduling estimate
  // (key_split_pays) says it finishes first: causal grids of about two
  // query tiles per SM or fewer, where the longest query tile's chain of key
  // steps, not the total work, sets the kernel time, and the split halves
  // that chain. Its rounding differs from the other forms' (key tiles summed
  // in another order), so the choice is made on the whole problem (plan_bh)
  // when a caller launches it in chunks.
  if (causal && prefill::key_split_pays(n_qt, plan_bh > 0 ? plan_bh : BH, sms))
    form = FA_PREFILL_FORM_KEY_SPLIT;
  // FA_PREFILL_FORM=paired|solo|split forces a form (measurement only).
  static const char *force = getenv("FA_PREFILL_FORM");
  if (force && *force) {
    form = !strcmp(force, "split")  ? FA_PREFILL_FORM_KEY_SPLIT
           : !strcmp(force, "solo") ? FA_PREFILL_FORM_SOLO
                                    : FA_PREFILL_FORM_PAIRED;
  }
  if (ctas) *ctas = static_cast<int>(form == FA_PREFILL_FORM_PAIRED ? n_pairs * BH
                                                                    : n_qt * BH);
  return form;
}

const void *prefill_solo_kernel_ptr(int dtype) {
  using prefill::prefill_kernel;
  return dtype == FA_DTYPE_BF16
             ? reinterpret_cast<const void *>(prefill_kernel<BF16, true>)
             : reinterpret_cast<const void *>(prefill_kernel<F16, true>);
}
int prefill_solo_smem_bytes() {
  return static_cast<int>(prefill::Form<true>::kSmemBytes);
}
int prefill_solo_threads() { return prefill::Form<true>::kThreads; }
const void *prefill_split_kernel_ptr(int dtype) {
  using prefill::prefill_kernel;
  return dtype == FA_DTYPE_BF16
             ? reinterpret_cast<const void *>(prefill_kernel<BF16, false, true>)
             : reinterpret_cast<const void *>(prefill_kernel<F16, false, true>);
}
int prefill_split_smem_bytes() {
  return static_cast<int>(prefill::Form<false, true>::kSmemBytes);
}
const void *prefill_kernel_ptr(int dtype) {
  return dtype == FA_DTYPE_BF16
             ? reinterpret_cast<const void *>(prefill::prefill_kernel<BF16>)
             : reinterpret_cast<const void *>(prefill::prefill_kernel<F16>);
}
int prefill_threads() { return prefill::Form<false>::kThreads; }
int prefill_smem_bytes() {
  return static_cast<int>(prefill::Form<false>::kSmemBytes);
}


cudaError_t launch_prefill_kernel(const CUtensorMap &tm_q,
                                  const CUtensorMap &tm_k,
                                  const CUtensorMap &tm_v, __half *out, int B,
                                  int H, int N, bool causal, float scale,
                                  int H_kv, int sms, int dtype,
                                  cudaStream_t stream, long long plan_bh) {
  static_assert(prefill::kBlockM == prefill::kBlockN,
                "causal tile skipping assumes square tiles");
  const int BH = B * H;
  const int n_qt = (N + prefill::kBlockM - 1) / prefill::kBlockM;
  const int n_pairs = (n_qt + 1) / 2;
  const unsigned grid =
      static_cast<unsigned>(n_pairs) * static_cast<unsigned>(BH);
  const float scale_log2 = scale * 1.4426950408889634f;
  // One wave of CTAs: zig-zag pairs of equal causal work, so the kernel
  // does not wait on the heaviest pair. Several waves: heaviest first.
  const int zigzag = causal && grid <= static_cast<unsigned>(sms) ? 2 : 0;
  const int form = prefill_form_of(BH, N, causal, sms, plan_bh, nullptr);
  const bool split = form == FA_PREFILL_FORM_KEY_SPLIT;
  const bool solo = form == FA_PREFILL_FORM_SOLO;
  if (split) {
    using prefill::prefill_kernel;
    auto kernel = dtype == FA_DTYPE_BF16 ? prefill_kernel<BF16, false, true>
                                         : prefill_kernel<F16, false, true>;
    kernel<<<static_cast<unsigned>(n_qt) * BH,
             prefill::Form<false, true>::kThreads,
             prefill::Form<false, true>::kSmemBytes, stream>>>(
        tm_q, tm_k, tm_v, out, N, BH, causal ? 1 : 0, scale_log2, H,
        H / H_kv, 0);
    return cudaGetLastError();
  }
  // Blocks of heads whose K/V (both tensors, all N rows) fit in about
  // kHeadBlockL2Bytes of L2, equal in size, for multi-wave grids.
  int head_block = 0;
  if (!zigzag) {
    const long long per_head = std::max(
        1LL, static_cast<long long>(N) * 2 * kHeadDim * 2 * H_kv / H);
    const long long budget = prefill::kHeadBlockL2Bytes;
    const int fit = static_cast<int>(std::max(1LL, budget / per_head));
    if (fit < BH) {
      const int blocks = (BH + fit - 1) / fit;
      head_block = (BH + blocks - 1) / blocks;
    }
  }
  if (solo) {
    using prefill::prefill_kernel;
    auto kernel = dtype == FA_DTYPE_BF16 ? prefill_kernel<BF16, true>
                                         : prefill_kernel<F16, true>;
    kernel<<<static_cast<unsigned>(n_qt) * BH, prefill::Form<true>::kThreads,
             prefill::Form<true>::kSmemBytes, stream>>>(
        tm_q, tm_k, tm_v, out, N, BH, causal ? 1 : 0, scale_log2, H,
        H / H_kv, head_block);
    return cudaGetLastError();
  }
  auto kernel = dtype == FA_DTYPE_BF16 ? prefill::prefill_kernel<BF16>
                                       : prefill::prefill_kernel<F16>;
  kernel<<<grid, prefill::Form<false>::kThreads,
           prefill::Form<false>::kSmemBytes, stream>>>(
      tm_q, tm_k, tm_v, out, N, BH, (causal ? 1 : 0) | zigzag, scale_log2, H,
      H / H_kv, head_block);
  return cudaGetLastError();
}

}  // namespace fa
