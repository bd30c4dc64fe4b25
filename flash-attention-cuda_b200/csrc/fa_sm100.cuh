// Device-side building blocks for the sm_100a attention kernels: mbarriers
// with bounded waits, TMA (tensor and bulk) loads, tcgen05 tensor-memory
// allocation / MMA / load / store, and the shared-memory matrix descriptors
// the tensor core reads its operands through.
//
// Everything here is hand-written inline PTX for sm_100a. No cluster-wide
// copies are used anywhere: every load lands in the issuing CTA's own shared
// memory.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "fa_b200.h"

namespace fa {

// The head dimension every kernel is specialised for (flash_common.h:11 in the
// reference pins the same value).
constexpr int kHeadDim = 64;
constexpr int kRowBytes = kHeadDim * 2;  // one fp16 row of K, V, Q or O

// Longest a single wait (on an mbarrier or a peer's counter) may spin before
// the kernel gives up, records FA_ERR_TIMEOUT and unwinds. Normal waits last
// microseconds. The default is 1 s; fa_set_wait_limit_ns changes it (tests
// shorten it to make a wait run out in milliseconds).
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s
__device__ unsigned long long g_fa_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ unsigned long long wait_limit_ns() {
  return *reinterpret_cast<volatile unsigned long long *>(&g_fa_wait_limit_ns);
}

// Device-wide error word, OR-ed with FA_ERR_* bits by any kernel that has to
// abandon its work. Read and cleared from the host by fa_take_device_error().
// The library is one translation unit (fa_all.cu), so this is its only
// definition.
__device__ unsigned int g_fa_error_word = 0;

__device__ __forceinline__ void record_error(unsigned int bits) {
  atomicOr(&g_fa_error_word, bits);
}

// True once any kernel has timed out since the host last read the error word.
// CTAs check it at entry and leave at once, so a failure costs one wait limit
// rather than one per CTA of a large grid. The host must read and clear the
// word (fa_take_device_error) to resume normal operation.
__device__ __forceinline__ bool device_failed() {
  return (*reinterpret_cast<volatile unsigned int *>(&g_fa_error_word) &
          FA_ERR_TIMEOUT) != 0;
}

// Optional cycle-stamp tracing of the pipeline (profiling builds only,
// compiled with -DFA_TRACE): the first 4 CTAs record clock64() at fixed slots.
#ifdef FA_TRACE
__device__ unsigned long long g_fa_trace[4 * 4096];
#define FA_TRACE_EVENT(slot)                                           \
  do {                                                                 \
    if (blockIdx.x < 4) g_fa_trace[blockIdx.x * 4096 + (slot)] = clock64(); \
  } while (0)
// Per-CTA global-timer stamps (8 slots per CTA, up to 2048 CTAs).
#define FA_TRACE_CTA(slot)                                               \
  do {                                                                   \
    if (blockIdx.x < 2048) g_fa_trace[blockIdx.x * 8 + (slot)] = global_timer_ns(); \
  } while (0)
#else
#define FA_TRACE_EVENT(slot) \
  do {                       \
  } while (0)
#define FA_TRACE_CTA(slot) \
  do {                     \
  } while (0)
#endif

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar,
                                                      uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of the phase. On sm_100 it answers an already completed
// phase in a few cycles, where try_wait costs about a hundred.
__device__ __forceinline__ bool mbar_test_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and
// records FA_ERR_TIMEOUT) if it has not completed within wait_limit_ns(), so a
// lost arrival turns into an error status instead of a hung GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_test_wait(addr, parity)) return true;
  if (mbar_try_wait(addr, parity)) return true;
  const unsigned long long t0 = global_timer_ns();
  const unsigned long long limit = wait_limit_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
      if (mbar_try_wait(addr, parity)) return true;
    }
    if (global_timer_ns() - t0 > limit) {
      record_error(FA_ERR_TIMEOUT);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// Copies into this CTA's shared memory
// ---------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
}

// 3-D tiled TMA load; coordinates are innermost first.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0),
      "r"(c1), "r"(c2)
      : "memory");
}

// Contiguous bulk copy global -> shared (both 16-byte aligned, size % 16 == 0),
// with an L2 eviction-priority hint for data that is read exactly once.
__device__ __forceinline__ void bulk_load(void *dst, const void *src,
                                          uint32_t bytes, uint64_t *bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(p));
  return p;
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (tensor core / TMA) reads of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Tensor memory (TMEM) and tcgen05
// ---------------------------------------------------------------------------
// Warp-wide: allocates `ncols` columns (power of two >= 32) and writes the
// TMEM base address into *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst)),
      "r"(ncols)
      : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, single-thread issue.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc,
                                          uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16: A (M x K, 16-bit) is read from
// tensor memory, lane = row, two elements per 32-bit column.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem,
                                          uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

// Warp-collective: thread t of the warp reads 32 consecutive 32-bit columns of
// TMEM lane (warp's lane quarter)*32 + t, starting at column (taddr & 0xffff).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr,
                                          const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Shared-memory matrix descriptors (sm_100 format, version 1)
//   bits  0-13 start address >> 4      bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4 bits 46-47 version (1)
//   bits 49-51 base offset (0: tiles are 1024-byte aligned)
//   bits 61-63 layout: 2 = 128-byte swizzle
// Every operand tile here is rows of 64 fp16 (128 bytes) written with the
// 128-byte swizzle, so 8 rows form one 1024-byte swizzle atom and the stride
// between atoms is 1024 bytes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>(1u) << 16) |        // LBO (unused by SW128)
         (static_cast<uint64_t>(1024u >> 4) << 32) |  // SBO: 8-row atom stride
         (static_cast<uint64_t>(1u) << 46) |        // descriptor version
         (static_cast<uint64_t>(2u) << 61);         // SWIZZLE_128B
}

// Instruction descriptor for kind::f16 with 16-bit A/B and fp32 accumulate.
//   bits 4-5 D format (1 = f32), 7-9 A format (0 = f16, 1 = bf16), 10-12 B
//   format (A and B always the same here), bit 15 A major (0 = K), bit 16 B
//   major (1 = MN), 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n,
                                                     bool b_mn_major,
                                                     uint32_t fmt = 0) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) |
         (static_cast<uint32_t>(b_mn_major) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Warp-level tensor-core operations (register operands)
// ---------------------------------------------------------------------------
// Four 8x8 16-bit matrices from shared memory; lanes 8i..8i+7 give the row
// addresses of matrix i. Lane t receives row t / 4, elements 2 (t % 4) and
// 2 (t % 4) + 1 of each matrix (the transposed variant: column t / 4, rows
// 2 (t % 4) and 2 (t % 4) + 1).
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(addr)
      : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr,
                                              uint32_t (&r)[4]) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(addr)
      : "memory");
}

// D (16x8 fp32) += A (16x16 bf16, row) * B (16x8 bf16, col).
__device__ __forceinline__ void mma_16816_bf16(float (&d)[4],
                                               const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D (16x8 fp32) += A (16x16 fp16, row) * B (16x8 fp16, col).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4],
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Math helpers
// ---------------------------------------------------------------------------
// 2^x with the MUFU approximation (hardware ex2, flush-to-zero).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Blackwell packed fp32 pair arithmetic (one instruction for two lanes of
// work) and the three-input max.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  return __ffma2_rn(a, b, c);
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  return __fadd2_rn(a, b);
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// fma with the result clamped to [0, 1] (the .sat modifier; there is no
// packed fp32x2 form of it).
__device__ __forceinline__ float fma_sat(float a, float b, float c) {
  float d;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for two values on the FMA pipe instead of the MUFU unit, the exponent
// given in clamped affine form: xs in [0, 1] stands for
// x = kExp2Lo + kExp2Span * xs, so the caller forms xs = saturate(s * a + b)
// with one scalar FMA per value and the clamp of x to [-126, 127] comes
// free with it (the range keeps the biased exponent written below inside
// 0..254). Cody-Waite style range reduction: x = j + f with j = round(x)
// and |f| <= 1/2, where j comes from the "add 1.5 * 2^23" rounding trick
// (the integer lands in the low mantissa bits of t). 2^f is a degree-3
// polynomial whose coefficients were fit for this project by iteratively
// reweighted least squares toward the minimax relative error on
// [-1/2, 1/2] (max relative error 7.5e-5, below half an fp16 ulp, which is
// all the result needs: it becomes a 16-bit P entry). Finally j is added
// to the exponent field.
constexpr float kExp2Lo = -126.f;
constexpr float kExp2Span = 253.f;
__device__ __forceinline__ float2 exp2_poly2_affine(float2 xs) {
  constexpr float kRoundLo = 12582912.0f + kExp2Lo;  // 1.5 * 2^23 - 126
  constexpr float kC0 = 0.99992806f;
  constexpr float kC1 = 0.69326097f;
  constexpr float kC2 = 0.24261113f;
  constexpr float kC3 = 0.05517166f;
  const float2 span = make_float2(kExp2Span, kExp2Span);
  const float2 t = ffma2(xs, span, make_float2(kRoundLo, kRoundLo));
  // -(j - kExp2Lo), so that f = kExp2Span * xs - (j - kExp2Lo) = x - j
  const float2 nr = ffma2(t, make_float2(-1.f, -1.f),
                          make_float2(kRoundLo, kRoundLo));
  const float2 f = ffma2(xs, span, nr);
  float2 p = ffma2(make_float2(kC3, kC3), f, make_float2(kC2, kC2));
  p = ffma2(p, f, make_float2(kC1, kC1));
  p = ffma2(p, f, make_float2(kC0, kC0));
  float2 out;
  out.x = __uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23));
  out.y = __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23));
  return out;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

// ---------------------------------------------------------------------------
// 16-bit element types. Tensors are 16-bit storage either way (the kernels'
// pointers are typed __half); the element type decides how values convert
// to and from fp32 and which format the tensor cores are given. Both MMA
// operands always have the same type.
// ---------------------------------------------------------------------------
struct F16 {
  static constexpr int kDtype = FA_DTYPE_F16;
  static constexpr uint32_t kFmt = 0;  // instruction-descriptor format
  __device__ static __forceinline__ uint32_t pack2(float lo, float hi) {
    return pack_half2(lo, hi);
  }
  __device__ static __forceinline__ float2 unpack2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&w));
  }
  __device__ static __forceinline__ void mma16816(float (&d)[4],
                                                  const uint32_t (&a)[4],
                                                  uint32_t b0, uint32_t b1) {
    mma_16816(d, a, b0, b1);
  }
};

struct BF16 {
  static constexpr int kDtype = FA_DTYPE_BF16;
  static constexpr uint32_t kFmt = 1;
  __device__ static __forceinline__ uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  __device__ static __forceinline__ float2 unpack2(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w));
  }
  __device__ static __forceinline__ void mma16816(float (&d)[4],
                                                  const uint32_t (&a)[4],
                                                  uint32_t b0, uint32_t b1) {
    mma_16816_bf16(d, a, b0, b1);
  }
};

// One output element in the tensor's 16-bit storage (run-time type: the
// rarely executed output paths of the decode kernels).
__device__ __forceinline__ __half store_elem(float x, int dtype) {
  return dtype == FA_DTYPE_BF16
             ? __ushort_as_half(__bfloat16_as_ushort(__float2bfloat16_rn(x)))
             : __float2half_rn(x);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a,
                                             uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a),
               "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Per-warpgroup register reallocation (all four warps of a warpgroup must
// execute the same one).
template <int kRegs>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}
template <int kRegs>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}

// True in exactly one lane of a fully active warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// Named barrier over a subset of the CTA's warps.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Arrive at a named barrier without waiting for the others.
__device__ __forceinline__ void named_bar_arrive(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// Softmax row helpers of the prefill kernels (one thread per 128-key S row).
// ---------------------------------------------------------------------------
// Bit i set: column pair i of every 8 takes its exponentials from the MUFU
// unit, the others from the polynomial on the FMA pipe. Five of eight
// balances the two pipes on the B200 (measured per-instruction costs: a warp
// ex2 holds the MUFU pipe 8 cycles, a packed FMA 2, and a polynomial pair
// costs about 18 FMA-pipe cycles against 16 MUFU cycles for a MUFU pair
// plus 4 on the FMA pipe); the fp16 pack and the row max run on a third
// pipe.
constexpr unsigned kMufuMask8 = 0x3B;

// Max of a 128-column S row: three-input max over 8 independent chains (one
// 127-long dependent chain would leave the two softmax warps of an SM
// sub-partition stalled on max latency).
__device__ __forceinline__ float row_max_128(const float (&s)[128]) {
  float mxp[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mxp[i] = s[i];
#pragma unroll
  for (int c = 8; c + 16 <= 128; c += 16) {  // columns 8..119
#pragma unroll
    for (int i = 0; i < 8; ++i) mxp[i] = fmax3(mxp[i], s[c + i], s[c + 8 + i]);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) mxp[i] = fmaxf(mxp[i], s[120 + i]);
  return fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]),
               fmaxf(mxp[6], mxp[7]));
}

// P = 2^(s * sl - m) for a 128-column row, packed to 16-bit pairs in pk;
// returns the row sum of the fp32 P values. The exponentials alternate
// between the MUFU unit (argument: one packed FMA per two columns) and the
// polynomial on the FMA pipe (argument: one saturating FMA per column, which
// also clamps it), so neither pipe bounds the step alone. The row sum uses
// four packed accumulators.
template <typename Dt>
__device__ __forceinline__ float exp_row(const float (&s)[128], float sl,
                                         float m, uint32_t (&pk)[2][32]) {
  const float2 sl2 = make_float2(sl, sl);
  const float2 nm2 = make_float2(-m, -m);
  const float a = sl * (1.f / kExp2Span);
  const float b = (-m - kExp2Lo) * (1.f / kExp2Span);
  float2 rs[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) rs[i] = make_float2(0.f, 0.f);
#pragma unroll
  for (int c = 0; c < 128; c += 2) {
    float2 p;
    if (!((kMufuMask8 >> ((c >> 1) & 7)) & 1)) {
      p = exp2_poly2_affine(
          make_float2(fma_sat(s[c], a, b), fma_sat(s[c + 1], a, b)));
    } else {
      const float2 x = ffma2(make_float2(s[c], s[c + 1]), sl2, nm2);
      p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
    }
    rs[(c >> 1) & 3] = fadd2(rs[(c >> 1) & 3], p);
    pk[c >> 6][(c >> 1) & 31] = Dt::pack2(p.x, p.y);
  }
  const float2 r = fadd2(fadd2(rs[0], rs[1]), fadd2(rs[2], rs[3]));
  return r.x + r.y;
}

}  // namespace fa
