// Single-head fp32 attention, O = softmax(Q K^T / sqrt(64)) V for (N, 64)
// tensors: the import-compatible replacement of the reference's v1 "legacy"
// kernels (csrc/legacy/legacy_ops.cu:39-51 exports legacy_naive,
// legacy_tiled and legacy_fused, three implementations of this one function).
// It keeps their fp32 contract; it is not on the hot path.
//
// CTA = 8 warps, one query row per warp. 64-key tiles of K and V are staged
// in shared memory (fp32, 16 KiB each) and shared by the 8 rows; lane l
// scores keys l and l + 32 against the row, the warp keeps an online
// softmax (max, sum) and lane l accumulates output dims 2l, 2l + 1.

#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "fa_kernels.h"
#include "fa_sm100.cuh"

namespace fa {
namespace legacy {

constexpr int kRowsPerCta = 8;
constexpr int kThreads = kRowsPerCta * 32;
constexpr int kKeys = 64;

__global__ void __launch_bounds__(kThreads)
    legacy_attention_kernel(const float *__restrict__ q,
                            const float *__restrict__ k,
                            const float *__restrict__ v,
                            float *__restrict__ o, int N) {
  __shared__ float ks[kKeys][kHeadDim + 1];  // +1: conflict-free column reads
  __shared__ float vs[kKeys][kHeadDim];
  __shared__ float qs[kRowsPerCta][kHeadDim];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowsPerCta + warp;
  const float scale = 0.125f;  // 1 / sqrt(64), as the v1 kernels fix it

  if (row < N) {
    qs[warp][lane] = q[static_cast<size_t>(row) * kHeadDim + lane] * scale;
    qs[warp][lane + 32] = q[static_cast<size_t>(row) * kHeadDim + lane + 32] * scale;
  }
  float m = -INFINITY, l = 0.f, acc0 = 0.f, acc1 = 0.f;

  for (int base = 0; base < N; base += kKeys) {
    __syncthreads();
    for (int i = threadIdx.x; i < kKeys * kHeadDim; i += kThreads) {
      const int r = i / kHeadDim, c = i % kHeadDim;
      const bool in = base + r < N;
      ks[r][c] = in ? k[static_cast<size_t>(base + r) * kHeadDim + c] : 0.f;
      vs[r][c] = in ? v[static_cast<size_t>(base + r) * kHeadDim + c] : 0.f;
    }
    __syncthreads();
    if (row >= N) continue;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 16
    for (int c = 0; c < kHeadDim; ++c) {
      const float qc = qs[warp][c];
      s0 = fmaf(qc, ks[lane][c], s0);
      s1 = fmaf(qc, ks[lane + 32][c], s1);
    }
    if (base + lane >= N) s0 = -INFINITY;
    if (base + lane + 32 >= N) s1 = -INFINITY;
    float mx = fmaxf(s0, s1);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m, mx);
    const float corr = expf(m - m_new);  // 0 on the first tile
    const float p0 = expf(s0 - m_new);
    const float p1 = expf(s1 - m_new);
    float ps = p0 + p1;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      ps += __shfl_xor_sync(0xffffffffu, ps, off);
    l = l * corr + ps;
    m = m_new;
    acc0 *= corr;
    acc1 *= corr;
    for (int j = 0; j < 32; ++j) {
      const float pj0 = __shfl_sync(0xffffffffu, p0, j);
      const float pj1 = __shfl_sync(0xffffffffu, p1, j);
      acc0 = fmaf(pj0, vs[j][2 * lane], fmaf(pj1, vs[j + 32][2 * lane], acc0));
      acc1 = fmaf(pj0, vs[j][2 * lane + 1],
                  fmaf(pj1, vs[j + 32][2 * lane + 1], acc1));
    }
  }
  if (row < N) {
    const float inv = 1.f / l;
    float2 r = make_float2(acc0 * inv, acc1 * inv);
    reinterpret_cast<float2 *>(o + static_cast<size_t>(row) * kHeadDim)[lane] = r;
  }
}

}  // namespace legacy

cudaError_t launch_legacy_kernel(const float *q, const float *k, const float *v,
                                 float *o, int N, cudaStream_t stream) {
  const int grid = (N + legacy::kRowsPerCta - 1) / legacy::kRowsPerCta;
  legacy::legacy_attention_kernel<<<grid, legacy::kThreads, 0, stream>>>(q, k, v,
                                                                        o, N);
  return cudaGetLastError();
}

}  // namespace fa
