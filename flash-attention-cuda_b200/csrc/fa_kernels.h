// Internal launch interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "fa_b200.h"

namespace fa {

// ---- prefill (prefill_sm100.cu) -------------------------------------------
const void *prefill_kernel_ptr(int dtype = FA_DTYPE_F16);
int prefill_threads();
const void *prefill_solo_kernel_ptr(int dtype = FA_DTYPE_F16);
int prefill_solo_smem_bytes();
int prefill_solo_threads();
const void *prefill_split_kernel_ptr(int dtype = FA_DTYPE_F16);
int prefill_split_smem_bytes();
const void *prefill_d128_solo_kernel_ptr(int dtype = FA_DTYPE_F16);
int prefill_d128_solo_smem_bytes();
const void *prefill_d128_wide_kernel_ptr(int dtype = FA_DTYPE_F16);
int prefill_d128_wide_smem_bytes();
int prefill_smem_bytes();
cudaError_t launch_prefill_kernel(const CUtensorMap &tm_q,
                                  const CUtensorMap &tm_k,
                                  const CUtensorMap &tm_v, __half *out, int B,
                                  int H, int N, bool causal, float scale,
                                  int H_kv, int sms, int dtype,
                                  cudaStream_t stream, long long plan_bh = 0);
// CTA form of the head_dim-64 prefill for BH (batch x head) pairs of N
// tokens (FA_PREFILL_FORM_*); *ctas (if given) receives the grid size.
// plan_bh > 0: the form of a chunk of a larger problem of plan_bh pairs.
int prefill_form_of(long long BH, int N, bool causal, int sms,
                    long long plan_bh, int *ctas);
// fa_prefill_ex for one chunk of a larger problem of plan_bh (batch x head)
// pairs: the CTA form is chosen for the whole problem, so a head's output
// does not depend on how the problem was cut into launches (capi.cu).
int prefill_chunk_ex(const void *q, const void *k, const void *v, void *o,
                     int B, int H, int H_kv, int N, int head_dim, int dtype,
                     int causal, float scale, void *stream, long long plan_bh);

// ---- prefill, head_dim 128 (prefill_d128_sm100.cu) -------------------------
const void *prefill_d128_kernel_ptr(int dtype = FA_DTYPE_F16);
int prefill_d128_smem_bytes();
cudaError_t launch_prefill_d128_kernel(const CUtensorMap &tm_q,
                                       const CUtensorMap &tm_k,
                                       const CUtensorMap &tm_v, __half *out,
                                       int B, int H, int N, bool causal,
                                       float scale, int H_kv, int sms,
                                       int dtype, cudaStream_t stream);

// ---- decode (decode_sm100.cu) ---------------------------------------------
struct DecodeArgs {
  const __half *q;
  const __half *k;
  const __half *v;
  const int32_t *seq_lens;
  __half *out;           // final fp16 output, or
  float *partial_out;    // (B, H, 68) log-sum-exp partials when non-null
  float *ws_partials;    // (B*H + grid) x 68 fp32
  uint32_t *ws_counters; // B*H arrival counters, zero between calls
  // fused append (null when not appending): the new token's K/V rows
  // (B, H_kv, 64), stored at row seq_lens[b] of the caches (written through
  // k_cache_w / v_cache_w, the same caches as k / v) and attended
  const __half *k_new;
  const __half *v_new;
  __half *k_cache_w;
  __half *v_cache_w;
  // cross-GPU exchange (null when not sharded): x_peers[r] is rank r's
  // exchange buffer, two epoch-parity banks of (x_world, B*H, 4 + D) fp32
  // partials then B*H uint32
  // arrival counters; each finished segment is sent to every rank and the
  // merged output written once all x_world partials of it are present
  // (counters reach x_epoch * x_world)
  float *const *x_peers;
  int x_rank, x_world;
  uint32_t x_epoch;
  int B, H, S_max;
  int H_kv;  // K/V heads; H / H_kv query heads share each
  float scale_log2;
  long long rows_per_cta;  // 0: balance the valid rows over the grid
  int grid;
  int dtype;  // FA_DTYPE_F16 or FA_DTYPE_BF16 (q, caches, new rows, out)
};

constexpr int kPartialFloats = 68;  // m, l, pad, pad, acc[64]

const void *decode_kernel_ptr(int dtype = FA_DTYPE_F16);
int decode_threads();
int decode_smem_bytes();
int decode_ctas_per_sm();
int decode_min_rows_per_cta();
cudaError_t launch_decode_kernel(const DecodeArgs &args, cudaStream_t stream);

// Grouped-query decode: K/V read once per group of query heads. The grid is
// one CTA per SM at most; segments are (b, K/V head, chunk of up to
// decode_gqa_max_heads() query heads).
// (decode_gqa_sm100.cu) head_dim 64 or 128; K/V TMA boxes of
// decode_gqa_box_rows(head_dim) rows; partials of 4 + head_dim floats.
const void *decode_gqa_kernel_ptr(int head_dim, int dtype = FA_DTYPE_F16);
int decode_gqa_smem_bytes(int head_dim);
int decode_gqa_max_heads();
// Partial records of one segment one round of the final merge gathers.
int decode_gqa_merge_batch(int head_dim, int heads_per_seg);
int decode_gqa_box_rows(int head_dim);
cudaError_t launch_decode_gqa_kernel(const DecodeArgs &args,
                                     const CUtensorMap &tm_k,
                                     const CUtensorMap &tm_v, int head_dim,
                                     cudaStream_t stream);

// head_dim 128 per-head decode (decode_d128_sm100.cu); partials are
// decode_d128_partial_floats() = 132 floats, grid as decode_kernel's.
const void *decode_d128_kernel_ptr(int dtype = FA_DTYPE_F16);
int decode_d128_smem_bytes();
int decode_d128_partial_floats();
cudaError_t launch_decode_d128_kernel(const DecodeArgs &args,
                                      cudaStream_t stream);

const void *merge_kernel_ptr();
int merge_threads();
cudaError_t launch_merge_kernel(const float *partials, int G, __half *out,
                                int B, int H, cudaStream_t stream);

// ---- single-head fp32 attention (legacy_sm100.cu) -------------------------
cudaError_t launch_legacy_kernel(const float *q, const float *k, const float *v,
                                 float *o, int N, cudaStream_t stream);

}  // namespace fa
