/*
 * CPU oracle for the head_dim-64 attention forward — TEST INFRASTRUCTURE ONLY.
 *
 * This file is a checker, never part of the product: only tests/, the smoke
 * check in __graft_entry__.py and bench.py's CPU-baseline leg may load it.
 * The library (flash-attention-cuda_b200/) never calls it and has no CPU
 * fallback.
 *
 * Plain C restatement of the reference's algorithm, in double precision on
 * inputs that the caller has already rounded to fp16:
 *   - oracle_prefill follows the reference's C++ CPU attention
 *     (src/main.cu:44-104: S = Q K^T * scale, row-max-subtracted softmax,
 *     O = P V) extended to (B, H) loops and the causal mask k <= q of the
 *     CUDA kernel (csrc/prefill.cu:268).
 *   - oracle_decode is the same computation for one query row over the first
 *     min(seq_lens[b], S_max) cache rows (csrc/decode.cu:69), with the
 *     reference's rule that a sequence with no rows outputs 0
 *     (csrc/decode.cu:164-172).
 * Layouts are the contiguous (B, H, rows, 64) arrays of the product API.
 */
#include <math.h>
#include <stddef.h>
#include <stdlib.h>

#define D 64

static void attend_row(const float *qrow, const float *k, const float *v,
                       int n_keys, double scale, double *scores,
                       float *out) {
  if (n_keys <= 0) {
    for (int d = 0; d < D; ++d) out[d] = 0.f;
    return;
  }
  double mx = -INFINITY;
  for (int j = 0; j < n_keys; ++j) {
    double dot = 0.0;
    const float *krow = k + (size_t)j * D;
    for (int d = 0; d < D; ++d) dot += (double)qrow[d] * (double)krow[d];
    scores[j] = dot * scale;
    if (scores[j] > mx) mx = scores[j];
  }
  double denom = 0.0;
  for (int j = 0; j < n_keys; ++j) {
    scores[j] = exp(scores[j] - mx);
    denom += scores[j];
  }
  double acc[D];
  for (int d = 0; d < D; ++d) acc[d] = 0.0;
  for (int j = 0; j < n_keys; ++j) {
    const float *vrow = v + (size_t)j * D;
    const double p = scores[j] / denom;
    for (int d = 0; d < D; ++d) acc[d] += p * (double)vrow[d];
  }
  for (int d = 0; d < D; ++d) out[d] = (float)acc[d];
}

/* q, k, v, o: (B, H, N, 64) fp32. Returns 0, or -1 on allocation failure. */
int oracle_prefill(const float *q, const float *k, const float *v, float *o,
                   int B, int H, int N, int causal, double scale) {
  double *scores = (double *)malloc(sizeof(double) * (size_t)(N > 0 ? N : 1));
  if (!scores) return -1;
  for (int bh = 0; bh < B * H; ++bh) {
    const size_t base = (size_t)bh * N * D;
    for (int i = 0; i < N; ++i) {
      const int n_keys = causal ? i + 1 : N;
      attend_row(q + base + (size_t)i * D, k + base, v + base, n_keys, scale,
                 scores, o + base + (size_t)i * D);
    }
  }
  free(scores);
  return 0;
}

/* q, o: (B, H, 1, 64); k, v: (B, H, S_max, 64); seq_lens: (B,). */
int oracle_decode(const float *q, const float *k, const float *v,
                  const int *seq_lens, float *o, int B, int H, int S_max,
                  double scale) {
  double *scores = (double *)malloc(sizeof(double) * (size_t)S_max);
  if (!scores) return -1;
  for (int b = 0; b < B; ++b) {
    int len = seq_lens[b];
    if (len < 0) len = 0;
    if (len > S_max) len = S_max;
    for (int h = 0; h < H; ++h) {
      const size_t g = (size_t)b * H + h;
      attend_row(q + g * D, k + g * S_max * D, v + g * S_max * D, len, scale,
                 scores, o + g * D);
    }
  }
  free(scores);
  return 0;
}
