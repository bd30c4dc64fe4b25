/*
 * fa_b200.h — C ABI of the B200 (sm_100a) attention forward: head_dim 64
 * fp16 as in the reference, plus head_dim 128, grouped K/V heads and bf16
 * through the entry points that say so.
 *
 * Every entry point takes plain device pointers (fa_prefill_host: host
 * pointers for q/k/v/o), sizes and a cudaStream_t passed as void*. No entry
 * point allocates memory, synchronises the stream
 * or touches a framework type; the Python package (flashattn_cuda._C) and any
 * other host language bind these symbols directly.
 *
 * Tensor layout (identical to the reference's pybind contract): every
 * q/k/v/o/cache tensor is a contiguous (B, H, rows, head_dim) array of
 * 16-bit elements (fp16 unless an entry point takes a dtype); row r of head
 * (b, h) starts at element ((b * H + h) * rows + r) * head_dim.
 *
 * Return value of every int-returning call: FA_OK (0) or one FA_E* code;
 * fa_status_string() names it. Argument errors are detected on the host
 * before anything is launched.
 */
#ifndef FA_B200_H_
#define FA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by the entry points. */
#define FA_OK 0
#define FA_EINVAL 1     /* bad size, count or scale                      */
#define FA_EALIGN 2     /* a pointer is not 16-byte aligned              */
#define FA_ECUDA 3      /* a CUDA runtime call or the launch failed      */
#define FA_ENOSPACE 4   /* caller's workspace is smaller than required   */
#define FA_EDEVICE 5    /* device is not sm_100 / driver entry missing   */

/* Bits of the device-side error word (fa_take_device_error). */
#define FA_ERR_TIMEOUT 1u   /* a pipeline wait exceeded its time limit   */
#define FA_ERR_SMEM_ALIGN 2u /* dynamic shared memory was not 1 KiB aligned */

/* Element types of q/k/v/o and the caches for the _ex entry points (every
 * other entry point is fp16). */
#define FA_DTYPE_F16 0
#define FA_DTYPE_BF16 1

/* head_dim every kernel is built for (reference flash_common.h:11). */
#define FA_HEAD_DIM 64

/*
 * Full-sequence attention forward, O = softmax(scale * Q K^T [+ causal mask]) V.
 * q, k, v, o: (B, H, N, 64) fp16 device arrays, 16-byte aligned; o is written.
 * causal != 0 masks key j > query i (same-length top-left causal mask).
 * Replaces the reference's prefill()/launch_prefill
 * (csrc/bindings.cpp:10-27, csrc/prefill.cu:347-373).
 */
int fa_prefill(const void *q, const void *k, const void *v, void *o, int B,
               int H, int N, int causal, float scale, void *stream);

/*
 * Grouped-query prefill: q, o are (B, H, N, 64), k, v are (B, H_kv, N, 64)
 * with H % H_kv == 0; query head h reads K/V head h / (H / H_kv). Same as
 * fa_prefill when H_kv == H, and equal to fa_prefill on K/V heads repeated
 * H / H_kv times, without materialising the repeat. No reference
 * counterpart (the reference's future work, README.md:398); the BASELINE
 * Qwen2.5-0.5B shapes have H=14, H_kv=2.
 */
int fa_prefill_gqa(const void *q, const void *k, const void *v, void *o, int B,
                   int H, int H_kv, int N, int causal, float scale,
                   void *stream);

/*
 * Prefill for head_dim 64 or 128: q, o (B, H, N, head_dim); k, v
 * (B, H_kv, N, head_dim) with H % H_kv == 0. head_dim 64 is fa_prefill_gqa;
 * head_dim 128 runs a kernel of its own (64-key tiles, 128-column O in
 * tensor memory). The reference is specialised to 64 and names 128 as its
 * next size (README "Engineering decisions"); no reference counterpart.
 */
int fa_prefill_hd(const void *q, const void *k, const void *v, void *o, int B,
                  int H, int H_kv, int N, int head_dim, int causal,
                  float scale, void *stream);

/*
 * Prefill for either 16-bit element type: q, k, v, o are fp16
 * (dtype = FA_DTYPE_F16) or bf16 (FA_DTYPE_BF16), all the same type, with
 * the shapes of fa_prefill_hd (head_dim 64 or 128, grouped K/V heads). The
 * arithmetic is the same (fp32 scores, accumulators and softmax); with bf16
 * the probabilities P enter the PV product as bf16 and O is rounded to
 * bf16. fa_prefill_hd is this call with FA_DTYPE_F16. The reference is
 * fp16-only and names bf16 as a next variant (README.md:229-231,397); no
 * reference counterpart.
 */
int fa_prefill_ex(const void *q, const void *k, const void *v, void *o, int B,
                  int H, int H_kv, int N, int head_dim, int dtype, int causal,
                  float scale, void *stream);

/*
 * Prefill with q, k, v and o in HOST memory (page-locked for the copies to
 * overlap; pageable memory works but serialises them). Same shapes and
 * result as fa_prefill_hd: every output element is bit-identical. The heads
 * are streamed through device staging slots in chunks of whole
 * (batch, K/V head) groups: the upload of chunk i+1, the kernel of chunk i
 * and the download of chunk i-1 run at the same time on two internal copy
 * streams and the caller's stream. The call only enqueues; o is complete
 * once `stream` reaches the point of the call (synchronise it before reading
 * o). workspace: device memory of at least fa_prefill_host_plan's
 * workspace_bytes, 256-byte aligned, owned by the caller. The two copy
 * streams and their events are created once per device on first use.
 * Replaces the reference's host-to-device round trip around prefill()
 * (tensors moved with .cuda() before csrc/bindings.cpp:10-27 and .cpu()
 * after); no single reference entry point.
 */
int fa_prefill_host(const void *q, const void *k, const void *v, void *o,
                    int B, int H, int H_kv, int N, int head_dim, int causal,
                    float scale, void *workspace, size_t workspace_bytes,
                    void *stream);

/* fa_prefill_host for either 16-bit element type (q, k, v, o all fp16 or
 * all bf16, dtype as fa_prefill_ex); fa_prefill_host is the fp16 case. */
int fa_prefill_host_ex(const void *q, const void *k, const void *v, void *o,
                       int B, int H, int H_kv, int N, int head_dim, int dtype,
                       int causal, float scale, void *workspace,
                       size_t workspace_bytes, void *stream);

/*
 * Plan of fa_prefill_host for this shape: the number of chunks (one kernel
 * launch each) and the device workspace it needs. Host-only.
 */
int fa_prefill_host_plan(int B, int H, int H_kv, int N, int head_dim,
                         int *chunks, size_t *workspace_bytes);

/*
 * Bytes of scratch memory fa_decode / fa_decode_partial need for this shape
 * and split choice (the log-sum-exp partials of segments split across CTAs).
 * It needs no initialisation. split_size <= 0 selects the automatic,
 * length-balanced schedule. Reference counterpart: the per-call
 * partial_acc/partial_ml allocation in launch_decode
 * (csrc/decode.cu:213-219), hoisted to the caller.
 */
size_t fa_decode_workspace_bytes(int B, int H, int S_max, int split_size,
                                 int device);

/*
 * Single-query attention against a KV cache (the decode step).
 * q, o: (B, H, 1, 64) fp16; k_cache, v_cache: (B, H, S_max, 64) fp16;
 * seq_lens: (B,) int32 device array, sequence b attends cache rows
 * [0, min(seq_lens[b], S_max)); a sequence with no rows gets an all-zero output.
 * split_size <= 0: automatic schedule; > 0: each CTA reduces at most
 * split_size cache rows (the reference's forced split, must be a multiple
 * of 4 as in the reference).
 * workspace: device scratch of at least fa_decode_workspace_bytes() bytes.
 * counters: device array of at least B*H uint32 that is zero before the
 * first call; every completed call leaves it zero again, so one array can
 * serve any sequence of calls and shapes (calls sharing workspace or
 * counters must be ordered on one stream; after a device error reported by
 * fa_take_device_error, zero it again).
 * Replaces decode()/_decode_with_split()/launch_decode
 * (csrc/bindings.cpp:36-76,127-129, csrc/decode.cu:194-240).
 */
int fa_decode(const void *q, const void *k_cache, const void *v_cache,
              const int32_t *seq_lens, void *o, int B, int H, int S_max,
              float scale, int split_size, void *workspace,
              size_t workspace_bytes, uint32_t *counters,
              size_t counter_count, void *stream);

/*
 * Decode for either 16-bit element type: q (B, H, 1, head_dim), caches
 * (B, H_kv, S_max, head_dim) and o, all fp16 (FA_DTYPE_F16) or all bf16
 * (FA_DTYPE_BF16); head_dim 64 or 128; H % H_kv == 0 (grouped K/V heads
 * read once per group). Automatic length-balanced split; seq_lens, clamping
 * and empty sequences as fa_decode. Scratch from
 * fa_decode_ex_workspace_bytes, counters as fa_decode (B * H, zero before
 * the first call, left at zero). No reference counterpart (the reference is
 * fp16-only; bf16 is its named next variant, README.md:229-231,397).
 */
int fa_decode_ex(const void *q, const void *k_cache, const void *v_cache,
                 const int32_t *seq_lens, void *o, int B, int H, int H_kv,
                 int S_max, int head_dim, int dtype, float scale,
                 void *workspace, size_t workspace_bytes, uint32_t *counters,
                 size_t counter_count, void *stream);

/*
 * fa_decode_append_hd for either 16-bit element type (q, new rows, caches
 * and o all fp16 or all bf16): stores each sequence's new K/V row at row
 * seq_lens[b] of the caches and attends seq_lens[b] + 1 rows, in one
 * launch. Scratch from fa_decode_ex_workspace_bytes. No reference
 * counterpart (see fa_decode_append and fa_decode_ex).
 */
int fa_decode_append_ex(const void *q, const void *k_new, const void *v_new,
                        void *k_cache, void *v_cache, const int32_t *seq_lens,
                        void *o, int B, int H, int H_kv, int S_max,
                        int head_dim, int dtype, float scale, void *workspace,
                        size_t workspace_bytes, uint32_t *counters,
                        size_t counter_count, void *stream);

/* Scratch bytes fa_decode_ex needs (the same for both element types). */
size_t fa_decode_ex_workspace_bytes(int B, int H, int H_kv, int S_max,
                                    int head_dim, int device);

/*
 * Scratch bytes fa_decode_gqa needs for this shape (0 on invalid arguments).
 * No reference counterpart.
 */
size_t fa_decode_gqa_workspace_bytes(int B, int H, int H_kv, int S_max,
                                     int device);

/*
 * Decode for head_dim 64 (same as fa_decode) or 128: q, o (B, H, 1,
 * head_dim), caches (B, H, S_max, head_dim), same schedule, rules and
 * counters as fa_decode; workspace of fa_decode_hd_workspace_bytes() bytes.
 * The reference is specialised to 64 and names 128 as its next size; no
 * reference counterpart.
 */
size_t fa_decode_hd_workspace_bytes(int B, int H, int S_max, int head_dim,
                                    int split_size, int device);
int fa_decode_hd(const void *q, const void *k_cache, const void *v_cache,
                 const int32_t *seq_lens, void *o, int B, int H, int S_max,
                 int head_dim, float scale, int split_size, void *workspace,
                 size_t workspace_bytes, uint32_t *counters,
                 size_t counter_count, void *stream);

/*
 * Sequence-sharded decode with the cross-GPU combine inside the kernel.
 * Rank r of `world` (one GPU each, world <= 32) holds a contiguous chunk of
 * every sequence's KV cache (caches (B, H, S_max, 64) of its chunk,
 * seq_lens = rows of the chunk). Each rank allocates one exchange buffer of
 * fa_exchange_bytes(B, H, world) bytes with fa_exchange_alloc (zeroed, with
 * a 64-byte IPC handle), sends the handle to the others and maps theirs
 * with fa_exchange_open; peer_buffers is a device array of the world
 * buffer pointers, index = rank. Every call passes the same epoch on all
 * ranks, starting at 1 and increasing by one per call. Each finished
 * (b, h) partial (m, l, acc[64]) is stored into every rank's buffer over
 * NVLink and counted; each rank then merges all ranks' partials (waits are
 * bounded) and writes the full (B, H, 1, 64) output. Partials of odd and
 * even epochs go to separate banks of the buffer, so a rank that has moved
 * on to the next call never overwrites a partial a slower peer still reads;
 * each rank must issue its calls in one stream order. Replaces the
 * reference-named exchange (decode_partial + NCCL all-gather + merge, the
 * (m, l, o) combine of csrc/decode.cu:143-175 across GPUs). After a
 * device error the buffers and epochs must be re-created.
 */
size_t fa_exchange_bytes(int B, int H, int world);
int fa_exchange_alloc(size_t bytes, void **buffer, void *ipc_handle);
int fa_exchange_open(const void *ipc_handle, void **peer_buffer);
int fa_exchange_close(void *peer_buffer);
int fa_exchange_free(void *buffer);
int fa_decode_exchange(const void *q, const void *k_cache, const void *v_cache,
                       const int32_t *seq_lens, void *o, int B, int H,
                       int S_max, float scale, void *workspace,
                       size_t workspace_bytes, uint32_t *counters,
                       size_t counter_count, float *const *peer_buffers,
                       int rank, int world, uint32_t epoch, void *stream);
/* fa_decode_exchange for either 16-bit element type (q, this rank's cache
 * chunk and o all fp16 or all bf16; dtype as fa_decode_ex) and head_dim 64
 * or 128 (one K/V head per query head). The exchanged partials are fp32
 * either way; peer_buffers sized by fa_exchange_bytes_hd. */
int fa_decode_exchange_ex(const void *q, const void *k_cache,
                          const void *v_cache, const int32_t *seq_lens,
                          void *o, int B, int H, int S_max, int head_dim,
                          int dtype, float scale, void *workspace,
                          size_t workspace_bytes, uint32_t *counters,
                          size_t counter_count, float *const *peer_buffers,
                          int rank, int world, uint32_t epoch, void *stream);

/* Exchange buffer bytes for head_dim 64 (= fa_exchange_bytes) or 128; the
 * buffers of one exchange are sized for the head_dim of the calls using
 * it. head_dim 128 decode scratch is fa_decode_hd_workspace_bytes. */
size_t fa_exchange_bytes_hd(int B, int H, int world, int head_dim);

/*
 * Grouped-query decode for head_dim 64 or 128 (64: as fa_decode_gqa); K/V
 * heads dividing the query heads, every K/V row read once per group;
 * workspace of fa_decode_gqa_hd_workspace_bytes() bytes. No reference
 * counterpart (kernel-side GQA and d = 128 are both the reference's named
 * next steps).
 */
size_t fa_decode_gqa_hd_workspace_bytes(int B, int H, int H_kv, int S_max,
                                        int head_dim, int device);
int fa_decode_gqa_hd(const void *q, const void *k_cache, const void *v_cache,
                     const int32_t *seq_lens, void *o, int B, int H, int H_kv,
                     int S_max, int head_dim, float scale, void *workspace,
                     size_t workspace_bytes, uint32_t *counters,
                     size_t counter_count, void *stream);

/*
 * Decode with the KV-cache append fused in: for every sequence b the new
 * token's k_new / v_new rows (B, H_kv, 1, 64) fp16 are stored at row
 * p = max(seq_lens[b], 0) of k_cache / v_cache (B, H_kv, S_max, 64) and the
 * query attends rows [0, p + 1). When p >= S_max the cache is full: nothing
 * is stored and rows [0, S_max) are attended. seq_lens is only read (the
 * caller advances it). H_kv == H or H % H_kv == 0 as for fa_decode_gqa;
 * workspace of fa_decode_gqa_workspace_bytes(B, H, H_kv, S_max) bytes,
 * counters as for fa_decode. The reference has no append; its callers write
 * the cache row with a separate copy before decode (the step named as the
 * caller of csrc/decode.cu:194-240).
 */
int fa_decode_append(const void *q, const void *k_new, const void *v_new,
                     void *k_cache, void *v_cache, const int32_t *seq_lens,
                     void *o, int B, int H, int H_kv, int S_max, float scale,
                     void *workspace, size_t workspace_bytes,
                     uint32_t *counters, size_t counter_count, void *stream);

/*
 * fa_decode_append for head_dim 64 (same as fa_decode_append) or 128 (k_new,
 * v_new (B, H_kv, 1, 128), caches (B, H_kv, S_max, 128)); workspace of
 * fa_decode_gqa_hd_workspace_bytes(B, H, H_kv, S_max, head_dim) bytes.
 */
int fa_decode_append_hd(const void *q, const void *k_new, const void *v_new,
                        void *k_cache, void *v_cache, const int32_t *seq_lens,
                        void *o, int B, int H, int H_kv, int S_max,
                        int head_dim, float scale, void *workspace,
                        size_t workspace_bytes, uint32_t *counters,
                        size_t counter_count, void *stream);

/*
 * Grouped-query decode: q, o (B, H, 1, 64); caches (B, H_kv, S_max, 64) with
 * H % H_kv == 0 (query head h reads K/V head h / (H / H_kv)); automatic
 * schedule; workspace of fa_decode_gqa_workspace_bytes() bytes; counters as
 * for fa_decode with the same B, H.
 * With H_kv < H every K/V row is read once for its whole group of query
 * heads (up to 16 per pass; larger groups take several passes).
 * No reference counterpart (see fa_prefill_gqa).
 */
int fa_decode_gqa(const void *q, const void *k_cache, const void *v_cache,
                  const int32_t *seq_lens, void *o, int B, int H, int H_kv,
                  int S_max, float scale, void *workspace,
                  size_t workspace_bytes, uint32_t *counters,
                  size_t counter_count, void *stream);

/*
 * Decode that stops before normalisation and writes, per (b, h), the
 * log-sum-exp partial {m, l, pad, pad, acc[64]} as 68 fp32 (m in log2 units
 * of scale*q.k; acc unnormalised). Used when the KV cache of one sequence is
 * sharded over GPUs: each GPU reduces its chunk, the partials are exchanged,
 * and fa_merge_partials finishes. No reference counterpart: the reference
 * has no multi-GPU path; the partial layout is its decode.cu:215-219
 * (m, l, acc) triple.
 */
int fa_decode_partial(const void *q, const void *k_cache, const void *v_cache,
                      const int32_t *seq_lens, float *partial_out, int B,
                      int H, int S_max, float scale, void *workspace,
                      size_t workspace_bytes, uint32_t *counters,
                      size_t counter_count, void *stream);

/*
 * Largest batch * heads that fa_decode_noalloc accepts; its scratch array is
 * sized for this many (batch, head) pairs.
 */
#define FA_NOALLOC_MAX_BH 8192

/*
 * fa_decode without caller-provided scratch, for callers that cannot
 * allocate GPU memory (a memory pool fixed at start-up, a plugin that only
 * receives its input and output pointers). Same arguments, layout and
 * results as fa_decode with the automatic schedule; no reference
 * counterpart (the reference allocates its scratch on every call).
 * The scratch lives in a fixed device array inside the library (about
 * 2.5 MB on every GPU that loads it, held until the process exits), so
 * nothing is allocated. Limits: B * H <= FA_NOALLOC_MAX_BH, else
 * FA_ENOSPACE before anything is launched. The first call on a device looks
 * up the array's device address (make it before any stream capture). All
 * calls share the array: calls that can overlap on the GPU (different
 * streams, or other devices' threads racing on one device) corrupt each
 * other's results; order them on one stream.
 */
int fa_decode_noalloc(const void *q, const void *k_cache, const void *v_cache,
                      const int32_t *seq_lens, void *o, int B, int H,
                      int S_max, float scale, void *stream);

/*
 * Log-sum-exp merge of G partial sets laid out (G, B, H, 68) fp32 into the
 * fp16 output o (B, H, 1, 64). Partials with l <= 0 are skipped and a row
 * with no keys anywhere is 0, as in the reference's merge pass
 * (csrc/decode.cu:143-175).
 */
int fa_merge_partials(const float *partials, int G, void *o, int B, int H,
                      void *stream);

/*
 * The reference's chunk-size rule: largest power of two in [128, 1024] with
 * batch*heads*ceil(max_seq/chunk) >= min_blocks, else 128
 * (csrc/decode.cu:183-192). Pure host function.
 */
int fa_choose_decode_split(int max_seq, int batch, int heads, int min_blocks);

/*
 * CTA form the head_dim-64 prefill launches for bh (batch x head) pairs of
 * n tokens on a device with `sms` SMs: one of FA_PREFILL_FORM_*; *ctas (if
 * not NULL) receives the grid size; -1 for a non-positive argument. Pure
 * host function. The reference's
 * launch_prefill (csrc/prefill.cu:347-373) has a single form with grid
 * (ceil(N/64), H, B); this reports which of the three B200 forms runs.
 */
#define FA_PREFILL_FORM_PAIRED 0    /* two query tiles of one head per CTA */
#define FA_PREFILL_FORM_SOLO 1      /* one query tile per CTA, 2 CTAs/SM */
#define FA_PREFILL_FORM_KEY_SPLIT 2 /* one query tile, key tiles split */
int fa_prefill_form(long long bh, int n, int causal, int sms, int *ctas);

/* One row of the occupancy report (reference csrc/flash_common.h:31-38). */
typedef struct fa_occupancy_entry {
  char name[64];
  int threads_per_block;
  int registers_per_thread;
  int shared_bytes_per_block;
  int max_active_blocks_per_sm;
  double theoretical_occupancy;
} fa_occupancy_entry;

/*
 * Fills up to max_entries rows for every kernel at its launch configuration
 * on the current device; *count receives the number of kernels.
 * Replaces occupancy_report() (csrc/bindings.cpp:80-97).
 */
int fa_occupancy(fa_occupancy_entry *out, int max_entries, int *count);

/*
 * Reads and clears the device-side error word of the current device
 * (FA_ERR_* bits, 0 when every kernel completed normally). Synchronises
 * the device. No reference counterpart: the reference kernels have no
 * bounded waits.
 */
int fa_take_device_error(unsigned int *bits);

/*
 * Sets how long any single device-side wait (a pipeline mbarrier, or a
 * peer's arrival counter in fa_decode_exchange) may spin on the current
 * device before the kernel records FA_ERR_TIMEOUT and unwinds; ns in
 * [1e3, 6e10], default 1e9 (1 s). Synchronises the device first. A host
 * that detects lost peers sooner, or a test that makes a wait run out on
 * purpose, shortens it. No reference counterpart (no bounded waits there).
 */
int fa_set_wait_limit_ns(unsigned long long ns);

/*
 * Single-head fp32 attention O = softmax(Q K^T / 8) V on (N, 64) fp32
 * device arrays (non-causal), the function behind the reference's v1
 * legacy_naive / legacy_tiled / legacy_fused exports
 * (csrc/legacy/legacy_ops.cu:39-51, csrc/bindings.cpp:131-133).
 */
int fa_legacy_attention_f32(const float *q, const float *k, const float *v,
                            float *o, int N, void *stream);

/* Name of a status code. */
const char *fa_status_string(int status);

/* Number of SMs of the current device (0 on failure). */
int fa_num_sms(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H_ */
