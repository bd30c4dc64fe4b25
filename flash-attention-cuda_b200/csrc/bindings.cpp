// flashattn_cuda._C — the PyTorch-facing operator layer over the C ABI in
// include/fa_b200.h. It keeps the reference's pybind surface (csrc/bindings.cpp
// in shrvan30/flash-attention-cuda): the same function names, argument names,
// validation order and error messages, so existing callers and tests see the
// same behaviour. Torch appears only here: tensors are checked, outputs are
// allocated from the caching allocator, and raw pointers plus the current
// stream go to the C ABI.

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>
#include <mutex>
#include <unordered_map>

#include "fa_b200.h"

namespace {

constexpr int kHeadDim = FA_HEAD_DIM;

// Message texts follow the reference's checks (csrc/flash_common.h:43-62) so
// callers matching on them keep working.
void check_cuda(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}
void check_half(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.scalar_type() == at::kHalf, name, " must be fp16 (got ",
              t.scalar_type(), ")");
}
void check_contiguous(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous row-major");
}
// (B, H, N, 64) fp16 CUDA tensor.
void check_bhnd(const at::Tensor &t, const char *name) {
  check_cuda(t, name);
  check_half(t, name);
  check_contiguous(t, name);
  TORCH_CHECK(t.dim() == 4, name, " must be 4-D (B, H, N, ", kHeadDim,
              "), got ", t.dim(), "-D");
  TORCH_CHECK(t.size(3) == kHeadDim, name, " must have head_dim == ",
              kHeadDim, ", got ", t.size(3));
}

// fp16, or bf16 where a kernel exists for it (prefill and decode).
void check_16bit(const at::Tensor &t, const char *name) {
  TORCH_CHECK(t.scalar_type() == at::kHalf || t.scalar_type() == at::kBFloat16,
              name, " must be fp16 or bf16 (got ", t.scalar_type(), ")");
}
int dtype_code(const at::Tensor &t) {
  return t.scalar_type() == at::kBFloat16 ? FA_DTYPE_BF16 : FA_DTYPE_F16;
}

// Prefill and per-head decode also take head_dim 128 (kernels of their own)
// and bf16 tensors.
void check_bhnd_any(const at::Tensor &t, const char *name) {
  check_cuda(t, name);
  check_16bit(t, name);
  check_contiguous(t, name);
  TORCH_CHECK(t.dim() == 4, name, " must be 4-D (B, H, N, ", kHeadDim,
              "), got ", t.dim(), "-D");
  TORCH_CHECK(t.size(3) == kHeadDim || t.size(3) == 128, name,
              " must have head_dim == ", kHeadDim, " (or 128), got ",
              t.size(3));
}

void check_status(int rc, const char *what) {
  TORCH_CHECK(rc == FA_OK, what, " failed: ", fa_status_string(rc));
}

int to_int(int64_t v, const char *what) {
  TORCH_CHECK(v >= 0 && v <= INT32_MAX, what, " out of range: ", v);
  return static_cast<int>(v);
}

void *current_stream() {
  return static_cast<void *>(at::cuda::getCurrentCUDAStream().stream());
}

// Decode scratch, cached per (device, stream): a partials buffer (no
// initialisation needed) and an arrival-counter array that fa_decode leaves
// at zero after every call, so it is zero-filled only when it is
// (re)allocated. Keying by stream keeps concurrent streams apart. The map is
// intentionally never destroyed (no CUDA frees during interpreter exit).
struct DecodeScratch {
  at::Tensor partials;  // uint8
  at::Tensor counters;  // int32, zero between calls
};

DecodeScratch &decode_scratch(const at::Tensor &like, size_t partial_bytes,
                              size_t n_counters) {
  static std::mutex mu;
  static auto *cache = new std::unordered_map<uint64_t, DecodeScratch>();
  const auto stream = at::cuda::getCurrentCUDAStream();
  const uint64_t key = (static_cast<uint64_t>(like.get_device()) << 56) ^
                       static_cast<uint64_t>(stream.id());
  std::lock_guard<std::mutex> lock(mu);
  DecodeScratch &s = (*cache)[key];
  if (!s.partials.defined() ||
      static_cast<size_t>(s.partials.numel()) < partial_bytes) {
    s.partials = at::empty({static_cast<int64_t>(partial_bytes)},
                           like.options().dtype(at::kByte));
  }
  if (!s.counters.defined() ||
      static_cast<size_t>(s.counters.numel()) < n_counters) {
    s.counters = at::zeros({static_cast<int64_t>(n_counters)},
                           like.options().dtype(at::kInt));
  }
  return s;
}

void check_decode_inputs(const at::Tensor &q, const at::Tensor &k_cache,
                         const at::Tensor &v_cache, const at::Tensor &seq_lens,
                         double scale) {
  check_bhnd_any(q, "q");
  check_bhnd_any(k_cache, "k_cache");
  check_bhnd_any(v_cache, "v_cache");
  TORCH_CHECK(q.scalar_type() == k_cache.scalar_type() &&
                  q.scalar_type() == v_cache.scalar_type(),
              "q and the caches must have the same dtype, got ",
              q.scalar_type(), ", ", k_cache.scalar_type(), " and ",
              v_cache.scalar_type());
  TORCH_CHECK(q.size(3) == k_cache.size(3),
              "q and the caches must have the same head_dim, got ", q.size(3),
              " and ", k_cache.size(3));
  TORCH_CHECK(q.size(2) == 1, "decode expects exactly one query row, got ",
              q.size(2));
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes(),
              "k_cache and v_cache must have identical shapes, got ",
              k_cache.sizes(), " and ", v_cache.sizes());
  TORCH_CHECK(q.size(0) == k_cache.size(0) && k_cache.size(1) > 0 &&
                  q.size(1) % k_cache.size(1) == 0,
              "q and the caches must agree on batch and head count, got q=",
              q.sizes(), " cache=", k_cache.sizes());
  TORCH_CHECK(k_cache.size(2) > 0, "cache length must be > 0");
  check_cuda(seq_lens, "seq_lens");
  check_contiguous(seq_lens, "seq_lens");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt,
              "seq_lens must be int32 (got ", seq_lens.scalar_type(), ")");
  TORCH_CHECK(seq_lens.dim() == 1 && seq_lens.size(0) == q.size(0),
              "seq_lens must be 1-D of length B=", q.size(0), ", got ",
              seq_lens.sizes());
  TORCH_CHECK(q.device() == k_cache.device() &&
                  q.device() == v_cache.device() &&
                  q.device() == seq_lens.device(),
              "q, caches and seq_lens must live on the same device");
  TORCH_CHECK(std::isfinite(scale), "scale must be finite");
}

}  // namespace

// prefill(q, k, v, causal, scale): reference csrc/bindings.cpp:10-27.
at::Tensor prefill(const at::Tensor &q, const at::Tensor &k,
                   const at::Tensor &v, bool causal, double scale) {
  check_bhnd_any(q, "q");
  check_bhnd_any(k, "k");
  check_bhnd_any(v, "v");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() &&
                  q.scalar_type() == v.scalar_type(),
              "q, k and v must have the same dtype, got ", q.scalar_type(),
              ", ", k.scalar_type(), " and ", v.scalar_type());
  // Identical shapes as in the reference; additionally k and v may have
  // fewer heads than q when they divide it (grouped-query attention).
  const bool same = q.sizes() == k.sizes() && q.sizes() == v.sizes();
  const bool grouped = k.sizes() == v.sizes() && q.size(0) == k.size(0) &&
                       q.size(2) == k.size(2) && q.size(3) == k.size(3) &&
                       k.size(1) > 0 && q.size(1) % k.size(1) == 0;
  TORCH_CHECK(same || grouped,
              "prefill expects q, k and v to have identical shapes, got q=",
              q.sizes(), " k=", k.sizes(), " v=", v.sizes());
  TORCH_CHECK(q.device() == k.device() && q.device() == v.device(),
              "q, k and v must live on the same device");
  TORCH_CHECK(q.size(2) > 0, "sequence length must be > 0");
  TORCH_CHECK(std::isfinite(scale), "scale must be finite");

  const c10::cuda::CUDAGuard guard(q.device());
  at::Tensor o = at::empty_like(q);
  check_status(fa_prefill_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                             o.data_ptr(), to_int(q.size(0), "batch"),
                             to_int(q.size(1), "heads"),
                             to_int(k.size(1), "kv heads"),
                             to_int(q.size(2), "sequence length"),
                             to_int(q.size(3), "head_dim"), dtype_code(q),
                             causal ? 1 : 0, static_cast<float>(scale),
                             current_stream()),
               "fa_prefill");
  return o;
}

// prefill_host(q, k, v, causal, scale, out=None, non_blocking=False): the
// prefill() contract with q/k/v (and the result) in host memory, streamed
// through the current CUDA device by fa_prefill_host. Page-locked inputs
// let the copies overlap the kernels. The result is a page-locked CPU
// tensor (or `out`); unless non_blocking, the call returns after the
// current stream has finished it, like Tensor.cpu().
at::Tensor prefill_host(const at::Tensor &q, const at::Tensor &k,
                        const at::Tensor &v, bool causal, double scale,
                        c10::optional<at::Tensor> out, bool non_blocking) {
  for (const auto *t : {&q, &k, &v}) {
    TORCH_CHECK(t->device().is_cpu(), "prefill_host expects CPU tensors");
    check_16bit(*t, "q/k/v");
    check_contiguous(*t, "q/k/v");
    TORCH_CHECK(t->dim() == 4 && (t->size(3) == kHeadDim || t->size(3) == 128),
                "q/k/v must be 4-D (B, H, N, 64 or 128), got ", t->sizes());
  }
  const bool same = q.sizes() == k.sizes() && q.sizes() == v.sizes();
  const bool grouped = k.sizes() == v.sizes() && q.size(0) == k.size(0) &&
                       q.size(2) == k.size(2) && q.size(3) == k.size(3) &&
                       k.size(1) > 0 && q.size(1) % k.size(1) == 0;
  TORCH_CHECK(same || grouped,
              "prefill expects q, k and v to have identical shapes, got q=",
              q.sizes(), " k=", k.sizes(), " v=", v.sizes());
  TORCH_CHECK(q.size(2) > 0, "sequence length must be > 0");
  TORCH_CHECK(std::isfinite(scale), "scale must be finite");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() &&
                  q.scalar_type() == v.scalar_type(),
              "q, k and v must have the same dtype");
  at::Tensor o;
  if (out.has_value()) {
    o = *out;
    TORCH_CHECK(o.device().is_cpu() && o.scalar_type() == q.scalar_type() &&
                    o.is_contiguous() && o.sizes() == q.sizes(),
                "out must be a contiguous CPU tensor of q's dtype and shape");
  } else {
    o = at::empty(q.sizes(), q.options().pinned_memory(true));
  }
  const int B = to_int(q.size(0), "batch"), H = to_int(q.size(1), "heads");
  const int H_kv = to_int(k.size(1), "kv heads");
  const int N = to_int(q.size(2), "sequence length");
  const int D = to_int(q.size(3), "head_dim");
  int chunks = 0;
  size_t ws_bytes = 0;
  check_status(fa_prefill_host_plan(B, H, H_kv, N, D, &chunks, &ws_bytes),
               "fa_prefill_host_plan");
  const auto dev_opts = at::TensorOptions()
                            .device(at::kCUDA, at::cuda::current_device())
                            .dtype(at::kByte);
  at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes)}, dev_opts);
  check_status(fa_prefill_host_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                               o.data_ptr(), B, H, H_kv, N, D, dtype_code(q),
                               causal ? 1 : 0,
                               static_cast<float>(scale), ws.data_ptr(),
                               ws_bytes, current_stream()),
               "fa_prefill_host");
  if (!non_blocking) {
    TORCH_CHECK(cudaStreamSynchronize(at::cuda::getCurrentCUDAStream()
                                          .stream()) == cudaSuccess,
                "prefill_host: stream synchronisation failed");
  }
  return o;
}

int64_t prefill_host_launches(int64_t B, int64_t H, int64_t H_kv, int64_t N,
                              int64_t head_dim) {
  int chunks = 0;
  check_status(fa_prefill_host_plan(to_int(B, "batch"), to_int(H, "heads"),
                                    to_int(H_kv, "kv heads"),
                                    to_int(N, "sequence length"),
                                    to_int(head_dim, "head_dim"), &chunks,
                                    nullptr),
               "fa_prefill_host_plan");
  return chunks;
}

// decode / _decode_with_split: reference csrc/bindings.cpp:36-76,127-129.
at::Tensor decode_impl(const at::Tensor &q, const at::Tensor &k_cache,
                       const at::Tensor &v_cache, const at::Tensor &seq_lens,
                       double scale, int64_t split_size) {
  check_decode_inputs(q, k_cache, v_cache, seq_lens, scale);
  if (split_size > 0) {
    TORCH_CHECK(split_size % 4 == 0,
                "decode split size must be a multiple of the warp count, got ",
                split_size);
  }
  const c10::cuda::CUDAGuard guard(q.device());
  const int B = to_int(q.size(0), "batch");
  const int H = to_int(q.size(1), "heads");
  const int S = to_int(k_cache.size(2), "cache length");
  const int split = split_size > 0 ? to_int(split_size, "split_size") : 0;
  at::Tensor o = at::empty_like(q);
  const int H_kv = to_int(k_cache.size(1), "kv heads");
  const int D = to_int(q.size(3), "head_dim");
  const bool bf16 = q.scalar_type() == at::kBFloat16;
  TORCH_CHECK(!bf16 || split == 0, "a forced split size needs fp16 tensors");
  const size_t bytes =
      H_kv != H
          ? fa_decode_gqa_hd_workspace_bytes(B, H, H_kv, S, D, q.get_device())
          : fa_decode_hd_workspace_bytes(B, H, S, D, split, q.get_device());
  TORCH_CHECK(bytes > 0, "fa_decode_workspace_bytes failed");
  DecodeScratch &ws = decode_scratch(q, bytes, static_cast<size_t>(B) * H);
  uint32_t *ctr = reinterpret_cast<uint32_t *>(ws.counters.data_ptr<int32_t>());
  if (bf16) {
    check_status(
        fa_decode_ex(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                     seq_lens.data_ptr<int32_t>(), o.data_ptr(), B, H, H_kv,
                     S, D, FA_DTYPE_BF16, static_cast<float>(scale),
                     ws.partials.data_ptr(),
                     static_cast<size_t>(ws.partials.numel()), ctr,
                     static_cast<size_t>(ws.counters.numel()),
                     current_stream()),
        "fa_decode");
  } else if (H_kv == H) {
    check_status(
        fa_decode_hd(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                     seq_lens.data_ptr<int32_t>(), o.data_ptr(), B, H, S, D,
                     static_cast<float>(scale), split, ws.partials.data_ptr(),
                     static_cast<size_t>(ws.partials.numel()), ctr,
                     static_cast<size_t>(ws.counters.numel()), current_stream()),
        "fa_decode");
  } else {
    TORCH_CHECK(split == 0, "a forced split size needs one K/V head per query head");
    check_status(
        fa_decode_gqa_hd(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                         seq_lens.data_ptr<int32_t>(), o.data_ptr(), B, H, H_kv,
                         S, D, static_cast<float>(scale), ws.partials.data_ptr(),
                         static_cast<size_t>(ws.partials.numel()), ctr,
                         static_cast<size_t>(ws.counters.numel()),
                         current_stream()),
        "fa_decode_gqa");
  }
  return o;
}

at::Tensor decode(const at::Tensor &q, const at::Tensor &k_cache,
                  const at::Tensor &v_cache, const at::Tensor &seq_lens,
                  double scale) {
  return decode_impl(q, k_cache, v_cache, seq_lens, scale, 0);
}

// Per-(b, h) log-sum-exp partials {m, l, 0, 0, acc[64]} of this device's part
// of the cache; used by the sequence-sharded multi-GPU decode.
at::Tensor decode_partial(const at::Tensor &q, const at::Tensor &k_cache,
                          const at::Tensor &v_cache,
                          const at::Tensor &seq_lens, double scale) {
  check_decode_inputs(q, k_cache, v_cache, seq_lens, scale);
  TORCH_CHECK(q.scalar_type() == at::kHalf, "decode_partial needs fp16 tensors");
  TORCH_CHECK(q.size(3) == kHeadDim, "decode_partial needs head_dim == ",
              kHeadDim);
  TORCH_CHECK(k_cache.size(1) == q.size(1),
              "decode_partial needs one K/V head per query head");
  const c10::cuda::CUDAGuard guard(q.device());
  const int B = to_int(q.size(0), "batch");
  const int H = to_int(q.size(1), "heads");
  const int S = to_int(k_cache.size(2), "cache length");
  at::Tensor part = at::empty({B, H, 68}, q.options().dtype(at::kFloat));
  const size_t bytes = fa_decode_workspace_bytes(B, H, S, 0, q.get_device());
  TORCH_CHECK(bytes > 0, "fa_decode_workspace_bytes failed");
  DecodeScratch &ws = decode_scratch(q, bytes, static_cast<size_t>(B) * H);
  check_status(
      fa_decode_partial(
          q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
          seq_lens.data_ptr<int32_t>(), part.data_ptr<float>(), B, H, S,
          static_cast<float>(scale), ws.partials.data_ptr(),
          static_cast<size_t>(ws.partials.numel()),
          reinterpret_cast<uint32_t *>(ws.counters.data_ptr<int32_t>()),
          static_cast<size_t>(ws.counters.numel()), current_stream()),
      "fa_decode_partial");
  return part;
}

// decode_append(q, k_new, v_new, k_cache, v_cache, seq_lens, scale): stores
// the new token's K/V rows at row seq_lens[b] of the caches (in place) and
// attends rows [0, seq_lens[b] + 1) in the same launch. No reference
// counterpart (its callers copy the row into the cache before decode()).
at::Tensor decode_append(const at::Tensor &q, const at::Tensor &k_new,
                         const at::Tensor &v_new, at::Tensor k_cache,
                         at::Tensor v_cache, const at::Tensor &seq_lens,
                         double scale) {
  check_decode_inputs(q, k_cache, v_cache, seq_lens, scale);
  check_bhnd_any(k_new, "k_new");
  check_bhnd_any(v_new, "v_new");
  TORCH_CHECK(k_new.scalar_type() == q.scalar_type() &&
                  v_new.scalar_type() == q.scalar_type(),
              "k_new and v_new must have the dtype of q and the caches");
  TORCH_CHECK(k_new.sizes() == v_new.sizes() && k_new.size(0) == k_cache.size(0) &&
                  k_new.size(1) == k_cache.size(1) && k_new.size(2) == 1 &&
                  k_new.size(3) == k_cache.size(3),
              "k_new and v_new must be (B, H_kv, 1, 64) matching the caches, got ",
              k_new.sizes(), " and ", v_new.sizes());
  TORCH_CHECK(k_new.device() == q.device() && v_new.device() == q.device(),
              "k_new and v_new must live on the device of q");
  const c10::cuda::CUDAGuard guard(q.device());
  const int B = to_int(q.size(0), "batch");
  const int H = to_int(q.size(1), "heads");
  const int H_kv = to_int(k_cache.size(1), "kv heads");
  const int S = to_int(k_cache.size(2), "cache length");
  at::Tensor o = at::empty_like(q);
  const int D = to_int(q.size(3), "head_dim");
  const size_t bytes =
      fa_decode_gqa_hd_workspace_bytes(B, H, H_kv, S, D, q.get_device());
  TORCH_CHECK(bytes > 0, "fa_decode_gqa_workspace_bytes failed");
  DecodeScratch &ws = decode_scratch(q, bytes, static_cast<size_t>(B) * H);
  check_status(
      fa_decode_append_ex(q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(),
                       k_cache.data_ptr(), v_cache.data_ptr(),
                       seq_lens.data_ptr<int32_t>(), o.data_ptr(), B, H, H_kv,
                       S, D, dtype_code(q), static_cast<float>(scale),
                       ws.partials.data_ptr(),
                       static_cast<size_t>(ws.partials.numel()),
                       reinterpret_cast<uint32_t *>(ws.counters.data_ptr<int32_t>()),
                       static_cast<size_t>(ws.counters.numel()), current_stream()),
      "fa_decode_append");
  return o;
}

// ---- sequence-sharded decode with the cross-GPU combine in the kernel ----
size_t exchange_bytes(int64_t B, int64_t H, int64_t world,
                      int64_t head_dim) {
  const size_t n = fa_exchange_bytes_hd(to_int(B, "batch"), to_int(H, "heads"),
                                        to_int(world, "world"),
                                        to_int(head_dim, "head_dim"));
  TORCH_CHECK(n > 0, "invalid exchange shape");
  return n;
}

py::tuple exchange_alloc(size_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void *p = nullptr;
  char handle[64];
  check_status(fa_exchange_alloc(bytes, &p, handle), "fa_exchange_alloc");
  return py::make_tuple(reinterpret_cast<uintptr_t>(p),
                        py::bytes(handle, sizeof(handle)));
}

uintptr_t exchange_open(py::bytes handle, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  const std::string h = handle;
  TORCH_CHECK(h.size() == 64, "an exchange handle is 64 bytes");
  void *p = nullptr;
  check_status(fa_exchange_open(h.data(), &p), "fa_exchange_open");
  return reinterpret_cast<uintptr_t>(p);
}

void exchange_close(uintptr_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  check_status(fa_exchange_close(reinterpret_cast<void *>(ptr)),
               "fa_exchange_close");
}

void exchange_free(uintptr_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  check_status(fa_exchange_free(reinterpret_cast<void *>(ptr)),
               "fa_exchange_free");
}

at::Tensor decode_exchange(const at::Tensor &q, const at::Tensor &k_cache,
                           const at::Tensor &v_cache,
                           const at::Tensor &seq_lens, double scale,
                           const at::Tensor &peers, int64_t rank,
                           int64_t world, int64_t epoch) {
  check_decode_inputs(q, k_cache, v_cache, seq_lens, scale);
  TORCH_CHECK(k_cache.size(1) == q.size(1),
              "sharded decode needs one K/V head per query head");
  check_cuda(peers, "peers");
  TORCH_CHECK(peers.scalar_type() == at::kLong && peers.dim() == 1 &&
                  peers.size(0) == world && peers.device() == q.device(),
              "peers must be an int64 CUDA tensor of world buffer pointers");
  TORCH_CHECK(epoch > 0 && epoch <= UINT32_MAX, "epoch out of range");
  const c10::cuda::CUDAGuard guard(q.device());
  const int B = to_int(q.size(0), "batch");
  const int H = to_int(q.size(1), "heads");
  const int S = to_int(k_cache.size(2), "cache length");
  at::Tensor o = at::empty_like(q);
  const int D = to_int(q.size(3), "head_dim");
  const size_t bytes = fa_decode_hd_workspace_bytes(B, H, S, D, 0, q.get_device());
  TORCH_CHECK(bytes > 0, "fa_decode_workspace_bytes failed");
  DecodeScratch &ws = decode_scratch(q, bytes, static_cast<size_t>(B) * H);
  check_status(
      fa_decode_exchange_ex(
          q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
          seq_lens.data_ptr<int32_t>(), o.data_ptr(), B, H, S, D, dtype_code(q),
          static_cast<float>(scale), ws.partials.data_ptr(),
          static_cast<size_t>(ws.partials.numel()),
          reinterpret_cast<uint32_t *>(ws.counters.data_ptr<int32_t>()),
          static_cast<size_t>(ws.counters.numel()),
          reinterpret_cast<float *const *>(peers.data_ptr<int64_t>()),
          to_int(rank, "rank"), to_int(world, "world"),
          static_cast<uint32_t>(epoch), current_stream()),
      "fa_decode_exchange");
  return o;
}

// Merges (G, B, H, 68) partials into the fp16 (B, H, 1, 64) output.
at::Tensor merge_partials(const at::Tensor &partials) {
  check_cuda(partials, "partials");
  check_contiguous(partials, "partials");
  TORCH_CHECK(partials.scalar_type() == at::kFloat,
              "partials must be fp32 (got ", partials.scalar_type(), ")");
  TORCH_CHECK(partials.dim() == 4 && partials.size(3) == 68,
              "partials must be (G, B, H, 68), got ", partials.sizes());
  const c10::cuda::CUDAGuard guard(partials.device());
  const int G = to_int(partials.size(0), "G");
  const int B = to_int(partials.size(1), "batch");
  const int H = to_int(partials.size(2), "heads");
  at::Tensor o = at::empty({B, H, 1, kHeadDim},
                           partials.options().dtype(at::kHalf));
  check_status(fa_merge_partials(partials.data_ptr<float>(), G, o.data_ptr(),
                                 B, H, current_stream()),
               "fa_merge_partials");
  return o;
}

int64_t choose_decode_split(int64_t max_seq, int64_t batch, int64_t heads,
                            int64_t min_blocks) {
  return fa_choose_decode_split(static_cast<int>(max_seq),
                                static_cast<int>(batch),
                                static_cast<int>(heads),
                                static_cast<int>(min_blocks));
}

// CTA form of the head_dim-64 prefill for bh (batch x head) pairs of n
// tokens on a device of `sms` SMs (host-only, no GPU needed).
py::dict prefill_form(int64_t bh, int64_t n, bool causal, int64_t sms) {
  int ctas = 0;
  const int form = fa_prefill_form(bh, static_cast<int>(n), causal ? 1 : 0,
                                   static_cast<int>(sms), &ctas);
  TORCH_CHECK(form >= 0, "prefill_form: bh, n and sms must be positive");
  static const char *names[] = {"paired", "solo", "key-split"};
  py::dict d;
  d["form"] = std::string(names[form]);
  d["ctas"] = ctas;
  d["ctas_per_sm"] = form == FA_PREFILL_FORM_SOLO ? 2 : 1;
  return d;
}

// occupancy_report(): reference csrc/bindings.cpp:80-97, same row keys.
py::list occupancy_report() {
  fa_occupancy_entry rows[8];
  int n = 0;
  check_status(fa_occupancy(rows, 8, &n), "fa_occupancy");
  py::list out;
  for (int i = 0; i < n && i < 8; ++i) {
    py::dict row;
    row["kernel"] = std::string(rows[i].name);
    row["threads_per_block"] = rows[i].threads_per_block;
    row["registers_per_thread"] = rows[i].registers_per_thread;
    row["shared_bytes_per_block"] = rows[i].shared_bytes_per_block;
    row["max_active_blocks_per_sm"] = rows[i].max_active_blocks_per_sm;
    row["theoretical_occupancy"] = rows[i].theoretical_occupancy;
    out.append(row);
  }
  return out;
}

// legacy_naive / legacy_tiled / legacy_fused: the reference's v1 exports
// (csrc/legacy/legacy_ops.cu:19-51), same checks and messages; all three
// run the one fp32 kernel.
at::Tensor legacy_attention(const at::Tensor &q, const at::Tensor &k,
                            const at::Tensor &v) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(),
              "legacy kernels expect CUDA tensors");
  TORCH_CHECK(q.scalar_type() == at::kFloat && k.scalar_type() == at::kFloat &&
                  v.scalar_type() == at::kFloat,
              "legacy kernels are fp32 only");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(),
              "legacy kernels expect contiguous tensors");
  TORCH_CHECK(q.dim() == 2 && k.dim() == 2 && v.dim() == 2,
              "legacy kernels are single-head: expected (N, ", kHeadDim,
              ") tensors");
  TORCH_CHECK(q.sizes() == k.sizes() && q.sizes() == v.sizes(),
              "legacy kernels expect identical q/k/v shapes");
  TORCH_CHECK(q.size(1) == kHeadDim, "legacy kernels expect head_dim == ",
              kHeadDim);
  const c10::cuda::CUDAGuard guard(q.device());
  at::Tensor o = at::empty_like(q);
  check_status(fa_legacy_attention_f32(q.data_ptr<float>(), k.data_ptr<float>(),
                                       v.data_ptr<float>(), o.data_ptr<float>(),
                                       to_int(q.size(0), "N"), current_stream()),
               "fa_legacy_attention_f32");
  return o;
}

// Reads and clears the device-side error word (0: every kernel completed).
int64_t take_device_error() {
  unsigned int bits = 0;
  check_status(fa_take_device_error(&bits), "fa_take_device_error");
  return bits;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) FlashAttention forward for head_dim=64";
  m.attr("head_dim") = kHeadDim;
  m.def("prefill", &prefill,
        "Full-sequence attention (fp16 in/out, fp32 accum)", py::arg("q"),
        py::arg("k"), py::arg("v"), py::arg("causal"), py::arg("scale"));
  m.def("prefill_host", &prefill_host,
        "prefill() with host-memory q/k/v/out, copies overlapped with compute",
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("causal"),
        py::arg("scale"), py::arg("out") = py::none(),
        py::arg("non_blocking") = false);
  m.def("_prefill_host_launches", &prefill_host_launches);
  m.def("_prefill_form", &prefill_form, py::arg("bh"), py::arg("n"),
        py::arg("causal"), py::arg("sms"));
  m.def("decode", &decode, "Single-query attention against a KV cache",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("seq_lens"), py::arg("scale"));
  m.def("occupancy_report", &occupancy_report,
        "Theoretical occupancy of each kernel at its launch configuration");
  m.def("choose_decode_split", &choose_decode_split,
        "Chunk size rule of the reference's split-K decode",
        py::arg("max_seq"), py::arg("batch"), py::arg("heads"),
        py::arg("min_blocks"));
  m.def("_decode_with_split", &decode_impl, py::arg("q"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("seq_lens"), py::arg("scale"),
        py::arg("split_size"));
  m.def("decode_partial", &decode_partial,
        "Log-sum-exp partials of decode over this device's cache rows",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("seq_lens"), py::arg("scale"));
  m.def("decode_append", &decode_append,
        "Decode with the new token's K/V row stored into the cache in the same launch",
        py::arg("q"), py::arg("k_new"), py::arg("v_new"), py::arg("k_cache"),
        py::arg("v_cache"), py::arg("seq_lens"), py::arg("scale"));
  m.def("_exchange_bytes", &exchange_bytes, py::arg("B"), py::arg("H"),
        py::arg("world"), py::arg("head_dim") = 64);
  m.def("_exchange_alloc", &exchange_alloc);
  m.def("_exchange_open", &exchange_open);
  m.def("_exchange_close", &exchange_close);
  m.def("_exchange_free", &exchange_free);
  m.def("decode_exchange", &decode_exchange,
        "Sequence-sharded decode, cross-GPU combine inside the kernel",
        py::arg("q"), py::arg("k_cache"), py::arg("v_cache"),
        py::arg("seq_lens"), py::arg("scale"), py::arg("peers"),
        py::arg("rank"), py::arg("world"), py::arg("epoch"));
  m.def("merge_partials", &merge_partials,
        "Merge (G, B, H, 68) decode partials into the fp16 output",
        py::arg("partials"));
  m.def("legacy_naive", &legacy_attention, "v1 single-head kernel (N, 64) fp32");
  m.def("legacy_tiled", &legacy_attention, "v1 single-head kernel (N, 64) fp32");
  m.def("legacy_fused", &legacy_attention, "v1 single-head kernel (N, 64) fp32");
  m.def("take_device_error", &take_device_error,
        "Read and clear the device-side error word");
}
