"""B200 (sm_100a) FlashAttention forward.

Drop-in for the reference package of the same name
(flashattn_cuda/__init__.py in shrvan30/flash-attention-cuda): the same
names with the same arguments for its head_dim-64 fp16 prefill and decode,
backed by hand-written sm_100a kernels in libfa_b200.so. The same calls also
take head_dim 128, bf16 tensors and K/V with fewer heads than Q; added are
decode_append (cache append fused into decode), prefill_host (inputs in host
memory, copies overlapped with the kernels), decode_partial / merge_partials
and flashattn_cuda.dist (multi-GPU sharding and the in-kernel NVLink decode
exchange). There is no CPU or eager fallback: importing fails loudly if the
compiled extension is missing.
"""

# The compiled extension links against libc10/libtorch, which are only on the
# loader's path once torch itself has been imported.
import torch as _torch  # noqa: F401

from ._C import (  # noqa: F401
    _decode_with_split,
    choose_decode_split,
    decode,
    decode_append,
    decode_partial,
    head_dim,
    legacy_fused,
    legacy_naive,
    legacy_tiled,
    merge_partials,
    occupancy_report,
    prefill,
    prefill_host,
    take_device_error,
)

__all__ = [
    "prefill",
    "prefill_host",
    "decode",
    "head_dim",
    "occupancy_report",
    "choose_decode_split",
    "legacy_naive",
    "legacy_tiled",
    "legacy_fused",
    "decode_append",
    "decode_partial",
    "merge_partials",
    "take_device_error",
]

__version__ = "2.0.0+b200"
