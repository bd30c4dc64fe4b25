"""B200 (sm_100a) FlashAttention forward for head_dim = 64.

Drop-in for the reference package of the same name
(flashattn_cuda/__init__.py in shrvan30/flash-attention-cuda): the same
names with the same arguments, backed by hand-written sm_100a kernels in
libfa_b200.so. There is no CPU or eager fallback: importing fails loudly if
the compiled extension is missing.
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
