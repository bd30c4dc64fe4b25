"""The prefill's CTA-form choice is a pure host function (no GPU): the
key-split form for causal grids whose longest query tile, not the total
work, sets the kernel time; solo or paired elsewhere. Cases are B200 shapes
(148 SMs) whose faster form was measured on the GPU."""

import ctypes
import os

import pytest
import torch  # noqa: F401  (loads libc10 for the extension)

from conftest import PKG_DIR

import flashattn_cuda

LIB = os.path.join(PKG_DIR, "flashattn_cuda", "libfa_b200.so")
SMS = 148


@pytest.mark.parametrize("bh,n,form", [
    (7, 4096, "key-split"),    # config 3 on 8 GPUs: 34.6 vs 44.6 us paired
    (10, 4096, "key-split"),   # 45.4 vs 46.6 us solo
    (12, 4096, "solo"),        # 48.1 vs 52.6 us key-split
    (56, 4096, "solo"),        # config 3 on one GPU
    (2, 16384, "key-split"),   # 99.3 vs 138.2 us paired
    (6, 8192, "key-split"),    # 79.8 vs 91.0 us paired
    (48, 8192, "paired"),      # 481.7 vs 549.4 us key-split
    (64, 512, "paired"),       # 15.9 vs 18.7 us key-split
    (40, 1024, "solo"),        # 20.2 vs 27.0 us key-split
    (96, 1024, "solo"),        # config 2
    (1, 100, "solo"),          # one query tile: nothing to split
])
def test_causal_form_follows_the_measured_winner(bh, n, form):
    got = flashattn_cuda._C._prefill_form(bh, n, True, SMS)
    assert got["form"] == form
    n_qt = -(-n // 128)
    assert got["ctas"] == (n_qt * bh if form != "paired"
                           else (n_qt + 1) // 2 * bh)
    assert got["ctas_per_sm"] == (2 if form == "solo" else 1)


@pytest.mark.parametrize("bh,n", [(7, 4096), (2, 16384), (1, 256)])
def test_full_attention_never_splits_keys(bh, n):
    assert flashattn_cuda._C._prefill_form(bh, n, False, SMS)["form"] != "key-split"


def test_c_abi_rejects_non_positive_arguments():
    lib = ctypes.CDLL(LIB)
    lib.fa_prefill_form.argtypes = [ctypes.c_longlong, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    assert lib.fa_prefill_form(0, 4096, 1, SMS, None) == -1
    assert lib.fa_prefill_form(7, 0, 1, SMS, None) == -1
    assert lib.fa_prefill_form(7, 4096, 1, 0, None) == -1
    ctas = ctypes.c_int(0)
    assert lib.fa_prefill_form(7, 4096, 1, SMS, ctypes.byref(ctas)) == 2
    assert ctas.value == 224
