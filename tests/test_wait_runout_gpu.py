"""A device-side wait that runs out ends in an error status, not a hang.

Every spin in the kernels (pipeline mbarriers, the cross-GPU arrival counters
of fa_decode_exchange) gives up after a time limit, records FA_ERR_TIMEOUT in
the device error word and unwinds. This test makes the exchange's counter
wait run out on one GPU without any fault: it calls fa_decode_exchange with
world = 2, where "rank 1's" buffer is a second local allocation that no
kernel ever merges from. Rank 0's counters then reach epoch x 1, never the
epoch x 2 the merge waits for. The limit is shortened to a few milliseconds
for the test and restored after; a normal decode afterwards must be correct.
"""

import ctypes
import math
import os
import time

import pytest
import torch

from conftest import PKG_DIR, requires_gpu

pytestmark = [pytest.mark.gpu, requires_gpu]

LIB = os.path.join(PKG_DIR, "flashattn_cuda", "libfa_b200.so")
FA_OK, FA_ERR_TIMEOUT = 0, 1
SCALE = 1.0 / math.sqrt(64)


def _lib():
    lib = ctypes.CDLL(LIB)
    vp, ci = ctypes.c_void_p, ctypes.c_int
    lib.fa_decode_exchange.argtypes = [vp, vp, vp, vp, vp, ci, ci, ci,
                                       ctypes.c_float, vp, ctypes.c_size_t,
                                       vp, ctypes.c_size_t, vp, ci, ci,
                                       ctypes.c_uint, vp]
    lib.fa_decode_workspace_bytes.argtypes = [ci] * 5
    lib.fa_decode_workspace_bytes.restype = ctypes.c_size_t
    lib.fa_exchange_bytes.argtypes = [ci] * 3
    lib.fa_exchange_bytes.restype = ctypes.c_size_t
    lib.fa_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
    lib.fa_take_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    return lib


def _take(lib):
    bits = ctypes.c_uint(0)
    assert lib.fa_take_device_error(ctypes.byref(bits)) == FA_OK
    return bits.value


def test_exchange_wait_runs_out_and_the_device_stays_usable():
    import flashattn_cuda

    lib = _lib()
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    torch.manual_seed(3)
    B, H, S = 2, 4, 3000
    q = torch.randn(B, H, 1, 64, device="cuda").half()
    k, v = (torch.randn(B, H, S, 64, device="cuda").half() for _ in range(2))
    lens = torch.tensor([S, 700], dtype=torch.int32, device="cuda")
    assert _take(lib) == 0

    xb = lib.fa_exchange_bytes(B, H, 2)
    own = torch.zeros(xb, dtype=torch.uint8, device="cuda")
    other = torch.zeros(xb, dtype=torch.uint8, device="cuda")
    peers = torch.tensor([own.data_ptr(), other.data_ptr()],
                         dtype=torch.int64, device="cuda")
    nbytes = lib.fa_decode_workspace_bytes(B, H, S, 0,
                                           torch.cuda.current_device())
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    counters = torch.zeros(B * H, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    assert lib.fa_set_wait_limit_ns(5_000_000) == FA_OK  # 5 ms
    try:
        t0 = time.perf_counter()
        assert lib.fa_decode_exchange(
            ptr(q), ptr(k), ptr(v), ptr(lens), ptr(out), B, H, S, SCALE,
            ptr(ws), nbytes, ptr(counters), B * H, ptr(peers), 0, 2, 1,
            stream) == FA_OK
        bits = _take(lib)  # synchronises: the launch has returned
        elapsed = time.perf_counter() - t0
    finally:
        assert lib.fa_set_wait_limit_ns(1_000_000_000) == FA_OK
    assert bits & FA_ERR_TIMEOUT, bits
    # One limit, not one per segment: later waits see the error and leave.
    assert elapsed < 0.5, elapsed
    # rank 0's counters (after both banks of partials) saw its own sends
    # only: 1 per segment, never the 2 the merge waits for
    n_part = 2 * 2 * B * H * 68 * 4
    own_ctr = own[n_part:n_part + 4 * B * H].view(torch.int32)
    assert torch.all(own_ctr == 1), own_ctr

    # the context is intact: a normal decode is correct afterwards
    got = flashattn_cuda.decode(q, k, v, lens, SCALE)
    torch.cuda.synchronize()
    assert _take(lib) == 0
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float(), v.float(), scale=SCALE,
        attn_mask=(torch.arange(S, device="cuda")[None, :] <
                   lens[:, None]).view(B, 1, 1, S))
    assert (got.float() - ref).abs().max().item() <= 2e-3
