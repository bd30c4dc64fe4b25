"""fa_decode_noalloc: the decode entry point for callers that cannot allocate.

Some hosts cannot hand the library scratch memory (a serving engine whose GPU
memory pool is fixed at start-up, a plugin that only receives pointers to its
inputs and outputs). fa_decode_noalloc serves them from a fixed device array
inside the library. These tests call it through the C ABI and check it
against fa_decode, which gets its scratch from the caller, on two calls in a
row with different inputs (the shared array keeps the previous call's
contents, which must not leak into the next result).

The file name sorts last so a run that stops at the first failure has run
every other test first; it also passes on its own in a fresh process.
"""

import ctypes
import os

import pytest
import torch

from conftest import PKG_DIR, requires_gpu

LIB = os.path.join(PKG_DIR, "flashattn_cuda", "libfa_b200.so")
SCALE = 0.125
TOL = 2e-3
FA_OK, FA_ENOSPACE = 0, 4
MAX_BH = 8192  # FA_NOALLOC_MAX_BH in include/fa_b200.h


def _lib():
    lib = ctypes.CDLL(LIB)
    vp = ctypes.c_void_p
    lib.fa_decode_noalloc.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int,
                                      ctypes.c_float, vp]
    lib.fa_decode.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_float, ctypes.c_int, vp,
                              ctypes.c_size_t, vp, ctypes.c_size_t, vp]
    lib.fa_decode_workspace_bytes.argtypes = [ctypes.c_int] * 5
    lib.fa_decode_workspace_bytes.restype = ctypes.c_size_t
    lib.fa_take_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    return lib


def test_noalloc_rejects_oversized_batch_before_launch():
    """B * H beyond the fixed array is refused on the host (no GPU needed)."""
    lib = _lib()
    p = ctypes.c_void_p(4096)
    assert lib.fa_decode_noalloc(p, p, p, p, p, MAX_BH + 1, 1, 8, SCALE,
                                 None) == FA_ENOSPACE
    assert lib.fa_decode_noalloc(p, p, p, p, p, 1024, 9, 8, SCALE,
                                 None) == FA_ENOSPACE


@pytest.mark.gpu
@requires_gpu
def test_noalloc_matches_fa_decode_on_consecutive_calls():
    lib = _lib()
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    gen = torch.Generator(device="cuda").manual_seed(123)
    # Two calls in a row with different shapes, lengths and values; the
    # second has many sequences split across CTAs so it reads the partials
    # and arrival counters the first call left in the shared array.
    cases = [(3, 12, 4096, [4096, 17, 2900]),
             (16, 8, 2048, [1 + (i * 331) % 2048 for i in range(16)])]
    for B, H, S, lens in cases:
        q = torch.randn(B, H, 1, 64, generator=gen, device="cuda").half()
        k = torch.randn(B, H, S, 64, generator=gen, device="cuda").half()
        v = torch.randn(B, H, S, 64, generator=gen, device="cuda").half()
        t_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")

        # existing entry point, scratch provided by the caller
        nbytes = lib.fa_decode_workspace_bytes(B, H, S, 0, torch.cuda.current_device())
        ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
        counters = torch.zeros(B * H, dtype=torch.int32, device="cuda")
        want = torch.full_like(q, float("nan"))
        assert lib.fa_decode(ptr(q), ptr(k), ptr(v), ptr(t_lens), ptr(want), B,
                             H, S, SCALE, 0, ptr(ws), nbytes, ptr(counters),
                             B * H, stream) == FA_OK

        got = torch.full_like(q, float("nan"))
        assert lib.fa_decode_noalloc(ptr(q), ptr(k), ptr(v), ptr(t_lens),
                                     ptr(got), B, H, S, SCALE,
                                     stream) == FA_OK
        torch.cuda.synchronize()
        assert not torch.isnan(got).any()
        assert (got.float() - want.float()).abs().max().item() <= TOL

    bits = ctypes.c_uint(1)
    assert lib.fa_take_device_error(ctypes.byref(bits)) == FA_OK
    assert bits.value == 0


@pytest.mark.gpu
@requires_gpu
def test_noalloc_at_the_array_limit():
    """B * H exactly at the limit uses the array's last counter and partial
    slots; the result must still equal fa_decode's."""
    lib = _lib()
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    gen = torch.Generator(device="cuda").manual_seed(7)
    B, H, S = 512, 16, 96
    assert B * H == MAX_BH
    q = torch.randn(B, H, 1, 64, generator=gen, device="cuda").half()
    k = torch.randn(B, H, S, 64, generator=gen, device="cuda").half()
    v = torch.randn(B, H, S, 64, generator=gen, device="cuda").half()
    lens = torch.randint(0, S + 1, (B,), generator=gen, device="cuda",
                         dtype=torch.int32)
    nbytes = lib.fa_decode_workspace_bytes(B, H, S, 0,
                                           torch.cuda.current_device())
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    counters = torch.zeros(B * H, dtype=torch.int32, device="cuda")
    want = torch.full_like(q, float("nan"))
    assert lib.fa_decode(ptr(q), ptr(k), ptr(v), ptr(lens), ptr(want), B, H,
                         S, SCALE, 0, ptr(ws), nbytes, ptr(counters), B * H,
                         stream) == FA_OK
    for _ in range(2):
        got = torch.full_like(q, float("nan"))
        assert lib.fa_decode_noalloc(ptr(q), ptr(k), ptr(v), ptr(lens),
                                     ptr(got), B, H, S, SCALE,
                                     stream) == FA_OK
        torch.cuda.synchronize()
        assert not torch.isnan(got).any()
        assert (got.float() - want.float()).abs().max().item() <= TOL
    bits = ctypes.c_uint(1)
    assert lib.fa_take_device_error(ctypes.byref(bits)) == FA_OK
    assert bits.value == 0


@pytest.mark.gpu
@requires_gpu
def test_noalloc_rejects_bad_pointers_and_sizes():
    """Misaligned pointers and empty caches are refused with the same codes
    fa_decode gives; the checks run before the shared counters are cleared."""
    lib = _lib()
    q = torch.zeros(2, 2, 1, 64, device="cuda").half()
    kv = torch.zeros(2, 2, 8, 64, device="cuda").half()
    lens = torch.full((2,), 8, dtype=torch.int32, device="cuda")
    bad = ctypes.c_void_p(q.data_ptr() + 2)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    assert lib.fa_decode_noalloc(bad, p(kv), p(kv), p(lens), p(q), 2, 2, 8,
                                 SCALE, None) == 2  # FA_EALIGN
    assert lib.fa_decode_noalloc(p(q), p(kv), p(kv), p(lens), p(q), 2, 2, 0,
                                 SCALE, None) == 1  # FA_EINVAL (S_max 0)
