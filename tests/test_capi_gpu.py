"""The C ABI called directly through ctypes with device pointers (no torch
operator layer in between), on a B200."""

import ctypes
import math
import os

import numpy as np
import pytest
import torch

from conftest import PKG_DIR, requires_gpu

import oracle

pytestmark = [pytest.mark.gpu, requires_gpu]

LIB = os.path.join(PKG_DIR, "flashattn_cuda", "libfa_b200.so")
SCALE = 0.125


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(LIB)
    vp = ctypes.c_void_p
    lib.fa_prefill.argtypes = [vp, vp, vp, vp, ctypes.c_int, ctypes.c_int,
                               ctypes.c_int, ctypes.c_int, ctypes.c_float, vp]
    lib.fa_decode.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_float, ctypes.c_int, vp,
                              ctypes.c_size_t, vp, ctypes.c_size_t, vp]
    lib.fa_decode_workspace_bytes.argtypes = [ctypes.c_int] * 5
    lib.fa_decode_workspace_bytes.restype = ctypes.c_size_t
    lib.fa_take_device_error.argtypes = [ctypes.POINTER(ctypes.c_uint)]
    return lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_capi_prefill_matches_oracle(lib):
    torch.manual_seed(0)
    for causal in (0, 1):
        q, k, v = (torch.randn(2, 3, 300, 64, device="cuda").half() for _ in range(3))
        o = torch.full_like(q, float("nan"))
        rc = lib.fa_prefill(_ptr(q), _ptr(k), _ptr(v), _ptr(o), 2, 3, 300,
                            causal, SCALE, _stream())
        assert rc == 0
        torch.cuda.synchronize()
        ref = oracle.prefill_c(q.float().cpu().numpy(), k.float().cpu().numpy(),
                               v.float().cpu().numpy(), bool(causal), SCALE)
        assert np.abs(o.float().cpu().numpy() - ref).max() <= 2e-3
    bits = ctypes.c_uint(123)
    assert lib.fa_take_device_error(ctypes.byref(bits)) == 0
    assert bits.value == 0


def test_capi_decode_workspace_reuse(lib):
    """One zero-initialised counter array and one workspace serve consecutive
    calls of different shapes: the kernel leaves its counters at zero."""
    torch.manual_seed(1)
    nbytes = lib.fa_decode_workspace_bytes(64, 16, 5000, 4, 0)
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    ctr = torch.zeros(64 * 16, dtype=torch.int32, device="cuda")
    cases = [(3, 4, 5000, [5000, 1, 2500], 0), (3, 4, 5000, [17, 4999, 0], 8),
             (2, 16, 900, [900, 450], 0), (3, 4, 5000, [5000] * 3, 0),
             (5, 2, 700, [1, 2, 3, 699, 700], 4)]
    for B, H, S, lens, split in cases:
        q = torch.randn(B, H, 1, 64, device="cuda").half()
        k = torch.randn(B, H, S, 64, device="cuda").half()
        v = torch.randn(B, H, S, 64, device="cuda").half()
        need = lib.fa_decode_workspace_bytes(B, H, S, split, 0)
        assert 0 < need <= nbytes
        t = torch.tensor(lens, dtype=torch.int32, device="cuda")
        o = torch.full_like(q, float("nan"))
        # too small a workspace or counter array is refused
        assert lib.fa_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(t), _ptr(o), B, H,
                             S, SCALE, split, _ptr(ws), need - 1, _ptr(ctr),
                             B * H, _stream()) == 4
        assert lib.fa_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(t), _ptr(o), B, H,
                             S, SCALE, split, _ptr(ws), need, _ptr(ctr),
                             B * H - 1, _stream()) == 4
        rc = lib.fa_decode(_ptr(q), _ptr(k), _ptr(v), _ptr(t), _ptr(o), B, H, S,
                           SCALE, split, _ptr(ws), need, _ptr(ctr), ctr.numel(),
                           _stream())
        assert rc == 0
        torch.cuda.synchronize()
        ref = oracle.decode_c(q.float().cpu().numpy(), k.float().cpu().numpy(),
                              v.float().cpu().numpy(), np.array(lens), SCALE)
        assert np.abs(o.float().cpu().numpy() - ref).max() <= 2e-3
        assert int(ctr.abs().sum()) == 0
