"""prefill_host (fa_prefill_host): q/k/v in host memory streamed through the
device in chunks, copies overlapped with the kernels. Every output element
must be bit-identical to prefill() on the same inputs already on the
device: chunking only changes which launch computes a head, not how."""

import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]


def host_inputs(b, h, h_kv, n, d, seed, pinned=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, h, n, d, generator=g).half()
    k = torch.randn(b, h_kv, n, d, generator=g).half()
    v = torch.randn(b, h_kv, n, d, generator=g).half()
    if pinned:
        q, k, v = q.pin_memory(), k.pin_memory(), v.pin_memory()
    return q, k, v


# shapes: single chunk, ragged last chunk, several chunks (ring wraps),
# grouped K/V heads, head_dim 128, the config-3 shape
@pytest.mark.parametrize("b,h,h_kv,n,d", [
    (1, 1, 1, 1, 64), (1, 2, 2, 100, 64), (2, 5, 5, 1024, 64),
    (3, 7, 7, 2048, 64), (2, 14, 2, 1500, 64), (4, 14, 14, 4096, 64),
    (1, 5, 5, 1024, 128), (2, 8, 2, 777, 128)])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_host_equals_device_prefill(b, h, h_kv, n, d, causal):
    q, k, v = host_inputs(b, h, h_kv, n, d, seed=b * 100 + h * 10 + n + d)
    scale = d ** -0.5
    got = flashattn_cuda.prefill_host(q, k, v, causal, scale)
    assert got.device.type == "cpu" and got.is_pinned()
    assert got.shape == q.shape and got.dtype == torch.float16
    want = flashattn_cuda.prefill(q.cuda(), k.cuda(), v.cuda(), causal,
                                  scale).cpu()
    assert torch.equal(got, want)
    assert flashattn_cuda.take_device_error() == 0


def test_prefill_host_many_chunks():
    # 64 heads of 3 MiB input: chunks capped at 21 heads, the ring of 3
    # slots wraps several times
    q, k, v = host_inputs(2, 32, 32, 8192, 64, seed=3)
    got = flashattn_cuda.prefill_host(q, k, v, True, 0.125)
    want = flashattn_cuda.prefill(q.cuda(), k.cuda(), v.cuda(), True,
                                  0.125).cpu()
    assert torch.equal(got, want)


def test_prefill_host_pageable_inputs_and_out():
    q, k, v = host_inputs(2, 6, 3, 900, 64, seed=7, pinned=False)
    out = torch.full_like(q, float("nan"))
    got = flashattn_cuda.prefill_host(q, k, v, True, 0.125, out=out)
    assert got.data_ptr() == out.data_ptr()
    want = flashattn_cuda.prefill(q.cuda(), k.cuda(), v.cuda(), True,
                                  0.125).cpu()
    assert torch.equal(out, want)


def test_prefill_host_non_blocking_is_stream_ordered():
    q, k, v = host_inputs(2, 14, 14, 2048, 64, seed=11)
    out = flashattn_cuda.prefill_host(q, k, v, True, 0.125,
                                      non_blocking=True)
    torch.cuda.current_stream().synchronize()
    want = flashattn_cuda.prefill(q.cuda(), k.cuda(), v.cuda(), True,
                                  0.125).cpu()
    assert torch.equal(out, want)
    # back-to-back calls reuse the copy streams and events
    outs = [flashattn_cuda.prefill_host(q, k, v, True, 0.125,
                                        non_blocking=True) for _ in range(3)]
    torch.cuda.current_stream().synchronize()
    for o in outs:
        assert torch.equal(o, want)


def test_prefill_host_on_a_side_stream():
    q, k, v = host_inputs(1, 9, 9, 1024, 64, seed=5)
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        got = flashattn_cuda.prefill_host(q, k, v, False, 0.2)
    want = flashattn_cuda.prefill(q.cuda(), k.cuda(), v.cuda(), False,
                                  0.2).cpu()
    assert torch.equal(got, want)


def test_prefill_host_rejects_device_tensors():
    q = torch.zeros(1, 1, 8, 64, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="CPU tensors"):
        flashattn_cuda.prefill_host(q, q, q, True, 0.1)


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_host_bf16(d):
    g = torch.Generator().manual_seed(d)
    q = torch.randn(2, 8, 1500, d, generator=g).bfloat16().pin_memory()
    k = torch.randn(2, 2, 1500, d, generator=g).bfloat16().pin_memory()
    v = torch.randn(2, 2, 1500, d, generator=g).bfloat16().pin_memory()
    got = flashattn_cuda.prefill_host(q, k, v, True, d ** -0.5)
    assert got.dtype == torch.bfloat16 and got.is_pinned()
    want = flashattn_cuda.prefill(q.cuda(), k.cuda(), v.cuda(), True,
                                  d ** -0.5).cpu()
    assert torch.equal(got, want)
