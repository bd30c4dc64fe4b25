"""Grouped-query attention (query heads sharing K/V heads) without
materialising repeated K/V: equal to the same call on K/V repeated per
group (the BASELINE Qwen2.5-0.5B shapes pre-expand 2 K/V heads to 14)."""

import math

import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]
SCALE = 1.0 / math.sqrt(64)


def expand(t, group):
    return t.repeat_interleave(group, dim=1).contiguous()


@pytest.mark.parametrize("h,h_kv", [(14, 2), (12, 4), (8, 1), (6, 6)])
@pytest.mark.parametrize("n,causal", [(1000, True), (512, False), (129, True)])
def test_prefill_gqa_equals_expanded(h, h_kv, n, causal):
    torch.manual_seed(h * 100 + n)
    q = torch.randn(2, h, n, 64, device="cuda").half()
    k, v = (torch.randn(2, h_kv, n, 64, device="cuda").half() for _ in range(2))
    got = flashattn_cuda.prefill(q, k, v, causal, SCALE)
    want = flashattn_cuda.prefill(q, expand(k, h // h_kv), expand(v, h // h_kv),
                                  causal, SCALE)
    assert torch.equal(got, want)


@pytest.mark.parametrize("h,h_kv", [(14, 2), (12, 3), (8, 1)])
def test_decode_gqa_equals_expanded(h, h_kv):
    torch.manual_seed(h)
    b, s = 5, 3000
    q = torch.randn(b, h, 1, 64, device="cuda").half()
    k, v = (torch.randn(b, h_kv, s, 64, device="cuda").half() for _ in range(2))
    lens = torch.tensor([3000, 1, 0, 1777, 64], dtype=torch.int32, device="cuda")
    got = flashattn_cuda.decode(q, k, v, lens, SCALE)
    want = flashattn_cuda.decode(q, expand(k, h // h_kv), expand(v, h // h_kv),
                                 lens, SCALE)
    assert (got.float() - want.float()).abs().max().item() <= 1e-3


def test_gqa_rejects_non_dividing_heads():
    q = torch.randn(1, 6, 16, 64, device="cuda").half()
    k = torch.randn(1, 4, 16, 64, device="cuda").half()
    with pytest.raises(RuntimeError, match="identical shapes"):
        flashattn_cuda.prefill(q, k, k, True, SCALE)
    with pytest.raises(RuntimeError, match="agree on batch and head count"):
        flashattn_cuda.decode(q[:, :, :1].contiguous(), k, k,
                              torch.tensor([4], dtype=torch.int32, device="cuda"), SCALE)
    assert flashattn_cuda.take_device_error() == 0
