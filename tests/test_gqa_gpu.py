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


def decode_reference(q, k, v, lens, scale):
    """fp32 decode with grouped heads: query head h reads K/V head h // group."""
    b, h = q.shape[:2]
    group = h // k.shape[1]
    out = torch.zeros(b, h, 1, 64, dtype=torch.float32, device=q.device)
    for i in range(b):
        n = max(0, min(int(lens[i]), k.shape[2]))
        if n == 0:
            continue
        kk = k[i, :, :n].float().repeat_interleave(group, dim=0)
        vv = v[i, :, :n].float().repeat_interleave(group, dim=0)
        s = (q[i].float() @ kk.transpose(1, 2)) * scale
        out[i] = torch.softmax(s, dim=-1) @ vv
    return out


@pytest.mark.parametrize("h,h_kv", [(14, 2), (12, 3), (8, 1), (16, 1), (32, 1),
                                    (40, 2), (4, 2)])
def test_decode_gqa_matches_fp32(h, h_kv):
    """Grouped decode (K/V read once per group, up to 16 query heads per pass,
    more passes above that) against an fp32 evaluation, ragged lengths
    including empty, single-row and clamped sequences."""
    torch.manual_seed(h * 7 + h_kv)
    b, s = 6, 2500
    q = torch.randn(b, h, 1, 64, device="cuda").half()
    k, v = (torch.randn(b, h_kv, s, 64, device="cuda").half() for _ in range(2))
    lens = torch.tensor([2500, 1, 0, 1311, 130, 9999], dtype=torch.int32,
                        device="cuda")
    got = flashattn_cuda.decode(q, k, v, lens, SCALE)
    want = decode_reference(q, k, v, lens, SCALE)
    assert (got.float() - want).abs().max().item() <= 2e-3
    assert torch.all(got[2] == 0)
    assert flashattn_cuda.take_device_error() == 0


def test_decode_gqa_long_sequence_split_across_ctas():
    """One long sequence per K/V head: its rows are spread over every CTA and
    the per-CTA partials are merged by the last one to finish."""
    torch.manual_seed(5)
    h, h_kv, s = 14, 2, 65536
    q = torch.randn(1, h, 1, 64, device="cuda").half()
    k, v = (torch.randn(1, h_kv, s, 64, device="cuda").half() for _ in range(2))
    lens = torch.tensor([s - 3], dtype=torch.int32, device="cuda")
    for _ in range(2):  # the arrival counters are clean for the next call
        got = flashattn_cuda.decode(q, k, v, lens, SCALE)
        want = decode_reference(q, k, v, lens, SCALE)
        assert (got.float() - want).abs().max().item() <= 2e-3
    assert flashattn_cuda.take_device_error() == 0


def test_decode_gqa_scale_sign_and_extremes():
    torch.manual_seed(9)
    h, h_kv, s = 8, 2, 700
    q = (torch.randn(3, h, 1, 64, device="cuda") * 4).half()
    k, v = (torch.randn(3, h_kv, s, 64, device="cuda").half() for _ in range(2))
    lens = torch.tensor([700, 300, 5], dtype=torch.int32, device="cuda")
    for scale in (SCALE, -SCALE, 0.0, 1.0):
        got = flashattn_cuda.decode(q, k, v, lens, scale)
        want = decode_reference(q, k, v, lens, scale)
        assert (got.float() - want).abs().max().item() <= 2e-3, scale
