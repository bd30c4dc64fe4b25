"""Prefill at head_dim 128 (the reference's named next size): against fp32
attention at the north star's 2e-3 tolerance, causal and full, ragged
lengths, grouped K/V heads, unusual scales."""

import math

import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]


def reference(q, k, v, causal, scale):
    group = q.shape[1] // k.shape[1]
    kf = k.float().repeat_interleave(group, dim=1)
    vf = v.float().repeat_interleave(group, dim=1)
    return torch.nn.functional.scaled_dot_product_attention(
        q.float(), kf, vf, is_causal=causal, scale=scale)


@pytest.mark.parametrize("b,h,n", [(2, 3, 1000), (1, 4, 4096), (2, 2, 513),
                                   (1, 1, 1), (3, 2, 129), (1, 2, 64),
                                   (1, 1, 65), (2, 5, 256)])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_d128_matches_fp32(b, h, n, causal):
    torch.manual_seed(b * 1000 + h * 10 + n)
    q, k, v = (torch.randn(b, h, n, 128, device="cuda").half() for _ in range(3))
    scale = 1.0 / math.sqrt(128)
    got = flashattn_cuda.prefill(q, k, v, causal, scale)
    assert got.shape == q.shape and got.dtype == torch.float16
    want = reference(q, k, v, causal, scale)
    assert (got.float() - want).abs().max().item() <= 2e-3
    assert flashattn_cuda.take_device_error() == 0


def test_prefill_d128_grouped_heads():
    torch.manual_seed(11)
    q = torch.randn(2, 8, 777, 128, device="cuda").half()
    k, v = (torch.randn(2, 2, 777, 128, device="cuda").half() for _ in range(2))
    got = flashattn_cuda.prefill(q, k, v, True, 0.0883883)
    want = reference(q, k, v, True, 0.0883883)
    assert (got.float() - want).abs().max().item() <= 2e-3


@pytest.mark.parametrize("scale,tol", [(0.0, 2e-3), (-0.09, 2e-3), (0.5, 4e-3)])
def test_prefill_d128_scales(scale, tol):
    """The 2e-3 bound is stated for scale = 1/sqrt(d); at 0.5 the logits are
    5.7x wider, the softmax is peakier and the fp16 rounding of P and of the
    output weighs more, so that case gets twice the bound."""
    torch.manual_seed(12)
    q, k, v = (torch.randn(1, 3, 300, 128, device="cuda").half() for _ in range(3))
    for causal in (True, False):
        got = flashattn_cuda.prefill(q, k, v, causal, scale)
        want = reference(q, k, v, causal, scale)
        assert (got.float() - want).abs().max().item() <= tol, (scale, causal)


def test_prefill_d128_single_key_rows_are_exact():
    """Causal row 0 attends one key: its output is that value row."""
    torch.manual_seed(13)
    q, k, v = (torch.randn(2, 2, 200, 128, device="cuda").half() for _ in range(3))
    got = flashattn_cuda.prefill(q, k, v, True, 0.088)
    assert torch.equal(got[:, :, 0], v[:, :, 0])


def decode_reference(q, k, v, lens, scale):
    b, h = q.shape[:2]
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    for i in range(b):
        n = max(0, min(int(lens[i]), k.shape[2]))
        if n == 0:
            continue
        s = (q[i].float() @ k[i, :, :n].float().transpose(1, 2)) * scale
        out[i] = torch.softmax(s, dim=-1) @ v[i, :, :n].float()
    return out


@pytest.mark.parametrize("b,h,s,lens", [
    (5, 8, 3000, [3000, 1, 0, 1777, 64]),
    (1, 14, 65536, [65533]),
    (64, 4, 700, None),
])
def test_decode_d128_matches_fp32(b, h, s, lens):
    torch.manual_seed(b + h)
    q = torch.randn(b, h, 1, 128, device="cuda").half()
    k, v = (torch.randn(b, h, s, 128, device="cuda").half() for _ in range(2))
    if lens is None:
        g = torch.Generator().manual_seed(2)
        lens = torch.randint(0, s + 20, (b,), generator=g, dtype=torch.int32)
    lens = torch.as_tensor(lens, dtype=torch.int32).cuda()
    scale = 128 ** -0.5
    for _ in range(2):  # counters are clean for the next call
        got = flashattn_cuda.decode(q, k, v, lens, scale)
        want = decode_reference(q, k, v, lens, scale)
        assert (got.float() - want).abs().max().item() <= 2e-3
    empty = (lens <= 0).nonzero().flatten()
    assert torch.all(got[empty] == 0)
    assert flashattn_cuda.take_device_error() == 0


def test_decode_d128_equals_prefill_row():
    """decode of token t == causal prefill row t, at head_dim 128."""
    torch.manual_seed(21)
    b, h, n = 2, 3, 900
    q, k, v = (torch.randn(b, h, n, 128, device="cuda").half() for _ in range(3))
    scale = 128 ** -0.5
    pre = flashattn_cuda.prefill(q, k, v, True, scale)
    for t in (0, 1, 127, 128, 899):
        lens = torch.full((b,), t + 1, dtype=torch.int32, device="cuda")
        dec = flashattn_cuda.decode(q[:, :, t:t + 1].contiguous(), k, v, lens, scale)
        assert (dec.float() - pre[:, :, t:t + 1].float()).abs().max().item() <= 2e-3


@pytest.mark.parametrize("split", [128, 256, 1024])
def test_decode_d128_split_invariance(split):
    torch.manual_seed(22)
    q = torch.randn(2, 4, 1, 128, device="cuda").half()
    k, v = (torch.randn(2, 4, 5000, 128, device="cuda").half() for _ in range(2))
    lens = torch.tensor([5000, 2501], dtype=torch.int32, device="cuda")
    auto = flashattn_cuda.decode(q, k, v, lens, 0.088)
    forced = flashattn_cuda._decode_with_split(q, k, v, lens, 0.088, split)
    assert (auto.float() - forced.float()).abs().max().item() <= 1e-3


@pytest.mark.parametrize("h,h_kv", [(32, 8), (14, 2), (40, 2), (8, 1)])
def test_decode_d128_grouped_matches_fp32(h, h_kv):
    """Grouped decode at head_dim 128 (e.g. 32 query heads on 8 K/V heads):
    every K/V row read once per group, groups above 16 in two passes."""
    torch.manual_seed(h + h_kv)
    b, s = 5, 2500
    q = torch.randn(b, h, 1, 128, device="cuda").half()
    k, v = (torch.randn(b, h_kv, s, 128, device="cuda").half() for _ in range(2))
    lens = torch.tensor([2500, 1, 0, 1311, 9999], dtype=torch.int32, device="cuda")
    scale = 128 ** -0.5
    for _ in range(2):
        got = flashattn_cuda.decode(q, k, v, lens, scale)
        kk = k.repeat_interleave(h // h_kv, dim=1)
        vv = v.repeat_interleave(h // h_kv, dim=1)
        want = decode_reference(q, kk, vv, lens, scale)
        assert (got.float() - want).abs().max().item() <= 2e-3
    assert torch.all(got[2] == 0)
    assert flashattn_cuda.take_device_error() == 0


def test_decode_d128_grouped_long_sequence():
    torch.manual_seed(23)
    q = torch.randn(1, 32, 1, 128, device="cuda").half()
    k, v = (torch.randn(1, 8, 50000, 128, device="cuda").half() for _ in range(2))
    lens = torch.tensor([49999], dtype=torch.int32, device="cuda")
    got = flashattn_cuda.decode(q, k, v, lens, 0.088)
    want = decode_reference(q, k.repeat_interleave(4, 1), v.repeat_interleave(4, 1),
                            lens, 0.088)
    assert (got.float() - want).abs().max().item() <= 2e-3


def test_decode_d128_limits():
    q = torch.randn(1, 4, 1, 128, device="cuda").half()
    k = torch.randn(1, 2, 16, 128, device="cuda").half()
    lens = torch.tensor([4], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim"):
        flashattn_cuda.decode(q[..., :64].contiguous(), k, k, lens, 0.1)
