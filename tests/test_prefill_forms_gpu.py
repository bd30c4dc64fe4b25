"""Prefill in all three CTA forms against fp32 attention. The key-split
form (one query tile per CTA, its key tiles alternating between two
softmax warpgroups whose partial rows merge at the end) runs causal grids
of about two query tiles per SM or fewer; the solo form (one query tile
per CTA, two CTAs per SM) runs every other sequence of up to 48 query tiles
whose paired grid exceeds one wave of SMs; the paired form (two tiles of
one head per CTA) runs the rest: one-wave grids (zig-zag pairs) and long
sequences. flashattn_cuda._C._prefill_form reports the choice. Edges:
short and ragged N, odd (batch, head) counts, grouped K/V heads, both
dtypes, causal and full, and the sequence lengths on either side of each
switch."""

import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]


def reference(q, k, v, causal, scale):
    group = q.shape[1] // k.shape[1]
    return torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float().repeat_interleave(group, 1),
        v.float().repeat_interleave(group, 1), is_causal=causal, scale=scale)


@pytest.mark.parametrize("dtype,tol", [(torch.float16, 2e-3),
                                       (torch.bfloat16, 1.5e-2)])
@pytest.mark.parametrize("b,h,h_kv", [(1, 1, 1), (3, 5, 5), (2, 7, 1),
                                      (4, 6, 3), (64, 32, 32), (5, 31, 31),
                                      (3, 50, 10)])
@pytest.mark.parametrize("n", [1, 64, 100, 128, 300, 384, 640, 896])
@pytest.mark.parametrize("causal", [True, False])
def test_short_prefill_matches_fp32(dtype, tol, b, h, h_kv, n, causal):
    torch.manual_seed(b * 100 + h * 10 + n)
    q = torch.randn(b, h, n, 64, device="cuda").to(dtype)
    k = torch.randn(b, h_kv, n, 64, device="cuda").to(dtype)
    v = torch.randn(b, h_kv, n, 64, device="cuda").to(dtype)
    got = flashattn_cuda.prefill(q, k, v, causal, 0.125)
    err = (got.float() - reference(q, k, v, causal, 0.125)).abs().max().item()
    assert err <= tol, err
    assert flashattn_cuda.take_device_error() == 0


@pytest.mark.parametrize("dtype,tol", [(torch.float16, 2e-3),
                                       (torch.bfloat16, 1.5e-2)])
@pytest.mark.parametrize("b,h,h_kv", [(1, 1, 1), (3, 5, 5), (64, 32, 32),
                                      (5, 31, 31), (3, 50, 10)])
@pytest.mark.parametrize("n", [1, 64, 65, 100, 128, 300, 384, 640])
@pytest.mark.parametrize("causal", [True, False])
def test_short_prefill_d128_matches_fp32(dtype, tol, b, h, h_kv, n, causal):
    """head_dim 128 with an odd number of query tiles (1, 3 or 5). With one
    tile above one wave of SMs the kernel takes query tile 0 of two heads
    per CTA (one or two 64-key K/V tiles per head); longer sequences keep
    one head per CTA, whose last CTA holds a lone tile."""
    torch.manual_seed(b * 100 + h * 10 + n + 1)
    q = torch.randn(b, h, n, 128, device="cuda").to(dtype)
    k = torch.randn(b, h_kv, n, 128, device="cuda").to(dtype)
    v = torch.randn(b, h_kv, n, 128, device="cuda").to(dtype)
    scale = 128 ** -0.5
    got = flashattn_cuda.prefill(q, k, v, causal, scale)
    err = (got.float() - reference(q, k, v, causal, scale)).abs().max().item()
    assert err <= tol, err
    assert flashattn_cuda.take_device_error() == 0


@pytest.mark.parametrize("b,h,n", [
    (1, 7, 4096),    # causal: 224 tiles, key-split; full: zig-zag pairs
    (1, 1, 129),     # causal key-split: warpgroup 1 holds only the diagonal
    (1, 3, 257),     # three key tiles: two on warpgroup 0, one on 1
    (1, 10, 4096),   # causal: 320 tiles, still key-split; full: solo
    (1, 14, 4096),   # causal: 448 tiles, solo
    (1, 64, 512),    # causal: zig-zag pairs (a key split does not pay)
    (2, 7, 4096),    # 224 pairs: solo
    (1, 2, 6144),    # causal key-split; full: 48 pairs in one wave, paired
    (2, 4, 6144),    # 48 tiles, 192 pairs: solo
    (2, 4, 6145),    # 49 tiles: causal key-split, full paired
    (1, 4, 16384),   # long: causal key-split, full paired
])
@pytest.mark.parametrize("causal", [True, False])
def test_form_switch_lengths_match_fp32(b, h, n, causal):
    torch.manual_seed(n + h)
    q = torch.randn(b, h, n, 64, device="cuda").half()
    k = torch.randn(b, h, n, 64, device="cuda").half()
    v = torch.randn(b, h, n, 64, device="cuda").half()
    got = flashattn_cuda.prefill(q, k, v, causal, 0.125)
    err = (got.float() - reference(q, k, v, causal, 0.125)).abs().max().item()
    assert err <= 2e-3, err


@pytest.mark.parametrize("b,h,h_kv,n,d,causal,dtype", [
    (4, 14, 14, 4096, 64, True, torch.float16),    # 56 MB of K/V: 2 blocks of 28
    (3, 13, 13, 4096, 64, False, torch.float16),   # 39 heads: uneven blocks
    (2, 24, 6, 8192, 64, True, torch.float16),     # grouped K/V heads in blocks
    (4, 14, 14, 4096, 64, True, torch.bfloat16),
    (4, 7, 7, 4096, 128, True, torch.float16),     # d128: 2 MB per head
    (3, 11, 11, 4096, 128, False, torch.bfloat16),
])
def test_head_block_launch_order_matches_fp32(b, h, h_kv, n, d, causal, dtype):
    """Grids whose K/V exceed the L2 budget launch in blocks of heads; every
    (head, query tile) must still be computed once, for every block size."""
    torch.manual_seed(b * h + n + d)
    q = torch.randn(b, h, n, d, device="cuda").to(dtype)
    k = torch.randn(b, h_kv, n, d, device="cuda").to(dtype)
    v = torch.randn(b, h_kv, n, d, device="cuda").to(dtype)
    scale = d ** -0.5
    got = flashattn_cuda.prefill(q, k, v, causal, scale)
    tol = 2e-3 if dtype == torch.float16 else 1.5e-2
    for bi in range(b):  # per batch entry keeps the fp32 reference small
        ref = reference(q[bi:bi + 1], k[bi:bi + 1], v[bi:bi + 1], causal, scale)
        err = (got[bi:bi + 1].float() - ref).abs().max().item()
        assert err <= tol, (bi, err)
