"""Decode with the KV-cache append fused in (decode_append): the new token's
K/V rows land at row seq_lens[b] of the caches and are attended in the same
launch. Equal to writing the rows first and calling decode() with
seq_lens + 1, for per-head and grouped caches, at the cache edges."""

import math

import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]
SCALE = 1.0 / math.sqrt(64)


def append_reference(q, k_new, v_new, k, v, lens, scale=SCALE):
    """Cache update and fp32 attention done separately."""
    k, v = k.clone(), v.clone()
    s_max = k.shape[2]
    new_lens = []
    for b, n in enumerate(lens.tolist()):
        p = max(n, 0)
        if p < s_max:
            k[b, :, p] = k_new[b, :, 0]
            v[b, :, p] = v_new[b, :, 0]
        new_lens.append(min(p + 1, s_max))
    group = q.shape[1] // k.shape[1]
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    for b, n in enumerate(new_lens):
        kk = k[b, :, :n].float().repeat_interleave(group, dim=0)
        vv = v[b, :, :n].float().repeat_interleave(group, dim=0)
        out[b] = torch.softmax(q[b].float() @ kk.transpose(1, 2) * scale, -1) @ vv
    return out, k, v, torch.tensor(new_lens, dtype=torch.int32, device=q.device)


@pytest.mark.parametrize("h,h_kv", [(12, 12), (14, 2), (40, 2), (8, 1)])
def test_decode_append_matches_separate_steps(h, h_kv):
    torch.manual_seed(h + h_kv)
    b, s = 7, 1500
    q = torch.randn(b, h, 1, 64, device="cuda").half()
    k = torch.randn(b, h_kv, s, 64, device="cuda").half()
    v = torch.randn(b, h_kv, s, 64, device="cuda").half()
    k_new = torch.randn(b, h_kv, 1, 64, device="cuda").half()
    v_new = torch.randn(b, h_kv, 1, 64, device="cuda").half()
    # empty, negative, middle, last free row, full cache, past capacity
    lens = torch.tensor([0, -3, 700, s - 1, s, s + 9, 128], dtype=torch.int32,
                        device="cuda")
    want, k_want, v_want, lens_after = append_reference(q, k_new, v_new, k, v, lens)
    k_c, v_c = k.clone(), v.clone()
    got = flashattn_cuda.decode_append(q, k_new, v_new, k_c, v_c, lens, SCALE)
    assert torch.equal(k_c, k_want) and torch.equal(v_c, v_want)
    assert (got.float() - want).abs().max().item() <= 2e-3
    # identical to decode() over the updated cache with the advanced lengths
    again = flashattn_cuda.decode(q, k_c, v_c, lens_after, SCALE)
    assert torch.equal(got, again)
    assert torch.equal(lens.cpu(), torch.tensor([0, -3, 700, s - 1, s, s + 9, 128],
                                                dtype=torch.int32))
    assert flashattn_cuda.take_device_error() == 0


@pytest.mark.parametrize("h,h_kv", [(14, 14), (14, 2)])
def test_generation_loop(h, h_kv):
    """Token-by-token decoding from an empty cache: each step appends and
    attends; the cache ends up holding every generated row."""
    torch.manual_seed(3)
    b, s, steps = 3, 300, 40
    k_c = torch.zeros(b, h_kv, s, 64, device="cuda").half()
    v_c = torch.zeros_like(k_c)
    k_all = torch.randn(b, h_kv, steps, 64, device="cuda").half()
    v_all = torch.randn(b, h_kv, steps, 64, device="cuda").half()
    lens = torch.tensor([0, 5, 17], dtype=torch.int32, device="cuda")
    start = lens.clone()
    for t in range(steps):
        q = torch.randn(b, h, 1, 64, device="cuda").half()
        k_new = k_all[:, :, t:t + 1].contiguous()
        v_new = v_all[:, :, t:t + 1].contiguous()
        want, _, _, _ = append_reference(q, k_new, v_new, k_c, v_c, lens)
        got = flashattn_cuda.decode_append(q, k_new, v_new, k_c, v_c, lens, SCALE)
        assert (got.float() - want).abs().max().item() <= 2e-3, t
        lens = lens + 1
    for i in range(b):
        p0 = int(start[i])
        assert torch.equal(k_c[i, :, p0:p0 + steps], k_all[i])
        assert torch.equal(v_c[i, :, p0:p0 + steps], v_all[i])
    assert flashattn_cuda.take_device_error() == 0


def test_decode_append_rejects_bad_shapes():
    q = torch.randn(2, 4, 1, 64, device="cuda").half()
    k = torch.randn(2, 2, 32, 64, device="cuda").half()
    lens = torch.tensor([3, 4], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="k_new and v_new"):
        flashattn_cuda.decode_append(q, k[:, :, :2].contiguous(), k[:, :, :2].contiguous(),
                                     k, k.clone(), lens, SCALE)


@pytest.mark.parametrize("h,h_kv", [(8, 8), (32, 8), (20, 1)])
def test_decode_append_head_dim_128(h, h_kv):
    torch.manual_seed(31 + h)
    b, s = 5, 900
    scale = 128 ** -0.5
    q = torch.randn(b, h, 1, 128, device="cuda").half()
    k = torch.randn(b, h_kv, s, 128, device="cuda").half()
    v = torch.randn(b, h_kv, s, 128, device="cuda").half()
    k_new = torch.randn(b, h_kv, 1, 128, device="cuda").half()
    v_new = torch.randn(b, h_kv, 1, 128, device="cuda").half()
    lens = torch.tensor([0, 899, 900, 77, 450], dtype=torch.int32, device="cuda")
    want, k_want, v_want, lens_after = append_reference(q, k_new, v_new, k, v,
                                                        lens, scale)
    k_c, v_c = k.clone(), v.clone()
    got = flashattn_cuda.decode_append(q, k_new, v_new, k_c, v_c, lens, scale)
    assert torch.equal(k_c, k_want) and torch.equal(v_c, v_want)
    assert (got.float() - want).abs().max().item() <= 2e-3
    assert torch.equal(got, flashattn_cuda.decode(q, k_c, v_c, lens_after, scale))
    assert flashattn_cuda.take_device_error() == 0
