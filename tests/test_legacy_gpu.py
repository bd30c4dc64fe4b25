"""The reference's v1 exports legacy_naive / legacy_tiled / legacy_fused:
single-head fp32 (N, 64) non-causal attention with scale 1/8 (reference
csrc/legacy/legacy_ops.cu:19-51), checked against fp32 SDPA."""

import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]


@pytest.mark.parametrize("n", [1, 37, 64, 65, 256, 1000, 2048])
@pytest.mark.parametrize("name", ["legacy_naive", "legacy_tiled", "legacy_fused"])
def test_legacy_matches_fp32_sdpa(n, name):
    torch.manual_seed(n)
    q, k, v = (torch.randn(n, 64, device="cuda") for _ in range(3))
    out = getattr(flashattn_cuda, name)(q, k, v)
    ref = torch.nn.functional.scaled_dot_product_attention(
        q[None], k[None], v[None], scale=0.125)[0]
    assert (out - ref).abs().max().item() <= 1e-4


def test_legacy_rejects_bad_inputs():
    q = torch.randn(8, 64, device="cuda")
    with pytest.raises(RuntimeError, match="fp32 only"):
        flashattn_cuda.legacy_naive(q.half(), q.half(), q.half())
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        flashattn_cuda.legacy_tiled(q.cpu(), q.cpu(), q.cpu())
    with pytest.raises(RuntimeError, match="single-head"):
        flashattn_cuda.legacy_fused(q[None], q[None], q[None])
    with pytest.raises(RuntimeError, match="head_dim"):
        b = torch.randn(8, 32, device="cuda")
        flashattn_cuda.legacy_fused(b, b, b)
    with pytest.raises(RuntimeError, match="identical"):
        flashattn_cuda.legacy_fused(q, q[:4].contiguous(), q)
    assert flashattn_cuda.take_device_error() == 0
