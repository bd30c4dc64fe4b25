"""Our kernels against the reference's own CUDA kernels on the same inputs
(B200, -m gpu). The reference extension is built from its unmodified sources
by oracle/build_ref.py; the test is skipped where that library is absent."""

import math
import os

import pytest
import torch

from conftest import ORACLE_DIR, requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]
SCALE = 1.0 / math.sqrt(64)
TOL = 2e-3


@pytest.fixture(scope="module")
def ref():
    import build_ref
    if not os.path.exists(build_ref.out_path()):
        pytest.skip("reference kernels not built (oracle/build_ref.py)")
    return build_ref.load()


@pytest.mark.parametrize("b,h,n", [(2, 12, 256), (8, 12, 1024), (1, 14, 4096), (2, 5, 1023)])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_matches_reference_kernel(ref, b, h, n, causal):
    torch.manual_seed(b * 1000 + n)
    q, k, v = (torch.randn(b, h, n, 64, device="cuda").half() for _ in range(3))
    ours = flashattn_cuda.prefill(q, k, v, causal, SCALE)
    theirs = ref.prefill(q, k, v, causal, SCALE)
    # the reference tests' oracle: fp32 SDPA cast back to fp16
    exact = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float(), v.float(), is_causal=causal, scale=SCALE).half().float()
    # ours is held to the 2e-3 bound; the reference kernel's own error bounds
    # how far apart the two outputs may be
    err_ours = (ours.float() - exact).abs().max().item()
    err_theirs = (theirs.float() - exact).abs().max().item()
    assert err_ours <= TOL
    assert (ours.float() - theirs.float()).abs().max().item() <= err_ours + err_theirs + 1e-6


@pytest.mark.parametrize("lens", [[1, 2, 512, 4096], [4096, 1, 2048, 7], [3000, 3001, 17, 0]])
def test_decode_matches_reference_kernel(ref, lens):
    torch.manual_seed(len(lens) + sum(lens))
    b, h, cap = len(lens), 12, 4096
    q = torch.randn(b, h, 1, 64, device="cuda").half()
    k, v = (torch.randn(b, h, cap, 64, device="cuda").half() for _ in range(2))
    t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    ours = flashattn_cuda.decode(q, k, v, t, SCALE)
    theirs = ref.decode(q, k, v, t, SCALE)
    assert (ours.float() - theirs.float()).abs().max().item() <= 2 * TOL
