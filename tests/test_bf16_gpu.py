"""bf16 q/k/v/o (and caches) for prefill and decode, head_dim 64 and 128,
one or several query heads per K/V head, against fp32 attention computed
from the same bf16 values.

Tolerance: 1.5e-2 absolute. bf16 keeps 8 significant bits, so rounding the
output alone costs up to half an ulp, 2^-8 (3.9e-3) for values in [1, 2);
the probabilities enter the PV product as bf16 (relative error up to 2^-9
each). fp16 calls keep their 2e-3 bar in the other test files."""

import ctypes
import os

import pytest
import torch

from conftest import PKG_DIR, requires_gpu

import flashattn_cuda

pytestmark = [pytest.mark.gpu, requires_gpu]
TOL = 1.5e-2


def bf(*shape):
    return torch.randn(*shape, device="cuda").to(torch.bfloat16)


def prefill_reference(q, k, v, causal, scale):
    group = q.shape[1] // k.shape[1]
    kf = k.float().repeat_interleave(group, dim=1)
    vf = v.float().repeat_interleave(group, dim=1)
    return torch.nn.functional.scaled_dot_product_attention(
        q.float(), kf, vf, is_causal=causal, scale=scale)


def decode_reference(q, k, v, lens, scale):
    b, h = q.shape[:2]
    group = h // k.shape[1]
    out = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
    for i in range(b):
        n = max(0, min(int(lens[i]), k.shape[2]))
        if n == 0:
            continue
        kf = k[i, :, :n].float().repeat_interleave(group, dim=0)
        vf = v[i, :, :n].float().repeat_interleave(group, dim=0)
        s = (q[i].float() @ kf.transpose(1, 2)) * scale
        out[i] = torch.softmax(s, dim=-1) @ vf
    return out


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("b,h,h_kv,n", [(2, 3, 3, 1000), (1, 4, 4, 4096),
                                        (2, 14, 2, 513), (1, 1, 1, 1),
                                        (3, 2, 2, 129), (1, 8, 1, 2048)])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_bf16_matches_fp32(d, b, h, h_kv, n, causal):
    torch.manual_seed(d + b * 100 + h * 10 + n)
    q, k, v = bf(b, h, n, d), bf(b, h_kv, n, d), bf(b, h_kv, n, d)
    scale = d ** -0.5
    got = flashattn_cuda.prefill(q, k, v, causal, scale)
    assert got.dtype == torch.bfloat16 and got.shape == q.shape
    want = prefill_reference(q, k, v, causal, scale)
    assert (got.float() - want).abs().max().item() <= TOL
    assert flashattn_cuda.take_device_error() == 0


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("b,h,h_kv,s,lens", [
    (5, 8, 8, 3000, [3000, 1, 0, 1777, 64]),
    (1, 14, 14, 131072, [131072]),
    (1, 14, 2, 65536, [65533]),
    (64, 12, 4, 700, None),
    (8, 32, 8, 4096, None),
    (3, 6, 6, 512, [600, 512, 257]),   # lengths past the capacity clamp
])
def test_decode_bf16_matches_fp32(d, b, h, h_kv, s, lens):
    torch.manual_seed(d + b + h + s)
    q = bf(b, h, 1, d)
    k, v = bf(b, h_kv, s, d), bf(b, h_kv, s, d)
    if lens is None:
        g = torch.Generator().manual_seed(b)
        lens = torch.randint(0, s + 20, (b,), generator=g, dtype=torch.int32)
    lens = torch.as_tensor(lens, dtype=torch.int32).cuda()
    scale = d ** -0.5
    got = flashattn_cuda.decode(q, k, v, lens, scale)
    assert got.dtype == torch.bfloat16
    want = decode_reference(q, k, v, lens.cpu(), scale)
    assert (got.float() - want).abs().max().item() <= TOL
    # a sequence with no rows gives exactly zero
    for i in range(b):
        if int(lens[i]) <= 0:
            assert torch.count_nonzero(got[i]).item() == 0
    assert flashattn_cuda.take_device_error() == 0


def test_bf16_and_fp16_agree_on_the_same_values():
    """Inputs exactly representable in both types: the bf16 and fp16 paths
    compute the same attention to within the bf16 output rounding."""
    torch.manual_seed(7)
    q, k, v = (torch.randint(-8, 9, (2, 4, 777, 64), device="cuda").float() / 8
               for _ in range(3))
    out16 = flashattn_cuda.prefill(q.half(), k.half(), v.half(), True, 0.125)
    outbf = flashattn_cuda.prefill(q.bfloat16(), k.bfloat16(), v.bfloat16(),
                                   True, 0.125)
    assert (out16.float() - outbf.float()).abs().max().item() <= TOL


def test_mixed_dtypes_are_rejected():
    q = bf(1, 2, 64, 64)
    with pytest.raises(RuntimeError, match="same dtype"):
        flashattn_cuda.prefill(q, q.half(), q.half(), True, 0.1)
    lens = torch.tensor([64], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="same dtype"):
        flashattn_cuda.decode(bf(1, 2, 1, 64), q.half(), q.half(), lens, 0.1)
    with pytest.raises(RuntimeError, match="needs fp16"):
        flashattn_cuda.decode_partial(bf(1, 2, 1, 64), q, q, lens, 0.1)
    with pytest.raises(RuntimeError, match="dtype of q"):
        flashattn_cuda.decode_append(bf(1, 2, 1, 64),
                                     bf(1, 2, 1, 64).half(), bf(1, 2, 1, 64),
                                     q.clone(), q.clone(), lens, 0.1)


def test_c_abi_bf16_entry_points():
    """fa_prefill_ex / fa_decode_ex called directly, as a C host would."""
    lib = ctypes.CDLL(os.path.join(PKG_DIR, "flashattn_cuda", "libfa_b200.so"))
    vp, ci = ctypes.c_void_p, ctypes.c_int
    lib.fa_prefill_ex.argtypes = [vp] * 4 + [ci] * 7 + [ctypes.c_float, vp]
    lib.fa_decode_ex.argtypes = [vp] * 5 + [ci] * 6 + [
        ctypes.c_float, vp, ctypes.c_size_t, vp, ctypes.c_size_t, vp]
    lib.fa_decode_ex_workspace_bytes.restype = ctypes.c_size_t
    lib.fa_decode_ex_workspace_bytes.argtypes = [ci] * 6
    stream = vp(torch.cuda.current_stream().cuda_stream)
    torch.manual_seed(3)
    q, k, v = bf(2, 6, 300, 64), bf(2, 3, 300, 64), bf(2, 3, 300, 64)
    o = torch.empty_like(q)
    assert lib.fa_prefill_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                             o.data_ptr(), 2, 6, 3, 300, 64, 1, 1, 0.125,
                             stream) == 0
    torch.cuda.synchronize()
    assert (o.float() - prefill_reference(q, k, v, True, 0.125)).abs().max() <= TOL
    qd = bf(2, 6, 1, 128)
    kc, vc = bf(2, 3, 1000, 128), bf(2, 3, 1000, 128)
    lens = torch.tensor([1000, 333], dtype=torch.int32, device="cuda")
    od = torch.empty_like(qd)
    ws_bytes = lib.fa_decode_ex_workspace_bytes(2, 6, 3, 1000, 128, 0)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    ctr = torch.zeros(12, dtype=torch.int32, device="cuda")
    for _ in range(2):  # counters are left at zero for the next call
        assert lib.fa_decode_ex(qd.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                lens.data_ptr(), od.data_ptr(), 2, 6, 3, 1000,
                                128, 1, 128 ** -0.5, ws.data_ptr(), ws_bytes,
                                ctr.data_ptr(), 12, stream) == 0
        torch.cuda.synchronize()
        want = decode_reference(qd, kc, vc, lens.cpu(), 128 ** -0.5)
        assert (od.float() - want).abs().max().item() <= TOL
    assert int(ctr.abs().sum()) == 0


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("h,h_kv", [(12, 12), (14, 2)])
def test_decode_append_bf16(d, h, h_kv):
    """The new rows land at seq_lens[b] of bf16 caches (bit copies) and are
    attended in the same launch; a full cache attends its old rows only."""
    torch.manual_seed(d + h)
    b, s_max = 4, 1500
    q = bf(b, h, 1, d)
    k, v = bf(b, h_kv, s_max, d), bf(b, h_kv, s_max, d)
    k_new, v_new = bf(b, h_kv, 1, d), bf(b, h_kv, 1, d)
    lens = torch.tensor([0, 700, s_max - 1, s_max], dtype=torch.int32,
                        device="cuda")
    k_want, v_want = k.clone(), v.clone()
    new_lens = []
    for i, n in enumerate(lens.tolist()):
        if n < s_max:
            k_want[i, :, n] = k_new[i, :, 0]
            v_want[i, :, n] = v_new[i, :, 0]
        new_lens.append(min(n + 1, s_max))
    got = flashattn_cuda.decode_append(q, k_new, v_new, k, v, lens, d ** -0.5)
    assert got.dtype == torch.bfloat16
    assert torch.equal(k, k_want) and torch.equal(v, v_want)
    want = decode_reference(q, k_want, v_want, new_lens, d ** -0.5)
    assert (got.float() - want).abs().max().item() <= TOL
    assert flashattn_cuda.take_device_error() == 0
