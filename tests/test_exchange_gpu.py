"""Sequence-sharded decode with the cross-GPU combine inside the kernel
(dist.PeerExchange + sharded_decode_fused). One rank exercises the whole
path on a single GPU (send to itself, count, merge); two ranks, when the
box has two GPUs, check the NVLink exchange against the unsharded decode."""

import math
import os

import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda
from flashattn_cuda import dist as fadist

pytestmark = [pytest.mark.gpu, requires_gpu]
SCALE = 1.0 / math.sqrt(64)


def test_single_rank_exchange_equals_decode():
    torch.manual_seed(0)
    b, h, s = 4, 14, 5000
    q = torch.randn(b, h, 1, 64, device="cuda").half()
    k, v = (torch.randn(b, h, s, 64, device="cuda").half() for _ in range(2))
    lens = torch.tensor([5000, 0, 1, 2345], dtype=torch.int32, device="cuda")
    xchg = fadist.PeerExchange(b, h)
    try:
        for _ in range(3):  # epochs advance, counters keep counting
            got = fadist.sharded_decode_fused(q, k, v, lens, SCALE, xchg)
            want = flashattn_cuda.decode(q, k, v, lens, SCALE)
            assert torch.equal(got, want)
        assert torch.all(got[1] == 0)
    finally:
        xchg.close()
    assert flashattn_cuda.take_device_error() == 0


def test_single_rank_exchange_bf16_equals_decode():
    torch.manual_seed(1)
    b, h, s = 3, 14, 3000
    q = torch.randn(b, h, 1, 64, device="cuda").bfloat16()
    k, v = (torch.randn(b, h, s, 64, device="cuda").bfloat16() for _ in range(2))
    lens = torch.tensor([3000, 17, 0], dtype=torch.int32, device="cuda")
    xchg = fadist.PeerExchange(b, h)
    try:
        for _ in range(2):
            got = fadist.sharded_decode_fused(q, k, v, lens, SCALE, xchg)
            assert got.dtype == torch.bfloat16
            want = flashattn_cuda.decode(q, k, v, lens, SCALE)
            assert torch.equal(got, want)
    finally:
        xchg.close()
    assert flashattn_cuda.take_device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_single_rank_exchange_d128_equals_decode(dtype):
    torch.manual_seed(2)
    b, h, s = 3, 8, 4000
    q = torch.randn(b, h, 1, 128, device="cuda").to(dtype)
    k, v = (torch.randn(b, h, s, 128, device="cuda").to(dtype) for _ in range(2))
    lens = torch.tensor([4000, 0, 333], dtype=torch.int32, device="cuda")
    xchg = fadist.PeerExchange(b, h, head_dim=128)
    try:
        for _ in range(3):
            got = fadist.sharded_decode_fused(q, k, v, lens, 128 ** -0.5, xchg)
            want = flashattn_cuda.decode(q, k, v, lens, 128 ** -0.5)
            assert torch.equal(got, want)
        assert torch.all(got[1] == 0)
        with pytest.raises(ValueError, match="head_dim"):
            fadist.sharded_decode_fused(q[..., :64].contiguous(),
                                        k[..., :64].contiguous(),
                                        v[..., :64].contiguous(), lens, 0.1,
                                        xchg)
    finally:
        xchg.close()
    assert flashattn_cuda.take_device_error() == 0


def _two_rank_worker(rank, world, port, result):
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        err = 0.0
        for d in (64, 128):  # head_dim 64 and 128 through the same exchange code
            g = torch.Generator().manual_seed(1)
            b, h, s = 2, 14, 20000
            q = torch.randn(b, h, 1, d, generator=g).half().cuda()
            k = torch.randn(b, h, s, d, generator=g).half()
            v = torch.randn(b, h, s, d, generator=g).half()
            lens = torch.tensor([20000, 7000], dtype=torch.int32)
            c0, c1 = fadist.seq_shard(s, world, rank)
            kl = k[:, :, c0:c1].contiguous().cuda()
            vl = v[:, :, c0:c1].contiguous().cuda()
            ll = torch.as_tensor(fadist.local_seq_lens(lens.tolist(), c0, c1),
                                 dtype=torch.int32).cuda()
            xchg = fadist.PeerExchange(b, h, head_dim=d)
            outs = [fadist.sharded_decode_fused(q, kl, vl, ll, d ** -0.5, xchg)
                    for _ in range(3)]
            torch.cuda.synchronize()
            xchg.close()
            want = flashattn_cuda.decode(q, k.cuda(), v.cuda(), lens.cuda(),
                                         d ** -0.5)
            err = max([err] + [(o.float() - want.float()).abs().max().item()
                               for o in outs])
        result[rank] = err if flashattn_cuda.take_device_error() == 0 else -1.0
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_exchange_equals_unsharded():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_two_rank_worker, args=(2, 29617, result), nprocs=2,
                       start_method="spawn")
    assert sorted(result.keys()) == [0, 1]
    for r in (0, 1):
        assert 0.0 <= result[r] <= 1e-3, result[r]


def _many_epochs_worker(rank, world, port, result):
    """Back-to-back epochs with no host sync between them, new queries and
    lengths every epoch, and sequences that have no rows on one rank (their
    partials are sent before streaming, merged after): a rank that runs
    ahead must never overwrite a partial a slower peer still merges."""
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("nccl", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(5)
        b, h, s, steps = 6, 8, 8192, 24
        k = torch.randn(b, h, s, 64, generator=g).half()
        v = torch.randn(b, h, s, 64, generator=g).half()
        c0, c1 = fadist.seq_shard(s, world, rank)
        kl = k[:, :, c0:c1].contiguous().cuda()
        vl = v[:, :, c0:c1].contiguous().cuda()
        qs, ls, outs = [], [], []
        xchg = fadist.PeerExchange(b, h)
        for step in range(steps):
            q = torch.randn(b, h, 1, 64, generator=g).half().cuda()
            # short sequences live on rank 0 only; long ones span both
            lens = torch.randint(1, s + 1, (b,), generator=g, dtype=torch.int32)
            lens[step % b] = 1 + step
            lens[(step + 1) % b] = 0
            ll = torch.as_tensor(fadist.local_seq_lens(lens.tolist(), c0, c1),
                                 dtype=torch.int32).cuda()
            qs.append(q)
            ls.append(lens)
            outs.append(fadist.sharded_decode_fused(q, kl, vl, ll, SCALE, xchg))
        torch.cuda.synchronize()
        xchg.close()
        kc, vc = k.cuda(), v.cuda()
        err = 0.0
        for q, lens, o in zip(qs, ls, outs):
            want = flashattn_cuda.decode(q, kc, vc, lens.cuda(), SCALE)
            err = max(err, (o.float() - want.float()).abs().max().item())
        result[rank] = err if flashattn_cuda.take_device_error() == 0 else -1.0
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_exchange_many_back_to_back_epochs():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_many_epochs_worker, args=(2, 29619, result), nprocs=2,
                       start_method="spawn")
    assert sorted(result.keys()) == [0, 1]
    for r in (0, 1):
        assert 0.0 <= result[r] <= 1e-3, result[r]
