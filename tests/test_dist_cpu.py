"""Multi-GPU host logic on CPU: sharding plans, the sequence-sharded decode
exchange and merge over a world-size-2 gloo group, and failure detection
(a rank that leaves makes the other's next collective fail, not hang)."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from flashattn_cuda import dist as fdist
import oracle

SCALE = 0.125
LOG2E = 1.4426950408889634


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def host_partials(q, k, v, lens, scale):
    """Per-(b, h) {m, l, 0, 0, acc[64]} over the given rows (the layout of
    fa_decode_partial), in float64."""
    B, H = q.shape[:2]
    out = np.zeros((B, H, fdist.PARTIAL_FLOATS))
    out[..., 0] = -1e30
    for b in range(B):
        n = int(lens[b])
        if n <= 0:
            continue
        for h in range(H):
            x = (k[b, h, :n].astype(np.float64) @ q[b, h, 0].astype(np.float64)) * scale * LOG2E
            m = x.max()
            p = np.exp2(x - m)
            out[b, h, 0], out[b, h, 1] = m, p.sum()
            out[b, h, 4:] = p @ v[b, h, :n].astype(np.float64)
    return out


def test_shard_units_cover_everything_once():
    for total in (1, 7, 56, 64):
        for world in (1, 2, 4, 8):
            got = [fdist.shard_units(total, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [e - s for s, e in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        fdist.shard_units(8, 2, 2)


def test_lpt_partition_balances_ragged_lengths():
    rng = np.random.default_rng(0)
    lens = rng.integers(1, 8193, 64).tolist()
    for world in (2, 4, 8):
        bins = fdist.lpt_partition(lens, world)
        assert sorted(i for b in bins for i in b) == list(range(64))
        loads = [sum(lens[i] for i in b) for b in bins]
        assert max(loads) - min(loads) <= max(lens)
        assert max(loads) <= sum(lens) / world * 1.1


def test_merge_of_shard_partials_equals_unsharded_decode():
    rng = np.random.default_rng(1)
    B, H, S = 3, 2, 300
    q = rng.standard_normal((B, H, 1, 64)).astype(np.float16).astype(np.float32)
    k = rng.standard_normal((B, H, S, 64)).astype(np.float16).astype(np.float32)
    v = rng.standard_normal((B, H, S, 64)).astype(np.float16).astype(np.float32)
    lens = np.array([300, 100, 0], dtype=np.int32)
    want = oracle.decode_c(q, k, v, lens, SCALE)[:, :, 0]
    for world in (1, 2, 3, 4):
        parts = []
        for r in range(world):
            s, e = fdist.seq_shard(S, world, r)
            ll = fdist.local_seq_lens(lens, s, e)
            parts.append(host_partials(q, k[:, :, s:e], v[:, :, s:e], ll, SCALE))
        got = fdist.merge_partials_host(np.stack(parts))
        np.testing.assert_allclose(got, want, atol=1e-5)
        assert np.all(got[2] == 0)  # empty sequence


def _exchange_worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    fdist.init(backend="gloo", timeout_s=20)
    rng = np.random.default_rng(7)
    B, H, S = 2, 3, 512
    q = rng.standard_normal((B, H, 1, 64)).astype(np.float32)
    k = rng.standard_normal((B, H, S, 64)).astype(np.float32)
    v = rng.standard_normal((B, H, S, 64)).astype(np.float32)
    lens = np.array([512, 200], dtype=np.int32)
    s, e = fdist.seq_shard(S, world, rank)
    part = torch.from_numpy(host_partials(q, k[:, :, s:e], v[:, :, s:e],
                                          fdist.local_seq_lens(lens, s, e), SCALE))
    gathered = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(gathered, part)
    got = fdist.merge_partials_host(torch.stack(gathered).numpy())
    want = oracle.decode_ref(q, k, v, lens, SCALE)[:, :, 0]
    err = float(np.abs(got - want).max())
    if rank == 0:
        with open(result_path, "w") as f:
            f.write(repr(err))
    dist.destroy_process_group()


def test_gloo_world2_sequence_sharded_exchange(tmp_path):
    out = tmp_path / "err.txt"
    mp.start_processes(_exchange_worker, args=(2, free_port(), str(out)),
                       nprocs=2, join=True, start_method="spawn")
    assert float(out.read_text()) < 1e-5


def _failure_worker(rank, world, port, result_path):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                      RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    fdist.init(backend="gloo", timeout_s=3)
    t = torch.ones(4)
    dist.all_reduce(t)  # one healthy step
    if rank == 1:
        os._exit(0)  # this rank leaves between steps, nothing in flight
    try:
        dist.all_reduce(t)
        outcome = "completed"
    except Exception as ex:  # timeout or connection loss
        outcome = "raised:" + type(ex).__name__
    with open(result_path, "w") as f:
        f.write(outcome)
    os._exit(0)


def test_gloo_lost_rank_is_detected_not_hung(tmp_path):
    out = tmp_path / "outcome.txt"
    ctx = mp.start_processes(_failure_worker, args=(2, free_port(), str(out)),
                             nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(60)
        assert not p.is_alive(), "a rank hung"
    assert out.read_text().startswith("raised:")
