"""Multi-GPU layer: one process per GPU, torch.distributed for the plumbing.

The reference is single-GPU; its work shards naturally:
  * prefill: the B*H (batch, head) units are independent — each rank takes a
    contiguous range (`shard_units`), no communication;
  * batched decode: sequences are independent — ranks take batch entries
    balanced by cached length (`lpt_partition`), no communication;
  * single-sequence long decode: the KV cache is split by contiguous sequence
    chunks (`seq_shard`); each rank reduces its chunk to per-(b, h)
    log-sum-exp partials {m, l, acc[64]} (the reference's split-K triple,
    csrc/decode.cu:215-219), the partials (68 fp32 per (b, h): 3,808 B at
    H=14) are all-gathered over NCCL and merged with the reference's merge
    rule (csrc/decode.cu:143-175) by `sharded_decode`.

Failure handling: collectives run under the process group's timeout (set it
short with `init(timeout_s=...)`); a rank that dies or never joins turns into
an exception on the others at their next collective, never a device hang.
"""

import datetime
import os

import numpy as np

PARTIAL_FLOATS = 68  # m, l, pad, pad, acc[64]


# ---------------------------------------------------------------------------
# Sharding plans (pure host logic)
# ---------------------------------------------------------------------------
def shard_units(total, world, rank):
    """Contiguous [start, end) share of `total` units for `rank`; the first
    total % world ranks get one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def lpt_partition(weights, world):
    """Longest-processing-time-first assignment of items to `world` bins
    (each item to the currently lightest bin, heaviest items first).
    Returns the sorted item indices of every bin."""
    order = sorted(range(len(weights)), key=lambda i: (-weights[i], i))
    loads = [0] * world
    bins = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        bins[r].append(i)
        loads[r] += weights[i]
    return [sorted(b) for b in bins]


def seq_shard(seq_len, world, rank):
    """Cache rows [start, end) held by `rank` when one sequence's KV cache is
    split into contiguous chunks."""
    return shard_units(seq_len, world, rank)


def local_seq_lens(seq_lens, start, end):
    """Valid rows of each sequence inside the chunk [start, end): lengths are
    clamped to the chunk (numpy or torch int32 arrays)."""
    try:
        import torch
        if isinstance(seq_lens, torch.Tensor):
            return torch.clamp(seq_lens - start, 0, end - start).to(torch.int32)
    except ImportError:  # pragma: no cover
        pass
    return np.clip(np.asarray(seq_lens) - start, 0, end - start).astype(np.int32)


def merge_partials_host(partials):
    """Host restatement of the device merge (fa_merge_partials): partials
    (G, ..., 68) -> output (..., 64). Skips l <= 0; no keys anywhere -> 0."""
    p = np.asarray(partials, dtype=np.float64)
    m, l, acc = p[..., 0], p[..., 1], p[..., 4:]
    valid = l > 0
    m_all = np.where(valid, m, -np.inf).max(axis=0)
    m_all = np.where(np.isfinite(m_all), m_all, 0.0)
    f = np.where(valid, np.exp2(m - m_all[None]), 0.0)
    l_all = (l * f).sum(axis=0)
    a_all = (acc * f[..., None]).sum(axis=0)
    out = np.where(l_all[..., None] > 0, a_all / np.where(l_all > 0, l_all, 1)[..., None], 0.0)
    return out.astype(np.float32)


# ---------------------------------------------------------------------------
# Process-group plumbing
# ---------------------------------------------------------------------------
def init(backend="nccl", timeout_s=60.0):
    """Joins the job launched by torchrun (RANK / WORLD_SIZE / MASTER_* env)
    with a bounded collective timeout. Returns (rank, world, local_rank)."""
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s),
                                **kw)
    return rank, world, local


def sharded_decode(q, k_local, v_local, seq_lens_local, scale, group=None):
    """Decode of sequences whose KV caches are split across the ranks of
    `group` by sequence chunk: every rank passes the full q and its own chunk
    (with lengths already clamped to the chunk, see local_seq_lens) and gets
    the full fp16 output. One NCCL all-gather of the partials, then the
    device merge."""
    import torch
    import torch.distributed as dist

    from . import decode, decode_partial, merge_partials

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return decode(q, k_local, v_local, seq_lens_local, scale)
    part = decode_partial(q, k_local, v_local, seq_lens_local, scale)
    gathered = torch.empty((world,) + tuple(part.shape), dtype=part.dtype,
                           device=part.device)
    dist.all_gather_into_tensor(gathered, part, group=group)
    return merge_partials(gathered)


class PeerExchange:
    """Exchange buffers for sharded_decode_fused on one process group.

    Each rank allocates one device buffer (fa_exchange_alloc), the 64-byte
    IPC handles are all-gathered on the host, and every rank maps the
    others' buffers; the kernel then stores its finished partials straight
    into every rank's buffer over NVLink. One instance serves any number of
    calls with this (B, H) and head_dim; all ranks must call in the same
    order."""

    def __init__(self, batch, heads, group=None, device=None, head_dim=64):
        import torch
        import torch.distributed as dist

        from . import _C

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.cuda.current_device() if device is None else device
        self.shape = (batch, heads)
        self.head_dim = head_dim
        nbytes = _C._exchange_bytes(batch, heads, self.world, head_dim)
        self._own, handle = _C._exchange_alloc(nbytes, self.device)
        handles = [handle]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
        self._opened = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
            else:
                p = _C._exchange_open(h, self.device)
                self._opened.append(p)
                ptrs.append(p)
        self.peers = torch.tensor(ptrs, dtype=torch.int64,
                                  device=torch.device("cuda", self.device))
        self.epoch = 0

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (after a barrier
        so no peer still writes into it)."""
        import torch
        import torch.distributed as dist

        from . import _C

        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for p in self._opened:
            _C._exchange_close(p, self.device)
        self._opened = []
        if self._own:
            _C._exchange_free(self._own, self.device)
            self._own = 0


def sharded_decode_fused(q, k_local, v_local, seq_lens_local, scale, xchg):
    """sharded_decode with the combine inside the decode kernel: every rank
    passes the full q and its own KV chunk (lengths clamped to the chunk, see
    local_seq_lens) and gets the full output (fp16 or bf16, the dtype of q
    and the cache) from one launch."""
    from . import _C

    if tuple(q.shape[:2]) != xchg.shape or q.shape[3] != xchg.head_dim:
        raise ValueError(f"exchange was sized for {xchg.shape} at head_dim "
                         f"{xchg.head_dim}, got {tuple(q.shape)}")
    xchg.epoch += 1
    return _C.decode_exchange(q, k_local, v_local, seq_lens_local, scale,
                              xchg.peers, xchg.rank, xchg.world, xchg.epoch)
