"""GPU parity of the sm_100a kernels (run on a B200 with -m gpu).

Mirrors the reference's tests/test_correctness.py contract: the same shapes,
the same 2e-3 max-abs tolerance, the same consistency and error-message
checks. The checkers are (a) the CPU oracle (oracle/, pinned to the
reference's outputs by tests/test_oracle.py) on sizes it finishes in
seconds, (b) the committed golden vectors, and (c) at full sizes the
reference tests' own oracle, fp32 SDPA on upcast inputs, plus size-independent
properties (decode of token t == causal prefill row t, split invariance,
sharded-merge == unsharded).
"""

import math

import numpy as np
import pytest
import torch

from conftest import requires_gpu

import flashattn_cuda
import oracle
from golden.make_golden import (C1, DECODE_CASES, PREFILL_CASES, inputs)

HEAD_DIM = flashattn_cuda.head_dim
SCALE = 1.0 / math.sqrt(HEAD_DIM)
TOL = 2e-3  # max-abs error bound of the north star and the reference tests

pytestmark = [pytest.mark.gpu, requires_gpu]


def rand(*shape, seed=None):
    if seed is not None:
        torch.manual_seed(seed)
    return torch.randn(*shape, device="cuda", dtype=torch.float16)


def sdpa_reference(q, k, v, causal, scale=SCALE):
    """fp32 SDPA on upcast inputs, cast back to fp16 (the reference tests'
    oracle, tests/test_correctness.py:29-34)."""
    out = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float(), v.float(), is_causal=causal, scale=scale)
    return out.half()


def decode_reference(q, k_cache, v_cache, seq_lens, scale=SCALE):
    """fp32 single-query attention over the valid part of each cache
    (tests/test_correctness.py:37-44), with the kernel's clamp/empty rules."""
    out = torch.zeros_like(q)
    for b in range(q.shape[0]):
        n = min(max(int(seq_lens[b]), 0), k_cache.shape[2])
        if n == 0:
            continue
        scores = (q[b].float() @ k_cache[b, :, :n].float().transpose(-1, -2)) * scale
        out[b] = (torch.softmax(scores, dim=-1) @ v_cache[b, :, :n].float()).half()
    return out


def max_abs_diff(a, b):
    return (a.float() - b.float()).abs().max().item()


def to_np(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def no_device_errors():
    yield
    assert flashattn_cuda.take_device_error() == 0


# ---------------------------------------------------------------------------
# Prefill
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("batch", [1, 4])
@pytest.mark.parametrize("heads", [8, 12, 14])
@pytest.mark.parametrize("seq", [128, 512, 1024, 2048, 4096])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_matches_sdpa(batch, heads, seq, causal):
    q = rand(batch, heads, seq, HEAD_DIM, seed=0)
    k = rand(batch, heads, seq, HEAD_DIM)
    v = rand(batch, heads, seq, HEAD_DIM)
    out = flashattn_cuda.prefill(q, k, v, causal, SCALE)
    ref = sdpa_reference(q, k, v, causal)
    assert max_abs_diff(out, ref) <= TOL


@pytest.mark.parametrize("seq", [1, 37, 65, 127, 128, 129, 130, 255, 1023])
@pytest.mark.parametrize("causal", [True, False])
def test_prefill_ragged_lengths_match_oracle(seq, causal):
    """Lengths that are not a multiple of the 128-row tile, against the C
    oracle on the same fp16 inputs."""
    q = rand(2, 5, seq, HEAD_DIM, seed=1)
    k = rand(2, 5, seq, HEAD_DIM)
    v = rand(2, 5, seq, HEAD_DIM)
    out = flashattn_cuda.prefill(q, k, v, causal, SCALE)
    ref = oracle.prefill_c(to_np(q), to_np(k), to_np(v), causal, SCALE)
    assert np.abs(to_np(out) - ref).max() <= TOL


@pytest.mark.parametrize("case", PREFILL_CASES, ids=[c[0] for c in PREFILL_CASES])
def test_prefill_golden_vectors(case, golden):
    name, b, h, n, causal, seed = case
    q, k, v = (torch.from_numpy(x).cuda() for x in inputs((b, h, n, HEAD_DIM), seed))
    out = flashattn_cuda.prefill(q, k, v, causal, SCALE)
    assert np.abs(to_np(out) - golden[name + "_sdpa"]).max() <= TOL


def test_c1_config_golden(golden):
    _, b, h, n, seed = C1
    q, k, v = (torch.from_numpy(x).cuda() for x in inputs((b, h, n, HEAD_DIM), seed))
    out = flashattn_cuda.prefill(q, k, v, True, SCALE)
    rows = golden["c1_prefill_rows"]
    assert np.abs(to_np(out)[:, :, rows] - golden["c1_prefill"]).max() <= TOL
    lens = torch.full((b,), n, dtype=torch.int32, device="cuda")
    d = flashattn_cuda.decode(q[:, :, n - 1:n].contiguous(), k, v, lens, SCALE)
    assert np.abs(to_np(d) - golden["c1_decode_last"]).max() <= TOL


@pytest.mark.parametrize("scale", [0.0, -0.125, 0.5, 1e-3])
def test_prefill_unusual_scales(scale):
    q = rand(1, 3, 200, HEAD_DIM, seed=8)
    k = rand(1, 3, 200, HEAD_DIM)
    v = rand(1, 3, 200, HEAD_DIM)
    for causal in (False, True):
        out = flashattn_cuda.prefill(q, k, v, causal, scale)
        ref = oracle.prefill_c(to_np(q), to_np(k), to_np(v), causal, scale)
        assert np.abs(to_np(out) - ref).max() <= TOL


def test_prefill_large_logits_rescale_path():
    """Inputs scaled up so row maxima move by many powers of two between key
    tiles, exercising the O rescale in tensor memory."""
    torch.manual_seed(3)
    q = (torch.randn(1, 2, 1024, HEAD_DIM, device="cuda") * 4).half()
    k = (torch.randn(1, 2, 1024, HEAD_DIM, device="cuda") * 4).half()
    # keys grow along the sequence so later tiles raise the max
    k = (k.float() * torch.linspace(0.2, 1.0, 1024, device="cuda")[None, None, :, None]).half()
    v = rand(1, 2, 1024, HEAD_DIM)
    for causal in (False, True):
        out = flashattn_cuda.prefill(q, k, v, causal, SCALE)
        ref = sdpa_reference(q, k, v, causal)
        assert max_abs_diff(out, ref) <= TOL


def test_prefill_config3_qwen_shape():
    """B=4, H=14, N=4096, causal."""
    q = rand(4, 14, 4096, HEAD_DIM, seed=42)
    k = rand(4, 14, 4096, HEAD_DIM)
    v = rand(4, 14, 4096, HEAD_DIM)
    out = flashattn_cuda.prefill(q, k, v, True, SCALE)
    ref = sdpa_reference(q, k, v, True)
    assert max_abs_diff(out, ref) <= TOL


def test_prefill_is_deterministic():
    q = rand(2, 4, 777, HEAD_DIM, seed=9)
    k = rand(2, 4, 777, HEAD_DIM)
    v = rand(2, 4, 777, HEAD_DIM)
    a = flashattn_cuda.prefill(q, k, v, True, SCALE)
    b = flashattn_cuda.prefill(q, k, v, True, SCALE)
    assert torch.equal(a, b)


# ---------------------------------------------------------------------------
# Decode
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("position", [0, 1, 17, 127, 128, 511, 1024, 2047])
def test_decode_matches_causal_prefill_row(position):
    """Decoding position t must reproduce row t of the causal prefill."""
    batch, heads, seq = 2, 12, 2048
    q = rand(batch, heads, seq, HEAD_DIM, seed=2)
    k = rand(batch, heads, seq, HEAD_DIM)
    v = rand(batch, heads, seq, HEAD_DIM)
    full = flashattn_cuda.prefill(q, k, v, True, SCALE)
    q_step = q[:, :, position:position + 1, :].contiguous()
    seq_lens = torch.full((batch,), position + 1, dtype=torch.int32, device="cuda")
    out = flashattn_cuda.decode(q_step, k, v, seq_lens, SCALE)
    assert max_abs_diff(out, full[:, :, position:position + 1, :]) <= TOL


@pytest.mark.parametrize(
    "seq_lens",
    [
        [1, 2, 512, 4096],
        [513, 1023, 1024, 3000],
        [64, 65, 127, 129],
        [4096, 1, 2048, 7],
    ],
)
def test_decode_ragged_batch(seq_lens):
    batch, heads, cache = len(seq_lens), 8, 4096
    q = rand(batch, heads, 1, HEAD_DIM, seed=3)
    k_cache = rand(batch, heads, cache, HEAD_DIM)
    v_cache = rand(batch, heads, cache, HEAD_DIM)
    lens = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    out = flashattn_cuda.decode(q, k_cache, v_cache, lens, SCALE)
    ref = decode_reference(q, k_cache, v_cache, lens)
    assert max_abs_diff(out, ref) <= TOL


@pytest.mark.parametrize("seq_lens,heads", [
    ([1, 128, 129, 255, 256], 12),   # every segment fits two stages: one CTA each
    ([256] * 40, 16),                # more whole segments than the grid has CTAs
    ([0, 256, 3, 200], 2),           # an empty sequence among short ones
    ([256, 257, 100], 12),           # one sequence just past the whole-segment limit
])
def test_decode_short_sequences_whole_segments(seq_lens, heads):
    """Sequences of at most two 128-row stages are streamed whole by one
    CTA (no cross-CTA merge); mixed with longer ones the usual split runs."""
    batch, cache = len(seq_lens), 257
    q = rand(batch, heads, 1, HEAD_DIM, seed=11)
    k_cache = rand(batch, heads, cache, HEAD_DIM)
    v_cache = rand(batch, heads, cache, HEAD_DIM)
    lens = torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    out = flashattn_cuda.decode(q, k_cache, v_cache, lens, SCALE)
    ref = decode_reference(q, k_cache, v_cache, lens)
    assert max_abs_diff(out, ref) <= TOL


@pytest.mark.parametrize("cache", [1, 63, 512, 513, 2048])
def test_decode_cache_lengths(cache):
    batch, heads = 3, 12
    q = rand(batch, heads, 1, HEAD_DIM, seed=4)
    k_cache = rand(batch, heads, cache, HEAD_DIM)
    v_cache = rand(batch, heads, cache, HEAD_DIM)
    lens = torch.full((batch,), cache, dtype=torch.int32, device="cuda")
    out = flashattn_cuda.decode(q, k_cache, v_cache, lens, SCALE)
    ref = decode_reference(q, k_cache, v_cache, lens)
    assert max_abs_diff(out, ref) <= TOL


def test_decode_clamp_and_empty_sequences():
    """seq_lens beyond the cache are clamped; zero/negative lengths give 0."""
    q = rand(5, 4, 1, HEAD_DIM, seed=12)
    k = rand(5, 4, 300, HEAD_DIM)
    v = rand(5, 4, 300, HEAD_DIM)
    lens = torch.tensor([0, 1000, -5, 300, 17], dtype=torch.int32, device="cuda")
    out = flashattn_cuda.decode(q, k, v, lens, SCALE)
    ref = oracle.decode_c(to_np(q), to_np(k), to_np(v), lens.cpu().numpy(), SCALE)
    assert np.abs(to_np(out) - ref).max() <= TOL
    assert torch.all(out[0] == 0) and torch.all(out[2] == 0)


@pytest.mark.parametrize("case", DECODE_CASES, ids=[c[0] for c in DECODE_CASES])
def test_decode_golden_vectors(case, golden):
    name, b, h, s_max, lens, seed = case
    q = torch.from_numpy(inputs((b, h, 1, HEAD_DIM), seed, 1)[0]).cuda()
    k, v = (torch.from_numpy(x).cuda()
            for x in inputs((b, h, s_max, HEAD_DIM), seed + 1000, 2))
    t_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    out = flashattn_cuda.decode(q, k, v, t_lens, SCALE)
    assert np.abs(to_np(out) - golden[name + "_ref"]).max() <= TOL


@pytest.mark.parametrize("cache", [512, 1024, 2048])
def test_decode_is_invariant_to_split_size(cache):
    batch, heads = 2, 12
    q = rand(batch, heads, 1, HEAD_DIM, seed=7)
    k_cache = rand(batch, heads, cache, HEAD_DIM)
    v_cache = rand(batch, heads, cache, HEAD_DIM)
    lens = torch.tensor([cache, cache // 2 + 1], dtype=torch.int32, device="cuda")
    chosen = flashattn_cuda.decode(q, k_cache, v_cache, lens, SCALE)
    ref = decode_reference(q, k_cache, v_cache, lens)
    assert max_abs_diff(chosen, ref) <= TOL
    for split in (4, 36, 128, 256, 512, 1024):
        forced = flashattn_cuda._decode_with_split(q, k_cache, v_cache, lens,
                                                   SCALE, split)
        assert max_abs_diff(forced, ref) <= TOL
        assert max_abs_diff(forced, chosen) <= 1e-3


def test_decode_config4_ragged_batch():
    """B=64, H=12, capacity 8192, lengths U[1, 8192]."""
    g = torch.Generator().manual_seed(0)
    lens = torch.randint(1, 8193, (64,), generator=g, dtype=torch.int32).cuda()
    q = rand(64, 12, 1, HEAD_DIM, seed=44)
    k = rand(64, 12, 8192, HEAD_DIM)
    v = rand(64, 12, 8192, HEAD_DIM)
    out = flashattn_cuda.decode(q, k, v, lens, SCALE)
    ref = decode_reference(q, k, v, lens)
    assert max_abs_diff(out, ref) <= TOL
    again = flashattn_cuda.decode(q, k, v, lens, SCALE)
    assert torch.equal(out, again)  # fixed merge order: deterministic


def test_decode_config5_long_context_and_sharded_merge():
    """B=1, H=14, S=131072, plus the sequence-sharded
    path emulated on one GPU: per-shard partials merged == unsharded."""
    S = 131072
    q = rand(1, 14, 1, HEAD_DIM, seed=55)
    k = rand(1, 14, S, HEAD_DIM)
    v = rand(1, 14, S, HEAD_DIM)
    lens = torch.tensor([S], dtype=torch.int32, device="cuda")
    out = flashattn_cuda.decode(q, k, v, lens, SCALE)
    ref = decode_reference(q, k, v, lens)
    assert max_abs_diff(out, ref) <= TOL
    for shards in (2, 4, 8):
        chunk = S // shards
        parts = []
        for r in range(shards):
            ks = k[:, :, r * chunk:(r + 1) * chunk].contiguous()
            vs = v[:, :, r * chunk:(r + 1) * chunk].contiguous()
            ls = torch.clamp(lens - r * chunk, 0, chunk).to(torch.int32)
            parts.append(flashattn_cuda.decode_partial(q, ks, vs, ls, SCALE))
        merged = flashattn_cuda.merge_partials(torch.stack(parts))
        assert max_abs_diff(merged, ref) <= TOL
        assert max_abs_diff(merged, out) <= 1e-3


def test_decode_partial_with_empty_shard():
    q = rand(2, 3, 1, HEAD_DIM, seed=60)
    k = rand(2, 3, 256, HEAD_DIM)
    v = rand(2, 3, 256, HEAD_DIM)
    lens = torch.tensor([100, 256], dtype=torch.int32, device="cuda")
    full = flashattn_cuda.decode(q, k, v, lens, SCALE)
    p0 = flashattn_cuda.decode_partial(q, k[:, :, :128].contiguous(),
                                       v[:, :, :128].contiguous(),
                                       torch.clamp(lens, 0, 128), SCALE)
    p1 = flashattn_cuda.decode_partial(q, k[:, :, 128:].contiguous(),
                                       v[:, :, 128:].contiguous(),
                                       torch.clamp(lens - 128, 0, 128).int(), SCALE)
    assert float(p1[0, :, 1].max()) == 0.0  # sequence 0 has no rows in shard 1
    merged = flashattn_cuda.merge_partials(torch.stack([p0, p1]))
    assert max_abs_diff(merged, full) <= 1e-3


def test_decode_split_choice_targets_the_device():
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    target = 2 * sms
    for batch, heads, seq in [(1, 12, 2048), (8, 12, 2048), (4, 12, 1024)]:
        split = flashattn_cuda.choose_decode_split(seq, batch, heads, target)
        assert split in (128, 256, 512, 1024)
        if batch * heads * -(-seq // 128) < target:
            assert split == 128
            continue
        assert batch * heads * -(-seq // split) >= target
        if split < 1024:
            assert batch * heads * -(-seq // (split * 2)) < target
    assert flashattn_cuda.choose_decode_split(512, 1, 12, target) == 128


# ---------------------------------------------------------------------------
# Input validation (message contract of the reference)
# ---------------------------------------------------------------------------
def test_prefill_rejects_bad_inputs():
    q = rand(1, 2, 8, HEAD_DIM, seed=5)
    with pytest.raises(RuntimeError, match="must be fp16"):
        flashattn_cuda.prefill(q.float(), q.float(), q.float(), True, SCALE)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        flashattn_cuda.prefill(q.cpu(), q.cpu(), q.cpu(), True, SCALE)
    with pytest.raises(RuntimeError, match="must be 4-D"):
        flashattn_cuda.prefill(q[0], q[0], q[0], True, SCALE)
    with pytest.raises(RuntimeError, match="must be contiguous"):
        flashattn_cuda.prefill(q[:, :, ::2], q, q, True, SCALE)
    with pytest.raises(RuntimeError, match="head_dim"):
        bad = rand(1, 2, 8, 32)
        flashattn_cuda.prefill(bad, bad, bad, True, SCALE)
    with pytest.raises(RuntimeError, match="identical shapes"):
        flashattn_cuda.prefill(q, q[:, :, :4].contiguous(), q, True, SCALE)
    with pytest.raises(RuntimeError, match="scale must be finite"):
        flashattn_cuda.prefill(q, q, q, True, float("nan"))


def test_decode_rejects_bad_inputs():
    q = rand(1, 2, 1, HEAD_DIM, seed=6)
    cache = rand(1, 2, 8, HEAD_DIM)
    lens = torch.tensor([4], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="exactly one query row"):
        flashattn_cuda.decode(cache, cache, cache, lens, SCALE)
    with pytest.raises(RuntimeError, match="seq_lens must be int32"):
        flashattn_cuda.decode(q, cache, cache, lens.long(), SCALE)
    with pytest.raises(RuntimeError, match="seq_lens must be 1-D"):
        flashattn_cuda.decode(q, cache, cache, lens.repeat(3), SCALE)
    with pytest.raises(RuntimeError, match="identical shapes"):
        flashattn_cuda.decode(q, cache, cache[:, :, :4].contiguous(), lens, SCALE)
    with pytest.raises(RuntimeError, match="multiple of the warp count"):
        flashattn_cuda._decode_with_split(q, cache, cache, lens, SCALE, 6)


def test_occupancy_report_rows():
    rows = flashattn_cuda.occupancy_report()
    names = {r["kernel"] for r in rows}
    assert {"prefill_kernel", "decode_kernel", "merge_kernel"} <= names
    for r in rows:
        assert set(r) == {"kernel", "threads_per_block", "registers_per_thread",
                          "shared_bytes_per_block", "max_active_blocks_per_sm",
                          "theoretical_occupancy"}
        assert r["max_active_blocks_per_sm"] >= 1
    by = {r["kernel"]: r for r in rows}
    # the paired prefill form fills an SM (all registers, 512 tensor-memory
    # columns); the solo form is sized for two per SM (half of each), which
    # the occupancy API reports as 1 for kernels that allocate tensor
    # memory, although two run side by side (per-CTA SM stamps on a B200)
    assert by["prefill_kernel"]["max_active_blocks_per_sm"] == 1
    assert by["prefill_solo_kernel"]["registers_per_thread"] <= 128
    assert by["prefill_solo_kernel"]["shared_bytes_per_block"] * 2 + 2048 <= 228 * 1024


def test_prefill_causal_single_key_rows_are_exact():
    """Causal row 0 attends to key 0 only, so its output is v[0] exactly
    whatever the logits (regression: a row-max that read past the 128
    columns of the S tile made P != 1 there)."""
    torch.manual_seed(2256)
    q = rand(2, 12, 256, HEAD_DIM)
    k = rand(2, 12, 256, HEAD_DIM)
    v = (torch.randn(2, 12, 256, HEAD_DIM, device="cuda") * 3).half()
    out = flashattn_cuda.prefill(q, k, v, True, SCALE)
    assert torch.equal(out[:, :, 0], v[:, :, 0])
    # every query tile's first row attends to a full prefix; the last row of
    # a non-causal single-key sequence too
    one = flashattn_cuda.prefill(q[:, :, :1].contiguous(), k[:, :, :1].contiguous(),
                                 v[:, :, :1].contiguous(), False, SCALE)
    assert torch.equal(one[:, :, 0], v[:, :, 0])
