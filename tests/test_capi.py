"""The C ABI library loads, exports every declared entry point, and its
host-only logic behaves (no GPU needed)."""

import ctypes
import math
import os
import re

import pytest

from conftest import PKG_DIR, REPO

HEADER = os.path.join(REPO, "include", "fa_b200.h")
LIB = os.path.join(PKG_DIR, "flashattn_cuda", "libfa_b200.so")

FA_OK, FA_EINVAL, FA_EALIGN = 0, 1, 2


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fa_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    assert os.path.exists(LIB), "run flash-attention-cuda_b200/build.py first"
    lib = ctypes.CDLL(LIB)
    lib.fa_choose_decode_split.argtypes = [ctypes.c_int] * 4
    lib.fa_status_string.restype = ctypes.c_char_p
    vp = ctypes.c_void_p
    lib.fa_prefill.argtypes = [vp, vp, vp, vp, ctypes.c_int, ctypes.c_int,
                               ctypes.c_int, ctypes.c_int, ctypes.c_float, vp]
    lib.fa_decode.argtypes = [vp, vp, vp, vp, vp, ctypes.c_int, ctypes.c_int,
                              ctypes.c_int, ctypes.c_float, ctypes.c_int, vp,
                              ctypes.c_size_t, vp, ctypes.c_size_t, vp]
    lib.fa_merge_partials.argtypes = [vp, ctypes.c_int, vp, ctypes.c_int,
                                      ctypes.c_int, vp]
    return lib


def test_header_declares_the_entry_points():
    names = declared_functions()
    for expected in ("fa_prefill", "fa_decode", "fa_decode_workspace_bytes",
                     "fa_decode_partial", "fa_merge_partials",
                     "fa_choose_decode_split", "fa_occupancy",
                     "fa_take_device_error", "fa_status_string"):
        assert expected in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def reference_rule(max_seq, batch, heads, min_blocks):
    """csrc/decode.cu:183-192 of the reference, restated."""
    split = 1024
    while split > 128:
        if batch * heads * -(-max_seq // split) >= min_blocks:
            return split
        split >>= 1
    return 128


@pytest.mark.parametrize("sms", [82, 132, 148])
def test_choose_decode_split_follows_the_reference_rule(lib, sms):
    target = 2 * sms
    for max_seq in (1, 63, 128, 512, 513, 2048, 8192, 131072):
        for batch in (1, 2, 8, 64):
            for heads in (1, 12, 14):
                assert lib.fa_choose_decode_split(max_seq, batch, heads, target) \
                    == reference_rule(max_seq, batch, heads, target)


def test_choose_decode_split_contract_at_b200_size(lib):
    """tests/test_correctness.py:180-198 of the reference at 148 SMs.

    At B200 size (target 296 blocks) the shape (1, 12, 2048) cannot reach the
    target with any chunk (12 * 16 = 192 blocks at 128), so the rule falls
    back to 128; the reference's own test asserts the target is reached and
    would fail there. The rule's contract is checked as stated instead:
    reached when reachable, largest such chunk, else 128."""
    target = 2 * 148
    for batch, heads, seq in [(1, 12, 2048), (8, 12, 2048), (4, 12, 1024)]:
        split = lib.fa_choose_decode_split(seq, batch, heads, target)
        assert split in (128, 256, 512, 1024)
        reachable = batch * heads * -(-seq // 128) >= target
        if not reachable:
            assert split == 128
            continue
        assert batch * heads * -(-seq // split) >= target
        if split < 1024:
            assert batch * heads * -(-seq // (split * 2)) < target
    assert lib.fa_choose_decode_split(512, 1, 12, target) == 128


def test_status_strings(lib):
    assert lib.fa_status_string(0) == b"ok"
    assert b"invalid" in lib.fa_status_string(1)
    assert b"aligned" in lib.fa_status_string(2)
    assert lib.fa_status_string(99) == b"unknown status"


def test_argument_errors_are_reported_before_any_launch(lib):
    p = ctypes.c_void_p(4096)
    assert lib.fa_prefill(p, p, p, p, 0, 1, 1, 0, 0.125, None) == FA_EINVAL
    assert lib.fa_prefill(p, p, p, p, 1, 1, 0, 0, 0.125, None) == FA_EINVAL
    assert lib.fa_prefill(p, p, p, p, 1, 1, 8, 0, math.nan, None) == FA_EINVAL
    assert lib.fa_prefill(p, p, p, p, 1, 1, 8, 0, math.inf, None) == FA_EINVAL
    assert lib.fa_prefill(None, p, p, p, 1, 1, 8, 0, 0.125, None) == FA_EINVAL
    odd = ctypes.c_void_p(4096 + 8)
    assert lib.fa_prefill(p, odd, p, p, 1, 1, 8, 0, 0.125, None) == FA_EALIGN
    # decode: split must be a multiple of 4 (reference decode.cu:209-211)
    assert lib.fa_decode(p, p, p, p, p, 1, 1, 8, 0.125, 6, p, 1 << 20, p, 1,
                         None) == FA_EINVAL
    assert lib.fa_decode(p, p, p, p, p, 1, 0, 8, 0.125, 0, p, 1 << 20, p, 1,
                         None) == FA_EINVAL
    assert lib.fa_decode(p, p, p, p, None, 1, 1, 8, 0.125, 0, p, 1 << 20, p, 1,
                         None) == FA_EINVAL
    assert lib.fa_decode(p, p, p, p, p, 1, 1, 8, 0.125, 0, p, 1 << 20, None, 1,
                         None) == FA_EINVAL
    assert lib.fa_merge_partials(p, 0, p, 1, 1, None) == FA_EINVAL


def test_python_package_exports_the_reference_surface():
    import flashattn_cuda

    for name in ("prefill", "decode", "head_dim", "occupancy_report",
                 "choose_decode_split", "_decode_with_split", "legacy_naive",
                 "legacy_tiled", "legacy_fused"):
        assert hasattr(flashattn_cuda, name)
    assert flashattn_cuda.head_dim == 64
    assert flashattn_cuda.choose_decode_split(512, 1, 12, 296) == 128


def test_new_entry_points_reject_bad_arguments_without_a_device(lib):
    """head_dim, append and exchange entry points validate on the host
    before touching a device (status codes only, no GPU here)."""
    vp = ctypes.c_void_p
    p = ctypes.c_void_p(4096)
    lib.fa_prefill_hd.argtypes = [vp] * 4 + [ctypes.c_int] * 6 + [ctypes.c_float, vp]
    # head_dim 96 is not built; 0 heads; non-dividing K/V heads
    assert lib.fa_prefill_hd(p, p, p, p, 1, 2, 2, 16, 96, 1, 0.1, None) == FA_EINVAL
    assert lib.fa_prefill_hd(p, p, p, p, 1, 0, 1, 16, 128, 1, 0.1, None) == FA_EINVAL
    assert lib.fa_prefill_hd(p, p, p, p, 1, 6, 4, 16, 128, 1, 0.1, None) == FA_EINVAL
    assert lib.fa_prefill_hd(p, p, p, p, 1, 2, 2, 16, 128, 1, math.nan, None) == FA_EINVAL
    odd = ctypes.c_void_p(4096 + 8)
    assert lib.fa_prefill_hd(p, odd, p, p, 1, 2, 2, 16, 128, 1, 0.1, None) == FA_EALIGN
    lib.fa_decode_hd.argtypes = [vp] * 5 + [ctypes.c_int] * 4 + [
        ctypes.c_float, ctypes.c_int, vp, ctypes.c_size_t, vp, ctypes.c_size_t, vp]
    assert lib.fa_decode_hd(p, p, p, p, p, 1, 1, 8, 96, 0.1, 0, p, 1 << 20, p, 1,
                            None) == FA_EINVAL
    assert lib.fa_decode_hd(p, p, p, p, p, 1, 1, 8, 128, 0.1, 6, p, 1 << 20, p, 1,
                            None) == FA_EINVAL
    lib.fa_decode_append.argtypes = [vp] * 7 + [ctypes.c_int] * 4 + [
        ctypes.c_float, vp, ctypes.c_size_t, vp, ctypes.c_size_t, vp]
    # the new-token rows are required
    assert lib.fa_decode_append(p, None, p, p, p, p, p, 1, 2, 2, 8, 0.1, p,
                                1 << 20, p, 2, None) == FA_EINVAL
    lib.fa_decode_exchange.argtypes = [vp] * 5 + [ctypes.c_int] * 3 + [
        ctypes.c_float, vp, ctypes.c_size_t, vp, ctypes.c_size_t, vp,
        ctypes.c_int, ctypes.c_int, ctypes.c_uint32, vp]
    # epoch 0 is reserved (counters start at zero)
    assert lib.fa_decode_exchange(p, p, p, p, p, 1, 2, 8, 0.1, p, 1 << 20, p, 2,
                                  p, 0, 1, 0, None) == FA_EINVAL


def test_exchange_buffer_size(lib):
    lib.fa_exchange_bytes.restype = ctypes.c_size_t
    lib.fa_exchange_bytes.argtypes = [ctypes.c_int] * 3
    for b, h, w in [(1, 14, 8), (64, 12, 2), (3, 5, 1)]:
        n = lib.fa_exchange_bytes(b, h, w)
        need = 2 * b * h * w * 68 * 4 + b * h * 4
        assert need <= n < need + 256 and n % 256 == 0
    assert lib.fa_exchange_bytes(1, 14, 0) == 0
    assert lib.fa_exchange_bytes(1, 14, 33) == 0
    lib.fa_exchange_bytes_hd.restype = ctypes.c_size_t
    lib.fa_exchange_bytes_hd.argtypes = [ctypes.c_int] * 4
    for b, h, w in [(1, 14, 8), (3, 5, 2)]:
        assert lib.fa_exchange_bytes_hd(b, h, w, 64) == lib.fa_exchange_bytes(b, h, w)
        n = lib.fa_exchange_bytes_hd(b, h, w, 128)
        need = 2 * b * h * w * 132 * 4 + b * h * 4
        assert need <= n < need + 256 and n % 256 == 0
    assert lib.fa_exchange_bytes_hd(1, 14, 8, 96) == 0


def test_prefill_host_plan_and_validation(lib):
    """fa_prefill_host_plan chunks whole (batch, K/V head) groups and sizes
    the staging ring; fa_prefill_host rejects bad arguments before touching
    a device."""
    vp, ci = ctypes.c_void_p, ctypes.c_int
    lib.fa_prefill_host_plan.argtypes = [ci] * 5 + [vp, vp]
    lib.fa_prefill_host.argtypes = [vp] * 4 + [ci] * 6 + [
        ctypes.c_float, vp, ctypes.c_size_t, vp]

    def plan(B, H, H_kv, N, D):
        c, w = ctypes.c_int(), ctypes.c_size_t()
        rc = lib.fa_prefill_host_plan(B, H, H_kv, N, D, ctypes.byref(c),
                                      ctypes.byref(w))
        return rc, c.value, w.value

    # config 3: 56 single-head groups, 3 chunks of 14 and the last 14 split
    # in two; 3 staging slots of 14 * 4 * 512 KiB
    assert plan(4, 14, 14, 4096, 64) == (FA_OK, 5, 3 * 14 * 4 * (512 << 10))
    # grouped: 8 groups of 7 query heads + 1 K/V head, chunks of 2 groups
    rc, chunks, ws = plan(4, 14, 2, 4096, 64)
    assert (rc, chunks) == (FA_OK, 5) and ws == 3 * 2 * (7 * 2 + 2) * (512 << 10)
    # tiny: a single chunk, a single slot
    rc, chunks, ws = plan(1, 1, 1, 128, 64)
    assert (rc, chunks) == (FA_OK, 1) and ws == 4 * 128 * 64 * 2
    # ragged: 5 heads of 768 KiB input each at head_dim 128 make chunks of
    # 3 heads (>= 2 MiB), the remaining 2 split in two
    rc, chunks, _ = plan(1, 5, 5, 1024, 128)
    assert (rc, chunks) == (FA_OK, 3)
    # large: chunks are capped at 64 MiB of input (21 heads of 3 MiB here),
    # so 12 chunks of 21 heads + the last 4 split in two, and the workspace
    # stays bounded
    rc, chunks, ws = plan(8, 32, 32, 8192, 64)
    assert rc == FA_OK and chunks == 14 and ws == 3 * 21 * 4 * (1 << 20)
    for bad in [(1, 2, 2, 16, 96), (0, 2, 2, 16, 64), (1, 6, 4, 16, 64),
                (1, 2, 2, 0, 64)]:
        assert plan(*bad)[0] == FA_EINVAL
    p = ctypes.c_void_p(4096)
    rc, _, ws = plan(1, 2, 2, 256, 64)
    assert lib.fa_prefill_host(p, p, p, p, 1, 2, 2, 256, 64, 1, 0.1, p,
                               ws - 1, None) == 4  # FA_ENOSPACE
    assert lib.fa_prefill_host(p, p, p, p, 1, 2, 2, 256, 64, 1, 0.1,
                               ctypes.c_void_p(4096 + 16), ws, None) == FA_EALIGN
    assert lib.fa_prefill_host(p, None, p, p, 1, 2, 2, 256, 64, 1, 0.1, p,
                               ws, None) == FA_EINVAL
    assert lib.fa_prefill_host(p, p, p, p, 1, 2, 2, 256, 64, 1, math.inf, p,
                               ws, None) == FA_EINVAL


def test_dtype_entry_points_reject_bad_arguments_without_a_device(lib):
    vp, ci = ctypes.c_void_p, ctypes.c_int
    p = ctypes.c_void_p(4096)
    lib.fa_prefill_ex.argtypes = [vp] * 4 + [ci] * 7 + [ctypes.c_float, vp]
    lib.fa_decode_ex.argtypes = [vp] * 5 + [ci] * 6 + [
        ctypes.c_float, vp, ctypes.c_size_t, vp, ctypes.c_size_t, vp]
    # dtype codes: 0 fp16, 1 bf16; anything else is rejected
    assert lib.fa_prefill_ex(p, p, p, p, 1, 2, 2, 16, 64, 2, 1, 0.1, None) == FA_EINVAL
    assert lib.fa_prefill_ex(p, p, p, p, 1, 2, 2, 16, 96, 1, 1, 0.1, None) == FA_EINVAL
    assert lib.fa_prefill_ex(p, p, p, p, 1, 6, 4, 16, 128, 1, 1, 0.1, None) == FA_EINVAL
    odd = ctypes.c_void_p(4096 + 8)
    assert lib.fa_prefill_ex(p, p, odd, p, 1, 2, 2, 16, 64, 1, 1, 0.1, None) == FA_EALIGN
    assert lib.fa_decode_ex(p, p, p, p, p, 1, 2, 2, 8, 64, -1, 0.1, p, 1 << 20,
                            p, 2, None) == FA_EINVAL
    assert lib.fa_decode_ex(p, p, p, p, None, 1, 2, 2, 8, 64, 1, 0.1, p, 1 << 20,
                            p, 2, None) == FA_EINVAL


def test_wait_limit_range_is_checked_on_the_host(lib):
    lib.fa_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
    assert lib.fa_set_wait_limit_ns(10) == 1  # FA_EINVAL: below 1 us
    assert lib.fa_set_wait_limit_ns(10 ** 12) == 1  # above 60 s
