"""The CPU oracle pinned against the reference's own outputs (no GPU).

The golden vectors in tests/golden/golden.npz were produced from the
reference's src/attention_cpu.py and the oracles of its
tests/test_correctness.py (see tests/golden/make_golden.py). Both oracle
restatements (numpy and C) must reproduce them before they are trusted as
the checker of the GPU kernels.
"""

import os

import numpy as np
import pytest

import oracle
from golden.make_golden import (C1, DECODE_CASES, HEAD_DIM, PREFILL_CASES,
                                SCALE, inputs)

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
ORACLE_TOL = 2e-5  # fp32 reference path vs fp64 oracle on the same inputs


@pytest.mark.parametrize("case", PREFILL_CASES, ids=[c[0] for c in PREFILL_CASES])
@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_prefill_oracle_matches_reference(case, impl):
    name, b, h, n, causal, seed = case
    q, k, v = inputs((b, h, n, HEAD_DIM), seed)
    fn = oracle.prefill_ref if impl == "numpy" else oracle.prefill_c
    got = fn(q, k, v, causal, SCALE)
    np.testing.assert_allclose(got, GOLDEN[name + "_sdpa"], atol=ORACLE_TOL, rtol=0)
    if not causal:
        np.testing.assert_allclose(got, GOLDEN[name + "_cpu"], atol=ORACLE_TOL,
                                   rtol=0)


@pytest.mark.parametrize("case", DECODE_CASES, ids=[c[0] for c in DECODE_CASES])
@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_decode_oracle_matches_reference(case, impl):
    name, b, h, s_max, lens, seed = case
    q = inputs((b, h, 1, HEAD_DIM), seed, 1)[0]
    k, v = inputs((b, h, s_max, HEAD_DIM), seed + 1000, 2)
    fn = oracle.decode_ref if impl == "numpy" else oracle.decode_c
    got = fn(q, k, v, np.array(lens, dtype=np.int32), SCALE)
    # The reference's decode_reference casts its fp32 result to fp16
    # (tests/test_correctness.py:43), so the golden values are fp16-rounded:
    # the oracle, rounded the same way, must agree to one fp16 ulp.
    gold = GOLDEN[name + "_ref"]
    ulp = np.spacing(np.abs(gold).astype(np.float16)).astype(np.float32)
    diff = np.abs(got.astype(np.float16).astype(np.float32) - gold)
    assert np.all(diff <= ulp), float((diff - ulp).max())


def test_c1_config_oracle():
    """BASELINE config 1 (B2 H12 N256 causal + decode of the last token)."""
    _, b, h, n, seed = C1
    q, k, v = inputs((b, h, n, HEAD_DIM), seed)
    full = oracle.prefill_c(q, k, v, True, SCALE)
    rows = GOLDEN["c1_prefill_rows"]
    np.testing.assert_allclose(full[:, :, rows], GOLDEN["c1_prefill"],
                               atol=ORACLE_TOL, rtol=0)
    last = oracle.decode_c(q[:, :, n - 1:n], k, v,
                           np.full(b, n, dtype=np.int32), SCALE)
    np.testing.assert_allclose(last, GOLDEN["c1_decode_last"], atol=ORACLE_TOL,
                               rtol=0)
    # decode of token t == causal prefill row t (reference
    # tests/test_correctness.py:94-110), inside the oracle itself.
    np.testing.assert_allclose(last[:, :, 0], full[:, :, n - 1], atol=1e-6, rtol=0)


def test_oracle_decode_equals_causal_prefill_rows():
    q, k, v = inputs((1, 2, 70, HEAD_DIM), 5)
    full = oracle.prefill_c(q, k, v, True, SCALE)
    for t in (0, 1, 33, 69):
        d = oracle.decode_c(q[:, :, t:t + 1], k, v, np.array([t + 1], np.int32),
                            SCALE)
        np.testing.assert_allclose(d[:, :, 0], full[:, :, t], atol=1e-6, rtol=0)


def test_oracle_edge_rules():
    """seq_lens clamp (decode.cu:69) and empty -> 0 (decode.cu:164-172)."""
    q = inputs((3, 1, 1, HEAD_DIM), 9, 1)[0]
    k, v = inputs((3, 1, 8, HEAD_DIM), 10, 2)
    lens = np.array([0, -3, 50], dtype=np.int32)
    got = oracle.decode_c(q, k, v, lens, SCALE)
    assert np.all(got[0] == 0) and np.all(got[1] == 0)
    full = oracle.decode_c(q[2:], k[2:], v[2:], np.array([8], np.int32), SCALE)
    np.testing.assert_array_equal(got[2:], full)


def test_oracle_softmax_invariances():
    """Shift invariance of softmax and convexity of the output."""
    q, k, v = inputs((1, 1, 40, HEAD_DIM), 3)
    o = oracle.prefill_ref(q, k, v, False, SCALE)
    vf = v.astype(np.float32)
    o_shift = oracle.prefill_ref(q, k, vf + 1.0, False, SCALE)
    np.testing.assert_allclose(o_shift, o + 1.0, atol=1e-6)
    assert np.all(o <= vf.max(axis=2, keepdims=True) + 1e-6)
    assert np.all(o >= vf.min(axis=2, keepdims=True) - 1e-6)
