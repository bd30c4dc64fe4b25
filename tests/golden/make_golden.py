"""Generates the golden vectors in tests/golden/ from the reference itself.

Run where the reference checkout is available (its path in FA_REFERENCE);
the outputs are committed, so tests never need the reference at run time:

    FA_REFERENCE=/path/to/flash-attention-cuda python tests/golden/make_golden.py

Sources of truth, all taken from the reference's own code:
  * src/attention_cpu.py `attention_cpu` — the reference's CPU path
    (non-causal, one (N, d) head), imported from the checkout;
  * tests/test_correctness.py `sdpa_reference` and `decode_reference` — the
    oracles the reference's GPU tests compare against (fp32 torch SDPA and a
    per-sequence fp32 softmax loop). Their source is read from the test file
    and executed on CPU tensors (the test module itself imports the CUDA
    extension, so it is not imported).

Inputs are regenerated from the seeds below with numpy's PCG64 generator
(`inputs()`), so only outputs are stored.
"""

import ast
import importlib.util
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
HEAD_DIM = 64
SCALE = 1.0 / math.sqrt(HEAD_DIM)

# (name, B, H, N, causal, seed) prefill cases and decode cases.
PREFILL_CASES = [
    ("p_n1", 1, 1, 1, False, 11),
    ("p_n37", 1, 2, 37, False, 12),
    ("p_n128", 1, 1, 128, False, 13),
    ("p_n130_causal", 2, 3, 130, True, 14),
    ("p_n65_causal", 1, 5, 65, True, 15),
    ("p_n256_full", 1, 2, 256, False, 16),
]
# (name, B, H, S_max, seq_lens, seed)
DECODE_CASES = [
    ("d_ragged", 4, 3, 300, [1, 2, 150, 300], 21),
    ("d_clamp_empty", 3, 2, 64, [0, 64, 100], 22),
]
# B=2, H=12, N=256, causal, plus decode of the last token.
C1 = ("c1", 2, 12, 256, 31)


def inputs(shape, seed, count=3):
    """fp16 N(0,1) tensors from a seeded PCG64 stream (stable across numpy)."""
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
            for _ in range(count)]


def _load_reference(ref_root):
    spec = importlib.util.spec_from_file_location(
        "ref_attention_cpu", os.path.join(ref_root, "src", "attention_cpu.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    import torch
    src = open(os.path.join(ref_root, "tests", "test_correctness.py")).read()
    tree = ast.parse(src)
    wanted = {"sdpa_reference", "decode_reference"}
    fns = [n for n in tree.body
           if isinstance(n, ast.FunctionDef) and n.name in wanted]
    ns = {"torch": torch, "SCALE": SCALE}
    exec(compile(ast.Module(body=fns, type_ignores=[]), "test_correctness",
                 "exec"), ns)
    return mod.attention_cpu, ns["sdpa_reference"], ns["decode_reference"]


def main():
    import torch
    # $FA_REFERENCE, else a "reference" checkout beside this repository.
    here = os.path.dirname(os.path.abspath(__file__))
    ref_root = os.environ.get(
        "FA_REFERENCE",
        os.path.normpath(os.path.join(here, *[os.pardir] * 3, "reference")))
    attention_cpu, sdpa_reference, decode_reference = _load_reference(ref_root)
    out = {}

    for name, b, h, n, causal, seed in PREFILL_CASES:
        q, k, v = inputs((b, h, n, HEAD_DIM), seed)
        if not causal:
            # The reference's CPU path, head by head, in fp32 as it runs.
            o = np.empty((b, h, n, HEAD_DIM), dtype=np.float32)
            for bi in range(b):
                for hi in range(h):
                    o[bi, hi] = attention_cpu(
                        q[bi, hi].astype(np.float32), k[bi, hi].astype(np.float32),
                        v[bi, hi].astype(np.float32), SCALE)
            out[name + "_cpu"] = o
        # The reference tests' SDPA oracle, before its final .half() cast.
        t = [torch.from_numpy(x) for x in (q, k, v)]
        ref = torch.nn.functional.scaled_dot_product_attention(
            t[0].float(), t[1].float(), t[2].float(), is_causal=causal,
            scale=SCALE)
        out[name + "_sdpa"] = ref.numpy().astype(np.float32)

    for name, b, h, s_max, lens, seed in DECODE_CASES:
        q = inputs((b, h, 1, HEAD_DIM), seed, 1)[0]
        k, v = inputs((b, h, s_max, HEAD_DIM), seed + 1000, 2)
        lens_t = torch.tensor(lens, dtype=torch.int32)
        # decode_reference slices [:n] with n = seq_lens[b] (no clamp, and an
        # empty slice gives NaN from softmax over nothing); the reference
        # kernel clamps to S_max and writes 0 for empty rows
        # (csrc/decode.cu:69,164-172), so compute the oracle on the clamped
        # lengths and apply the empty rule.
        clamped = torch.clamp(lens_t, 0, s_max)
        tq, tk, tv = (torch.from_numpy(x) for x in (q, k, v))
        o = torch.zeros(b, h, 1, HEAD_DIM)
        nonempty = [i for i in range(b) if int(clamped[i]) > 0]
        if nonempty:
            idx = torch.tensor(nonempty)
            sub = decode_reference(tq[idx].float(), tk[idx], tv[idx],
                                   clamped[idx])
            o[idx] = sub.float()
        out[name + "_ref"] = o.numpy().astype(np.float32)

    name, b, h, n, seed = C1
    q, k, v = inputs((b, h, n, HEAD_DIM), seed)
    t = [torch.from_numpy(x).float() for x in (q, k, v)]
    full = torch.nn.functional.scaled_dot_product_attention(
        t[0], t[1], t[2], is_causal=True, scale=SCALE).numpy()
    rows = list(range(0, n, 8)) + [n - 1]
    out["c1_prefill_rows"] = np.array(rows, dtype=np.int32)
    out["c1_prefill"] = full[:, :, rows].astype(np.float32)
    last = np.empty((b, h, 1, HEAD_DIM), dtype=np.float32)
    for bi in range(b):
        for hi in range(h):
            last[bi, hi] = attention_cpu(
                q[bi, hi, n - 1:n].astype(np.float32),
                k[bi, hi].astype(np.float32), v[bi, hi].astype(np.float32),
                SCALE)
    out["c1_decode_last"] = last

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {sorted(out)}")


if __name__ == "__main__":
    sys.exit(main())
