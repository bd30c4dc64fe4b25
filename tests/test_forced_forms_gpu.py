"""Every prefill CTA form, forced, against fp32 attention. The launch rule
picks one form per grid, so some forms are reached by few shapes (the
key-split form only by small causal grids; the 64-key head_dim-128 form by
none since the 128-key form replaced it). The measurement overrides
FA_PREFILL_FORM (head_dim 64: paired, solo, split) and FA_PREFILL_D128_FORM
(head_dim 128: paired) are read once per process, so each case runs in a
child process on the same GPU."""

import json
import os
import subprocess
import sys

import pytest

from conftest import PKG_DIR, requires_gpu

pytestmark = [pytest.mark.gpu, requires_gpu]

CHILD = r'''
import json, sys, torch
import flashattn_cuda as fa
out = {}
for (b, h, h_kv, n, d, causal, dt) in json.loads(sys.argv[1]):
    dtype = torch.bfloat16 if dt == "bf16" else torch.float16
    torch.manual_seed(b * 1000 + h * 10 + n + d)
    q = torch.randn(b, h, n, d, device="cuda").to(dtype)
    k = torch.randn(b, h_kv, n, d, device="cuda").to(dtype)
    v = torch.randn(b, h_kv, n, d, device="cuda").to(dtype)
    scale = d ** -0.5
    got = fa.prefill(q, k, v, bool(causal), scale)
    g = h // h_kv
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float().repeat_interleave(g, 1),
        v.float().repeat_interleave(g, 1), is_causal=bool(causal), scale=scale)
    out[str((b, h, h_kv, n, d, causal, dt))] = (got.float() - ref).abs().max().item()
out["device_error"] = fa.take_device_error()
print(json.dumps(out))
'''

# (b, h, h_kv, n, d, causal, dtype)
CASES = [
    (1, 3, 3, 1000, 64, 1, "f16"), (2, 5, 5, 777, 64, 0, "f16"),
    (1, 7, 1, 2048, 64, 1, "f16"), (2, 4, 2, 513, 64, 1, "bf16"),
    (1, 2, 2, 129, 64, 1, "f16"), (1, 1, 1, 1, 64, 1, "f16"),
]
CASES_D128 = [
    (1, 3, 3, 1000, 128, 1, "f16"), (2, 4, 2, 777, 128, 0, "f16"),
    (1, 2, 2, 2048, 128, 1, "bf16"),
]


def run_child(env_extra, cases):
    env = dict(os.environ)
    env.update(env_extra)
    env["PYTHONPATH"] = PKG_DIR + os.pathsep + env.get("PYTHONPATH", "")
    res = subprocess.run([sys.executable, "-c", CHILD, json.dumps(cases)],
                         env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    return json.loads(res.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("form", ["paired", "solo", "split"])
def test_forced_head_dim_64_form_matches_fp32(form):
    out = run_child({"FA_PREFILL_FORM": form}, CASES)
    assert out.pop("device_error") == 0
    for case, err in out.items():
        tol = 1.5e-2 if "bf16" in case else 2e-3
        assert err <= tol, (form, case, err)


def test_forced_head_dim_128_paired_form_matches_fp32():
    out = run_child({"FA_PREFILL_D128_FORM": "paired"}, CASES_D128)
    assert out.pop("device_error") == 0
    for case, err in out.items():
        tol = 1.5e-2 if "bf16" in case else 2e-3
        assert err <= tol, (case, err)
