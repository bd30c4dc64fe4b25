"""Fixed workloads for profiling one kernel under ncu.

    python flash-attention-cuda_b200/profile_workload.py --case prefill_c3
    ncu --set full --clock-control none -k regex:prefill_kernel -s 2 -c 1 \
        python flash-attention-cuda_b200/profile_workload.py --case prefill_c3

Each case runs `--iters` launches of one kernel on seeded synthetic inputs
(the BASELINE configurations); the first launches are warm-up, so skip them
with ncu's -s. Inputs stay well under a few GB of device memory.
"""

import argparse
import math
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import flashattn_cuda as fa  # noqa: E402

SCALE = 1.0 / math.sqrt(64)

CASES = {
    # name: (kind, shape, causal, K/V heads (None: as many as query heads))
    "prefill_c3": ("prefill", (4, 14, 4096), True, None),
    "prefill_c2_causal": ("prefill", (8, 12, 1024), True, None),
    "prefill_c2_full": ("prefill", (8, 12, 1024), False, None),
    "prefill_small": ("prefill", (1, 8, 2048), True, None),
    # one GPU's share of config 3 on eight GPUs: key-split form
    "prefill_c3_shard8": ("prefill", (1, 7, 4096), True, None),
    # two heads per CTA: one query tile each (N <= 128), and three tiles
    "prefill_pairs_n128": ("prefill", (64, 32, 128), True, None),
    "prefill_pairs_n384": ("prefill", (64, 32, 384), True, None),
    "prefill_d128_pairs_n128": ("prefill_d128", (64, 32, 128), True, None),
    # config 3's shape at head_dim 128
    "prefill_d128_c3": ("prefill_d128", (4, 14, 4096), True, None),
    "decode_c4": ("decode", (64, 12, 8192), None, None),
    "decode_c5": ("decode", (1, 14, 131072), None, None),
    # Qwen2.5-0.5B's real 2 K/V heads, and a wider grouped batch
    "decode_gqa_c5": ("decode", (1, 14, 131072), None, 2),
    "decode_gqa_b8": ("decode", (8, 32, 32768), None, 8),
    "decode_append_c4": ("decode_append", (64, 12, 8192), None, None),
    # head_dim 128: config 4 per head, and 32 query heads on 8 K/V heads
    "decode_d128_c4": ("decode_d128", (64, 12, 8192), None, None),
    "decode_gqa_d128_b8": ("decode_d128", (8, 32, 32768), None, 8),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=sorted(CASES), required=True)
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    kind, (b, h, n), causal, h_kv = CASES[args.case]
    h_kv = h_kv or h
    g = torch.Generator(device="cuda").manual_seed(0)
    if kind in ("prefill", "prefill_d128"):
        d = 128 if kind == "prefill_d128" else 64
        q, k, v = (torch.randn(b, h, n, d, generator=g, device="cuda",
                               dtype=torch.float16) for _ in range(3))
        fn = lambda: fa.prefill(q, k, v, causal, d ** -0.5)
    else:
        d = 128 if kind == "decode_d128" else 64
        q = torch.randn(b, h, 1, d, generator=g, device="cuda", dtype=torch.float16)
        k, v = (torch.randn(b, h_kv, n, d, generator=g, device="cuda",
                            dtype=torch.float16) for _ in range(2))
        cpu_gen = torch.Generator().manual_seed(0)
        if b > 1:
            lens = torch.randint(1, n + 1, (b,), generator=cpu_gen, dtype=torch.int32)
        else:
            lens = torch.full((b,), n, dtype=torch.int32)
        lens = lens.cuda()
        if kind == "decode_append":
            kn, vn = (torch.randn(b, h_kv, 1, 64, generator=g, device="cuda",
                                  dtype=torch.float16) for _ in range(2))
            lens = (lens - 1).contiguous()
            fn = lambda: fa.decode_append(q, kn, vn, k, v, lens, SCALE)
        else:
            fn = lambda: fa.decode(q, k, v, lens, d ** -0.5)
    for _ in range(args.iters):
        fn()
    torch.cuda.synchronize()
    assert fa.take_device_error() == 0
    print(f"{args.case}: {args.iters} launches ok")


if __name__ == "__main__":
    main()
