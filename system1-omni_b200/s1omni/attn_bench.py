"""Micro-benchmark of cs1_attention_gated_batch of an ABI-9 library.

    cd system1-omni_b200 && python -m s1omni.attn_bench --lengths 4096 [--hq 24 --hk 4]
        [--lib PATH] [--reps 10] [--once]

Packed sequences of the given lengths (comma-separated; `bench32` is the bench's batch of 32
prompts), head dim 256, gated, causal.
Times `reps` calls with CUDA events on the calling stream after three warm-up calls and
prints one JSON line: TFLOP/s at the causal algorithmic count 4*Hq*256*sum(T(T+1)/2)
(QK^T and PV). `--once` makes exactly one call (for a profiler capture). Works with any
library exporting the ABI (this build's, or a build of the reference's sources, which
accepts at most 16 sequences per call).
"""
import argparse
import json

import numpy as np
import torch

from .cs1 import Cs1


def flops(lengths, hq, dh=256):
    return 4.0 * hq * dh * sum(t * (t + 1) / 2 for t in lengths)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--lib", default=None)
    ap.add_argument("--lengths", default="4096")
    ap.add_argument("--hq", type=int, default=24)
    ap.add_argument("--hk", type=int, default=4)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--once", action="store_true")
    a = ap.parse_args()
    lib = Cs1(a.lib)
    if a.lengths == "bench32":  # the bench's batch of 32 prompts
        import os
        import sys
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
        import bench
        lengths = [len(r) for r in bench.pool(32)]
    else:
        lengths = [int(x) for x in a.lengths.split(",")]
    T, Hq, Hk, D = sum(lengths), a.hq, a.hk, 256
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(T, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(T, Hk, D, device="cuda", generator=g).to(torch.bfloat16)
    ldv = Hk * D + 64  # V read from a wider row, as from the stacked projection output
    v = torch.randn(T, ldv, device="cuda", generator=g).to(torch.bfloat16)
    gate = torch.randn(T, Hq, D, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(T, Hq, D, device="cuda", dtype=torch.bfloat16)
    lens = np.asarray(lengths, dtype=np.uintp)
    stream = torch.cuda.current_stream().cuda_stream
    scale = D ** -0.5

    def call():
        lib.cs1_attention_gated_batch(q, k, v, ldv, gate, out, lens.ctypes.data, len(lengths), Hq, Hk, D, scale,
                                      stream)

    if a.once:
        call()
        torch.cuda.synchronize()
        print(json.dumps({"lengths": lengths, "hq": Hq, "hk": Hk, "calls": 1}))
        return
    for _ in range(3):
        call()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(a.reps):
        call()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / a.reps
    print(json.dumps({"lengths": lengths if len(lengths) <= 8 else f"{len(lengths)} sequences, {T} tokens",
                      "hq": Hq, "hk": Hk, "ms": ms, "tflops": flops(lengths, Hq) / ms / 1e9,
                      "finite": bool(torch.isfinite(out.float()).all()), "lib": lib.path}))


if __name__ == "__main__":
    main()
