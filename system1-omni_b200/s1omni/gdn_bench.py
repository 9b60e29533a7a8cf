"""Micro-benchmark of the bf16 GDN prefill of an ABI-9 library.

    cd system1-omni_b200 && python -m s1omni.gdn_bench --lengths 936 [--h 48 --hk 16]
        [--lib PATH] [--reps 10] [--once]

Packed sequences of the given lengths (comma-separated; `bench32` is the bench's batch of
32 prompts), head dim 128: one `cs1_gdn_prefill_batch_x` call over all of them when the
library has it, else one `cs1_gdn_prefill` per sequence (the reference library: its batched
entry point takes at most 16 sequences). Inputs q, k, v ~ N(0,1), g ~ -U(0, 0.25),
beta ~ U(0,1), seeded. Times `reps` calls with CUDA events on the calling stream after
three warm-up calls and prints one JSON line with the fraction of the HBM bound (q, k,
v, o, g and beta bytes once, against the measured copy bandwidth of MEASURED_PEAKS.json).
`--once` makes exactly one call (for a profiler capture).
"""
import argparse
import ctypes
import json
import os

import numpy as np
import torch

from .cs1 import Cs1


def hbm_gbs():
    """The measured copy bandwidth (MEASURED_PEAKS.json at the repository root), else the
    pool's earlier measurement."""
    try:
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def algorithmic_bytes(T, H, HK, d=128):
    return T * (2 * HK * d * 2 + 2 * H * d * 2 + H * 4 + H * 2)


def bench32():
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    import bench
    return [len(r) for r in bench.pool(32)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--lib", default=None)
    ap.add_argument("--lengths", default="936")
    ap.add_argument("--h", type=int, default=48)
    ap.add_argument("--hk", type=int, default=16)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--once", action="store_true")
    a = ap.parse_args()
    lib = Cs1(a.lib)
    lengths = bench32() if a.lengths == "bench32" else [int(x) for x in a.lengths.split(",")]
    T, H, HK, D = sum(lengths), a.h, a.hk, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(T, HK, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(T, HK, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(T, H, D, device="cuda", generator=g).to(torch.bfloat16)
    gl = -torch.rand(T, H, device="cuda", generator=g) * 0.25
    beta = torch.rand(T, H, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty(T, H, D, device="cuda", dtype=torch.bfloat16)
    lens = np.asarray(lengths, dtype=np.uintp)
    stream = torch.cuda.current_stream().cuda_stream
    scale = ctypes.c_float(D ** -0.5)
    batched = "cs1_gdn_prefill_batch_x" not in lib.missing
    nws = lib.cs1_gdn_workspace_floats(max(lengths), H) if not batched else 64
    ws = torch.empty(nws, dtype=torch.float32, device="cuda")
    offs = np.concatenate([[0], np.cumsum(lengths)])

    def call():
        if batched:
            rc = lib.raw.cs1_gdn_prefill_batch_x(q.data_ptr(), k.data_ptr(), v.data_ptr(), gl.data_ptr(),
                                                 beta.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel() * 4,
                                                 lens.ctypes.data, len(lengths), H, HK, scale, None, 0, None, stream)
            assert rc == 0, rc
            return
        for i, L in enumerate(lengths):
            o = int(offs[i])
            rc = lib.raw.cs1_gdn_prefill(q.data_ptr() + o * HK * D * 2, k.data_ptr() + o * HK * D * 2,
                                         v.data_ptr() + o * H * D * 2, gl.data_ptr() + o * H * 4,
                                         beta.data_ptr() + o * H * 2, out.data_ptr() + o * H * D * 2, ws.data_ptr(),
                                         L, H, HK, scale, stream)
            assert rc == 0, rc

    if a.once:
        call()
        torch.cuda.synchronize()
        print(json.dumps({"lengths": lengths if len(lengths) <= 8 else f"{len(lengths)} sequences, {T} tokens",
                          "h": H, "hk": HK, "calls": 1}))
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
    byt = algorithmic_bytes(T, H, HK)
    print(json.dumps({"lengths": lengths if len(lengths) <= 8 else f"{len(lengths)} sequences, {T} tokens",
                      "h": H, "hk": HK, "ms": ms, "gbs": byt / ms / 1e6, "frac_hbm": byt / ms / 1e6 / hbm_gbs(),
                      "finite": bool(torch.isfinite(out.float()).all()), "lib": lib.path}))


if __name__ == "__main__":
    main()
