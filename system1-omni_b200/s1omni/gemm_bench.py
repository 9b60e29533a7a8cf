"""Micro-benchmark of the cs1_gemm entry points of an ABI-9 library.

    cd system1-omni_b200 && python -m s1omni.gemm_bench --m 2048 --n 16480 --k 5120 [--lib PATH]
        [--epi store|residual|swiglu] [--reps 10] [--once]

Times `reps` calls with CUDA events on the calling stream after three warm-up calls and
prints one JSON line (TFLOP/s at 2*M*N*K). `--once` makes exactly one call (for a
profiler capture). Works with any library exporting the cs1_gemm ABI (this build's, or a
build of the reference's sources).
"""
import argparse
import json

import torch

from .cs1 import Cs1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--lib", default=None)
    ap.add_argument("--m", type=int, required=True)
    ap.add_argument("--n", type=int, required=True)
    ap.add_argument("--k", type=int, required=True)
    ap.add_argument("--epi", default="store", choices=["store", "residual", "swiglu"])
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--once", action="store_true")
    a = ap.parse_args()
    lib = Cs1(a.lib)
    M, N, K = a.m, a.n, a.k
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    out_n = N // 2 if a.epi == "swiglu" else N
    y = torch.zeros(M, out_n, device="cuda", dtype=torch.bfloat16)
    h = lib.cs1_gemm_create(32 << 20)
    stream = torch.cuda.current_stream().cuda_stream

    def call():
        if a.epi == "swiglu":
            lib.cs1_gemm_swiglu(h, x, w, y, M, N // 2, K, out_n, stream)
        elif a.epi == "residual":
            lib.cs1_gemm_residual(h, x, w, y, M, N, K, out_n, stream)
        else:
            lib.cs1_gemm(h, x, w, y, M, N, K, out_n, stream)

    if a.once:
        call()
        torch.cuda.synchronize()
        print(json.dumps({"m": M, "n": N, "k": K, "epi": a.epi, "calls": 1}))
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
    lib.cs1_gemm_destroy(h)
    print(json.dumps({"m": M, "n": N, "k": K, "epi": a.epi, "ms": ms, "tflops": 2.0 * M * N * K / ms / 1e9,
                      "lib": lib.path}))


if __name__ == "__main__":
    main()
