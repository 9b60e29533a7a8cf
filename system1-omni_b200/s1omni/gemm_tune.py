"""Time every projection-GEMM kernel of libqwen3_5_cuda.so on the 27B projection shapes.

    cd system1-omni_b200 && python -m s1omni.gemm_tune [--m 300,771,2048] [--reps 10] [--lib PATH]

For each M and shape, one handle per kernel option (S1_GEMM_KERNEL = pair | row256 |
row128 | swap | swap2 with S1_GEMM_NT = 64..256, set before cs1_gemm_create) and the default
handle (the library's wave model); CUDA-event time per call after three warm-up calls.
Prints one JSON line per (M, shape) with every option's milliseconds, the fastest
option and the model's time. Used to calibrate the kernel choice.
"""
import argparse
import json
import os

import torch

from .cs1 import Cs1

SHAPES = [("swiglu", 34816, 5120), ("store", 16480, 5120), ("store", 14336, 5120), ("residual", 5120, 17408),
          ("residual", 5120, 6144)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", default="300,771,2048")
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--lib", default=None, help="another build of the library (default: this package's)")
    a = ap.parse_args()
    lib = Cs1(a.lib)
    st = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(0)
    opts = [("model", {}), ("pair", {"S1_GEMM_KERNEL": "pair"}), ("row256", {"S1_GEMM_KERNEL": "row256"}),
            ("row128", {"S1_GEMM_KERNEL": "row128"})]
    opts += [(f"swap{nt}", {"S1_GEMM_KERNEL": "swap", "S1_GEMM_NT": str(nt)}) for nt in (64, 96, 128, 160, 192, 224, 256)]
    opts += [(f"pswap{nt}", {"S1_GEMM_KERNEL": "swap2", "S1_GEMM_NT": str(nt)})
             for nt in range(64, 257, 16)]
    for M in [int(x) for x in a.m.split(",")]:
        for epi, N, K in SHAPES:
            x = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
            w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
            out_n = N // 2 if epi == "swiglu" else N
            y = torch.zeros(M, out_n, device="cuda", dtype=torch.bfloat16)
            res = {}
            for name, env in opts:
                if epi == "swiglu" and (name == "row128" or (name.startswith("swap") and int(name[4:]) > 128)):
                    continue
                for k in ("S1_GEMM_KERNEL", "S1_GEMM_NT"):
                    os.environ.pop(k, None)
                os.environ.update(env)
                h = lib.cs1_gemm_create(0)

                def call():
                    if epi == "swiglu":
                        lib.cs1_gemm_swiglu(h, x, w, y, M, N // 2, K, out_n, st)
                    elif epi == "residual":
                        lib.cs1_gemm_residual(h, x, w, y, M, N, K, out_n, st)
                    else:
                        lib.cs1_gemm(h, x, w, y, M, N, K, out_n, st)
                for _ in range(3):
                    call()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                s.record()
                for _ in range(a.reps):
                    call()
                e.record()
                torch.cuda.synchronize()
                res[name] = round(s.elapsed_time(e) / a.reps, 4)
                lib.cs1_gemm_destroy(h)
            for k in ("S1_GEMM_KERNEL", "S1_GEMM_NT"):
                os.environ.pop(k, None)
            best = min((v, k) for k, v in res.items() if k != "model")
            print(json.dumps({"m": M, "epi": epi, "n": N, "k": K, "best": best[1], "best_ms": best[0],
                              "model_ms": res["model"], "ms": res}), flush=True)


if __name__ == "__main__":
    main()
