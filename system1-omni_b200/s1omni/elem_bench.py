"""Bandwidth micro-benchmark of the HBM-bound cs1_* kernels at the 27B prefill shapes.

    cd system1-omni_b200 && python -m s1omni.elem_bench [--tokens 29122] [--lib PATH]
        [--reps 20] [--once]

For each op: CUDA-event time per call (after three warm-up calls, on the calling stream)
and the algorithmic bytes it must move (every input read once, every output written
once; weights and tables included), so GB/s = bytes / time and frac = GB/s / the measured
HBM peak of MEASURED_PEAKS.json (the profiling fallback 6650 GB/s without it). All
tensors exceed L2 (126 MB) at the default 29,122 tokens. `--once` calls every op once
(for a profiler capture). Prints one JSON line per op.
"""
import argparse
import ctypes
import json
import os

import torch

from .cs1 import Cs1

H, HK, HV, HQ, HKV = 5120, 16, 48, 24, 4
KEY, VAL = HK * 128, HV * 128          # 2048, 6144
GDN_IN = 2 * KEY + VAL + VAL + 2 * HV  # q k v | z | b a = 16480
ATTN_IN = HQ * 512 + 2 * HKV * 256      # q+gate | k | v = 14336


def peak():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=29122)
    ap.add_argument("--lib", default=None)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--once", action="store_true")
    a = ap.parse_args()
    lib = Cs1(a.lib)
    T = a.tokens
    dev = "cuda"
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).to(bf)

    st = torch.cuda.current_stream().cuda_stream
    x = rnd(T, H)
    w = rnd(H, scale=0.1)
    out = torch.empty(T, H, device=dev, dtype=bf)
    res = rnd(T, H)
    gdn_in = rnd(T, GDN_IN)
    conv_w = rnd(2 * KEY + VAL, 4, scale=0.3)
    q = torch.empty(T, KEY, device=dev, dtype=bf)
    k = torch.empty(T, KEY, device=dev, dtype=bf)
    v = torch.empty(T, VAL, device=dev, dtype=bf)
    o = rnd(T, HV, 128)
    gw = rnd(128, scale=0.1)
    go = torch.empty(T, HV * 128, device=dev, dtype=bf)
    attn_in = rnd(T, ATTN_IN)
    qw, kw = rnd(256, scale=0.1), rnd(256, scale=0.1)
    cos, sin = rnd(T, 32), rnd(T, 32)
    aq = torch.empty(T, HQ, 256, device=dev, dtype=bf)
    agate = torch.empty(T, HQ, 256, device=dev, dtype=bf)
    ak = torch.empty(T, HKV, 256, device=dev, dtype=bf)
    I_ = 17408
    gu = rnd(T, 2 * I_)
    act = torch.empty(T, I_, device=dev, dtype=bf)
    rnq = torch.empty(T, HK, device=dev)
    rnk = torch.empty(T, HK, device=dev)
    A_log, dt_bias = rnd(HV, scale=0.5), rnd(HV, scale=0.5)
    beta = torch.empty(T, HV, device=dev, dtype=bf)
    gf = torch.empty(T, HV, device=dev)
    lens = (ctypes.c_size_t * 1)(T)
    boff = 2 * KEY + 2 * VAL

    ops = {
        "rms_norm": (lambda: lib.cs1_rms_norm(x, w, out, T, H, 1e-6, st), T * H * 2 * 2 + H * 2),
        "add_rms_norm": (lambda: lib.cs1_add_rms_norm(res, x, w, out, T, H, 1e-6, st), T * H * 2 * 4 + H * 2),
        "gdn_conv": (lambda: lib.cs1_gdn_conv(gdn_in, GDN_IN, conv_w, q, k, v, T, KEY, VAL, st),
                     T * (2 * KEY + VAL) * 2 * 2 + (2 * KEY + VAL) * 8),
        # the fused front end: conv + SiLU, q/k inverse norms, gates (reads the gate columns too)
        "gdn_front": (lambda: lib.cs1_gdn_front_batch(gdn_in, None, GDN_IN, conv_w, q, k, v, rnq, rnk,
                                                      gdn_in[:, boff:], gdn_in[:, boff + HV:], A_log, dt_bias, beta, gf,
                                                      HV, ctypes.addressof(lens), 1, KEY, VAL, st),
                      T * (2 * KEY + VAL) * 2 * 2 + (2 * KEY + VAL) * 8 + T * (2 * HK * 4 + HV * (2 + 2 + 2 + 4))),
        "gated_rms_norm": (lambda: lib.cs1_gated_rms_norm(o, gdn_in[:, 2 * KEY + VAL:], GDN_IN, gw, go, T, HV, 128,
                                                          1e-6, st), T * HV * 128 * 2 * 3 + 256),
        "attn_prep": (lambda: lib.cs1_attn_prep(attn_in, attn_in[:, HQ * 512:], ATTN_IN, qw, kw, cos, sin, aq, agate, ak,
                                                T, HQ, HKV, 256, 32, 1e-6, st),
                      T * (HQ * 512 + HKV * 256) * 2 * 2 + T * 64 * 2 + 1024),
        "silu_mul": (lambda: lib.cs1_silu_mul(gu, 2 * I_, act, T, I_, st), T * I_ * 2 * 3),
    }
    pk, kind = peak()
    for name, (call, nbytes) in ops.items():
        if a.once:
            call()
            continue
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
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"op": name, "tokens": T, "ms": round(ms, 4), "bytes": nbytes, "gbs": round(gbs, 1),
                          "frac": round(gbs / pk, 3), "peak_gbs": pk, "peak_kind": kind}), flush=True)
    if a.once:
        torch.cuda.synchronize()
        print(json.dumps({"ops": list(ops), "calls": 1}))


if __name__ == "__main__":
    main()
