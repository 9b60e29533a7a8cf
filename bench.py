"""Prefill benchmark of the 27B-shaped Qwen3.5 hybrid decision scorer on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--ref-cuda]

A step is one packed prefill of 32 single-candidate requests per GPU (workload (a) of the
27B benchmark configuration: prompt lengths log-normal, median 800, sigma 0.6, clipped to
1..8192; synthetic uniform token ids; random-init bf16 weights of the 27B shape) through
the C++ host and the sm_100a kernels, scored by the 8-label head on each final token.
Weak scaling: one pool of 32 x N requests is drawn from one seed and dispatched over the
N ranks longest-processing-time first by token cost (s1omni.dispatch); every rank holds a
full weight replica and no collective sits on the hot path. Prints one JSON line on rank 0.
Rank 0 also times workload (b), one 32,768-token prefill (`long_prefill`; `--no-long`
skips it); with N > 1 GPUs every rank then runs the same prompt context-parallel, one piece
per GPU with the per-layer state passed rank to rank over NCCL (`long_prefill_cp`, with
`cp_bit_exact`: its logits equal the one-GPU logits bit for bit). `c3` is configuration C3
(9B shape, 256 requests of a log-normal prompt and 4 candidates each, the candidates
continuing from the shared prompt), the 256 requests dispatched over the N ranks (strong
scaling; `--no-c3` skips it).

`--impl reference` times the reference's CPU path on the host cores instead: Transformers'
own Qwen3.5 decoder layers (the reference's CPU parity anchor, FLA and causal-conv1d off,
float32) on one 771-token prompt (the median of the concurrency-1 workload) through one
4-layer period of the 27B shape, extrapolated x16 to 64 layers; every host thread is used.
`--ref-cuda` times the reference's own CUDA library (built from its sources by
oracle/Makefile) through the same C++ host on the same GPU instead, and prints its own line
with `gdn_same_box`: the complete GDN prefill call of both libraries at the reference's own
GDN benchmark points (`--gdn-only` prints that table alone).
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "system1-omni_b200"))

import numpy as np  # noqa: E402

METRIC = "prefill tokens/s (27B-shape hybrid scorer, batch of 32 requests per GPU)"
UNIT = "tokens/s"
BATCH = 32


LONG = 32768  # workload (b) of the 27B benchmark configuration: one 32,768-token prefill


def long_request(seed=5):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 151936, LONG).astype(np.int32)


def pool(n, seed=4):
    """n requests of workload (a): log-normal lengths (median 800, sigma 0.6, 1..8192)."""
    rng = np.random.default_rng(seed)
    x = np.exp(rng.normal(np.log(800.0), 0.6, n))
    lens = np.clip(np.round(x), 1, 8192).astype(np.int64)
    return [rng.integers(0, 151936, int(L)).astype(np.int32) for L in lens]


def requests(rank, world=1):
    """This rank's share of one pool of 32 x world requests, dispatched over the ranks
    longest processing time first by token cost (s1omni.dispatch)."""
    from s1omni import preset, request_cost, shard
    reqs = pool(BATCH * world)
    if world == 1:
        return reqs
    cfg = preset("27b")
    return shard(reqs, [request_cost(cfg, len(r)) for r in reqs], world, rank)


C3_REQUESTS = 256


def c3_pool(seed=3):
    """Configuration C3: 256 requests, prompt lengths clip(round(exp(N(ln 600, 0.6))), 64,
    4096), 4 candidates of U{16..64} tokens each; uniform token ids."""
    rng = np.random.default_rng(seed)
    lens = np.clip(np.round(np.exp(rng.normal(np.log(600.0), 0.6, C3_REQUESTS))), 64, 4096).astype(np.int64)
    cands = rng.integers(16, 65, (C3_REQUESTS, 4))
    return [(rng.integers(0, 151936, int(L)).astype(np.int32),
             [rng.integers(0, 151936, int(c)).astype(np.int32) for c in cands[i]]) for i, L in enumerate(lens)]


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = [s for s in self.samples if len(s) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["hbm_gbs"], "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0, "fallback"


# ------------------------------------------------------------------ CPU arm ----
CPU_TOKENS = 771  # median prompt of the concurrency-1 workload (single_requests)
_HF = {}


def host_threads():
    """Every host thread this process may run on (torchrun sets OMP_NUM_THREADS=1; the
    CPU arm overrides it explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def hf_period():
    """Transformers' own Qwen3.5 text model with one 4-layer period of the 27B shape (3
    Gated DeltaNet + 1 gated attention layer, SwiGLU 17,408), float32, FLA and
    causal-conv1d forced off as the reference's HF baseline does. Weights are filled from
    a seeded block of N(0, 0.02) values (A_log = log U(1, 16), dt_bias 1, norms at their
    identity values): a timing model, built once per process."""
    if "m" in _HF:
        return _HF["m"]
    import torch
    import transformers.utils.import_utils as iu
    iu.is_flash_linear_attention_available = lambda *a, **k: False
    iu.is_causal_conv1d_available = lambda *a, **k: False
    from transformers import Qwen3_5TextConfig
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M
    config = Qwen3_5TextConfig(
        vocab_size=16, hidden_size=5120, intermediate_size=17408, num_hidden_layers=4, num_attention_heads=24,
        num_key_value_heads=4, head_dim=256, linear_num_key_heads=16, linear_num_value_heads=48,
        linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
        layer_types=["linear_attention"] * 3 + ["full_attention"], rms_norm_eps=1e-6, max_position_embeddings=40000,
        rope_parameters={"rope_type": "default", "rope_theta": 1e7, "partial_rotary_factor": 0.25,
                         "mrope_section": [11, 11, 10], "mrope_interleaved": True})
    config._attn_implementation = "eager"
    with torch.device("meta"):
        model = M.Qwen3_5TextModel(config)
    model = model.to_empty(device="cpu").eval()
    g = torch.Generator().manual_seed(0)
    block = torch.randn(1 << 20, generator=g) * 0.02
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("A_log"):
                p.uniform_(1.0, 16.0, generator=g).log_()
            elif name.endswith("dt_bias") or name.endswith("linear_attn.norm.weight"):
                p.fill_(1.0)
            elif name.endswith("norm.weight") or name.endswith("layernorm.weight"):
                p.zero_()  # zero-centred RMSNorm: scale 1 + w
            elif "conv1d" in name:
                p.uniform_(-0.5, 0.5, generator=g)
            else:
                flat = p.view(-1)
                for i in range(0, flat.numel(), block.numel()):
                    n = min(block.numel(), flat.numel() - i)
                    flat[i:i + n].copy_(block[:n])
    model.rotary_emb = M.Qwen3_5TextRotaryEmbedding(config=config)  # its buffers, computed on the host
    _HF["m"] = model
    _HF["versions"] = f"transformers {__import__('transformers').__version__}, torch {torch.__version__}"
    return model


def cpu_sample(tokens=CPU_TOKENS, seed=0):
    """Time one `tokens`-token prompt through the 27B-shape period of Transformers' model on
    every host thread; return (tokens/s extrapolated to 64 layers, seconds, threads)."""
    import torch
    threads = host_threads()
    torch.set_num_threads(threads)
    model = hf_period()
    x = torch.randn(1, tokens, 5120, generator=torch.Generator().manual_seed(seed)) * 0.02
    with torch.no_grad():
        t0 = time.perf_counter()
        model(inputs_embeds=x)
        dt = time.perf_counter() - t0
    return tokens / (dt * 16), dt, threads


def cpu_sample_desc(tokens=CPU_TOKENS):
    return (f"one {tokens}-token prompt through one 4-layer period (3 GDN + 1 attention + MLPs) of the 27B shape, "
            f"Transformers Qwen3_5TextModel float32 eager (FLA off; {_HF.get('versions', '')}), "
            f"x16 periods (extrapolated to 64 layers)")


def run_reference(args, rank, world):
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup):
        cpu_sample()
    threads = host_threads()
    for _ in range(args.steps):
        v, dt, threads = cpu_sample()
        vals.append(v)
    value = float(np.median(vals))
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "27b-a-batch32", "model": "qwen3.5-27b-shape", "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                         "sample": cpu_sample_desc()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def gdn_same_box(torch, stream, ref_path, points=(107, 936, 3399), H=48, HK=16, calls=100, seed=20261003):
    """The complete GDN prefill call (`cs1_gdn_prefill`, batch 1, 16 q/k heads, 48 value
    heads, head dim 128) through this build's library and the reference's (oracle/_ref) on
    the same GPU, same stream, same device inputs and workspace size, at the token counts
    of the reference's own GDN benchmark (benchmarks/gdn/README.md:56-61): per point and
    arm one excluded feasibility call, ten excluded warm-ups, then two passes of `calls`
    calls (the second pass in reversed arm order), wall time per call with eager
    submission included and the CUDA event span beside it. Inputs: q ~ N(0,1), k = 0.6 q
    + 0.8 N(0,1) (correlated q/k), v ~ N(0,1), beta ~ U(0,1), weak decay g ~ -U(0, 0.05),
    seeded; synthetic, as the reference's are."""
    import ctypes
    from s1omni import Cs1
    libs = {"ours": Cs1(), "reference": Cs1(ref_path)}
    gen = torch.Generator(device="cuda").manual_seed(seed)
    rows = []
    for T in points:
        q32 = torch.randn(T, HK, 128, device="cuda", generator=gen)
        k = (0.6 * q32 + 0.8 * torch.randn(T, HK, 128, device="cuda", generator=gen)).to(torch.bfloat16)
        q = q32.to(torch.bfloat16)
        v = torch.randn(T, H, 128, device="cuda", generator=gen).to(torch.bfloat16)
        g = -torch.rand(T, H, device="cuda", generator=gen) * 0.05
        beta = torch.rand(T, H, device="cuda", generator=gen).to(torch.bfloat16)
        nws = max(lib.cs1_gdn_workspace_floats(T, H) for lib in libs.values())
        ws = torch.empty(nws, dtype=torch.float32, device="cuda")
        outs = {a: torch.empty(T, H, 128, device="cuda", dtype=torch.bfloat16) for a in libs}

        def call(a):
            return libs[a].raw.cs1_gdn_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(),
                                               beta.data_ptr(), outs[a].data_ptr(), ws.data_ptr(), T, H, HK,
                                               ctypes.c_float(128 ** -0.5), stream)
        wall = {a: [] for a in libs}
        event = {a: [] for a in libs}
        for a in libs:
            assert call(a) == 0
            for _ in range(10):
                call(a)
        torch.cuda.synchronize()
        for order in (("reference", "ours"), ("ours", "reference")):
            for a in order:
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                s.record(torch.cuda.current_stream())
                for _ in range(calls):
                    call(a)
                e.record(torch.cuda.current_stream())
                torch.cuda.synchronize()
                wall[a].append((time.perf_counter() - t0) * 1e3 / calls)
                event[a].append(s.elapsed_time(e) / calls)
        o_ours, o_ref = outs["ours"].float(), outs["reference"].float()
        rows.append({"tokens": T, "ms_wall": {a: [round(x, 6) for x in wall[a]] for a in libs},
                     "ms_event": {a: [round(x, 6) for x in event[a]] for a in libs},
                     "speedup_wall": round(min(wall["reference"]) / min(wall["ours"]), 3),
                     "max_diff_rel": float((o_ours - o_ref).abs().max() / o_ref.abs().max())})
    return {"heads": [HK, H], "calls_per_pass": calls, "points": rows,
            "published_h200_ms": {"107": 0.050957, "936": 0.214178, "3399": 0.697262}}


def run_reference_cuda(args, rank, world, local):
    """The reference's own CUDA library (built from its sources by oracle/Makefile into
    oracle/_ref/, recompiled for sm_100a: cuBLASLt GEMMs, mma.sync attention and GDN)
    driven by the same C++ host on the same GPU, on rank 0's requests split into launches
    the way the reference executor packs them (<= 16 prompts, <= 4096 tokens,
    open_jev batching.rs:9-25), eager, wall clock around synchronous calls."""
    if rank != 0:
        return
    ref = os.path.join(ROOT, "oracle", "_ref", "libqwen3_5_cuda.so")
    if not os.path.exists(ref):
        print(json.dumps({"impl": "reference-cuda-same-gpu", "unavailable": "oracle/_ref not built"}), flush=True)
        return
    import torch
    from s1omni import Model, lib_path, pack_ranges, preset
    torch.cuda.set_device(local)
    gdn = gdn_same_box(torch, torch.cuda.current_stream().cuda_stream, ref)
    if args.gdn_only:
        print(json.dumps({"impl": "reference-cuda-same-gpu", "gdn_same_box": gdn}), flush=True)
        return
    cfg = preset("27b")
    seqs = requests(0)
    tokens = int(sum(len(s) for s in seqs))
    ranges = pack_ranges([len(s) for s in seqs], 16, 4096)
    cap = max(max(sum(len(s) for s in seqs[a:b]) for a, b in ranges), 0 if args.no_long else LONG) + 64
    m = Model(cfg, device=local, max_tokens=cap, max_seqs=16, cs1_library=ref + ";" + lib_path())
    m.init_random(seed=1234, std=0.02)

    def step():
        return np.concatenate([m.forward(seqs[a:b]) for a, b in ranges])
    logits = step()
    for _ in range(max(1, args.warmup - 1)):
        step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    n = max(1, min(args.steps, 3))
    for _ in range(n):
        step()
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1e3 / n
    lat = latency(m, args)
    long = None
    if not args.no_long:
        seq = long_request()
        m.forward([seq])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(2):
            m.forward([seq])
        torch.cuda.synchronize()
        lms = (time.perf_counter() - t0) * 1e3 / 2
        long = {"workload": "27b-b-32k", "tokens": LONG, "value": LONG / (lms * 1e-3), "unit": UNIT,
                "ms_per_step": lms, "timing": "wall clock around synchronous forward calls"}
    m.close()
    print(json.dumps({
        "impl": "reference-cuda-same-gpu", "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": UNIT,
        "ms_per_step": ms, "launch_ranges": len(ranges), "p50_decision_latency_ms": lat, "long_prefill": long,
        "library": "reference src/backends/cuda/qwen3_5 built for sm_100a (oracle/Makefile)",
        "host": "this build's C++ host, eager, host-side scorer head (the reference's executor path)",
        "timing": "wall clock around synchronous forward calls (host copies included)",
        "logits_sample": logits[:4].round(4).tolist(), "gdn_same_box": gdn}), flush=True)


# ------------------------------------------------------------------ GPU arm ----
# DRAM traffic of one gemm_pair_kernel<SWIGLU> launch at M = 29,122 (N = 34,816, K = 5,120),
# dram__bytes_read.sum + dram__bytes_write.sum from the ncu capture summarised in
# profiles/gemm_swiglu_29122x34816x5120.md; scaled by rows for another M.
SWIGLU_TRAFFIC = {"m": 29122, "bytes": 8526523904 + 1024200192}


def gemm_roofline(cs1, cfg, M, stream, torch):
    """Time the projection GEMMs of one GDN layer, one attention layer and the MLP at the
    workload's M with CUDA events on the launching stream; return the set's TFLOP/s, ms,
    FLOPs and, per shape, (kind, N, K, ms)."""
    H, I_ = cfg.hidden, cfg.intermediate
    kd, vd, hv = cfg.lin_k_heads * 128, cfg.lin_v_heads * 128, cfg.lin_v_heads
    shapes = [((2 * kd + vd) + vd + 2 * hv, H, "store"), (H, vd, "residual"),
              (2 * cfg.heads * 256 + 2 * cfg.kv_heads * 256, H, "store"), (H, cfg.heads * 256, "residual"),
              (2 * I_, H, "swiglu"), (H, I_, "residual")]
    h = cs1.cs1_gemm_create(0)
    x = torch.randn(M, max(I_, H), device="cuda").to(torch.bfloat16) * 0.5
    flops = 0.0
    ms = 0.0
    per_shape = []
    for N, K, kind in shapes:
        w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
        out_n = N // 2 if kind == "swiglu" else N
        y = torch.zeros(M, out_n, device="cuda", dtype=torch.bfloat16)
        xs = x[:, :K].contiguous()

        def call():
            if kind == "swiglu":
                cs1.cs1_gemm_swiglu(h, xs, w, y, M, N // 2, K, out_n, stream)
            elif kind == "residual":
                cs1.cs1_gemm_residual(h, xs, w, y, M, N, K, out_n, stream)
            else:
                cs1.cs1_gemm(h, xs, w, y, M, N, K, out_n, stream)
        for _ in range(3):
            call()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        reps = 10
        torch.cuda.synchronize()
        s.record(torch.cuda.current_stream())
        for _ in range(reps):
            call()
        e.record(torch.cuda.current_stream())
        torch.cuda.synchronize()
        t = s.elapsed_time(e) / reps
        ms += t
        flops += 2.0 * M * N * K
        per_shape.append((kind, N, K, t))
        del w, y, xs
    cs1.cs1_gemm_destroy(h)
    return flops / (ms * 1e-3) / 1e12, ms, flops, per_shape


def op_rooflines(cs1, cfg, lens, stream, torch, peak_tf, peak_bw, reps=10):
    """The GDN prefill and the gated attention at the workload's packed lengths, timed alone
    with CUDA events on the launching stream (after 3 warm-up calls; inputs ~N(0,1) or
    U(0,1) as in the reference's tests), against their algorithmic bounds: GDN bytes
    q, k (2 HK 128 2), v, o (2 H 128 2), g (4 H), beta (2 H) and the front end's inverse norms
    of q and k (2 HK 4) per token against the HBM peak (its 6.7 MFLOP per token at 27B are
    under the ridge); attention 4 Hq 256 T(T+1)/2 FLOP per sequence against the bf16 peak.
    The GDN runs as the forward runs it: `cs1_gdn_prefill_batch_xn`, taking the norms the
    front end computes."""
    import ctypes
    T, n = int(sum(lens)), len(lens)
    arr = np.asarray(lens, dtype=np.uintp)
    H, HK, hq, hkv = cfg.lin_v_heads, cfg.lin_k_heads, cfg.heads, cfg.kv_heads
    out = {}

    def timed(call):
        for _ in range(3):
            assert call() == 0
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record(torch.cuda.current_stream())
        for _ in range(reps):
            call()
        e.record(torch.cuda.current_stream())
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps

    q = torch.randn(T, HK, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(T, HK, 128, device="cuda").to(torch.bfloat16)
    v = torch.randn(T, H, 128, device="cuda").to(torch.bfloat16)
    g = -torch.rand(T, H, device="cuda") * 0.25
    beta = torch.rand(T, H, device="cuda").to(torch.bfloat16)
    o = torch.empty(T, H, 128, device="cuda", dtype=torch.bfloat16)
    rnq = torch.rsqrt((q.float() ** 2).sum(-1) + 1e-6).contiguous()
    rnk = torch.rsqrt((k.float() ** 2).sum(-1) + 1e-6).contiguous()
    ms = timed(lambda: cs1.raw.cs1_gdn_prefill_batch_xn(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), beta.data_ptr(), rnq.data_ptr(), rnk.data_ptr(),
        o.data_ptr(), arr.ctypes.data, n, H, HK, ctypes.c_float(128 ** -0.5), None, 0, None, stream))
    byt = T * (2 * HK * 128 * 2 + 2 * H * 128 * 2 + H * 4 + H * 2 + 2 * HK * 4)
    gbs = byt / (ms * 1e-3) / 1e9
    out["gdn"] = {"kernel": "gdn_fused (preparation and scan of each head and sequence in one CTA)",
                  "ms_per_launch": ms, "bound": "hbm", "algorithmic_bytes_per_launch": byt, "achieved": gbs,
                  "peak": peak_bw, "unit": "GB/s", "frac": gbs / peak_bw}
    del q, k, v, g, beta, o, rnq, rnk
    qa = torch.randn(T, hq, 256, device="cuda").to(torch.bfloat16)
    ka = torch.randn(T, hkv, 256, device="cuda").to(torch.bfloat16)
    va = torch.randn(T, hkv, 256, device="cuda").to(torch.bfloat16)
    ga = torch.randn(T, hq, 256, device="cuda").to(torch.bfloat16)
    oa = torch.empty(T, hq, 256, device="cuda", dtype=torch.bfloat16)
    ms = timed(lambda: cs1.raw.cs1_attention_gated_batch(
        qa.data_ptr(), ka.data_ptr(), va.data_ptr(), hkv * 256, ga.data_ptr(), oa.data_ptr(), arr.ctypes.data, n, hq,
        hkv, 256, ctypes.c_float(256 ** -0.5), stream))
    fl = sum(4.0 * hq * 256 * L * (L + 1) / 2 for L in lens)
    tf = fl / (ms * 1e-3) / 1e12
    out["attention"] = {"kernel": "flash_tc (S, P, O in TMEM)", "ms_per_launch": ms, "bound": "tensor",
                        "algorithmic_flops_per_launch": fl, "achieved": tf, "peak": peak_tf, "unit": "TFLOP/s",
                        "frac": tf / peak_tf}
    return out


def long_prefill(model, torch, stream, steps=3):
    """Workload (b): one 32,768-token prefill, staged in HBM, CUDA-graph replay timed with
    CUDA events on the model's stream."""
    seq = long_request()
    model.set_graphs(True)
    model.stage([seq])
    for _ in range(3):
        model.run_staged()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record(stream)
    for _ in range(steps):
        model.run_staged()
    e.record(stream)
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    logits = model.fetch_logits()
    return {"workload": "27b-b-32k", "tokens": LONG, "value": LONG / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms,
            "steps": steps, "warmup": 3, "seed": 5, "finite": bool(np.isfinite(logits).all()),
            "logits": logits[0].round(4).tolist(), "_raw": logits[0].copy()}


def long_prefill_cp(model, torch, dist, rank, world, stream, one_gpu=None, steps=3):
    """Workload (b) over every rank of a multi-GPU run: the same 32,768-token prompt split in
    order into one piece per GPU (64-token boundaries, sized for equal estimated work per
    rank), context-parallel (per-layer GDN
    state, conv history and attention K/V passed rank to rank over NCCL). Host ids in, the
    last rank's logits out; CUDA events on each model stream, max over ranks. On rank 0,
    `one_gpu` holds the one-GPU logits of the same prompt: `cp_bit_exact` says whether the
    context-parallel logits equal them bit for bit (they should: pieces start on 64-token
    boundaries, where the chunked GDN restarts)."""
    from s1omni import cp_pieces, cp_unique_id, preset
    seq = long_request()
    lengths = cp_pieces(preset("27b"), LONG, world)  # work-balanced pieces on 64-token boundaries
    start = sum(lengths[:rank])
    piece = seq[start:start + lengths[rank]]
    uid = [cp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    model.cp_init(rank, world, uid[0])
    model.forward_cp(piece, start)  # warm-up
    times, out = [], None
    for _ in range(steps):
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        out = model.forward_cp(piece, start)
        e.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times.append(float(t))
    logits = torch.tensor(out if out is not None else np.zeros(8, np.float32), device="cuda")
    dist.broadcast(logits, src=world - 1)
    ms = float(np.median(times))
    lg = logits.cpu().numpy()
    out = {"workload": "27b-b-32k", "parallelism": f"context-parallel x{world}", "tokens": LONG,
           "pieces": lengths, "value": LONG / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms, "steps": steps,
           "warmup": 1, "seed": 5, "timing": "CUDA events on each rank's model stream, max over ranks, median",
           "finite": bool(np.isfinite(lg).all()), "logits": lg.round(4).tolist()}
    if one_gpu is not None:
        out["cp_bit_exact"] = bool(np.array_equal(lg, one_gpu))
        out["max_abs_diff_vs_one_gpu"] = float(np.abs(lg - one_gpu).max())
    return out


def c3_step(model, reqs):
    """One pass over this rank's C3 requests: each request's prompt runs once as a shared
    prefix and its 4 candidates continue from it in one packed pass (host ids in, logits
    out). Returns (tokens, logits of the first request)."""
    tokens, first = 0, None
    for prompt, cands in reqs:
        lg = model.forward_shared(prompt, cands)
        first = lg if first is None else first
        tokens += len(prompt) + sum(len(c) for c in cands)
    return tokens, first


def run_c3(torch, dist, rank, world, local, steps=2):
    """Configuration C3 (9B shape, random-init weights seed 1234): the 256 requests of
    c3_pool dispatched over the ranks longest-processing-time first by token cost; each
    rank serves its share request by request (eager, wall clock around synchronous calls,
    max over ranks). Strong scaling: the 256 requests are the whole job at every N."""
    from s1omni import Model, preset, request_cost, shard
    cfg = preset("9b")
    reqs = c3_pool()
    costs = [request_cost(cfg, len(p), [len(c) for c in cs]) for p, cs in reqs]
    mine = shard(reqs, costs, world, rank)
    total = sum(len(p) + sum(len(c) for c in cs) for p, cs in reqs)
    cap = max(len(p) for p, _ in reqs) + 4 * 64 + 64
    m = Model(cfg, device=local, max_tokens=cap, max_seqs=8)
    try:
        m.init_random(seed=1234, std=0.02)
        c3_step(m, mine[:4])  # warm-up
        times = []
        logits = None
        for _ in range(steps):
            if dist:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            _, lg = c3_step(m, mine)
            torch.cuda.synchronize()
            t = torch.tensor([time.perf_counter() - t0], device="cuda")
            if dist:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times.append(float(t))
            logits = lg if rank == 0 else logits
    finally:
        m.close()
    sec = float(np.median(times))
    return {"workload": "c3-9b-256x4", "model": "qwen3.5-9b-shape hybrid scorer (24 GDN + 8 attn)",
            "requests": C3_REQUESTS, "candidates_per_request": 4, "tokens": int(total),
            "requests_on_rank0": len(mine), "value": total / sec, "unit": UNIT, "seconds_per_step": sec,
            "steps": steps, "warmup": 1, "scaling": "strong", "dispatch": "longest processing time first by token cost",
            "timing": "wall clock around synchronous forward_shared calls (host ids in, logits out), max over ranks",
            "logits_first_request": None if logits is None else logits.round(4).tolist()}


def single_requests(n=16, seed=5):
    """Concurrency-1 workload (a) of the 27B benchmark configuration: one prompt per request."""
    rng = np.random.default_rng(seed)
    x = np.exp(rng.normal(np.log(800.0), 0.6, n))
    lens = np.clip(np.round(x), 1, 8192).astype(np.int64)
    return [rng.integers(0, 151936, int(L)).astype(np.int32) for L in lens]


def latency(model, args, repeats=3):
    """p50 / mean decision latency at concurrency 1: host ids in, 8 logits out, eager
    (each request has its own length), wall clock per request after one warm-up; each
    request is timed `repeats` times and its median kept (a single shot moves the p50
    of 16 requests by several percent)."""
    reqs = single_requests()
    model.set_graphs(False)
    model.forward([reqs[0]])
    ms = []
    for r in reqs:
        one = []
        for _ in range(repeats):
            t0 = time.perf_counter()
            model.forward([r])
            one.append((time.perf_counter() - t0) * 1e3)
        ms.append(float(np.median(one)))
    return {"p50_ms": float(np.median(ms)), "mean_ms": float(np.mean(ms)), "requests": len(reqs),
            "repeats_per_request": repeats, "tokens_median": int(np.median([len(r) for r in reqs]))}


def latency_dynamic(model, repeats=3):
    """The same requests through device-side batching with CUDA graphs: one graph per
    capacity (rows rounded up to an eighth of their octave), captured once per capacity
    before the timing as a server does at start-up, then every request replays its
    capacity's graph whatever its length."""
    reqs = single_requests()
    model.set_graphs(True)
    model.set_dynamic(True)
    try:
        before = model.graph_count
        for r in reqs:  # warm: the first request of each capacity captures its graph
            model.forward([r])
        ms = []
        for r in reqs:
            one = []
            for _ in range(repeats):
                t0 = time.perf_counter()
                model.forward([r])
                one.append((time.perf_counter() - t0) * 1e3)
            ms.append(float(np.median(one)))
        return {"p50_ms": float(np.median(ms)), "mean_ms": float(np.mean(ms)), "requests": len(reqs),
                "repeats_per_request": repeats, "graphs": model.graph_count - before}
    finally:
        model.set_dynamic(False)
        model.set_graphs(False)


def run_ours(args, rank, world, local):
    import torch
    from s1omni import Cs1, Model, preset
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    cfg = preset("27b")
    seqs = requests(rank, world)
    tokens = int(sum(len(s) for s in seqs))
    cap = max(tokens, 0 if args.no_long else LONG) + 64
    model = Model(cfg, device=local, max_tokens=cap, max_seqs=BATCH)
    model.init_random(seed=1234, std=0.02)
    cs1 = Cs1()
    stream = torch.cuda.ExternalStream(model.stream)
    model.stage(seqs)
    model.run_staged()           # eager pass: counts the launches
    launches_per_step = model.last_launches
    model.set_graphs(True)
    for _ in range(max(args.warmup, 3)):
        model.run_staged()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    with clocks:
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            model.run_staged()
        end.record(stream)
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    logits = model.fetch_logits()
    ok = bool(np.isfinite(logits).all()) and Cs1().cs1_fault_status(1) == 0
    # end to end through the public API: host ids in, host logits out, every step
    e2e_ms = []
    for i in range(max(2, min(args.steps, 5))):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        model.forward(seqs)
        e2e_ms.append((time.perf_counter() - t0) * 1e3)
    e2e = float(np.median(e2e_ms[1:]))
    # the roofline kernels, timed alone on rank 0 right after the timed steps and before the
    # latency, long-prompt and C3 runs (which heat the GPU further)
    roof = None
    if rank == 0:
        peak_tf, peak_bw, peak_kind = measured_peaks()
        roof = (gemm_roofline(cs1, cfg, tokens, torch.cuda.current_stream().cuda_stream, torch),
                op_rooflines(cs1, cfg, [len(s) for s in seqs], torch.cuda.current_stream().cuda_stream, torch,
                             peak_tf, peak_bw))
    lat = latency(model, args)
    lat["dynamic_graphs"] = latency_dynamic(model)
    long = long_prefill(model, torch, stream) if rank == 0 and not args.no_long else None
    one_gpu = long.pop("_raw") if long else None
    long_cp = long_prefill_cp(model, torch, dist, rank, world, stream, one_gpu) if dist and not args.no_long else None
    c3 = None
    if not args.no_c3:
        model.close()  # the 9B replica of C3 takes its place
        model = None
        c3 = run_c3(torch, dist, rank, world, local)
    h2d = tokens * 4 + tokens * 32 * 2 * 2 + len(seqs) * 4  # ids, rotary rows, last-row indices
    d2h = len(seqs) * cfg.labels * 4
    tmax = torch.tensor([ms, e2e], device="cuda")
    tok = torch.tensor([float(tokens)], device="cuda")
    if dist:
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        dist.all_reduce(tok, op=dist.ReduceOp.SUM)
    ms_max, e2e_max = float(tmax[0]), float(tmax[1])
    total_tokens = float(tok[0])
    result = None
    if rank == 0:
        (tflops, gms, gflops, per_shape), ops = roof
        _, sw_n, sw_k, sw_ms = next(x for x in per_shape if x[0] == "swiglu")
        sw_flops = 2.0 * tokens * sw_n * sw_k
        sw_tf = sw_flops / (sw_ms * 1e-3) / 1e12
        sw_traffic = (SWIGLU_TRAFFIC["bytes"] * tokens / SWIGLU_TRAFFIC["m"]) if SWIGLU_TRAFFIC["bytes"] else None
        value = total_tokens / (ms_max * 1e-3)
        proj = cfg.projection_flops_per_token() * tokens
        # the CPU baseline is timed at N = 1 only (rank 0 of a multi-GPU job skips it)
        use_cpu = world == 1 and not args.no_cpu
        cpu_v, cpu_dt, cpu_threads = cpu_sample() if use_cpu else (None, 0.0, 0)
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (uniform token ids, random-init weights)",
            "config": {"workload": "27b-a-batch32", "model": "qwen3.5-27b-shape hybrid scorer (48 GDN + 16 attn)",
                       "requests_per_gpu": BATCH, "tokens_rank0": tokens, "tokens_total": int(total_tokens),
                       "global_batch": BATCH * world, "dispatch": "one pool of 32 x N requests, longest processing "
                       "time first by token cost (s1omni.dispatch)",
                       "seq_len": "log-normal median 800 sigma 0.6 clip 1..8192", "parallelism": f"replica x{world}",
                       "l2": "weights (54 GB) and activations exceed L2 every step", "cuda_graphs": True},
            "e2e": {"value": total_tokens / (e2e_max * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": int(launches_per_step * args.steps),
            "roofline": {"bound": "tensor",
                         "kernel": f"gemm_pair_kernel<SWIGLU> (MLP gate/up + SwiGLU), M={tokens} N={sw_n} K={sw_k}",
                         "achieved": sw_tf, "peak": peak_tf, "unit": "TFLOP/s", "frac": sw_tf / peak_tf,
                         "peak_kind": peak_kind + " burst bf16", "ms_per_launch": sw_ms,
                         "algorithmic_flops_per_launch": sw_flops, "traffic": sw_traffic,
                         "traffic_unit": "bytes per launch (ncu dram read + write)",
                         "projection_set": {"shapes": len(per_shape), "tflops": tflops, "frac": tflops / peak_tf,
                                            "per_shape": [{"epilogue": k, "n": n_, "k": k_, "ms": round(t_, 4),
                                                           "tflops": round(2.0 * tokens * n_ * k_ / (t_ * 1e-3) / 1e12, 1)}
                                                          for k, n_, k_, t_ in per_shape]},
                         "forward_projection_tflops": proj / (ms_max * 1e-3) / 1e12,
                         "operators": ops},
            "cpu_baseline": {"value": cpu_v, "unit": UNIT, "cores": cpu_threads, "kind": "reference",
                             "sample": cpu_sample_desc()} if use_cpu else None,
            "p50_decision_latency_ms": lat,
            "long_prefill": long,
            "long_prefill_cp": long_cp,
            "c3": c3,
            "clocks": clocks.summary(),
            "checks": {"finite_logits_no_fault": ok, "logits_sample": logits[:4].round(4).tolist()},
        }
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if model is not None:
        model.close()
    if result:
        print(json.dumps(result), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-cuda", action="store_true",
                    help="time the reference's own CUDA library (oracle/_ref) through the same host, same GPU")
    ap.add_argument("--gdn-only", action="store_true",
                    help="with --ref-cuda: only the same-GPU GDN operator table against the reference library")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-long", action="store_true", help="skip workload (b), the 32,768-token prefill")
    ap.add_argument("--no-c3", action="store_true", help="skip configuration C3 (9B, 256 requests x 4 candidates)")
    args = ap.parse_args()
    if args.gpus > 1 and "WORLD_SIZE" not in os.environ:
        # one process per GPU: relaunch under torch.distributed.run on this node
        import socket
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={args.gpus}",
               "--master-addr=127.0.0.1", f"--master-port={port}", os.path.abspath(__file__)] + sys.argv[1:]
        sys.exit(subprocess.call(cmd))
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.ref_cuda:
        run_reference_cuda(args, rank, world, local)
    elif args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
