"""One packed prefill of a preset model with random-init weights, timed (or run once for a
profiler capture).

    cd system1-omni_b200 && python -m s1omni.forward_bench --preset 27b --lengths 771 \
        [--graphs] [--steps 5] [--once] [--lib PATH]

`--lengths` lists the prompt lengths packed into the one forward (uniform token ids,
seed 0). Without `--graphs` every step is an eager forward through the C++ host (host ids
in, host logits out), the concurrency-1 serving path; with `--graphs` the staged batch is
replayed from a CUDA graph. Prints one JSON line (ms per forward, tokens/s, launches per
forward). `--once` runs exactly one eager forward after the weight fill. `--lib` loads another
build of libqwen3_5_cuda.so under the same host (A/B timing of two kernel builds).
"""
import argparse
import json
import time

import numpy as np
import torch

from .model import Model, preset


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="27b")
    ap.add_argument("--lengths", default="771")
    ap.add_argument("--graphs", action="store_true")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--once", action="store_true")
    ap.add_argument("--lib", default=None)
    a = ap.parse_args()
    cfg = preset(a.preset)
    lengths = [int(x) for x in a.lengths.split(",")]
    rng = np.random.default_rng(0)
    seqs = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in lengths]
    m = Model(cfg, device=0, max_tokens=sum(lengths) + 64, max_seqs=max(len(seqs), 1), cs1_library=a.lib)
    try:
        m.init_random(seed=1234, std=0.02)
        if a.once:
            m.forward(seqs)
            torch.cuda.synchronize()
            print(json.dumps({"preset": a.preset, "lengths": lengths, "forwards": 1, "launches": m.last_launches}))
            return
        if a.graphs:
            m.stage(seqs)
            m.run_staged()
            launches = m.last_launches
            m.set_graphs(True)
            for _ in range(3):
                m.run_staged()
            stream = torch.cuda.ExternalStream(m.stream)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            s.record(stream)
            for _ in range(a.steps):
                m.run_staged()
            e.record(stream)
            torch.cuda.synchronize()
            ms = s.elapsed_time(e) / a.steps
        else:
            m.set_graphs(False)
            for _ in range(2):
                m.forward(seqs)
            launches = m.last_launches
            ts = []
            for _ in range(a.steps):
                t0 = time.perf_counter()
                m.forward(seqs)
                ts.append((time.perf_counter() - t0) * 1e3)
            ms = float(np.median(ts))
        print(json.dumps({"preset": a.preset, "lengths": lengths if len(lengths) <= 8 else f"{len(lengths)} prompts",
                          "tokens": sum(lengths), "graphs": a.graphs, "ms": ms,
                          "tokens_per_s": sum(lengths) / ms * 1e3, "launches": launches}))
    finally:
        m.close()


if __name__ == "__main__":
    main()
