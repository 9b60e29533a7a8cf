"""Context-parallel prefill of one long prompt over the ranks of a torch.distributed.run
launch (one GPU each), 27B shape, random-init weights.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P -m s1omni.cp_bench [--tokens 32768] [--steps 3]

The prompt is split into pieces on 64-token boundaries (rank order = prompt order), sized
so that every rank's estimated work is about the same (`cp_pieces`; `--equal` for equal
pieces);
each step is one forward_cp on every rank, timed by wall clock between barriers (host
ids in, the last rank's logits out), max over ranks. Prints one JSON line on rank 0.
"""
import argparse
import json
import os
import time
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

from .model import Model, cp_pieces, cp_unique_id, preset


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--preset", default="27b")
    ap.add_argument("--equal", action="store_true", help="equal pieces instead of work-balanced ones")
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    cfg = preset(a.preset)
    lengths = cp_pieces(cfg, a.tokens, world) if not a.equal else \
        [(a.tokens // world) // 64 * 64] * (world - 1) + [a.tokens - (a.tokens // world) // 64 * 64 * (world - 1)]
    start = sum(lengths[:rank])
    ids = np.random.default_rng(5).integers(0, cfg.vocab, a.tokens).astype(np.int32)
    m = Model(cfg, device=local, max_tokens=lengths[rank] + 64, max_seqs=4)
    m.init_random(seed=1234, std=0.02)
    uid = [cp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    m.cp_init(rank, world, uid[0])
    piece = ids[start:start + lengths[rank]]
    m.forward_cp(piece, start)  # warm-up
    times = []
    out = None
    for _ in range(a.steps):
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = m.forward_cp(piece, start)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        t = torch.tensor([dt])
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        times.append(float(t))
    logits = torch.tensor(out if out is not None else np.zeros(cfg.labels, np.float32))
    dist.broadcast(logits, src=world - 1)
    if rank == 0:
        ms = float(np.median(times)) * 1e3
        print(json.dumps({"workload": f"{a.preset}-cp-{a.tokens}", "gpus": world, "tokens": a.tokens,
                          "pieces": lengths, "ms": ms, "tokens_per_s": a.tokens / (ms * 1e-3),
                          "timing": "wall clock between barriers, max over ranks, median of steps",
                          "finite": bool(np.isfinite(logits.numpy()).all()),
                          "logits": [round(float(x), 4) for x in logits.numpy()]}), flush=True)
    m.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
