"""One rank of the two-GPU context-parallel test (launched by tests/test_cp_gpu.py through
torch.distributed.run): the tiny hybrid model, one prompt split into pieces on 64-token
boundaries, each rank running its piece with the previous rank's per-layer state; the
last rank compares its logits and final hidden row with the whole prompt run on one GPU
(bit for bit) and with the numpy oracle, and prints one JSON line."""
import json
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "system1-omni_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from oracle import model as OM  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    from s1omni import Cs1, Model, cp_unique_id, preset
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    lengths = [int(x) for x in os.environ.get("CP_PIECES", "256,192").split(",")]
    assert len(lengths) == world
    ids = np.random.default_rng(9).integers(0, cfg.vocab, sum(lengths)).astype(np.int32)
    starts = np.concatenate([[0], np.cumsum(lengths)[:-1]]).astype(int)
    m = Model(preset("tiny"), device=local, max_tokens=2048, max_seqs=4)
    m.load(W)
    uid = [cp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    m.cp_init(rank, world, uid[0])
    a, n = int(starts[rank]), lengths[rank]
    res = None
    for _ in range(2):  # twice: buffers and the communicator are reused
        res = m.forward_cp(ids[a:a + n], a, hidden=True)
    dist.barrier()
    if rank == world - 1:
        logits, hidden = res
        one = Model(preset("tiny"), device=local, max_tokens=2048, max_seqs=4)
        one.load(W)
        ref_logits, ref_hidden = one.forward([ids], hidden=True)
        one.close()
        oracle = OM.forward_batch(cfg, W, [ids], gdn_mode="bf16")[1][0]
        print(json.dumps({
            "bit_exact_logits": bool(np.array_equal(logits, ref_logits[0])),
            "bit_exact_hidden": bool(np.array_equal(hidden, ref_hidden[0])),
            "max_abs_vs_oracle": float(np.abs(logits - oracle).max()),
            "fault": int(Cs1().cs1_fault_status(1)),
            "pieces": lengths}), flush=True)
    m.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
