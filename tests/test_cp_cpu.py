"""The multi-rank host logic on CPU (gloo, three ranks on 127.0.0.1).

* Context-parallel semantics with the oracle: rank r continues the prompt from the
  per-layer prefix state rank r - 1 sends it (GDN fp32 state, conv history, attention K/V
  of every earlier piece, the oracle's PrefixState), captures its own continuation and
  sends it on; the last rank's logits match the whole prompt run in one pass (the chunked
  GDN restarts at 64-token boundaries, so only float32 summation order differs).
* The handshake of the GPU path: rank 0's NCCL id reaches every rank unchanged, and every
  rank derives the same work-balanced pieces (`cp_pieces`), contiguous and in order.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, pieces, out):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "system1-omni_b200"))
    from datetime import timedelta

    import torch.distributed as dist

    from oracle import model as OM
    from s1omni import cp_pieces, cp_unique_id, preset

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120))
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    ids = np.random.default_rng(9).integers(0, cfg.vocab, sum(pieces)).astype(np.int64)
    starts = np.concatenate([[0], np.cumsum(pieces)[:-1]]).astype(int)
    a, n = int(starts[rank]), pieces[rank]
    # context-parallel chain: receive the prefix state, continue, capture, send on
    box = [None]
    if rank > 0:
        dist.recv_object_list(box, src=rank - 1)
    hidden, state = OM.run_sequence(cfg, W, ids[a:a + n], prefix=box[0], capture=rank < world - 1,
                                    gdn_mode="fp32")
    if rank < world - 1:
        dist.send_object_list([state], dst=rank + 1)
    # handshake of the GPU path
    uid = [cp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    mine = cp_pieces(preset("27b"), 32768, world)
    all_pieces = [None] * world
    dist.all_gather_object(all_pieces, mine)
    ids_seen = [None] * world
    dist.all_gather_object(ids_seen, uid[0])
    if rank == world - 1:
        logits = OM.head(cfg, W, hidden[-1:])[0]
        full_hidden, _ = OM.run_sequence(cfg, W, ids, gdn_mode="fp32")
        full = OM.head(cfg, W, full_hidden[-1:])[0]
        out.put({"diff": float(np.abs(logits - full).max()), "ids_equal": all(x == ids_seen[0] for x in ids_seen),
                 "id_len": len(ids_seen[0]), "pieces_equal": all(p == all_pieces[0] for p in all_pieces),
                 "pieces": all_pieces[0]})
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("pieces", [[192, 128, 128], [64, 64, 200]])
def test_context_parallel_chain_on_gloo(pieces):
    world = len(pieces)
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, pieces, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res["diff"] <= 1e-3, res
    assert res["ids_equal"] and res["id_len"] == 128
    assert res["pieces_equal"] and sum(res["pieces"]) == 32768 and len(res["pieces"]) == world
    assert all(x % 64 == 0 for x in res["pieces"][:-1])
