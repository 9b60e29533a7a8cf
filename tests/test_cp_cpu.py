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


def _agree_rank(rank, world, port, case, out):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "system1-omni_b200"))
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from s1omni import cp_agree, cp_piece_status

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    vocab, pieces = 1000, [128, 64, 100]
    starts = [0, 128, 192]
    ids = np.random.default_rng(rank).integers(0, vocab, pieces[rank]).astype(np.int32)
    start = starts[rank]
    if case == "bad_id" and rank == 1:
        ids[7] = vocab
    if case == "gap" and rank == 2:
        start = 256
    status = cp_piece_status(ids, start, rank, world, vocab, 4096)
    # the same exchange forward_cp makes over NCCL, here over gloo
    mine = torch.tensor([status, start, len(ids), 0], dtype=torch.int64)
    rows = [torch.zeros(4, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(rows, mine)
    rc, why = cp_agree(torch.stack(rows).numpy())
    out.put((rank, status, rc, why))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("case", ["good", "bad_id", "gap"])
def test_context_parallel_ranks_refuse_together(case):
    """forward_cp's agreement step on three gloo ranks: each rank checks its own piece,
    the (status, start, len) rows are all-gathered, and every rank reaches the same verdict,
    so a rank with a bad token id, or pieces that do not follow one another, make every rank
    return the same error before any transfer (none is left waiting in a send or receive)."""
    world = 3
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_rank, args=(r, world, port, case, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(out.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    verdicts = {(rc, why) for _, _, rc, why in res}
    assert len(verdicts) == 1, res
    rc, why = verdicts.pop()
    if case == "good":
        assert rc == 0 and all(st == 0 for _, st, _, _ in res)
    elif case == "bad_id":
        assert rc == -1 and "rank 1" in why and "token id" in why
        assert [st for _, st, _, _ in res] == [0, -6, 0]
    else:
        assert rc == -1 and "rank 2 starts at 256" in why


def test_piece_status_codes():
    from s1omni import cp_piece_status
    ok = np.zeros(64, np.int32)
    assert cp_piece_status(ok, 0, 0, 2, 10, 4096) == 0
    assert cp_piece_status(np.zeros(0, np.int32), 0, 0, 2, 10, 4096) == -1
    assert cp_piece_status(np.zeros(32, np.int32), 0, 0, 2, 10, 4096) == -2
    assert cp_piece_status(ok, 64, 1, 2, 10, 32) == -2
    assert cp_piece_status(ok, 65, 1, 2, 10, 4096) == -3
    assert cp_piece_status(np.zeros(65, np.int32), 0, 0, 2, 10, 4096) == -4
    assert cp_piece_status(np.zeros(65, np.int32), 64, 1, 2, 10, 4096) == 0
    assert cp_piece_status(ok, 64, 0, 2, 10, 4096) == -5
    assert cp_piece_status(ok, 0, 1, 2, 10, 4096) == -5
    bad = ok.copy()
    bad[3] = -1
    assert cp_piece_status(bad, 0, 0, 2, 10, 4096) == -6
