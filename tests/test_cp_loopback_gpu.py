"""Context-parallel prefill (s1_model_forward_cp) on ONE GPU: the ranks are threads of this
process, each with its own model (same weights) and stream, joined through a loopback
stand-in for the NCCL calls the host makes (tests/loopback_nccl/loopback_nccl.cpp:
stream-ordered device-to-device copies in NCCL's rendezvous order, host waits bounded).
This runs the host's whole context-parallel path where only one GPU exists: the piece
agreement before any transfer, then per layer the conv history, GDN state and attention
K/V handed from rank to rank. The last rank's logits and final hidden row equal those of
the whole prompt on one model bit for bit (as on several GPUs, tests/test_cp_gpu.py); a
piece with an out-of-range token id makes every rank return an error, and a later call
with valid pieces still succeeds."""
import os
import subprocess
import threading

import numpy as np
import pytest

from oracle import model as OM

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def loopback(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("loopback") / "libloopback_nccl.so")
    src = os.path.join(HERE, "loopback_nccl", "loopback_nccl.cpp")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-I/usr/local/cuda/include", src,
           "-L/usr/local/cuda/lib64", "-lcudart", "-Wl,-rpath,/usr/local/cuda/lib64", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def _ranks(models, pieces, ids, lib, hidden=True):
    """forward_cp of every rank in its own thread; returns per rank (result, exception)."""
    starts = np.concatenate([[0], np.cumsum(pieces)[:-1]]).astype(int)
    res = [None] * len(models)

    def work(r):
        try:
            a = int(starts[r])
            res[r] = (models[r].forward_cp(ids[r][a:a + pieces[r]], a, hidden=hidden), None)
        except Exception as e:  # noqa: BLE001 - reported per rank
            res[r] = (None, e)

    th = [threading.Thread(target=work, args=(r,)) for r in range(len(models))]
    for t in th:
        t.start()
    for t in th:
        t.join(300)
    assert not any(t.is_alive() for t in th), "a rank did not return"
    return res


@pytest.mark.parametrize("pieces", [[256, 192], [64, 321], [128, 64, 192, 100]])
def test_context_parallel_on_one_gpu_equals_whole_prompt(cs1, loopback, pieces):
    from s1omni import Model, cp_unique_id, preset
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    world = len(pieces)
    ids = np.random.default_rng(9).integers(0, cfg.vocab, sum(pieces)).astype(np.int32)
    models = []
    try:
        for _ in range(world):
            m = Model(preset("tiny"), device=0, max_tokens=2048, max_seqs=4)
            m.load(W)
            models.append(m)
        uid = cp_unique_id(loopback)
        for r, m in enumerate(models):
            m.cp_init(r, world, uid, loopback)
        for _ in range(2):  # twice: buffers and the communicator are reused
            out = _ranks(models, pieces, [ids] * world, loopback)
            for r, (_, e) in enumerate(out):
                assert e is None, (r, e)
        logits, hidden = out[-1][0]
        one = Model(preset("tiny"), device=0, max_tokens=2048, max_seqs=4)
        one.load(W)
        ref_logits, ref_hidden = one.forward([ids], hidden=True)
        one.close()
        assert np.array_equal(logits, ref_logits[0])
        assert np.array_equal(hidden, ref_hidden[0])
        assert cs1.cs1_fault_status(1) == 0
    finally:
        for m in models:
            m.close()


def test_context_parallel_refusal_reaches_every_rank(cs1, loopback):
    from s1omni import Model, cp_unique_id, preset
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    pieces = [128, 100]
    ids = np.random.default_rng(3).integers(0, cfg.vocab, sum(pieces)).astype(np.int32)
    bad = ids.copy()
    bad[150] = cfg.vocab  # inside rank 1's piece
    models = []
    try:
        for _ in range(2):
            m = Model(preset("tiny"), device=0, max_tokens=1024, max_seqs=4)
            m.load(W)
            models.append(m)
        uid = cp_unique_id(loopback)
        for r, m in enumerate(models):
            m.cp_init(r, 2, uid, loopback)
        out = _ranks(models, pieces, [ids, bad], loopback)
        assert all(e is not None for _, e in out), out  # rank 0's own piece was fine
        out = _ranks(models, pieces, [ids, ids], loopback)
        assert all(e is None for _, e in out), out
        one = Model(preset("tiny"), device=0, max_tokens=1024, max_seqs=4)
        one.load(W)
        ref_logits, _ = one.forward([ids], hidden=True)
        one.close()
        assert np.array_equal(out[-1][0][0], ref_logits[0])
        assert cs1.cs1_fault_status(1) == 0
    finally:
        for m in models:
            m.close()
