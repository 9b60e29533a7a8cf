"""Whole-forward parity of the B200 prefill host + kernels against the oracle.

* logits of the seeded tiny hybrid model (3 GDN + 1 attention layer) within 2e-2
  absolute of the numpy oracle (the benchmark's bf16 logit tolerance) and of Transformers'
  own forward (golden hidden rows through the same head);
* packed candidates == each candidate alone, bit for bit (per-sequence state isolation);
* shared-prefix suffixes == the full prompt, bit for bit at a 64-aligned prefix;
* CUDA-graph replay == eager.
"""
import numpy as np
import pytest

from oracle import fixtures
from oracle import model as OM

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(cs1):
    from s1omni import Model, preset
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    m = Model(preset("tiny"), device=0, max_tokens=2048, max_seqs=32)
    m.load(W)
    yield cfg, W, m
    m.close()


def test_tiny_model_logits_match_oracle(tiny):
    cfg, W, m = tiny
    seqs = fixtures.tiny_prompts(cfg)
    logits, hidden = m.forward(seqs, hidden=True)
    ref_last, ref_logits = OM.forward_batch(cfg, W, seqs, gdn_mode="bf16")
    assert np.abs(logits - ref_logits).max() <= 2e-2, np.abs(logits - ref_logits).max()
    gold = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "tiny_model.npz"))
    hf_logits = OM.head(cfg, W, gold["last"])
    assert np.abs(logits - hf_logits).max() <= 4e-2, np.abs(logits - hf_logits).max()


def test_packed_candidates_equal_single_runs(tiny):
    cfg, W, m = tiny
    rng = np.random.default_rng(3)
    seqs = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (1, 63, 64, 65, 129, 200, 7)]
    packed = m.forward(seqs)
    for i, s in enumerate(seqs):
        assert np.array_equal(m.forward([s])[0], packed[i]), i


def test_shared_prefix_equals_full_prompt(tiny):
    cfg, W, m = tiny
    rng = np.random.default_rng(4)
    prefix = rng.integers(0, cfg.vocab, 256).astype(np.int32)
    suffixes = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (32, 1, 70)]
    shared = m.forward_shared(prefix, suffixes)
    for i, s in enumerate(suffixes):
        full = m.forward([np.concatenate([prefix, s])])[0]
        assert np.array_equal(shared[i], full), (i, np.abs(shared[i] - full).max())
    ref = OM.forward_shared_prefix(cfg, W, prefix, suffixes)[1]
    assert np.abs(shared - ref).max() <= 2e-2


def test_graph_replay_equals_eager(tiny):
    cfg, W, m = tiny
    rng = np.random.default_rng(5)
    seqs = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (10, 90)]
    eager = m.forward(seqs)
    m.set_graphs(True)
    try:
        first = m.forward(seqs)    # eager run + capture
        second = m.forward(seqs)   # replay
        other = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (10, 90)]
        replay_other = m.forward(other)
    finally:
        m.set_graphs(False)
    assert np.array_equal(first, eager) and np.array_equal(second, eager)
    assert np.array_equal(replay_other, m.forward(other))


def test_out_of_range_token_ids_are_refused(tiny):
    """An id outside [0, vocab) would index past the embedding table on the device: the
    host refuses the batch before any copy or launch, on every entry point, and the model
    stays usable."""
    cfg, W, m = tiny
    rng = np.random.default_rng(6)
    good = rng.integers(0, cfg.vocab, 40).astype(np.int32)
    before = m.forward([good])
    for bad_id in (cfg.vocab, -1):
        bad = good.copy()
        bad[17] = bad_id
        with pytest.raises(RuntimeError, match="outside"):
            m.forward([good, bad])
        with pytest.raises(RuntimeError, match="outside"):
            m.forward_shared(bad, [good])
    from s1omni import Cs1
    assert Cs1().cs1_fault_status(1) == 0
    assert np.array_equal(m.forward([good]), before)


def test_refused_stage_keeps_the_staged_batch(tiny):
    """s1_model_stage refuses a batch with an out-of-range id before any copy, so the batch
    staged before it still runs and gives the same logits."""
    cfg, W, m = tiny
    rng = np.random.default_rng(8)
    good = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (33, 70)]
    m.stage(good)
    m.run_staged()
    before = m.fetch_logits()
    bad = good[1].copy()
    bad[5] = cfg.vocab
    with pytest.raises(RuntimeError, match="outside"):
        m.stage([good[0], bad])
    m.run_staged()
    assert np.array_equal(m.fetch_logits(), before)
    assert np.array_equal(before, m.forward(good))


def test_graphs_survive_prefix_reallocation(tiny):
    """A longer shared prefix reallocates the prefix buffers; graphs captured for suffix
    passes on the old buffers are dropped with them, so a later suffix pass with the
    earlier prefix length captures afresh and equals eager (prefix 128 -> 256 -> 128)."""
    cfg, W, m = tiny
    rng = np.random.default_rng(9)
    suffixes = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (20, 45)]
    p1 = rng.integers(0, cfg.vocab, 128).astype(np.int32)
    p2 = rng.integers(0, cfg.vocab, 256).astype(np.int32)
    eager1 = m.forward_shared(p1, suffixes)
    eager2 = m.forward_shared(p2, suffixes)
    m.set_graphs(True)
    try:
        got = []
        for p in (p1, p1, p2, p2, p1, p1):
            got.append(m.forward_shared(p, suffixes))
    finally:
        m.set_graphs(False)
    for i, p in enumerate((p1, p1, p2, p2, p1, p1)):
        assert np.array_equal(got[i], eager1 if p is p1 else eager2), i
    from s1omni import Cs1
    assert Cs1().cs1_fault_status(1) == 0


def test_run_layers_composes_to_the_forward(tiny):
    """s1_model_run_layers from the embedding through every layer, one layer at a time,
    gives the forward's final hidden rows bit for bit, and one layer from a given residual
    stream matches the oracle's layer within the bf16 tolerance."""
    cfg, W, m = tiny
    from oracle.bf16 import bits, from_bits
    from oracle import ops
    rng = np.random.default_rng(10)
    seqs = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (65, 30)]
    _, hidden = m.forward(seqs, hidden=True)
    ids = np.concatenate(seqs)
    res = bits(W["embed"][ids])
    whole = m.run_layers(seqs, 0, len(cfg.layer_types), res)
    for layer in range(len(cfg.layer_types)):
        res = m.run_layers(seqs, layer, layer + 1, res)
    assert np.array_equal(res, whole)
    last = np.cumsum([len(s) for s in seqs]) - 1
    final = ops.rms_norm(from_bits(res)[last], W["final_norm"], cfg.eps)
    # the final RMSNorm restated on the host: within one bf16 ulp of the kernel's
    assert (np.abs(final - hidden) <= np.abs(hidden) * 2.0 ** -7 + 1e-30).all()
    # one layer, teacher-forced, against the oracle's layer on the first sequence
    h = bits(W["embed"][seqs[0]])
    got = from_bits(m.run_layers([seqs[0]], 0, 2, h))
    want = OM.run_layers(cfg, W, seqs[0], 0, 2, from_bits(h))
    upd = np.abs(want - from_bits(h)).max()
    assert np.abs(got - want).max() <= 2e-2 * upd, np.abs(got - want).max() / upd


def test_shared_prefix_off_the_64_grid_equals_full_prompt(tiny):
    """A prefix that is not a multiple of 64 tokens: the host shares its first 64k tokens
    and prepends the rest to every suffix, so each candidate equals its full prompt bit for
    bit; a prefix under 64 tokens is not shared at all."""
    cfg, W, m = tiny
    rng = np.random.default_rng(11)
    for plen in (100, 30):
        prefix = rng.integers(0, cfg.vocab, plen).astype(np.int32)
        suffixes = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (5, 64, 17)]
        shared = m.forward_shared(prefix, suffixes)
        for i, s in enumerate(suffixes):
            full = m.forward([np.concatenate([prefix, s])])[0]
            assert np.array_equal(shared[i], full), (plen, i)
