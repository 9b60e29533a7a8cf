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
