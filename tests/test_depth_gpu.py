"""Parity at full depth: the 27B benchmark model (64 layers) against the reference's own
CUDA library, and config C1 (4B, 32 layers, 1,024 tokens) against the reference library,
the numpy restatement and its float64 ("precise") form.

What is gated, and why. At full depth no two bf16 implementations agree to the 2e-2 logit
tolerance on these random-init networks, the reference's library and its own restatement
included: a difference of one bf16 ulp in some outputs of the first layer grows through
the residual stream (about 30x over 64 layers), so the final logits of any two faithful
bf16 forwards differ by ~0.1 (C1) to ~0.3 (27B), and each sits ~0.15 (C1) from the exact
forward. The tests therefore hold, at every layer and at the end:
* teacher-forced, per layer: from the same input residual stream, this build's layer
  output is within 2e-2 (RMS, relative to the layer's own update of the stream) of the
  reference library's layer and of the restatement's layer;
* substitution: running the reference library's layer 0 and this build's layers 1..L-1
  moves the logits by as much as the whole gap between the two libraries (the gap is
  the amplified first-layer ulp difference, not an op that drifts);
* free running: this build's logits are no further from the precise forward (C1) than
  the reference library's own logits are, plus 2e-2.
Skipped where the reference library was not built (make -C oracle).
"""
import os

import numpy as np
import pytest

from layerwise import embed_bits, head_logits, local_rel
from oracle import model as OM
from oracle.bf16 import from_bits

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "libqwen3_5_cuda.so")
TOL = 2e-2


def _pair(name, tokens, seqs_max=8):
    if not os.path.exists(REF):
        pytest.skip("reference library not built (make -C oracle)")
    from s1omni import Model, lib_path, preset
    cfg = preset(name)
    ours = Model(cfg, device=0, max_tokens=tokens + 64, max_seqs=seqs_max)
    ref = Model(cfg, device=0, max_tokens=tokens + 64, max_seqs=seqs_max, cs1_library=REF + ";" + lib_path())
    for m in (ours, ref):
        m.init_random(seed=1234, std=0.02)
    return cfg, ours, ref


def test_27b_full_depth_layer_by_layer_against_reference_library(cs1):
    """27B shape, all 64 layers, two prompts packed (the bench's weights, seed 1234)."""
    rng = np.random.default_rng(4)
    seqs = [rng.integers(0, 151936, n).astype(np.int32) for n in (300, 129)]
    cfg, ours, ref = _pair("27b", sum(len(s) for s in seqs))
    try:
        ocfg = OM.preset("27b")
        W = {n: ours.get_weight(n, sh) for n, sh in (("final_norm", (cfg.hidden,)), ("head_w", (cfg.labels, cfg.hidden)),
                                                     ("head_b", (cfg.labels,)))}
        last = np.cumsum([len(s) for s in seqs]) - 1
        h0 = embed_bits(ours, cfg, np.concatenate(seqs))
        a, b, c = h0, h0, None
        worst = 0.0
        for layer in range(len(cfg.layer_types)):
            nxt = ours.run_layers(seqs, layer, layer + 1, a)
            theirs = ref.run_layers(seqs, layer, layer + 1, a)
            rel = local_rel(from_bits(nxt), from_bits(theirs), from_bits(a))
            worst = max(worst, rel)
            assert rel <= TOL, (layer, rel)
            b = ref.run_layers(seqs, layer, layer + 1, b)
            c = theirs if layer == 0 else ours.run_layers(seqs, layer, layer + 1, c)
            a = nxt
        la, lb, lc = (head_logits(cfg, ocfg, W, x, last) for x in (a, b, c))
        gap, gap_sub = float(np.abs(la - lb).max()), float(np.abs(la - lc).max())
        # the forward's own logits are the host restatement's, bit for bit or within one bf16 ulp
        assert np.abs(ours.forward(seqs) - la).max() <= 2e-2
        print({"worst_layer_rel": worst, "gap_ours_vs_reference": gap, "gap_reference_layer0_only": gap_sub})
        assert gap <= 2.0 * gap_sub + TOL, (gap, gap_sub)
    finally:
        ours.close()
        ref.close()


def test_c1_4b_full_depth_against_oracle_and_reference_library(cs1):
    """C1: 4B, 32 layers, one 1,024-token prompt (ids seed 1)."""
    seq = np.random.default_rng(1).integers(0, 151936, 1024).astype(np.int32)
    cfg, ours, ref = _pair("4b", 1024, 2)
    try:
        ocfg = OM.preset("4b")
        W = {n: ours.get_weight(n, sh) for n, sh, _ in OM.weight_shapes(ocfg) if n != "embed"}
        h0 = embed_bits(ours, cfg, seq)
        a, b = h0, h0
        o32 = from_bits(h0)
        o64 = from_bits(h0)
        for layer in range(len(cfg.layer_types)):
            nxt = ours.run_layers([seq], layer, layer + 1, a)
            theirs = ref.run_layers([seq], layer, layer + 1, a)
            assert local_rel(from_bits(nxt), from_bits(theirs), from_bits(a)) <= TOL, layer
            # the restatement's layer from the same input (bf16 rounding points, float32 sums)
            mine = OM.run_layers(ocfg, W, seq, layer, layer + 1, from_bits(a))
            assert local_rel(from_bits(nxt), mine, from_bits(a)) <= TOL, layer
            b = ref.run_layers([seq], layer, layer + 1, b)
            o64 = OM.run_layers(ocfg, W, seq, layer, layer + 1, o64, precise=True)
            a = nxt
        la, lb = (head_logits(cfg, ocfg, W, x, [-1]) for x in (a, b))
        from oracle import ops
        lp = OM.head(ocfg, W, ops.rms_norm(o64[-1:], W["final_norm"], cfg.eps))
        assert np.abs(ours.forward([seq]) - la).max() <= 1e-2  # kernel final norm vs its restatement
        d_ours, d_ref = float(np.abs(la - lp).max()), float(np.abs(lb - lp).max())
        print({"ours_vs_precise": d_ours, "reference_vs_precise": d_ref,
               "ours_vs_reference": float(np.abs(la - lb).max())})
        assert d_ours <= d_ref + TOL, (d_ours, d_ref)
    finally:
        ours.close()
        ref.close()
