"""Whole-forward parity at the layer widths of the three benchmark models (4B, 9B, 27B) over one 4-layer
period (3 GDN + 1 attention): 27B (hidden 5120, SwiGLU 17408, GDN 16/48 heads, attention
24/4 heads x 256), 9B (4096, 12288, 16/32, 16/4) and 4B (2560, 9216, 16/32, 16/4).
Config C2's shape (a 2,048-token shared prefix and 8 candidates of 32 tokens) is run at
the 4B widths through the shared-prefix path.

The weights are drawn on the device by s1_model_init_random and read back with
s1_model_get_weight, so the numpy oracle runs on exactly the weights the kernels use.

Gates. At these widths the bf16 forward has a noise floor of the same size as the benchmark's
2e-2 logit tolerance: the numpy restatement itself moves by up to 0.028 when only its
GEMM accumulation changes from float32 to float64 (same weights and prompts, logits up
to 3.8), and the reference's own CUDA library differs from it by 0.039 (9B widths) to
0.044 (27B widths); a change of the fp32 reduction order inside one row normalisation
moves the 9B-width logits by about that much too. The distance between the reference
library and the restatement -- two faithful implementations of the same bf16 rounding
points -- is therefore measured in every run and used as the floor:
* logits within max(2e-2, floor + 5e-3) absolute of the reference's own CUDA library
  (built from its sources by oracle/Makefile) driven by the same host with the same
  weights -- the benchmark's 2e-2 wherever the forward itself is that stable;
* logits no further from the numpy restatement than the reference library is, plus 1e-2
  (or within 6e-2 when the reference library was not built).
"""
import os

import numpy as np
import pytest

from oracle import model as OM

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "libqwen3_5_cuda.so")


WIDTHS = {"27b": (5120, 17408, 16, 48, 24, 4), "9b": (4096, 12288, 16, 32, 16, 4), "4b": (2560, 9216, 16, 32, 16, 4)}


def _cfgs(name):
    from s1omni import Config
    layers = ["gdn", "gdn", "gdn", "attn"]
    H, I, hk, hv, hq, hkv = WIDTHS[name]
    ours = Config(H, I, layers, hk, hv, hq, hkv, 4096, name=name + "-period")
    oracle = OM.Config(H, I, layers, hk, hv, hq, hkv, 4096, name=name + "-period")
    return ours, oracle


@pytest.fixture(scope="module", params=["27b", "9b", "4b"])
def period(cs1, request):
    from s1omni import Model
    cfg, ocfg = _cfgs(request.param)
    m = Model(cfg, device=0, max_tokens=1024, max_seqs=8)
    m.init_random(seed=99, std=0.02)
    W = {name: m.get_weight(name, shape) for name, shape, _ in OM.weight_shapes(ocfg)}
    yield cfg, ocfg, m, W
    m.close()


def _prompts(vocab):
    rng = np.random.default_rng(5)
    return [rng.integers(0, vocab, n).astype(np.int32) for n in (100, 65, 1)]


def test_fullwidth_period_matches_oracle_and_reference(period):
    cfg, ocfg, m, W = period
    seqs = _prompts(cfg.vocab)
    ours = m.forward(seqs)
    _, oracle = OM.forward_batch(ocfg, W, seqs, gdn_mode="bf16")
    d_oracle = float(np.abs(ours - oracle).max())
    report = {"ours_vs_oracle": d_oracle, "logit_max": float(np.abs(oracle).max())}
    if os.path.exists(REF):
        from s1omni import Model, lib_path
        r = Model(cfg, device=0, max_tokens=1024, max_seqs=8, cs1_library=REF + ";" + lib_path())
        try:
            r.init_random(seed=99, std=0.02)
            theirs = r.forward(seqs)
        finally:
            r.close()
        report["ours_vs_reference"] = float(np.abs(ours - theirs).max())
        report["reference_vs_oracle"] = float(np.abs(theirs - oracle).max())
    print(report)
    if "ours_vs_reference" in report:
        floor = report["reference_vs_oracle"]
        assert report["ours_vs_reference"] <= max(2e-2, floor + 5e-3), report
        assert d_oracle <= floor + 1e-2, report
    else:
        assert d_oracle <= 6e-2, report


def test_c2_shared_prefix_candidates_at_4b_width(cs1):
    """C2's shape at the 4B widths: 8 candidates of 32 tokens after one 2,048-token
    prefix. The shared-prefix pass (prefix once, GDN state / conv rows / K-V forked) must
    equal each full prompt run on its own, bit for bit, and stay within the noise floor of
    the oracle's shared-prefix forward."""
    from s1omni import Model
    cfg, ocfg = _cfgs("4b")
    rng = np.random.default_rng(2)
    prefix = rng.integers(0, cfg.vocab, 2048).astype(np.int32)
    suffixes = [rng.integers(0, cfg.vocab, 32).astype(np.int32) for _ in range(8)]
    m = Model(cfg, device=0, max_tokens=2048 + 8 * 32 + 64, max_seqs=16)
    try:
        m.init_random(seed=7, std=0.02)
        shared = m.forward_shared(prefix, suffixes)
        for i, sfx in enumerate(suffixes):
            full = m.forward([np.concatenate([prefix, sfx])])[0]
            assert np.array_equal(shared[i], full), (i, np.abs(shared[i] - full).max())
        W = {name: m.get_weight(name, shape) for name, shape, _ in OM.weight_shapes(ocfg)}
    finally:
        m.close()
    ref = OM.forward_shared_prefix(ocfg, W, prefix, suffixes)[1]
    d = float(np.abs(shared - ref).max())
    print({"c2_ours_vs_oracle": d, "logit_max": float(np.abs(ref).max())})
    assert d <= 6e-2
