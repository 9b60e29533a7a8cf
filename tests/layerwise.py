"""Layer-by-layer comparison helpers for the full-depth parity tests.

A bf16 forward through many layers of a random-init hybrid network amplifies any
ulp-level difference of its first layer: two faithful bf16 implementations (this build,
the reference's own CUDA library, the numpy restatement) drift apart by the same amount
whichever of them introduces the first difference. So the tests compare what each layer
computes from the same input (teacher-forced: the residual stream entering layer l is
handed to every implementation), and compare the free-running results with the distance
of the reference's own library from the exact (float64) forward.
"""
import numpy as np

from oracle.bf16 import bits, from_bits


def rms(x):
    x = np.asarray(x, np.float64)
    return float(np.sqrt((x * x).mean()))


def local_rel(out, other, inp):
    """|out - other| / |out - inp| (RMS): the difference of two layers' outputs relative
    to the layer's own update of the residual stream."""
    out, other, inp = (np.asarray(x, np.float64) for x in (out, other, inp))
    return rms(out - other) / rms(out - inp)


def embed_bits(model, cfg, ids):
    """bf16 bits of the embedding rows of `ids` (the residual stream entering layer 0)."""
    E = model.get_weight("embed", (cfg.vocab, cfg.hidden))
    return bits(E[np.asarray(ids, np.int64)])


def head_logits(cfg, ocfg, W, res_bits, last_rows):
    """Final RMSNorm (restated) and the scorer head on the last rows of a residual stream."""
    from oracle import model as OM
    from oracle import ops
    x = ops.rms_norm(from_bits(res_bits)[last_rows], W["final_norm"], cfg.eps)
    return OM.head(ocfg, W, x)
