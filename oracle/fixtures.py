"""Seeded synthetic inputs shared by the golden generator, the tests and the
bench (test infrastructure only). The benchmark workloads name no public suite;
these seeded generators stand in with its shapes and value distributions.
"""
import numpy as np

from .bf16 import rnd


def c0_inputs(seed=0, T=512, H=16, HK=16, D=128):
    """C0, the standalone GDN operator: q, k ~ N(0,1) then L2-normalised per head,
    v ~ N(0,1), beta = sigmoid(N(0,1)), g = -softplus(N(0,1)) * exp(A_log) with
    A_log ~ U(log 1, log 16) per head; float32, batch dimension dropped."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((T, HK, D), dtype=np.float32)
    k = rng.standard_normal((T, HK, D), dtype=np.float32)
    q = q / np.sqrt((q * q).sum(-1, keepdims=True))
    k = k / np.sqrt((k * k).sum(-1, keepdims=True))
    v = rng.standard_normal((T, H, D), dtype=np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal((T, H), dtype=np.float32)))).astype(np.float32)
    a_log = rng.uniform(np.log(1.0), np.log(16.0), H).astype(np.float32)
    x = rng.standard_normal((T, H), dtype=np.float32)
    g = (-np.log1p(np.exp(x)) * np.exp(a_log)[None, :]).astype(np.float32)
    return q.astype(np.float32), k.astype(np.float32), v, g, beta


def grouped_inputs(seed, T, H, HK, D=128, decay=0.25):
    """The reference test's operator inputs (`tests/qwen3_5/test_gdn_fp32.py:57-68`):
    bf16-valued q, k, v ~ N(0,1), g = -U(0,1)*decay (float32), beta ~ U(0,1) bf16."""
    rng = np.random.default_rng(seed)
    q = rnd(rng.standard_normal((T, HK, D), dtype=np.float32))
    k = rnd(rng.standard_normal((T, HK, D), dtype=np.float32))
    v = rnd(rng.standard_normal((T, H, D), dtype=np.float32))
    g = (-rng.random((T, H), dtype=np.float32) * np.float32(decay)).astype(np.float32)
    beta = rnd(rng.random((T, H), dtype=np.float32))
    return q, k, v, g, beta


def tiny_prompts(cfg, seed=11, lengths=(1, 70, 130)):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in lengths]


def lognormal_lengths(rng, n, median, sigma, lo, hi):
    """Prompt lengths L = clip(round(exp(N(ln median, sigma))), lo, hi)."""
    x = np.exp(rng.normal(np.log(median), sigma, n))
    return np.clip(np.round(x), lo, hi).astype(np.int64)
