"""Same-GPU parity against the reference's own CUDA library.

`make -C oracle` builds the reference's src/backends/cuda/qwen3_5/*.cu (cuBLASLt GEMMs,
mma.sync attention and GDN kernels) for sm_100a into oracle/_ref/. Both libraries export
the same cs1_* ABI, so each operation runs on identical device inputs through both and
the whole tiny model runs through the same C++ host over each. Tolerances: bf16 ops
within one bf16 ulp of each other; GEMM, GDN and attention within the gates of their
own parity tests; logits within 2e-2. Skipped when the reference library was not built.
"""
import os

import numpy as np
import pytest
import torch

from helpers import dev_bf16, dev_f32, empty_bf16, host, max_rel, rel_l2
from oracle import fixtures
from oracle import model as OM
from oracle.bf16 import rnd

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "libqwen3_5_cuda.so")
ULP = 2.0 ** -7


@pytest.fixture(scope="module")
def ref(cs1):
    if not os.path.exists(REF):
        pytest.skip("reference library not built (make -C oracle)")
    from s1omni import Cs1
    return Cs1(REF)


def _r(shape, seed, scale=1.0):
    return rnd(np.random.default_rng(seed).standard_normal(shape).astype(np.float32) * np.float32(scale))


def test_norms_conv_gates_silu_match_reference_kernels(cs1, ref, stream):
    T, H = 77, 2560
    r, d, w = _r((T, H), 1), _r((T, H), 2), _r((H,), 3, 0.1)
    outs = []
    for lib in (cs1, ref):
        res, out = dev_bf16(r), empty_bf16(T, H)
        lib.cs1_add_rms_norm(res, dev_bf16(d), dev_bf16(w), out, T, H, 1e-6, stream)
        outs.append((host(res), host(out)))
    assert np.array_equal(outs[0][0], outs[1][0])
    assert max_rel(outs[0][1], outs[1][1]) <= ULP
    kd, vd = 256, 512
    ld = 2 * kd + vd + 2 * 4 + vd
    qkv = _r((T, ld), 4)
    cw = rnd(np.random.default_rng(5).uniform(-0.5, 0.5, (2 * kd + vd, 4)).astype(np.float32))
    convs = []
    for lib in (cs1, ref):
        q, k, v = empty_bf16(T, kd), empty_bf16(T, kd), empty_bf16(T, vd)
        lib.cs1_gdn_conv(dev_bf16(qkv), ld, dev_bf16(cw), q, k, v, T, kd, vd, stream)
        convs.append([host(q), host(k), host(v)])
    for a, b in zip(*convs):
        assert max_rel(a, b) <= ULP
    gates = []
    for lib in (cs1, ref):
        beta, g = empty_bf16(T, 4), torch.empty(T, 4, dtype=torch.float32, device="cuda")
        src = dev_bf16(qkv)
        lib.cs1_gdn_gates(src[:, 2 * kd + vd:], src[:, 2 * kd + vd + 4:], ld, dev_bf16(_r((4,), 6)),
                          dev_bf16(_r((4,), 7)), beta, g, T, 4, stream)
        gates.append((host(beta), host(g)))
    assert np.array_equal(gates[0][0], gates[1][0]) and np.allclose(gates[0][1], gates[1][1], rtol=1e-6)
    gu = _r((T, 2048), 8)
    silus = []
    for lib in (cs1, ref):
        out = empty_bf16(T, 1024)
        lib.cs1_silu_mul(dev_bf16(gu), 2048, out, T, 1024, stream)
        silus.append(host(out))
    assert max_rel(silus[0], silus[1]) <= ULP


def test_gemm_matches_cublaslt_reference(cs1, ref, stream):
    M, N, K = 777, 5120, 6144
    x, w = dev_bf16(_r((M, K), 9)), dev_bf16(_r((N, K), 10, 0.05))
    ys = []
    for lib in (cs1, ref):
        h = lib.cs1_gemm_create(32 << 20)
        y = empty_bf16(M, N)
        lib.cs1_gemm(h, x, w, y, M, N, K, N, stream)
        ys.append(host(y))
        lib.cs1_gemm_destroy(h)
    assert max_rel(ys[0], ys[1]) <= 1e-2 and rel_l2(ys[0], ys[1]) <= 4e-3


@pytest.mark.parametrize("T,H,HK", [(107, 48, 16), (936, 48, 16), (200, 4, 2)])
def test_gdn_matches_reference_kernel(cs1, ref, stream, T, H, HK):
    q, k, v, g, beta = fixtures.grouped_inputs(T, T, H, HK)
    outs = []
    for lib in (cs1, ref):
        ws = torch.empty(lib.cs1_gdn_workspace_floats(T, H), dtype=torch.float32, device="cuda")
        o = empty_bf16(T, H, 128)
        lib.cs1_gdn_prefill(dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta), o, ws, T, H, HK,
                            128 ** -0.5, stream)
        outs.append(host(o))
    assert rel_l2(outs[0], outs[1]) <= 1e-2
    assert np.abs(outs[0] - outs[1]).max() <= 2e-2 * np.abs(outs[1]).max()


def test_attention_matches_reference_kernel(cs1, ref, stream):
    T, Hq, Hk = 700, 24, 4
    rng = np.random.default_rng(11)
    q = rnd(rng.standard_normal((T, Hq, 256)).astype(np.float32))
    k = rnd(rng.standard_normal((T, Hk, 256)).astype(np.float32))
    v = rnd(rng.standard_normal((T, Hk * 256)).astype(np.float32))
    gate = rnd(rng.standard_normal((T, Hq * 256)).astype(np.float32))
    outs = []
    for lib in (cs1, ref):
        o = empty_bf16(T, Hq, 256)
        lib.cs1_attention_gated(dev_bf16(q), dev_bf16(k), dev_bf16(v), Hk * 256, dev_bf16(gate), o, T, Hq, Hk, 256,
                                256 ** -0.5, stream)
        outs.append(host(o).reshape(T, -1))
    rowrel = (np.abs(outs[0] - outs[1]).max(1) / np.maximum(np.abs(outs[1]).max(1), 1e-30)).max()
    assert rowrel <= 1.6e-2


def test_tiny_model_same_host_over_both_libraries(cs1, ref):
    from s1omni import Model, preset
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    seqs = fixtures.tiny_prompts(cfg)
    logits = []
    for path in (None, REF):
        m = Model(preset("tiny"), device=0, max_tokens=1024, max_seqs=16, cs1_library=path)
        m.load(W)
        logits.append(m.forward(seqs))
        m.close()
    assert np.abs(logits[0] - logits[1]).max() <= 2e-2
