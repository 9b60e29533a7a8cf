"""GPU parity of the Gated DeltaNet chunked prefill (tcgen05 scan) and the FP32 operator.

Gates, as in the reference's own tests:
* bf16 kernel vs the float64 token-by-token recurrence: max|err| <= 2e-2 * max|ref|
  (tests/qwen3_5/kernels.rs:1190), and vs the numpy restatement of the same
  bf16-intermediate chunk form (oracle.gdn.chunk_bf16), relative L2 <= 1e-2;
* FP32 operator vs Transformers' chunk form (oracle.gdn.chunk_fp32, pinned to
  torch_chunk_gated_delta_rule by the golden vectors): relative L2 <= 1e-4
  (tests/qwen3_5/test_gdn_fp32.py:89);
* continuation from an fp32 state at a 64-token boundary, packed vs one-by-one
  sequences, and replay after a poisoned workspace: bit-exact.
"""
import numpy as np
import pytest
import torch

from helpers import dev_bf16, dev_f32, empty_bf16, host, max_rel, rel_l2
from oracle import fixtures
from oracle import gdn as G
from oracle.bf16 import rnd

pytestmark = pytest.mark.gpu
SCALE = 128 ** -0.5


def _inputs(T, H, HK, seed, decay=0.25, amp=1.0):
    q, k, v, g, beta = fixtures.grouped_inputs(seed, T, H, HK, decay=decay)
    return rnd(q * np.float32(amp)), rnd(k * np.float32(amp)), v, g, beta


def _run(cs1, stream, q, k, v, g, beta, H, HK, s_in=None, want_state=False):
    T = v.shape[0]
    ws = torch.empty(cs1.cs1_gdn_workspace_floats(T, H), dtype=torch.float32, device="cuda")
    o = empty_bf16(T, H, 128)
    s_out = torch.empty(H, 128, 128, dtype=torch.float32, device="cuda") if want_state else None
    cs1.cs1_gdn_prefill_x(dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta), o, ws, T, H, HK, SCALE,
                          None if s_in is None else dev_f32(s_in), s_out, stream)
    torch.cuda.synchronize()
    assert cs1.cs1_fault_status(1) == 0
    return host(o), (host(s_out) if want_state else None)


# (4096, 4, 2): 64 chunks, many turns of the double-buffered operand slots and of the single
# v buffer that loads on its own barrier
@pytest.mark.parametrize("T,H,HK", [(1, 4, 2), (16, 4, 2), (63, 4, 2), (64, 4, 4), (65, 4, 2), (129, 8, 4),
                                    (300, 4, 2), (936, 48, 16), (4096, 4, 2)])
def test_gdn_matches_float64_recurrence(cs1, stream, T, H, HK):
    q, k, v, g, beta = _inputs(T, H, HK, seed=T)
    o, s = _run(cs1, stream, q, k, v, g, beta, H, HK, want_state=True)
    ref, ref_s = G.recurrent_f64(q, k, v, g, beta, SCALE)
    assert np.abs(o - ref).max() <= 2e-2 * np.abs(ref).max()
    assert max_rel(s, ref_s) <= 2e-2
    if T * H <= 20000:
        ob, _ = G.chunk_bf16(q, k, v, g, beta, SCALE)
        assert rel_l2(o, ob) <= 1e-2


@pytest.mark.parametrize("amp,decay", [(1e-9, 0.25), (1.0, 4.0), (1.0, 1e-4)])
def test_gdn_tiny_amplitudes_and_decays(cs1, stream, amp, decay):
    q, k, v, g, beta = _inputs(150, 4, 2, seed=5, decay=decay, amp=amp)
    o, _ = _run(cs1, stream, q, k, v, g, beta, 4, 2)
    ref, _ = G.recurrent_f64(q, k, v, g, beta, SCALE)
    assert np.isfinite(o).all()
    assert np.abs(o - ref).max() <= 2e-2 * max(np.abs(ref).max(), 1e-30)


def test_gdn_continuation_is_bit_exact(cs1, stream):
    """State at a 64-token boundary reproduces the one-shot pass (ops.h:129-136)."""
    T, H, HK = 256, 4, 2
    q, k, v, g, beta = _inputs(T, H, HK, seed=9)
    full, s_full = _run(cs1, stream, q, k, v, g, beta, H, HK, want_state=True)
    a, s_a = _run(cs1, stream, q[:128], k[:128], v[:128], g[:128], beta[:128], H, HK, want_state=True)
    b, s_b = _run(cs1, stream, q[128:], k[128:], v[128:], g[128:], beta[128:], H, HK, s_in=s_a, want_state=True)
    assert np.array_equal(np.concatenate([a, b]), full)
    assert np.array_equal(s_b, s_full)


def test_gdn_empty_sequence_passes_state_through(cs1, stream):
    H = 4
    s_in = np.random.default_rng(1).standard_normal((H, 128, 128)).astype(np.float32)
    s_out = torch.zeros(H, 128, 128, dtype=torch.float32, device="cuda")
    p = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    cs1.cs1_gdn_prefill_x(p, p, p, p, p, p, p, 0, H, 2, SCALE, dev_f32(s_in), s_out, stream)
    assert np.array_equal(host(s_out), s_in)
    cs1.cs1_gdn_prefill_x(p, p, p, p, p, p, p, 0, H, 2, SCALE, None, s_out, stream)
    assert not host(s_out).any()


@pytest.mark.parametrize("lengths", [[1, 63, 64, 65, 129], [1] * 16, [78, 82, 200, 3], [600, 1]])
def test_gdn_batch_equals_serial(cs1, stream, lengths):
    H, HK = 6, 2
    T = sum(lengths)
    q, k, v, g, beta = _inputs(T, H, HK, seed=len(lengths))
    lens = np.asarray(lengths, dtype=np.uintp)
    floats = cs1.cs1_gdn_batch_workspace_floats(T, H, len(lengths))
    ws = torch.empty(floats, dtype=torch.float32, device="cuda")
    o = empty_bf16(T, H, 128)
    cs1.cs1_gdn_prefill_batch(dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta), o, ws, floats * 4,
                              lens.ctypes.data, len(lengths), H, HK, SCALE, stream)
    packed = host(o)
    off = 0
    for n in lengths:
        one, _ = _run(cs1, stream, q[off:off + n], k[off:off + n], v[off:off + n], g[off:off + n],
                      beta[off:off + n], H, HK)
        assert np.array_equal(packed[off:off + n], one)
        off += n


def test_gdn_batch_shared_state(cs1, stream):
    """Every suffix continues the same fp32 prefix state (cs1_gdn_prefill_batch_shared)."""
    H, HK = 4, 2
    P = 128
    lengths = [5, 64, 70]
    T = P + max(lengths)
    q, k, v, g, beta = _inputs(T, H, HK, seed=77)
    _, s_prefix = _run(cs1, stream, q[:P], k[:P], v[:P], g[:P], beta[:P], H, HK, want_state=True)
    sq = np.concatenate([q[P:P + n] for n in lengths])
    sk = np.concatenate([k[P:P + n] for n in lengths])
    sv = np.concatenate([v[P:P + n] for n in lengths])
    sg = np.concatenate([g[P:P + n] for n in lengths])
    sb = np.concatenate([beta[P:P + n] for n in lengths])
    lens = np.asarray(lengths, dtype=np.uintp)
    floats = cs1.cs1_gdn_batch_workspace_floats(int(lens.sum()), H, len(lengths))
    ws = torch.empty(floats, dtype=torch.float32, device="cuda")
    o = empty_bf16(int(lens.sum()), H, 128)
    cs1.cs1_gdn_prefill_batch_shared(dev_bf16(sq), dev_bf16(sk), dev_bf16(sv), dev_f32(sg), dev_bf16(sb), o, ws,
                                     floats * 4, lens.ctypes.data, len(lengths), H, HK, SCALE, dev_f32(s_prefix),
                                     stream)
    got = host(o)
    off = 0
    for n in lengths:
        full, _ = _run(cs1, stream, q[:P + n], k[:P + n], v[:P + n], g[:P + n], beta[:P + n], H, HK)
        assert np.array_equal(got[off:off + n], full[P:P + n])
        off += n


def test_gdn_poisoned_workspace_replays_identically(cs1, stream):
    T, H, HK = 200, 4, 2
    q, k, v, g, beta = _inputs(T, H, HK, seed=3)
    ws = torch.empty(cs1.cs1_gdn_workspace_floats(T, H), dtype=torch.float32, device="cuda")
    o = empty_bf16(T, H, 128)
    args = [dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta), o, ws, T, H, HK, SCALE, stream]
    cs1.cs1_gdn_prefill(*args)
    first = host(o).copy()
    ws.fill_(float("nan"))
    other = list(args)
    other[2] = dev_bf16(rnd(np.random.default_rng(5).standard_normal(v.shape).astype(np.float32)))
    cs1.cs1_gdn_prefill(*other)
    cs1.cs1_gdn_prefill(*args)
    assert np.array_equal(host(o), first)


def test_fp32_operator_matches_transformers_form(cs1, stream):
    """C0 inputs (bf16-rounded for the ABI) through cs1_gdn_prefill_fp32(_x) vs chunk_fp32."""
    q, k, v, g, beta = fixtures.c0_inputs(0)
    q, k, v, beta = rnd(q), rnd(k), rnd(v), rnd(beta)
    T, H, HK = 512, 16, 16
    ref, ref_s = G.chunk_fp32(q, k, v, g, beta, SCALE)
    ctx = cs1.cs1_gdn_fp32_create(32 << 20)
    assert ctx
    try:
        floats = cs1.cs1_gdn_fp32_workspace_floats(T, H)
        ws = torch.empty(floats, dtype=torch.float32, device="cuda")
        o32 = torch.empty(T, H, 128, dtype=torch.float32, device="cuda")
        s_out = torch.empty(H, 128, 128, dtype=torch.float32, device="cuda")
        cs1.cs1_gdn_prefill_fp32_x(ctx, dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta), o32, ws, T,
                                   H, HK, SCALE, None, s_out, stream)
        assert rel_l2(host(o32), ref) <= 1e-4
        assert rel_l2(host(s_out), ref_s) <= 1e-4
        ob = empty_bf16(T, H, 128)
        cs1.cs1_gdn_prefill_fp32(ctx, dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta), ob, ws, T, H,
                                 HK, SCALE, stream)
        assert rel_l2(host(ob), rnd(ref)) <= 1e-4
        # invalid shape / scale fail before any launch (test_gdn_fp32.py:107-111)
        p = ob.data_ptr()
        for T_, H_, HK_, sc in [(0, H, HK, SCALE), (T, H, 3, SCALE), (T, H, HK, float("nan")), (T, H, HK, 0.0)]:
            assert cs1.raw.cs1_gdn_prefill_fp32(ctx, p, p, p, p, p, p, ws.data_ptr(), T_, H_, HK_, sc, stream) != 0
    finally:
        cs1.cs1_gdn_fp32_destroy(ctx)
    for T_, H_ in [(0, 32), (-1, 32), (65537, 32), (1, 0), (1, 257)]:
        assert cs1.cs1_gdn_fp32_workspace_floats(T_, H_) == 0


@pytest.mark.parametrize("T,H,HK", [(1, 32, 16), (33, 32, 16), (129, 4, 2), (513, 32, 16)])
def test_fp32_operator_reference_shapes(cs1, stream, T, H, HK):
    q, k, v, g, beta = _inputs(T, H, HK, seed=141 + T)
    ref, _ = G.chunk_fp32(q, k, v, g, beta, SCALE)
    ctx = cs1.cs1_gdn_fp32_create(0)
    try:
        ws = torch.empty(cs1.cs1_gdn_fp32_workspace_floats(T, H), dtype=torch.float32, device="cuda")
        o = empty_bf16(T, H, 128)
        cs1.cs1_gdn_prefill_fp32(ctx, dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta), o, ws, T, H,
                                 HK, SCALE, stream)
        assert rel_l2(host(o), rnd(ref)) <= 1e-4
    finally:
        cs1.cs1_gdn_fp32_destroy(ctx)
