"""Device-side batching (the `cs1_*_dyn` entry points and s1_model_set_dynamic).

Each `_dyn` operation is launched for capacities larger than the batch (rows and
sequences) with the batch in a device descriptor (cs1_batch_desc_pack + one copy), and
must equal its host-length entry point bit for bit on the batch's rows; rows past the
batch are scratch. The GEMM runs at shapes where the wave model picks each kernel family
(CTA pair, 128 x 256, swapped, swapped pair) for the capacity. Then the model: with
graphs and device batching on, one captured graph per capacity serves several length
vectors, with the logits and hidden rows of the eager host-length forward, bit for bit,
for plain batches and shared-prefix suffix passes."""
import ctypes

import numpy as np
import pytest
import torch

from helpers import dev_bf16, dev_f32, empty_bf16, host
from oracle import fixtures
from oracle import model as OM

pytestmark = pytest.mark.gpu
LENS = [37, 100, 5, 64]  # 206 rows
CAP_ROWS, CAP_SEQS = 512, 8


def _desc(cs1, lengths):
    n = cs1.cs1_batch_desc_bytes()
    buf = np.zeros(n, np.uint8)
    arr = np.asarray(lengths, dtype=np.uintp)
    assert cs1.raw.cs1_batch_desc_pack(arr.ctypes.data, len(lengths), buf.ctypes.data, n) == 0
    return torch.from_numpy(buf).to("cuda")


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).to(torch.bfloat16)


def test_descriptor_refuses_bad_batches(cs1):
    n = cs1.cs1_batch_desc_bytes()
    buf = np.zeros(n, np.uint8)
    for lens in ([], [3, 0], [1] * 257):
        arr = np.asarray(lens or [1], dtype=np.uintp)
        assert cs1.raw.cs1_batch_desc_pack(arr.ctypes.data, len(lens), buf.ctypes.data, n) != 0
    arr = np.asarray([4], dtype=np.uintp)
    assert cs1.raw.cs1_batch_desc_pack(arr.ctypes.data, 1, buf.ctypes.data, n - 1) != 0


@pytest.mark.parametrize("M,cap,N,K,epi", [
    (206, 512, 5120, 1024, 0), (206, 512, 2048, 1024, 2), (771, 1024, 5120, 2048, 1), (3000, 4096, 4096, 1024, 0),
    (3000, 4096, 2048, 1024, 2), (2049, 4096, 1536, 512, 1), (17, 64, 1024, 512, 0)])
def test_gemm_dyn_equals_gemm(cs1, stream, M, cap, N, K, epi):
    h = cs1.cs1_gemm_create(0)
    try:
        x = _rand((cap, K), 1)
        w = _rand((N, K), 2, 0.05)
        out_n = N // 2 if epi == 2 else N
        res0 = _rand((cap, out_n), 3)
        desc = _desc(cs1, [M])
        y_ref = res0.clone() if epi == 1 else torch.zeros(cap, out_n, dtype=torch.bfloat16, device="cuda")
        y = res0.clone() if epi == 1 else torch.zeros(cap, out_n, dtype=torch.bfloat16, device="cuda")
        if epi == 0:
            assert cs1.raw.cs1_gemm(h, x.data_ptr(), w.data_ptr(), y_ref.data_ptr(), M, N, K, N, stream) == 0
        elif epi == 1:
            assert cs1.raw.cs1_gemm_residual(h, x.data_ptr(), w.data_ptr(), y_ref.data_ptr(), M, N, K, N, stream) == 0
        else:
            assert cs1.raw.cs1_gemm_swiglu(h, x.data_ptr(), w.data_ptr(), y_ref.data_ptr(), M, N // 2, K, N // 2,
                                           stream) == 0
        assert cs1.raw.cs1_gemm_dyn(h, x.data_ptr(), w.data_ptr(), y.data_ptr(), cap, N, K, out_n, epi, desc.data_ptr(),
                                    stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(y[:M], y_ref[:M])
        assert cs1.cs1_fault_status(1) == 0
    finally:
        cs1.cs1_gemm_destroy(h)


def test_norms_embed_gates_dyn_equal_host_length_ops(cs1, stream):
    T, D, H = sum(LENS), 2560, 32
    d = _desc(cs1, LENS)  # held until the launches have run
    desc = d.data_ptr()
    x, w = _rand((CAP_ROWS, D), 4), _rand((D,), 5, 0.1)
    a, b = empty_bf16(CAP_ROWS, D), empty_bf16(CAP_ROWS, D)
    assert cs1.raw.cs1_rms_norm(x.data_ptr(), w.data_ptr(), a.data_ptr(), T, D, ctypes.c_float(1e-6), stream) == 0
    assert cs1.raw.cs1_rms_norm_dyn(x.data_ptr(), w.data_ptr(), b.data_ptr(), CAP_ROWS, D, ctypes.c_float(1e-6), desc,
                                    stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(a[:T], b[:T])
    r1, r2, dl = _rand((CAP_ROWS, D), 6), None, _rand((CAP_ROWS, D), 7)
    r2 = r1.clone()
    assert cs1.raw.cs1_add_rms_norm(r1.data_ptr(), dl.data_ptr(), w.data_ptr(), a.data_ptr(), T, D, ctypes.c_float(1e-6),
                                    stream) == 0
    assert cs1.raw.cs1_add_rms_norm_dyn(r2.data_ptr(), dl.data_ptr(), w.data_ptr(), b.data_ptr(), CAP_ROWS, D,
                                        ctypes.c_float(1e-6), desc, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(a[:T], b[:T]) and torch.equal(r1[:T], r2[:T])
    # gated norm: o [rows, H, 128], z strided
    ldz = H * 128 + 64
    o, z, wn = _rand((CAP_ROWS, H, 128), 8), _rand((CAP_ROWS, ldz), 9), _rand((128,), 10, 0.1)
    ga, gb = empty_bf16(CAP_ROWS, H * 128), empty_bf16(CAP_ROWS, H * 128)
    assert cs1.raw.cs1_gated_rms_norm(o.data_ptr(), z.data_ptr(), ldz, wn.data_ptr(), ga.data_ptr(), T, H, 128,
                                      ctypes.c_float(1e-6), stream) == 0
    assert cs1.raw.cs1_gated_rms_norm_dyn(o.data_ptr(), z.data_ptr(), ldz, wn.data_ptr(), gb.data_ptr(), CAP_ROWS, H,
                                          128, ctypes.c_float(1e-6), desc, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(ga[:T], gb[:T])
    # embedding
    V = 1000
    table = _rand((V, D), 11)
    ids = torch.randint(0, V, (CAP_ROWS,), dtype=torch.int32, device="cuda")
    ea, eb = empty_bf16(CAP_ROWS, D), empty_bf16(CAP_ROWS, D)
    assert cs1.raw.cs1_embed(ids.data_ptr(), table.data_ptr(), ea.data_ptr(), T, D, stream) == 0
    assert cs1.raw.cs1_embed_dyn(ids.data_ptr(), table.data_ptr(), eb.data_ptr(), CAP_ROWS, D, desc, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(ea[:T], eb[:T])
    # gates
    ld = 2 * H + 16
    src = _rand((CAP_ROWS, ld), 12)
    A_log, dt = _rand((H,), 13, 0.5), _rand((H,), 14, 0.5)
    ba, bb = empty_bf16(CAP_ROWS, H), empty_bf16(CAP_ROWS, H)
    gf_a = torch.empty(CAP_ROWS, H, device="cuda")
    gf_b = torch.empty(CAP_ROWS, H, device="cuda")
    assert cs1.raw.cs1_gdn_gates(src.data_ptr(), src.data_ptr() + H * 2, ld, A_log.data_ptr(), dt.data_ptr(),
                                 ba.data_ptr(), gf_a.data_ptr(), T, H, stream) == 0
    assert cs1.raw.cs1_gdn_gates_dyn(src.data_ptr(), src.data_ptr() + H * 2, ld, A_log.data_ptr(), dt.data_ptr(),
                                     bb.data_ptr(), gf_b.data_ptr(), CAP_ROWS, H, desc, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(ba[:T], bb[:T]) and torch.equal(gf_a[:T], gf_b[:T])
    assert cs1.cs1_fault_status(1) == 0


@pytest.mark.parametrize("with_history", [False, True])
def test_conv_dyn_equals_conv_batch(cs1, stream, with_history):
    T, kd, vd = sum(LENS), 2048, 4096
    ld = 2 * kd + vd + 64
    qkv, w = _rand((CAP_ROWS, ld), 15), _rand((2 * kd + vd, 4), 16, 0.3)
    hist = _rand((3, ld), 17) if with_history else None
    d = _desc(cs1, LENS)
    outs = []
    for dyn in (False, True):
        q, k, v = empty_bf16(CAP_ROWS, kd), empty_bf16(CAP_ROWS, kd), empty_bf16(CAP_ROWS, vd)
        hp = hist.data_ptr() if hist is not None else None
        if dyn:
            rc = cs1.raw.cs1_gdn_conv_dyn(qkv.data_ptr(), hp, ld, w.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          CAP_ROWS, CAP_SEQS, kd, vd, d.data_ptr(), stream)
        else:
            arr = np.asarray(LENS, dtype=np.uintp)
            rc = cs1.raw.cs1_gdn_conv_batch(qkv.data_ptr(), hp, ld, w.data_ptr(), q.data_ptr(), k.data_ptr(),
                                            v.data_ptr(), arr.ctypes.data, len(LENS), kd, vd, stream)
        assert rc == 0
        torch.cuda.synchronize()
        outs.append((q[:T].clone(), k[:T].clone(), v[:T].clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("state", [False, True])
def test_gdn_dyn_equals_batch_x(cs1, stream, state):
    H, HK = 8, 4
    T = sum(LENS)
    q, k, v, g, beta = fixtures.grouped_inputs(5, CAP_ROWS, H, HK)
    dq, dk, dv, dg, db = dev_bf16(q), dev_bf16(k), dev_bf16(v), dev_f32(g), dev_bf16(beta)
    s_in = dev_f32(np.random.default_rng(6).standard_normal((H, 128, 128)).astype(np.float32) * 0.1) if state else None
    sp = s_in.data_ptr() if state else None
    ws = torch.empty(64, dtype=torch.float32, device="cuda")
    arr = np.asarray(LENS, dtype=np.uintp)
    oa, ob = empty_bf16(CAP_ROWS, H, 128), empty_bf16(CAP_ROWS, H, 128)
    d = _desc(cs1, LENS)
    assert cs1.raw.cs1_gdn_prefill_batch_x(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                           oa.data_ptr(), ws.data_ptr(), 256, arr.ctypes.data, len(LENS), H, HK,
                                           ctypes.c_float(128 ** -0.5), sp, 0, None, stream) == 0
    assert cs1.raw.cs1_gdn_prefill_dyn(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                       None, None, ob.data_ptr(), CAP_ROWS, CAP_SEQS, H, HK,
                                       ctypes.c_float(128 ** -0.5), sp, 0, None, d.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(oa[:T], ob[:T])
    # with inverse norms handed in (as the front end computes them): the same bits as the
    # host-length entry point given the same norms
    kf = torch.from_numpy(np.asarray(k, np.float32)).reshape(CAP_ROWS, HK, 128)
    qf = torch.from_numpy(np.asarray(q, np.float32)).reshape(CAP_ROWS, HK, 128)
    rnk = (1.0 / torch.sqrt((kf.double() ** 2).sum(-1) + 1e-6)).float().cuda().contiguous()
    rnq = (1.0 / torch.sqrt((qf.double() ** 2).sum(-1) + 1e-6)).float().cuda().contiguous()
    oc, od = empty_bf16(CAP_ROWS, H, 128), empty_bf16(CAP_ROWS, H, 128)
    assert cs1.raw.cs1_gdn_prefill_batch_xn(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                            rnq.data_ptr(), rnk.data_ptr(), oc.data_ptr(), arr.ctypes.data, len(LENS),
                                            H, HK, ctypes.c_float(128 ** -0.5), sp, 0, None, stream) == 0
    assert cs1.raw.cs1_gdn_prefill_dyn(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                       rnq.data_ptr(), rnk.data_ptr(), od.data_ptr(), CAP_ROWS, CAP_SEQS, H, HK,
                                       ctypes.c_float(128 ** -0.5), sp, 0, None, d.data_ptr(), stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(oc[:T], od[:T])
    # and within the GDN gate of the prefill's own norms
    a, c = host(oa[:T]), host(oc[:T])
    assert np.abs(a - c).max() <= 2e-2 * np.abs(a).max()
    assert cs1.cs1_fault_status(1) == 0


@pytest.mark.parametrize("with_history", [False, True])
def test_front_dyn_equals_front_batch(cs1, stream, with_history):
    T, kd, vd, H = sum(LENS), 2048, 4096, 32
    ld = 2 * kd + vd + 2 * H + 64
    qkv, w = _rand((CAP_ROWS, ld), 25), _rand((2 * kd + vd, 4), 26, 0.3)
    A_log, dt = _rand((H,), 27, 0.5), _rand((H,), 28, 0.5)
    hist = _rand((3, ld), 29) if with_history else None
    hp = hist.data_ptr() if hist is not None else None
    d = _desc(cs1, LENS)
    bptr = qkv.data_ptr() + (2 * kd + vd) * 2
    outs = []
    for dyn in (False, True):
        q, k, v = empty_bf16(CAP_ROWS, kd), empty_bf16(CAP_ROWS, kd), empty_bf16(CAP_ROWS, vd)
        rq = torch.empty(CAP_ROWS, kd // 128, device="cuda")
        rk = torch.empty(CAP_ROWS, kd // 128, device="cuda")
        beta, g = empty_bf16(CAP_ROWS, H), torch.empty(CAP_ROWS, H, device="cuda")
        common = (qkv.data_ptr(), hp, ld, w.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), rq.data_ptr(),
                  rk.data_ptr(), bptr, bptr + H * 2, A_log.data_ptr(), dt.data_ptr(), beta.data_ptr(), g.data_ptr(), H)
        if dyn:
            rc = cs1.raw.cs1_gdn_front_dyn(*common, CAP_ROWS, CAP_SEQS, kd, vd, d.data_ptr(), stream)
        else:
            arr = np.asarray(LENS, dtype=np.uintp)
            rc = cs1.raw.cs1_gdn_front_batch(*common, arr.ctypes.data, len(LENS), kd, vd, stream)
        assert rc == 0
        torch.cuda.synchronize()
        outs.append([t[:T].clone() for t in (q, k, v, rq, rk, beta, g)])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("prefix", [0, 128])
def test_attention_and_prep_dyn_equal_batch(cs1, stream, prefix):
    Hq, Hk, D = 8, 2, 256
    T = sum(LENS)
    ld = Hq * 2 * D + 2 * Hk * D  # [q+gate | k | v] rows of the stacked projection
    ain = _rand((CAP_ROWS, ld), 18)
    qw, kw = _rand((D,), 19, 0.1), _rand((D,), 20, 0.1)
    pos = np.concatenate([np.arange(n) + prefix for n in LENS] + [np.zeros(CAP_ROWS - T, int)])
    inv = 1.0 / (1e7 ** (np.arange(32) / 32.0))
    ang = pos[:, None] * inv[None, :]
    cos, sin = dev_bf16(np.cos(ang).astype(np.float32)), dev_bf16(np.sin(ang).astype(np.float32))
    kptr = ain.data_ptr() + Hq * 2 * D * 2
    vptr = kptr + Hk * D * 2
    pk = _rand((max(prefix, 1), Hk, D), 21) if prefix else None
    pv = _rand((max(prefix, 1), Hk, D), 22) if prefix else None
    d = _desc(cs1, LENS)
    res = []
    for dyn in (False, True):
        q, gate, k, out = (empty_bf16(CAP_ROWS, Hq, D), empty_bf16(CAP_ROWS, Hq, D), empty_bf16(CAP_ROWS, Hk, D),
                           empty_bf16(CAP_ROWS, Hq, D))
        desc = d.data_ptr()
        args = (ain.data_ptr(), kptr, ld, qw.data_ptr(), kw.data_ptr(), cos.data_ptr(), sin.data_ptr(), q.data_ptr(),
                gate.data_ptr(), k.data_ptr())
        if dyn:
            assert cs1.raw.cs1_attn_prep_dyn(*args, CAP_ROWS, Hq, Hk, D, 32, ctypes.c_float(1e-6), desc, stream) == 0
            assert cs1.raw.cs1_attention_dyn(q.data_ptr(), k.data_ptr(), vptr, ld, gate.data_ptr(), out.data_ptr(),
                                             pk.data_ptr() if prefix else None, pv.data_ptr() if prefix else None,
                                             prefix, CAP_ROWS, CAP_SEQS, Hq, Hk, D, ctypes.c_float(D ** -0.5), desc,
                                             stream) == 0
        else:
            assert cs1.raw.cs1_attn_prep(*args, T, Hq, Hk, D, 32, ctypes.c_float(1e-6), stream) == 0
            arr = np.asarray(LENS, dtype=np.uintp)
            assert cs1.raw.cs1_attention_gated_shared_batch(
                q.data_ptr(), k.data_ptr(), vptr, ld, gate.data_ptr(), out.data_ptr(),
                pk.data_ptr() if prefix else None, pv.data_ptr() if prefix else None, arr.ctypes.data, len(LENS), prefix,
                Hq, Hk, D, ctypes.c_float(D ** -0.5), stream) == 0
        torch.cuda.synchronize()
        res.append((q[:T].clone(), gate[:T].clone(), k[:T].clone(), out[:T].clone()))
    for a, b in zip(*res):
        assert torch.equal(a, b)
    assert cs1.cs1_fault_status(1) == 0


def test_head_dyn_scores_the_batch_only(cs1, stream):
    D, L, cap_n = 512, 8, 8
    hidden = _rand((300, D), 23)
    W = torch.randn(L, D, device="cuda") * 0.02
    bias = torch.randn(L, device="cuda")
    lens = [30, 50, 7]
    rows = torch.tensor(np.cumsum(lens) - 1, dtype=torch.int32, device="cuda")
    a = torch.full((cap_n, L), 7.0, device="cuda")
    b = torch.full((cap_n, L), 7.0, device="cuda")
    assert cs1.raw.cs1_head_score(hidden.data_ptr(), D, rows.data_ptr(), len(lens), W.data_ptr(), bias.data_ptr(), L,
                                  D, a.data_ptr(), stream) == 0
    d = _desc(cs1, lens)
    desc = d.data_ptr()
    assert cs1.raw.cs1_head_score_dyn(hidden.data_ptr(), D, None, cap_n, W.data_ptr(), bias.data_ptr(), L, D,
                                      b.data_ptr(), desc, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(a[:3], b[:3])
    assert bool((b[3:] == 7.0).all())  # candidates past the batch are not written


@pytest.fixture(scope="module")
def tiny_pair(cs1):
    from s1omni import Model, preset
    cfg = OM.preset("tiny")
    W = OM.make_weights(cfg, seed=7)
    ref = Model(preset("tiny"), device=0, max_tokens=2048, max_seqs=32)
    ref.load(W)
    dyn = Model(preset("tiny"), device=0, max_tokens=2048, max_seqs=32)
    dyn.load(W)
    dyn.set_graphs(True)
    dyn.set_dynamic(True)
    yield cfg, ref, dyn
    ref.close()
    dyn.close()


def test_one_graph_per_capacity_serves_every_length_vector(tiny_pair):
    cfg, ref, dyn = tiny_pair
    rng = np.random.default_rng(11)
    # every batch below has 193..256 rows and 3..4 sequences: one capacity (256 rows, 4 sequences)
    batches = [[100, 60, 40], [1, 64, 65, 70], [130, 60, 1, 2], [200, 30, 20], [64, 64, 64, 64]]
    before = dyn.graph_count
    for lens in batches:
        seqs = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in lens]
        for _ in range(2):  # the first call of a capacity captures, the second replays
            logits, hidden = dyn.forward(seqs, hidden=True)
            want_logits, want_hidden = ref.forward(seqs, hidden=True)
            assert np.array_equal(logits, want_logits), lens
            assert np.array_equal(hidden, want_hidden), lens
    assert dyn.graph_count - before == 1
    # another capacity: a second graph
    seqs = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in (500, 3)]
    assert np.array_equal(dyn.forward(seqs), ref.forward(seqs))
    assert dyn.graph_count - before == 2


def test_dynamic_shared_prefix_suffixes_match(tiny_pair):
    cfg, ref, dyn = tiny_pair
    rng = np.random.default_rng(12)
    prefix = rng.integers(0, cfg.vocab, 192).astype(np.int32)
    for lens in ((32, 1, 70), (5, 9), (40, 40, 40, 40)):
        suffixes = [rng.integers(0, cfg.vocab, n).astype(np.int32) for n in lens]
        assert np.array_equal(dyn.forward_shared(prefix, suffixes), ref.forward_shared(prefix, suffixes)), lens
