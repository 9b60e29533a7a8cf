"""CPU checks of the drop-in boundary: both libraries load without a GPU, export
every symbol their headers declare, report ABI version 9, and the host packing
policy matches the reference's own test vectors (tests/open_jev/batching.rs)."""
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"//.*", "", text)
    return sorted(set(re.findall(r"\b((?:cs1|s1)_[a-z0-9_]+)\s*\(", text)))


def _exported(lib):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_cs1_library_exports_every_declared_symbol():
    from s1omni import lib_path
    names = _declared("qwen3_5_ops.h")
    assert len(names) > 60
    exported = _exported(lib_path())
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    # nothing else leaks out of the library
    assert all(n.startswith("cs1_") for n in exported), sorted(n for n in exported if not n.startswith("cs1_"))


def test_model_library_exports_every_declared_symbol():
    from s1omni import lib_path
    names = _declared("s1_model.h") + _declared("s1_processing.h")
    assert "s1_processor_prepare" in names and "s1_tokenizer_encode" in names
    exported = _exported(lib_path("libs1_model.so"))
    missing = [n for n in names if n not in exported]
    assert not missing, missing


def test_abi_version_without_gpu():
    from s1omni import Cs1
    lib = Cs1()
    assert lib.cs1_abi_version() == 9
    assert lib.cs1_gdn_fp32_workspace_floats(0, 32) == 0
    assert lib.cs1_gdn_fp32_workspace_floats(65537, 32) == 0
    assert lib.cs1_gdn_fp32_workspace_floats(1, 257) == 0
    assert lib.cs1_gdn_batch_workspace_floats(100, 4, 0) == 0
    assert lib.cs1_gdn_workspace_floats(64, 4) > 0


def test_reference_loader_required_symbols_present():
    """Every symbol the reference's Rust loader requires (cuda.rs api! table)."""
    from s1omni import lib_path
    required = """cs1_abi_version cs1_error_string cs1_set_device cs1_get_device cs1_bf16_finite cs1_malloc cs1_free
    cs1_stream_create cs1_stream_sync cs1_stream_destroy cs1_graph_begin cs1_graph_end cs1_graph_launch
    cs1_graph_destroy cs1_upload cs1_download cs1_copy_dd cs1_copy2d cs1_embed cs1_rms_norm cs1_add_rms_norm
    cs1_gated_rms_norm cs1_gdn_conv cs1_gdn_gates cs1_gdn_workspace_floats cs1_gdn_prefill cs1_gdn_prefill_x
    cs1_attn_prep cs1_attention cs1_attention_gated cs1_attention_gated_prefix cs1_sigmoid_gate cs1_silu_mul
    cs1_gemm_create cs1_gemm_create_fixed cs1_gemm_destroy cs1_gemm cs1_vision_linear cs1_gemm_f32
    cs1_vision_norm cs1_vision_position cs1_vision_rope cs1_vision_attention cs1_vision_bias cs1_vision_gelu
    cs1_vision_add cs1_vision_to_float cs1_vision_lora_add cs1_reference_available""".split()
    required.remove("cs1_reference_available")  # optional (Reference::resolve), not required
    exported = _exported(lib_path())
    assert not [n for n in required if n not in exported]


def test_pack_ranges_reference_vectors():
    from s1omni import pack_ranges
    from oracle.packing import ranges
    lengths = [2048, 2048, 1, 5000, 3] + [4] * 17
    expect = [(0, 2), (2, 3), (3, 4), (4, 20), (20, 22)]
    assert pack_ranges(lengths) == expect
    assert ranges(lengths) == expect
    rng = np.random.default_rng(0)
    for _ in range(200):
        lens = rng.integers(1, 5000, rng.integers(1, 40)).tolist()
        assert pack_ranges(lens) == ranges(lens)
    assert pack_ranges([]) == []


def test_shared_prefix_reference_vectors():
    from s1omni import shared_prefix
    from oracle.packing import shared_prefix as oracle_sp
    a = np.ones(2100, np.int32)
    b = a.copy()
    b[2000] = 2
    for fn in (shared_prefix, oracle_sp):
        assert fn([a, b]) == 1984
    b[100] = 3
    for fn in (shared_prefix, oracle_sp):
        assert fn([a, b]) == 0
        assert fn([a, a]) == 2048
        assert fn([a]) == 0
        assert fn([a, a[:2048]]) == 0
        assert fn([a] * 17) == 0
    a = np.full(801, 42, np.int32)
    b = np.full(832, 42, np.int32)
    b[790] = 7
    for fn in (shared_prefix, oracle_sp):
        assert fn([a, b]) == 0
        assert fn([a, b], 512) == 768
        assert fn([a, b[:511]], 512) == 0
        assert fn([a, b[:512]], 512) == 0
        assert fn([a], 512) == 0
        assert fn([a] * 17, 512) == 0


def test_model_create_reports_missing_library():
    from s1omni import Model, preset
    with pytest.raises(RuntimeError, match="dlopen"):
        Model(preset("tiny"), cs1_library="/nonexistent/libqwen3_5_cuda.so")


def test_cp_pieces_balance_and_alignment():
    """Context-parallel piece sizes: in order, on 64-token boundaries, summing to the prompt,
    and each rank's estimated work (projections + causal attention) within one 64-token step
    of the mean (2% at 32k tokens)."""
    from s1omni import cp_pieces, preset
    cfg = preset("27b")
    lin = cfg.projection_flops_per_token()
    att = 4.0 * cfg.heads * cfg.head_dim * sum(1 for t in cfg.layer_types if t != "gdn")
    for tokens, world in ((32768, 2), (32768, 4), (32768, 8), (8192, 3)):
        lengths = cp_pieces(cfg, tokens, world)
        assert len(lengths) == world and sum(lengths) == tokens
        assert all(n % 64 == 0 for n in lengths[:-1]) and lengths[-1] >= 64
        starts = np.concatenate([[0], np.cumsum(lengths)[:-1]])
        cost = [lin * n + att * n * (s + n / 2) for s, n in zip(starts, lengths)]
        step = 64 / (tokens / world)  # relative size of one alignment step
        assert max(cost) / np.mean(cost) < 1 + max(0.02, step), (tokens, world, lengths)
    with pytest.raises(ValueError):
        cp_pieces(cfg, 200, 4)


def test_dispatch_lpt_balances_and_matches_restatement():
    """s1_dispatch_lpt (C++ host) against a plain restatement of longest-processing-time
    first, and its makespan against the 4/3 bound of the greedy, on log-normal costs."""
    from s1omni import dispatch, request_cost, preset
    rng = np.random.default_rng(0)
    cfg = preset("27b")
    lens = np.clip(np.round(np.exp(rng.normal(np.log(800.0), 0.6, 256))), 1, 8192).astype(int)
    costs = [request_cost(cfg, int(n)) for n in lens]
    for ranks in (1, 2, 3, 8):
        rank_of, loads = dispatch(costs, ranks)
        # restatement: decreasing cost (stable on index), least-loaded rank (lowest index on ties)
        order = sorted(range(len(costs)), key=lambda i: -costs[i])
        want, load = [0] * len(costs), [0.0] * ranks
        for i in order:
            r = min(range(ranks), key=lambda j: (load[j], j))
            want[i] = r
            load[r] += costs[i]
        assert rank_of == want
        assert np.allclose(loads, load)
        assert max(loads) <= (4.0 / 3.0) * max(sum(costs) / ranks, max(costs)) + 1e-6
    assert dispatch([], 4) == ([], [0.0] * 4)
    with pytest.raises(ValueError):
        dispatch([1.0, -1.0], 2)
    with pytest.raises(ValueError):
        dispatch([1.0], 0)


def test_request_cost_counts_candidates_over_the_prompt():
    from s1omni import request_cost, preset
    cfg = preset("9b")
    lin = cfg.projection_flops_per_token()
    assert request_cost(cfg, 100, [10, 20]) > request_cost(cfg, 100) + lin * 30
    assert request_cost(cfg, 0, [64]) == request_cost(cfg, 64)


def test_batch_descriptor_layout_and_work_index():
    """The capacity path's descriptor, packed on the host without a GPU: packed row
    offsets, sequences by decreasing length (stable), and the prefix sums of 128-row
    query blocks in that order that the attention kernel's CTAs search for their
    (sequence, query block)."""
    from s1omni import Cs1
    cs1 = Cs1()
    MAX = 256
    n = cs1.cs1_batch_desc_bytes()
    assert n == 4 * (4 + 2 + (MAX + 1) + MAX + (MAX + 1))
    rng = np.random.default_rng(11)
    for lengths in ([1], [128], [129], [37, 100, 5, 64, 100, 300], list(rng.integers(1, 3000, 256))):
        buf = np.zeros(n, np.uint8)
        arr = np.asarray(lengths, dtype=np.uintp)
        assert cs1.raw.cs1_batch_desc_pack(arr.ctypes.data, len(lengths), buf.ctypes.data, n) == 0
        w = buf.view(np.int32)
        rows, tab = w[0], w[4:]
        count, max_len = tab[0], tab[1]
        offset = tab[2:2 + MAX + 1]
        order = tab[2 + MAX + 1:2 + MAX + 1 + MAX]
        qcum = tab[2 + MAX + 1 + MAX:]
        c = len(lengths)
        assert (rows, count, max_len) == (sum(lengths), c, max(lengths))
        assert list(offset[:c + 1]) == [0] + list(np.cumsum(lengths))
        want_order = sorted(range(c), key=lambda i: (-lengths[i], i))
        assert list(order[:c]) == want_order
        blocks = [(lengths[i] + 127) // 128 for i in want_order]
        assert list(qcum[:c + 1]) == [0] + list(np.cumsum(blocks))
        # the kernel's search: the last i with qcum[i] <= target, block counted from the end
        for target in range(int(qcum[c])):
            lo, hi = 0, c
            while hi - lo > 1:
                mid = (lo + hi) // 2
                lo, hi = (mid, hi) if qcum[mid] <= target else (lo, mid)
            seq, qb = order[lo], qcum[lo + 1] - 1 - target
            assert 0 <= qb < (lengths[seq] + 127) // 128
        seen = set()
        for target in range(int(qcum[c])):
            lo = int(np.searchsorted(qcum[:c + 1], target, side="right")) - 1
            seen.add((int(order[lo]), int(qcum[lo + 1] - 1 - target)))
        assert seen == {(i, b) for i in range(c) for b in range((lengths[i] + 127) // 128)}
