"""Request dispatch over GPUs: one process per GPU, each with a full weight replica.

The reference serves one GPU per worker process and groups the requests queued at a
worker into launches (`src/runtime/src/batching.rs:94-125`, with the limits of
`src/models/open_jev/native/src/executor/batched.rs:28-31`). Across GPUs the work shards
by request (a request's candidates stay together: they share a prefix), so the one
decision left is which GPU serves which request. `dispatch` makes it by token cost,
longest processing time first (C++ host: `s1_dispatch_lpt`), so that every GPU finishes
at about the same time; `request_cost` is the cost model.
"""
import ctypes

import numpy as np

from .model import _get


def request_cost(cfg, prompt, candidates=()):
    """Estimated FLOPs of one request: the projection FLOPs of every token it runs
    (prompt once, then each candidate), plus causal attention, which grows with the keys
    each query sees (the prompt's own triangle, then each candidate over the prompt and
    its own earlier tokens). `prompt` and `candidates` are token counts."""
    lin = cfg.projection_flops_per_token()
    att = 4.0 * cfg.heads * cfg.head_dim * sum(1 for t in cfg.layer_types if t != "gdn")
    p = float(prompt)
    cost = lin * p + att * p * (p + 1) / 2.0
    for c in candidates:
        c = float(c)
        cost += lin * c + att * c * (p + (c + 1) / 2.0)
    return cost


def dispatch(costs, ranks):
    """Rank of each request (list of ints) and the per-rank cost totals, longest
    processing time first: requests in decreasing cost, each to the least-loaded rank."""
    lib = _get()
    lib.s1_dispatch_lpt.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_void_p,
                                    ctypes.c_void_p]
    c = np.ascontiguousarray(costs, dtype=np.float64)
    rank_of = np.zeros(len(c), np.int32)
    loads = np.zeros(max(ranks, 1), np.float64)
    if lib.s1_dispatch_lpt(c.ctypes.data if len(c) else None, len(c), ranks, rank_of.ctypes.data if len(c) else None,
                           loads.ctypes.data) != 0:
        raise ValueError("dispatch: ranks must be >= 1 and costs finite and non-negative")
    return rank_of.tolist(), loads.tolist()


def shard(items, costs, ranks, rank):
    """The items (in their original order) that `dispatch` gives to `rank`."""
    rank_of, _ = dispatch(costs, ranks)
    return [x for x, r in zip(items, rank_of) if r == rank]
