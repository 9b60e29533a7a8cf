"""Candidate packing, shared prefixes, positions and rotary tables
(test infrastructure only).

Restates the host-side integer and table logic of the reference:
* `ranges`         -- `src/models/open_jev/native/src/batching.rs:9-25`
* `shared_prefix`  -- `batching.rs:29-49` (common prefix floored to 64, >= 512)
* `layout`         -- the packed row layout of `model.rs:1548-1632`: per-sequence
                      offsets, positions restarting at 0 (or continuing at the
                      prefix length for shared-prefix suffixes, `model.rs:3240`)
                      and the final-token row of each sequence
* `rotary_tables`  -- `src/models/qwen3_5/native/src/inputs.rs:178-204`
"""
import numpy as np

from .bf16 import bits, rnd

MAX_SEQUENCES = 16
MAX_TOKENS = 4096


def ranges(lengths, max_sequences=MAX_SEQUENCES, max_tokens=MAX_TOKENS):
    """Order-keeping packing of candidate prompts into launches (batching.rs:9-25):
    a launch closes before a candidate that would make it hold max_sequences
    prompts or exceed max_tokens tokens; a long prompt runs alone."""
    out = []
    start = 0
    tokens = 0
    for i, n in enumerate(lengths):
        if i > start and (i - start == max_sequences or tokens + n > max_tokens):
            out.append((start, i))
            start = i
            tokens = 0
        tokens += n
    if start < len(lengths):
        out.append((start, len(lengths)))
    return out


def shared_prefix(inputs, minimum=MAX_TOKENS // 2 + 1):
    """Common prefix of 2..16 candidates, floored to a multiple of 64, or 0
    (batching.rs:29-49). `minimum` is 2049 for the long-candidate path and 512
    for the packed path (`packed_shared_prefix`)."""
    if not (2 <= len(inputs) <= MAX_SEQUENCES) or any(len(x) < minimum for x in inputs):
        return 0
    shortest = min(len(x) for x in inputs)
    common = 0
    for i in range(shortest - 1):
        if all(x[i] == inputs[0][i] for x in inputs):
            common += 1
        else:
            break
    aligned = common // 64 * 64
    return aligned if aligned >= 512 else 0


def layout(lengths, prefix=0):
    """Packed rows: offsets [n], positions [sum], last-token rows [n] (int64), as
    `forward_batch_layout` builds them (`src/models/qwen3_5/native/src/model.rs:1548-1632`);
    with a prefix, positions continue at its length (`model.rs:3240`)."""
    lengths = [int(x) for x in lengths]
    offsets = np.zeros(len(lengths), np.int64)
    if lengths:
        offsets[1:] = np.cumsum(lengths)[:-1]
    positions = np.concatenate([prefix + np.arange(n, dtype=np.int64) for n in lengths]) if lengths else np.zeros(0, np.int64)
    last = offsets + np.asarray(lengths, np.int64) - 1
    return offsets, positions, last


def rotary_tables(positions, half, theta):
    """bf16 cos/sin [T, half] (inputs.rs:178-204): float32 inverse frequencies
    1 / theta^(2i / 2half), float32 angle, float64 cos/sin rounded to float32
    then bfloat16. Returns (cos, sin) as float32 arrays of bf16 values."""
    i = np.arange(half, dtype=np.float32)
    inv = (np.float32(1) / np.power(np.float32(theta), (np.float32(2) * i) / np.float32(2 * half))).astype(np.float32)
    pos = np.asarray(positions, dtype=np.int64).astype(np.float32)
    ang = (pos[:, None] * inv[None, :]).astype(np.float32).astype(np.float64)
    return rnd(np.cos(ang).astype(np.float32)), rnd(np.sin(ang).astype(np.float32))


def rotary_bits(positions, half, theta):
    """Same tables as uint16 bf16 bit patterns (for byte-exact comparison)."""
    c, s = rotary_tables(positions, half, theta)
    return bits(c), bits(s)
