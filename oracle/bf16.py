"""bfloat16 rounding for the oracle (test infrastructure only).

Round-to-nearest-even from float32, the conversion `__float2bfloat16` performs
in the reference kernels (`src/backends/cuda/qwen3_5/common.cuh:14-15`) and
that PyTorch applies when it stores a bfloat16 result.
"""
import numpy as np


def bits(x):
    """float32 array -> uint16 bfloat16 bit patterns (RNE, NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def from_bits(b):
    """uint16 bfloat16 bit patterns -> float32."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def rnd(x):
    """Round a float array through bfloat16, returning float32."""
    return from_bits(bits(np.asarray(x, dtype=np.float32)))
