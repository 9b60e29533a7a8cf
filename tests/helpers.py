"""Shared helpers for the GPU parity tests: numpy <-> torch device tensors."""
import numpy as np
import torch


def dev_bf16(a):
    """numpy float32 (bf16-valued) -> cuda bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to("cuda").to(torch.bfloat16)


def dev_f32(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to("cuda")


def host(t):
    torch.cuda.synchronize()
    return t.detach().float().cpu().numpy()


def empty_bf16(*shape):
    return torch.empty(*shape, dtype=torch.bfloat16, device="cuda")


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
