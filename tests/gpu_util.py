"""Shared helpers of the GPU parity tests (seeded inputs, device buffers)."""
from __future__ import annotations

import numpy as np

import oracle as O

# fp32 outputs must match the oracle within 1e-3 relative (normwise: max abs
# error over max |reference|); bf16 tensor-core paths within 2e-2.
RTOL_F32 = 1e-3
RTOL_BF16 = 2e-2


def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        import pytest
        pytest.skip("no CUDA device")
    return torch


def to_dev(a: np.ndarray):
    torch = torch_cuda()
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t


def empty_dev(shape, dtype):
    torch = torch_cuda()
    return torch.empty(shape, dtype=dtype, device="cuda")


def rel_err(y: np.ndarray, ref: np.ndarray) -> float:
    ref = np.asarray(ref, dtype=np.float64)
    den = max(np.max(np.abs(ref)), 1e-30)
    return float(np.max(np.abs(np.asarray(y, dtype=np.float64) - ref)) / den)


def make_lowbit(rng, n, k, bits, n_groups, sz_f16=False, zp_mode="array", unsigned_mid=False):
    """Random packed weights in the reference layout with group scales.
    zp_mode: 'array' (float zero-points), 'int' (integer zero-points), 'none'."""
    w = rng.integers(0, 256, size=(n, O.row_bytes(k, bits)), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, size=(n, n_groups)).astype(np.float32)
    if zp_mode == "array":
        zp = rng.uniform(-2.0, 2.0, size=(n, n_groups)).astype(np.float32)
    elif zp_mode == "int":
        lo, hi = -(1 << (bits - 1)), (1 << (bits - 1)) - 1
        zp = rng.integers(lo, hi + 1, size=(n, n_groups)).astype(np.float32)
    else:
        zp = None
    if sz_f16:
        s = s.astype(np.float16)
        zp = zp.astype(np.float16) if zp is not None else None
    return w, s, zp


def dequant_np(w, n, k, bits, s, zp, n_groups, unsigned=False, zp_const=0.0):
    """Vectorized numpy dequant (pinned to the oracle by test_gpu_lowbit)."""
    codes = O.unpack_rows_np(w, n, k, bits, unsigned=unsigned).astype(np.float64)
    gi = np.minimum((np.arange(k) * n_groups) // k, n_groups - 1) if n_groups > 1 else np.zeros(k, dtype=np.int64)
    sv = np.asarray(s, dtype=np.float64).reshape(n, n_groups)[:, gi]
    zv = np.asarray(zp, dtype=np.float64).reshape(n, n_groups)[:, gi] if zp is not None else zp_const
    return (codes - zv) * sv
