"""Shared helpers of the GPU parity tests (not collected as tests)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import numerics

REL_TOL = 2e-2  # max |y - ref| / max |ref|, the reference's gate (verify_v3.py:26)


def rel_err(y, ref) -> float:
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = max(np.abs(ref).max(), 1e-30)
    return float(np.abs(y - ref).max() / den)


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def ulps(y, ref) -> np.ndarray:
    return numerics.ulp_diff_bf16(np.asarray(y, np.float32), np.asarray(ref, np.float32))


def dev() -> torch.device:
    return torch.device("cuda", torch.cuda.current_device())
