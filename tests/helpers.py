"""Numeric comparison helpers and fixture paths shared by the tests."""
from __future__ import annotations

import os

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_host.npz")
GOLDEN_SUBBLOCK = os.path.join(ROOT, "tests", "golden", "reference_subblock.npz")
GOLDEN_ROPE = os.path.join(ROOT, "tests", "golden", "reference_rope.npz")
GOLDEN_DDIM = os.path.join(ROOT, "tests", "golden", "reference_ddim.npz")
GOLDEN_TEMPORAL_MASK = os.path.join(ROOT, "tests", "golden", "reference_temporal_mask.npz")

# Parity bar of the benchmark spec for bf16 kernels against the fp32 oracle.
REL_L2_TOL = 1e-2
COS_TOL = 0.999


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().double().cpu().reshape(-1), b.detach().double().cpu().reshape(-1)
    return float(a @ b / (a.norm() * b.norm()).clamp_min(1e-30))
