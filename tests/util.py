"""Test helpers: numpy <-> torch conversions (bf16 as uint16 bit patterns)."""

from __future__ import annotations

import numpy as np
import torch


def bf16_t(bits: np.ndarray, device=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).astype(np.uint16).view(np.int16)).view(torch.bfloat16)
    return t.to(device) if device is not None else t


def u8_t(a: np.ndarray, device=None) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint8))
    return t.to(device) if device is not None else t


def np_f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def rel(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12))
