"""Helpers for the GPU parity tests: seeded golden-case inputs as CUDA
tensors, device pointer arrays, and byte digests of device buffers."""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from tests.golden import gen


def to_dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr_array(tensors) -> torch.Tensor:
    return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64, device="cuda")


def dsha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest()


class DeviceKV:
    """Paged layers of a golden case on the GPU (uint8, flat per layer)."""

    def __init__(self, case: dict, zero: bool = False, seed: int | None = None):
        self.case = case
        k, v = gen.paged_layers(case, seed=seed, zero=zero)
        self.k = [to_dev(a) for a in k]
        self.v = [to_dev(a) for a in v] if v is not None else None
        self.kp = ptr_array(self.k)
        self.vp = ptr_array(self.v) if self.v is not None else None

    def host(self):
        return ([t.cpu().numpy() for t in self.k],
                [t.cpu().numpy() for t in self.v] if self.v is not None else None)
