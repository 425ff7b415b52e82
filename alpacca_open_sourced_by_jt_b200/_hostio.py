"""Host <-> device copies for the NumPy-facing drop-in functions.

Uploads go through a pinned staging tensor so the copy is a real DMA from
page-locked memory; downloads return fresh NumPy arrays (the reference's
functions return fresh arrays, never views of shared buffers).
"""
from __future__ import annotations

import numpy as np
import torch


def _device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("the B200 attention path needs a CUDA device (no CPU fallback)")
    return torch.device("cuda", torch.cuda.current_device())


def to_device(a: np.ndarray) -> torch.Tensor:
    h = torch.from_numpy(np.ascontiguousarray(a))
    return h.pin_memory().to(_device(), non_blocking=True)


def to_host(t: torch.Tensor) -> np.ndarray:
    return t.detach().to("cpu").numpy().copy()
