"""numpy <-> torch helpers for the GPU tests (bf16 travels as uint16 bits)."""

import numpy as np
import torch


def to_dev(a, device="cuda"):
    if a is None:
        return None
    a = np.ascontiguousarray(a).reshape(np.shape(a))
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(device)
    return torch.from_numpy(a.copy()).to(device)


def to_np(t):
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()
