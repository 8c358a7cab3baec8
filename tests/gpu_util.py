"""Helpers shared by the GPU tests: bf16 bit patterns <-> CUDA tensors."""
import numpy as np
import torch


def to_dev_bf16(bits: np.ndarray, device="cuda:0") -> torch.Tensor:
    b = np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)
    return torch.from_numpy(b.copy()).to(device).view(torch.bfloat16)


def from_dev_bf16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_dev(a: np.ndarray, device="cuda:0") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).copy()).to(device)


def bf16_ulp_diff(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bf16 units of last place (sign-magnitude ordering)."""
    def key(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, -(x & 0x7FFF), x & 0x7FFF)
    return np.abs(key(a_bits) - key(b_bits))
