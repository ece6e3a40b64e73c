"""Helpers shared by the GPU tests: moving bf16 bit arrays to and from torch."""
import numpy as np


def torch_mod():
    import torch
    return torch


def dev(a: np.ndarray, device: str = "cuda:0"):
    """numpy uint16 (bf16 bits) / int32 / float32 -> CUDA tensor with the same bits."""
    torch = torch_mod()
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(device)
    return torch.from_numpy(a).to(device)


def host_u16(t) -> np.ndarray:
    return t.cpu().numpy().view(np.uint16)


def bf16_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def empty_u16(shape, device: str = "cuda:0"):
    torch = torch_mod()
    return torch.empty(shape, dtype=torch.int16, device=device)


def max_abs(a, b) -> float:
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0


def bf16_ulps(a_bits, b_bits) -> np.ndarray:
    """Distance in bf16 ulps between two bf16 bit arrays (sign-magnitude mapped
    to a monotone integer line, so +0/-0 and sign crossings count correctly)."""
    a = np.asarray(a_bits, np.uint16).astype(np.int32)
    b = np.asarray(b_bits, np.uint16).astype(np.int32)
    a = np.where(a & 0x8000, 0x8000 - (a & 0x7FFF), a + 0x8000)
    b = np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), b + 0x8000)
    return np.abs(a - b)


def f32_to_bf16_bits(x) -> np.ndarray:
    """Upper half of f32 values that hold bf16 values."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)
