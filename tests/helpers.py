"""Seeded synthetic inputs and comparison helpers shared by the tests."""

from __future__ import annotations

import numpy as np
import torch

DISTS = ("n05", "n1", "n1_outlier", "qk_div8", "zeros", "tiny", "huge")


def gen_bf16(
    shape: tuple[int, ...], dist: str, seed: int, dtype: torch.dtype = torch.bfloat16
) -> torch.Tensor:
    """bf16 (or ``dtype``) CPU tensor drawn from a named distribution with a fixed seed.

    n05: N(0, 0.5); n1: N(0, 1); n1_outlier: N(0, 1) with 1 % of entries x20
    (mask from the same generator); qk_div8: N(0, 1) / 8 (the reference's own
    FP8 test input, tests/test_attention_cuda.py:159-161); zeros; tiny: values
    around 1e-7 (amax below the 1e-6 floor); huge: N(0, 1) * 1e30.
    """
    g = torch.Generator().manual_seed(seed)
    if dist == "n05":
        x = torch.randn(shape, generator=g) * 0.5
    elif dist == "n1":
        x = torch.randn(shape, generator=g)
    elif dist == "n1_outlier":
        x = torch.randn(shape, generator=g)
        mask = torch.rand(shape, generator=g) < 0.01
        x = torch.where(mask, x * 20.0, x)
    elif dist == "qk_div8":
        x = torch.randn(shape, generator=g) / 8.0
    elif dist == "zeros":
        x = torch.zeros(shape)
    elif dist == "tiny":
        x = torch.randn(shape, generator=g) * 1e-7
    elif dist == "huge":
        x = torch.randn(shape, generator=g) * 1e30
    else:
        raise ValueError(dist)
    return x.to(dtype)


def bits(t: torch.Tensor) -> np.ndarray:
    """16-bit (bf16 / fp16) tensor -> uint16 bit patterns (CPU, contiguous)."""
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def fp8_bytes(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.uint8).numpy()


def bytes_equal_nan_aware(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Elementwise equality of e4m3 bytes where any two NaN encodings match."""
    nan_a = (a & 0x7F) == 0x7F
    nan_b = (b & 0x7F) == 0x7F
    return (a == b) | (nan_a & nan_b)


def scales_equal(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))
