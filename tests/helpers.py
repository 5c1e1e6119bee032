"""Seeded inputs and comparison helpers shared by the tests and the fixture scripts."""
from __future__ import annotations

import hashlib

import torch


def randn_half(shape, seed: int, scale: float = 1.0) -> torch.Tensor:
    """fp16 ~N(0, scale^2) from a CPU generator seeded with `seed`."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(tuple(shape), generator=g, dtype=torch.float32) * scale).to(torch.float16)


def sha256_of(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def fp16_ulp_diff(a: torch.Tensor, b: torch.Tensor) -> int:
    """Largest distance in fp16 units-in-the-last-place between a and b (same shape)."""
    def ordered(x):
        bits = x.contiguous().cpu().view(torch.int16).to(torch.int32)
        mag = bits & 0x7FFF
        return torch.where(bits < 0, -mag, mag)

    if a.numel() == 0:
        return 0
    return int((ordered(a) - ordered(b)).abs().max())


NAN16 = float("nan")
