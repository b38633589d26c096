"""Helpers shared by the tests (inputs, bf16 bit patterns, tolerances)."""
import numpy as np
import torch

# Parity bar of the target spec: max-abs error on bf16 O and on fp32 LSE.
O_TOL = 2e-2
LSE_TOL = 1e-3


def bf16_from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def seeded_bf16(shape, seed, dist="randn"):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) if dist == "randn" else torch.rand(*shape, generator=g)
    return x.bfloat16()
