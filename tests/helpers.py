"""Shared helpers for the GPU parity tests."""
import numpy as np
import torch


def bf16_from_bits(a: np.ndarray, device="cuda") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a, np.uint16).view(np.int16))
    return t.view(torch.bfloat16).to(device)


def bits_from_bf16(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def rand_bf16_bits(shape, seed, scale=1.0, quant=None) -> np.ndarray:
    """Seeded N(0, scale) values rounded to bf16 (optionally quantised to a grid,
    which creates many equal values)."""
    from oracle import ks_oracle as O

    rng = np.random.default_rng(seed)
    x = (rng.standard_normal(shape) * scale).astype(np.float32)
    if quant:
        x = (np.round(x * quant) / quant).astype(np.float32)
    return O.f32_to_bf16(x)
