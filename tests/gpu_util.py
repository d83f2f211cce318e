"""Helpers for GPU parity tests: bf16 <-> numpy bit patterns and seeded inputs."""

import numpy as np
import torch


def t2u(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor (any device) -> numpy uint16 bit patterns."""
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def u2t(u: np.ndarray, device="cuda") -> torch.Tensor:
    """numpy uint16 bf16 bit patterns -> bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(u).view(np.int16)).view(torch.bfloat16).to(device)


def randn_bf16(shape, gen: torch.Generator, std=1.0, mean=0.0) -> torch.Tensor:
    return (torch.randn(*shape, generator=gen) * std + mean).to(torch.bfloat16)


def np_(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()
