"""Helpers shared by the GPU parity tests: numpy <-> torch conversions and seeded inputs."""
import numpy as np
import torch

from oracle import oracle as O


def bf16_tensor(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(dev).view(torch.bfloat16)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def t(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def linear_inputs(seed, M, K, N, dev):
    x, w, ws, bias = O.make_linear_inputs(seed, M, K, N)
    return (x, w, ws, bias), (bf16_tensor(x, dev), t(w, dev), t(ws, dev), t(bias, dev))
