"""Regenerates tests/golden/torch_randn.npz: torch.randn(n, generator=torch.manual_seed(seed)) values that pin
the oracle's restatement of rng.rs TorchGen.  Run from the repo root: python tests/golden/gen_golden.py"""
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    cases = [(0, 8), (0, 16), (42, 37), (1234, 100), (7, 1000)]
    out = {}
    for seed, n in cases:
        g = torch.Generator().manual_seed(seed)
        out[f"s_{seed}_{n}"] = torch.randn(n, generator=g, dtype=torch.float32).numpy()
    np.savez(os.path.join(HERE, "torch_randn.npz"), **out)


if __name__ == "__main__":
    main()
