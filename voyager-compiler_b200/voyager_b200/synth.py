"""Seeded synthetic inputs for the benchmark configurations.

The reference names no dataset for this path; its configurations are
synthetic tensors of stated shapes and distributions.  Inputs are drawn with
numpy's PCG64 generator (bit-reproducible on every host that runs the same
numpy build), in float32, and rounded to bfloat16 nearest-even where the
configuration is bfloat16.  Arrays are returned as numpy (bfloat16 as uint16
bit patterns) so the same bytes feed the CUDA path, the CPU oracle and the
golden fixtures.
"""

from typing import Tuple

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns, nearest-even (NaN -> 0xFFFF)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r[nan] = 0xFFFF
    return r


def normal(shape: Tuple[int, ...], std: float, seed: int) -> np.ndarray:
    """float32 N(0, std^2) of ``shape`` from PCG64(seed)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal(size=shape, dtype=np.float32)
    if std != 1.0:
        x *= np.float32(std)
    return x


def c1_input(rows: int = 4096, cols: int = 4096) -> np.ndarray:
    """C1: N(0,1) with 1% of positions (seeded, uniform) scaled x50, bf16."""
    x = normal((rows, cols), 1.0, seed=0)
    n = x.size
    pos = np.random.Generator(np.random.PCG64(1)).permutation(n)[: n // 100]
    x.reshape(-1)[pos] *= np.float32(50.0)
    return f32_to_bf16_bits(x)


def c2_weight(rows: int = 11008, cols: int = 4096) -> np.ndarray:
    """C2: float32 weights N(0, 0.02^2)."""
    return normal((rows, cols), 0.02, seed=0)


def c3_operands(m: int = 8192, k: int = 4096, n: int = 11008):
    """C3: activations N(0,1) [M,K] and weights N(0,0.02^2) [N,K], bf16."""
    a = f32_to_bf16_bits(normal((m, k), 1.0, seed=0))
    w = f32_to_bf16_bits(normal((n, k), 0.02, seed=1))
    return a, w


def c4_operands(m: int, k: int, n: int):
    """C4: activations N(0,1) [M,K], weights N(0,0.02^2) [N,K], bf16."""
    a = f32_to_bf16_bits(normal((m, k), 1.0, seed=2))
    w = f32_to_bf16_bits(normal((n, k), 0.02, seed=3))
    return a, w
