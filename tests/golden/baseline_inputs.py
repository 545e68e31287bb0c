"""Seeded inputs of the BASELINE GEMM configurations, identical on every host.

Config 1 is C = A B with A[512 x 4096], B[4096 x 4096] (W = B^T [4096 x
4096] in nn.Linear layout), values N(0, 1) * K^-1/2 rounded to bf16, one
fault of +2^8 max|C| at ``random.Random(seed).randrange(M * N)`` (the index
scheme of pytorch/abft/injector.py:71). The fixtures store the reference's
check results and SHA-256 digests of these inputs, not the tensors: the
tests regenerate them and assert the digests first.

Values come from numpy's PCG64 generator (integer state, ziggurat normals)
and are rounded to bf16 by ``oracle.abft_oracle.f32_to_bf16_bits``; the
output C is the float64 product rounded to float32 and then to bf16, so a
GPU float64 GEMM gives the same bits (checked by the digest).
"""
from __future__ import annotations

import hashlib
import random
from typing import Tuple

import numpy as np

from oracle.abft_oracle import bf16_bits_to_f32, f32_to_bf16_bits

CONFIG1 = {"M": 512, "K": 4096, "N": 4096}


def sha256_bits(bits: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(bits, dtype="<u2").tobytes()).hexdigest()


def gemm_inputs(seed: int, m: int, k: int, n: int) -> Tuple[np.ndarray, np.ndarray]:
    """(A bits [m, k], W bits [n, k]) as uint16 bf16 storage."""
    rng = np.random.default_rng(seed)
    a = f32_to_bf16_bits((rng.standard_normal((m, k)) * k ** -0.5).astype(np.float32))
    w = f32_to_bf16_bits((rng.standard_normal((n, k)) * k ** -0.5).astype(np.float32))
    return a, w


def product_bits(a_bits: np.ndarray, w_bits: np.ndarray) -> np.ndarray:
    """bf16(float32(A W^T)) with the product in float64, on the CPU."""
    a = bf16_bits_to_f32(a_bits).astype(np.float64)
    w = bf16_bits_to_f32(w_bits).astype(np.float64)
    return f32_to_bf16_bits((a @ w.T).astype(np.float32))


def fault_for(seed: int, c_bits: np.ndarray) -> Tuple[int, float]:
    """(flat index, magnitude) of the seeded fault: 2^8 max|C| at
    random.Random(seed).randrange(M * N)."""
    idx = random.Random(seed).randrange(c_bits.size)
    mag = float(2.0 ** 8 * np.abs(bf16_bits_to_f32(c_bits)).max())
    return idx, mag
