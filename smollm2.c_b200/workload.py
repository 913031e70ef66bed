"""Seeded synthetic inputs with the shapes and value distributions of the
LoRA-on-lm_head workloads (the real SmolLM2 GGUF and datasets are not
available, so every run draws its inputs from a seed).

Distributions (N(mean, std) throughout):
  W  [V][d]  f16   N(0, 0.02)              tied token_embd / lm_head
  h  [T][d]  bf16  N(0, 1)                 post-final-RMSNorm hidden states
  A  [d][r]  fp32  N(0, 1/sqrt(d))         i.e. variance 1/d (unit-variance h.A)
  B  [r][V]  fp32  N(0, 1e-3)
  targets    int32 bounded Zipf(s=1.1) over ids 0..V-1 (p(k) ~ k^-1.1,
                   id = k-1), inverse-CDF sampling.
A and B are returned in the reference layouts (A[d*r + j], B[j*V + v],
src/train.c:35-36).
"""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + 0x7FFF
    return ((u + rounding) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f16_exact(h_f32: np.ndarray) -> np.ndarray:
    """The f32 values the tensor cores see after an RN conversion to f16."""
    return np.asarray(h_f32, np.float32).astype(np.float16).astype(np.float32)


def zipf_targets(rng: np.random.Generator, n: int, V: int, s: float = 1.1) -> np.ndarray:
    k = np.arange(1, V + 1, dtype=np.float64)
    cdf = np.cumsum(k ** (-s))
    cdf /= cdf[-1]
    u = rng.random(n)
    return np.minimum(np.searchsorted(cdf, u, side="right"), V - 1).astype(np.int32)


def make_weight(seed: int, V: int, d: int) -> np.ndarray:
    """W [V][d] as f16 bit patterns (uint16)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((V, d), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    return w.view(np.uint16)


def make_step_inputs(seed: int, T: int, V: int, d: int, r: int):
    """h (bf16 bits), targets, A [d][r], B [r][V] for one step."""
    rng = np.random.default_rng(seed + 1)
    h = f32_to_bf16_bits(rng.standard_normal((T, d), dtype=np.float32))
    A = (rng.standard_normal((r, d), dtype=np.float32) * np.float32(1.0 / np.sqrt(d))).T.copy()
    B = (rng.standard_normal((V, r), dtype=np.float32) * np.float32(1e-3)).T.copy()
    tgt = zipf_targets(rng, T, V)
    return h, tgt, A, B


def oracle_hidden(h_bf16: np.ndarray) -> np.ndarray:
    """Hidden rows as the kernels consume them (bf16 -> f16 RN), in f32."""
    return f16_exact(bf16_bits_to_f32(h_bf16))


def make_weight_q4k(seed: int, V: int, d: int) -> np.ndarray:
    """W [V][d] as Q4_K super-blocks over the flattened tensor
    (V*d/256 blocks of 144 bytes): d and dmin f16 drawn uniformly from
    [4e-5, 1.2e-4] (weights of about the spread of N(0, 0.02)), the 12 scale
    bytes (eight 6-bit scale / min pairs) and the
    128 quant bytes (4-bit values) uniform random bytes."""
    assert (V * d) % 256 == 0
    n = V * d // 256
    rng = np.random.default_rng(seed)
    blocks = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    dd = rng.uniform(4e-5, 1.2e-4, size=(n, 2)).astype(np.float16)
    blocks[:, 0:4] = dd.view(np.uint8).reshape(n, 4)
    return blocks


def q4k_dequant_np(blocks: np.ndarray) -> np.ndarray:
    """Q4_K -> f32 in numpy (float32 arithmetic, each product and the
    difference rounded separately): an independent restatement of the
    format used to cross-check the C restatement in the tests."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 144)
    n = b.shape[0]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    q = b[:, 4:16].astype(np.int32)
    sc = np.empty((n, 8), np.int32)
    mn = np.empty((n, 8), np.int32)
    sc[:, :4] = q[:, 0:4] & 63
    mn[:, :4] = q[:, 4:8] & 63
    sc[:, 4:] = (q[:, 8:12] & 15) | ((q[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (q[:, 8:12] >> 4) | ((q[:, 4:8] >> 6) << 4)
    qs = b[:, 16:144].reshape(n, 4, 32).astype(np.int32)
    nib = np.stack([qs & 15, qs >> 4], axis=2).reshape(n, 8, 32)  # sub-block 2c, 2c+1
    dsc = (d[:, None] * sc.astype(np.float32)).astype(np.float32)
    mm = (dmin[:, None] * mn.astype(np.float32)).astype(np.float32)
    p = (dsc[:, :, None] * nib.astype(np.float32)).astype(np.float32)
    return (p - mm[:, :, None]).astype(np.float32).reshape(-1)


def make_adam_inputs(seed: int, d: int, V: int, r: int, k: int):
    """An adapter and k steps of gradient sums for optimizer-only checks:
    A [d][r], B [r][V], gA [k][d][r], gB [k][r][V] with magnitudes spread
    over many decades (and some exact zeros), n_pred [k]."""
    rng = np.random.default_rng(seed)
    A = (rng.standard_normal((d, r)) / np.sqrt(d)).astype(np.float32)
    B = (rng.standard_normal((r, V)) * 1e-3).astype(np.float32)
    gA = (rng.standard_normal((k, d, r)) * 10.0 ** rng.uniform(-6, 2, (k, d, r))).astype(np.float32)
    gB = (rng.standard_normal((k, r, V)) * 10.0 ** rng.uniform(-9, 1, (k, r, V))).astype(np.float32)
    gB[:, :, ::97] = 0.0
    n_pred = rng.integers(1, 70000, k).astype(np.int32)
    return A, B, gA, gB, n_pred
