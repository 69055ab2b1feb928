"""Seeded synthetic GGUF weights and activations for the MUL_MAT workloads.

Distributions (per block):
  Q4_K: d, dmin = f16(|N(0,1)| * 2e-3) (round-to-nearest-even, so some land
        as f16 subnormals); 6-bit scales/mins uniform in 0..63; 4-bit quants
        uniform in 0..15. The 12 packed scale bytes and the 128 quant bytes
        are a bijection of those fields, so uniform fields are uniform bytes.
  Q6_K: 6-bit quants uniform in 0..63 (uniform ql/qh bytes), int8 scales
        uniform in -128..127, d = f16(|N(0,1)| * 2e-3).
  Q8_0: int8 quants uniform in -127..127, d = f16(|N(0,1)| * 1e-2).
  Q5_K: as Q4_K, with the 32 high-bit bytes uniform (5-bit quants uniform in
        0..31).
  Q4_0: 4-bit quants uniform in 0..15, d = f16(|N(0,1)| * 1e-2).
  IQ4_XS: 6-bit sub-block scales and 4-bit level indices uniform (uniform
        scale and quant bytes), d = f16(|N(0,1)| * 5e-4), which puts the
        weights (d (ls - 32) level, |level| <= 127) in the other types' range.
Activations are f32 N(0,1). No public dataset is involved.

Model shapes are the per-layer MUL_MATs (name, src0 type, M rows, K).
"""
from __future__ import annotations

import numpy as np

from .jsep import (BLOCK_GEOMETRY, GGML_TYPE_IQ4_XS, GGML_TYPE_Q4_0, GGML_TYPE_Q4_K, GGML_TYPE_Q5_K, GGML_TYPE_Q6_K,
                   GGML_TYPE_Q8_0)

Q4_K, Q6_K, Q8_0 = GGML_TYPE_Q4_K, GGML_TYPE_Q6_K, GGML_TYPE_Q8_0
Q5_K, Q4_0 = GGML_TYPE_Q5_K, GGML_TYPE_Q4_0
IQ4_XS = GGML_TYPE_IQ4_XS

# Llama-3.2-3B decode: hidden 3072, FFN 8192, 24 q heads / 8 kv heads x 128.
LLAMA32_3B_LAYER = [
    ("attn_q", Q4_K, 3072, 3072),
    ("attn_k", Q4_K, 1024, 3072),
    ("attn_v", Q6_K, 1024, 3072),
    ("attn_output", Q4_K, 3072, 3072),
    ("ffn_gate", Q4_K, 8192, 3072),
    ("ffn_up", Q4_K, 8192, 3072),
    ("ffn_down", Q6_K, 3072, 8192),
]
LLAMA32_3B_LAYERS = 28

# Qwen3-8B decode: hidden 4096, FFN 12288, 36 layers, Q6_K output 151936 x 4096.
QWEN3_8B_LAYER = [
    ("attn_q", Q4_K, 4096, 4096),
    ("attn_k", Q4_K, 1024, 4096),
    ("attn_v", Q4_K, 1024, 4096),
    ("attn_output", Q4_K, 4096, 4096),
    ("ffn_gate", Q4_K, 12288, 4096),
    ("ffn_up", Q4_K, 12288, 4096),
    ("ffn_down", Q4_K, 4096, 12288),
]
QWEN3_8B_LAYERS = 36
QWEN3_8B_OUTPUT = ("output", Q6_K, 151936, 4096)

# Llama-3-8B prefill, 512 tokens.
LLAMA3_8B_PREFILL = [
    ("attn_q", Q4_K, 4096, 4096),
    ("attn_kv", Q4_K, 1024, 4096),
    ("ffn_gate_up", Q4_K, 14336, 4096),
    ("ffn_down", Q4_K, 4096, 14336),
]

# Gemma-2-2B, Q8_0: hidden 2304, FFN 9216, vocab 256000.
GEMMA2_2B_SHAPES = [
    ("ffn_up", Q8_0, 9216, 2304),
    ("ffn_down", Q8_0, 2304, 9216),
    ("output", Q8_0, 256000, 2304),
    ("attn_proxy", Q8_0, 2304, 2304),
]


def row_bytes(qtype: int, K: int) -> int:
    be, bb = BLOCK_GEOMETRY[qtype]
    assert K % be == 0
    return K // be * bb


def algorithmic_bytes(qtype: int, M: int, K: int, N: int) -> int:
    """M*K*bpw + N*K*4 + N*M*4 (weights read once, x read, y written)."""
    return M * row_bytes(qtype, K) + 4 * N * K + 4 * N * M


def _f16_scale(rng: np.random.Generator, n: int, scale: float) -> np.ndarray:
    return (np.abs(rng.standard_normal(n)) * scale).astype(np.float16)


def q4_k_blocks(rng: np.random.Generator, M: int, K: int) -> np.ndarray:
    nb = M * (K // 256)
    blk = np.empty((nb, 144), dtype=np.uint8)
    blk[:, 0:2] = _f16_scale(rng, nb, 2e-3).view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = _f16_scale(rng, nb, 2e-3).view(np.uint8).reshape(nb, 2)
    blk[:, 4:] = rng.integers(0, 256, size=(nb, 140), dtype=np.uint8)
    return blk.reshape(M, -1)


def q6_k_blocks(rng: np.random.Generator, M: int, K: int) -> np.ndarray:
    nb = M * (K // 256)
    blk = np.empty((nb, 210), dtype=np.uint8)
    blk[:, :208] = rng.integers(0, 256, size=(nb, 208), dtype=np.uint8)
    blk[:, 208:210] = _f16_scale(rng, nb, 2e-3).view(np.uint8).reshape(nb, 2)
    return blk.reshape(M, -1)


def q8_0_blocks(rng: np.random.Generator, M: int, K: int) -> np.ndarray:
    nb = M * (K // 32)
    blk = np.empty((nb, 34), dtype=np.uint8)
    blk[:, 0:2] = _f16_scale(rng, nb, 1e-2).view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    return blk.reshape(M, -1)


def q5_k_blocks(rng: np.random.Generator, M: int, K: int) -> np.ndarray:
    nb = M * (K // 256)
    blk = np.empty((nb, 176), dtype=np.uint8)
    blk[:, 0:2] = _f16_scale(rng, nb, 2e-3).view(np.uint8).reshape(nb, 2)
    blk[:, 2:4] = _f16_scale(rng, nb, 2e-3).view(np.uint8).reshape(nb, 2)
    blk[:, 4:] = rng.integers(0, 256, size=(nb, 172), dtype=np.uint8)
    return blk.reshape(M, -1)


def q4_0_blocks(rng: np.random.Generator, M: int, K: int) -> np.ndarray:
    nb = M * (K // 32)
    blk = np.empty((nb, 18), dtype=np.uint8)
    blk[:, 0:2] = _f16_scale(rng, nb, 1e-2).view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = rng.integers(0, 256, size=(nb, 16), dtype=np.uint8)
    return blk.reshape(M, -1)


def iq4_xs_blocks(rng: np.random.Generator, M: int, K: int) -> np.ndarray:
    nb = M * (K // 256)
    blk = np.empty((nb, 136), dtype=np.uint8)
    blk[:, 0:2] = _f16_scale(rng, nb, 5e-4).view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = rng.integers(0, 256, size=(nb, 134), dtype=np.uint8)
    return blk.reshape(M, -1)


def weights(rng: np.random.Generator, qtype: int, M: int, K: int) -> np.ndarray:
    if qtype == Q4_K:
        return q4_k_blocks(rng, M, K)
    if qtype == Q5_K:
        return q5_k_blocks(rng, M, K)
    if qtype == Q4_0:
        return q4_0_blocks(rng, M, K)
    if qtype == Q6_K:
        return q6_k_blocks(rng, M, K)
    if qtype == Q8_0:
        return q8_0_blocks(rng, M, K)
    if qtype == IQ4_XS:
        return iq4_xs_blocks(rng, M, K)
    raise ValueError(f"unsupported type {qtype}")


def activations(rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    return rng.standard_normal((N, K), dtype=np.float32)


def activations_with_outliers(rng: np.random.Generator, N: int, K: int, value: float,
                              blocks: tuple[str, ...] = ("first", "middle", "last")) -> np.ndarray:
    """N(0,1) activations with 1-4 channels per named 256-element block set to
    +-value, the shape of real residual streams (a few channels 100-1000x the
    rest): within such a block every other element is small next to the
    block maximum that scales the GEMV's activation limbs."""
    x = rng.standard_normal((N, K), dtype=np.float32)
    nb = K // 256
    idx = {"first": 0, "middle": nb // 2, "last": nb - 1}
    for n in range(N):
        for name in blocks:
            b = idx[name]
            ch = rng.choice(256, size=int(rng.integers(1, 5)), replace=False)
            x[n, b * 256 + ch] = np.float32(value) * rng.choice(np.array([-1.0, 1.0], dtype=np.float32), size=len(ch))
    return x


def weights_torch(gen, qtype: int, M: int, K: int, device):
    """Same distributions as weights(), generated on the device with torch."""
    import torch

    be, bb = BLOCK_GEOMETRY[qtype]
    nb = M * (K // be)
    blk = torch.randint(0, 256, (nb, bb), dtype=torch.uint8, device=device, generator=gen)

    def f16(scale):
        v = (torch.randn(nb, device=device, generator=gen).abs() * scale).to(torch.float16)
        return v.view(torch.uint8).view(nb, 2)

    if qtype in (Q4_K, Q5_K):
        blk[:, 0:2] = f16(2e-3)
        blk[:, 2:4] = f16(2e-3)
    elif qtype == Q4_0:
        blk[:, 0:2] = f16(1e-2)
    elif qtype == Q6_K:
        blk[:, 208:210] = f16(2e-3)
    elif qtype == IQ4_XS:
        blk[:, 0:2] = f16(5e-4)
    elif qtype == Q8_0:
        blk[:, 0:2] = f16(1e-2)
        q = torch.randint(-127, 128, (nb, 32), dtype=torch.int16, device=device, generator=gen)
        blk[:, 2:] = q.to(torch.int8).view(torch.uint8)
    else:
        raise ValueError(f"unsupported type {qtype}")
    return blk.view(M, -1)
