"""Generate the committed golden fixtures for the quantized MUL_MAT path.

Run from the repository root (in a container that has the `gguf` package):

    python tests/golden/make_golden.py

Fixtures written next to this script:

q4k_kat.npz
    The reference's Q4_K known-answer test (tests/jsep-matmul-golden.test.ts:521-600,
    same vector as runQ4KSelfTest in smoke-test/p2-v2-spike.src.ts:154-253):
    one super-block with sc=[5,12,...,54], m=[3,7,...,31], nibbles[i]=i&15,
    d=0.05, dmin=0.01, src1[i]=((i%13)-6)*0.15, M=1, K=256, N=1. The reference
    computes its expected values at run time with its own JS helpers; they are
    restated below in numpy with the same arithmetic: the f16 encoder
    f32ToF16Bits truncates the mantissa and flushes subnormals
    (jsep-matmul-golden.test.ts:103-127), packQ4_K dequantizes in f64 and
    stores to a Float32Array (:200-254), cpuMatmul accumulates in f64 (JS
    numbers) and stores f32 (:67-90).
q4k_synth_64x2048.npz
    buildSyntheticQ4KMatrix(64, 2048) with the N=6 activations of
    runMatmulProductionSelfTest (smoke-test/p2-v2-spike.src.ts:287-330,340-360),
    expected dequant and the f64-accumulated reference product.
gguf_blocks.npz
    Random blocks of Q4_K, Q6_K, Q8_0, Q5_K, Q4_0 and IQ4_XS (seeded) with
    the dequantization of the third-party `gguf` python package 0.19.0
    (gguf.quants.dequantize), the published ggml block formats the
    reference's llama.cpp fork uses. The reference repository has no
    Q6_K/Q8_0/Q5_K/Q4_0/IQ4_XS code of its own.
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def f32_to_f16_bits_js(f: float) -> int:
    """f32ToF16Bits (jsep-matmul-golden.test.ts:103-127): truncating, FTZ."""
    u32 = int(np.array([f], dtype=np.float32).view(np.uint32)[0])
    sign = (u32 >> 31) & 1
    exp32 = (u32 >> 23) & 0xFF
    mant32 = u32 & 0x7FFFFF
    if exp32 == 0xFF:
        return (sign << 15) | 0x7C00 | (1 if mant32 else 0)
    exp16 = exp32 - 127 + 15
    if exp16 >= 0x1F:
        return (sign << 15) | 0x7C00
    if exp16 <= 0:
        return sign << 15
    return (sign << 15) | (exp16 << 10) | (mant32 >> 13)


def f16_bits_to_f64(bits: int) -> float:
    """f16BitsToF32 (jsep-matmul-golden.test.ts:256-272), a JS double."""
    sign = (bits >> 15) & 1
    exp = (bits >> 10) & 0x1F
    mant = bits & 0x3FF
    if exp == 0:
        v = 2.0 ** -14 * (mant / 1024)
    elif exp == 0x1F:
        v = float("nan") if mant else float("inf")
    else:
        v = 2.0 ** (exp - 15) * (1 + mant / 1024)
    return -v if sign else v


def pack_q4_k(d: float, dmin: float, sc, m, nibbles):
    """packQ4_K (jsep-matmul-golden.test.ts:200-254): 144 bytes + f32 dequant."""
    b = np.zeros(144, dtype=np.uint8)
    db, dminb = f32_to_f16_bits_js(d), f32_to_f16_bits_js(dmin)
    b[0], b[1] = db & 0xFF, db >> 8
    b[2], b[3] = dminb & 0xFF, dminb >> 8
    for j in range(4):
        b[4 + j] = (sc[j] & 0x3F) | (((sc[j + 4] >> 4) & 3) << 6)
        b[8 + j] = (m[j] & 0x3F) | (((m[j + 4] >> 4) & 3) << 6)
        b[12 + j] = (sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4)
    for p in range(4):
        for l in range(32):
            b[16 + 32 * p + l] = (nibbles[64 * p + l] & 0xF) | ((nibbles[64 * p + 32 + l] & 0xF) << 4)
    dd, dm = f16_bits_to_f64(db), f16_bits_to_f64(dminb)
    deq = np.zeros(256, dtype=np.float64)
    for p in range(4):
        d1, m1 = dd * sc[2 * p], dm * m[2 * p]
        d2, m2 = dd * sc[2 * p + 1], dm * m[2 * p + 1]
        for l in range(32):
            deq[64 * p + l] = d1 * nibbles[64 * p + l] - m1
            deq[64 * p + 32 + l] = d2 * nibbles[64 * p + 32 + l] - m2
    return b, deq.astype(np.float32)  # Float32Array store


def cpu_matmul_js(src0: np.ndarray, src1: np.ndarray, M: int, K: int, N: int) -> np.ndarray:
    """cpuMatmul (jsep-matmul-golden.test.ts:67-90): f64 accumulation, f32 store."""
    a = src0.astype(np.float64).reshape(M, K)
    x = src1.astype(np.float64).reshape(N, K)
    out = np.zeros((N, M), dtype=np.float64)
    for n in range(N):
        for mm in range(M):
            acc = 0.0
            for k in range(K):
                acc += a[mm, k] * x[n, k]
            out[n, mm] = acc
    return out.astype(np.float32)


def make_kat():
    sc = [5, 12, 19, 26, 33, 40, 47, 54]
    m = [3, 7, 11, 15, 19, 23, 27, 31]
    nib = [i & 0xF for i in range(256)]
    blk, deq = pack_q4_k(0.05, 0.01, sc, m, nib)
    src1 = np.array([((i % 13) - 6) * 0.15 for i in range(256)], dtype=np.float64).astype(np.float32)
    ref = cpu_matmul_js(deq, src1, 1, 256, 1)
    np.savez_compressed(os.path.join(HERE, "q4k_kat.npz"), block=blk, dequant=deq, src1=src1, dst=ref,
                        M=1, K=256, N=1, tol=1e-2)


def make_synth():
    """buildSyntheticQ4KMatrix (p2-v2-spike.src.ts:287-330) + N=6 activations."""
    M, K, N = 64, 2048, 6
    spr = K // 256
    w = np.zeros((M, spr * 144), dtype=np.uint8)
    deq = np.zeros((M, K), dtype=np.float32)
    for r in range(M):
        for sb in range(spr):
            d = 0.04 + 0.0001 * ((r + sb * 3) % 17)
            dmin = 0.008 + 0.0001 * ((r * 5 + sb) % 11)
            sc = [(4 + i * 7 + r + sb * 2) & 0x3F for i in range(8)]
            mm = [(2 + i * 5 + r * 3 + sb) & 0x3F for i in range(8)]
            nib = [(i + r + sb * 11) & 0xF for i in range(256)]
            blk, bdeq = pack_q4_k(d, dmin, sc, mm, nib)
            w[r, sb * 144:(sb + 1) * 144] = blk
            deq[r, sb * 256:(sb + 1) * 256] = bdeq
    src1 = np.zeros((N, K), dtype=np.float32)
    for n in range(N):
        for k in range(K):
            src1[n, k] = np.float32((((k * 13 + n * 7) % 31) - 15) * 0.1)
    ref = (deq.astype(np.float64) @ src1.astype(np.float64).T).T  # f64 accumulation
    np.savez_compressed(os.path.join(HERE, "q4k_synth_64x2048.npz"), weights=w, dequant=deq, src1=src1,
                        dst_f64=ref, M=M, K=K, N=N)


def make_gguf_blocks():
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    rng = np.random.default_rng(20261201)
    from importlib.metadata import version

    out = {"gguf_version": np.array(version("gguf"))}
    # (blocks of types added later come after the others: the earlier arrays
    # keep their random streams)
    scale_offsets = {T.Q4_K: (0, 2), T.Q5_K: (0, 2), T.Q6_K: (208,), T.Q8_0: (0,), T.Q4_0: (0,), T.IQ4_XS: (0,)}
    for name, t, bb in (("q4_k", T.Q4_K, 144), ("q6_k", T.Q6_K, 210), ("q8_0", T.Q8_0, 34), ("q5_k", T.Q5_K, 176),
                        ("q4_0", T.Q4_0, 18), ("iq4_xs", T.IQ4_XS, 136)):
        nblk = 64
        raw = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
        # finite f16 scales spanning normals and subnormals
        for off in scale_offsets[t]:
            mag = np.abs(rng.standard_normal(nblk)) * (1e-2 if t in (T.Q8_0, T.Q4_0) else 2e-3)
            mag[:4] = [0.0, 3e-8, 6e-6, 6.0e-5]  # zero and f16 subnormals
            raw[:, off:off + 2] = mag.astype(np.float16).view(np.uint8).reshape(nblk, 2)
        deq = quants.dequantize(raw.reshape(-1), t).astype(np.float32).reshape(-1)
        out[f"{name}_raw"] = raw
        out[f"{name}_dequant"] = deq
    np.savez_compressed(os.path.join(HERE, "gguf_blocks.npz"), **out)


if __name__ == "__main__":
    make_kat()
    make_synth()
    make_gguf_blocks()
    print("fixtures written to", HERE)
