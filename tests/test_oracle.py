"""Pins the CPU oracle against the reference's golden vectors (no GPU).

The oracle is the checker for every GPU parity test, so it is checked first:
  - the reference's Q4_K known-answer test (tests/jsep-matmul-golden.test.ts:521-600),
  - the reference's synthetic 64x2048 Q4_K matrix (smoke-test/p2-v2-spike.src.ts:287-330),
  - gguf 0.19.0's dequantization of random Q4_K/Q6_K/Q8_0 blocks,
  - every f16 bit pattern against numpy's f16 -> f32 conversion.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from webllm_b200 import synth


def test_f16_decode_exhaustive():
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([O.f16_to_f32(int(b)) for b in bits[::1]], dtype=np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(got[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert np.array_equal(np.isinf(got), np.isinf(ref))


def test_block_geometry():
    # src/models/gguf-parser.ts:282,286,288
    assert (O.block_elems(O.TYPE_Q4_K), O.block_bytes(O.TYPE_Q4_K)) == (256, 144)
    assert (O.block_elems(O.TYPE_Q6_K), O.block_bytes(O.TYPE_Q6_K)) == (256, 210)
    assert (O.block_elems(O.TYPE_Q8_0), O.block_bytes(O.TYPE_Q8_0)) == (32, 34)


def test_q4k_kat_dequant_bit_exact(golden):
    z = golden("q4k_kat.npz")
    got = O.dequantize(O.TYPE_Q4_K, z["block"], 256)
    assert np.array_equal(got.view(np.uint32), z["dequant"].view(np.uint32))
    # the first and last values the reference's self-test logs
    assert got[0] == np.float32(z["dequant"][0])


def test_q4k_kat_mul_mat(golden):
    z = golden("q4k_kat.npz")
    w = z["block"].reshape(1, 144)
    x = z["src1"].reshape(1, 256)
    r = O.mul_mat_f64(O.TYPE_Q4_K, w, x)
    # the reference's own bar (max-abs < 1e-2) and the tighter f64 one
    assert abs(float(r[0, 0]) - float(z["dst"][0, 0])) < float(z["tol"])
    assert abs(float(r[0, 0]) - float(z["dst"][0, 0])) <= 1e-6 * abs(float(z["dst"][0, 0]))
    y = O.mul_mat_f32(O.TYPE_Q4_K, w, x, threads=1)
    assert O.rel_error(y, r) < 1e-6


def test_q4k_kat_detects_scale_unpack_error(golden):
    """A planted mistake in the oracle's input (one flipped high scale bit,
    the bits get_scale_min_k4 moves for sub-blocks 4..7) must change the
    KAT output: the vector discriminates the 6-bit unpack."""
    z = golden("q4k_kat.npz")
    bad = z["block"].copy()
    bad[4 + 0] ^= 0x40  # high bits of scales[0] feed sc[4]
    got = O.dequantize(O.TYPE_Q4_K, bad, 256)
    assert not np.array_equal(got, z["dequant"])
    assert np.array_equal(got[:128], z["dequant"][:128])  # sub-blocks 0..3 untouched


def test_q4k_synth_matrix(golden):
    z = golden("q4k_synth_64x2048.npz")
    K = int(z["K"])
    deq = O.dequantize_matrix(O.TYPE_Q4_K, z["weights"], K)
    assert np.array_equal(deq.view(np.uint32), z["dequant"].view(np.uint32))
    r = O.mul_mat_f64(O.TYPE_Q4_K, z["weights"], z["src1"])
    assert O.rel_error(r, z["dst_f64"]) < 1e-12


@pytest.mark.parametrize("name,qtype,be", [("q4_k", O.TYPE_Q4_K, 256), ("q6_k", O.TYPE_Q6_K, 256),
                                            ("q8_0", O.TYPE_Q8_0, 32), ("q5_k", O.TYPE_Q5_K, 256),
                                            ("q4_0", O.TYPE_Q4_0, 32), ("iq4_xs", O.TYPE_IQ4_XS, 256)])
def test_dequant_matches_gguf(golden, name, qtype, be):
    z = golden("gguf_blocks.npz")
    raw = z[f"{name}_raw"]
    ref = z[f"{name}_dequant"]
    got = O.dequantize(qtype, raw.reshape(-1), raw.shape[0] * be)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), name


@pytest.mark.parametrize("qtype", [O.TYPE_Q4_K, O.TYPE_Q6_K, O.TYPE_Q8_0, O.TYPE_Q5_K, O.TYPE_Q4_0, O.TYPE_IQ4_XS])
def test_f32_baseline_close_to_f64(qtype):
    rng = np.random.default_rng(7)
    M, K, N = 37, 1024, 3
    w = synth.weights(rng, qtype, M, K)
    x = synth.activations(rng, N, K)
    r = O.mul_mat_f64(qtype, w, x)
    for t in (1, 4):
        y = O.mul_mat_f32(qtype, w, x, threads=t)
        assert O.rel_error(y, r) < 1e-5


def test_bad_arguments():
    with pytest.raises(ValueError):
        O.dequantize(O.TYPE_Q4_K, np.zeros(144, np.uint8), 255)
    with pytest.raises(ValueError):
        O.dequantize(99, np.zeros(144, np.uint8), 256)


def test_synth_distributions():
    rng = np.random.default_rng(1)
    w = synth.q4_k_blocks(rng, 256, 4096)
    d = w.reshape(-1, 144)[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    sub = np.mean((d != 0) & (np.abs(d) < 6.103515625e-05))
    assert 0.01 < sub < 0.04  # |N(0,1)|*2e-3 lands ~2.4% in f16 subnormals
    q8 = synth.q8_0_blocks(rng, 64, 2304).reshape(-1, 34)[:, 2:].view(np.int8)
    assert q8.min() >= -127 and q8.max() <= 127
    # algorithmic bytes of the single-GEMV workload: 4096x4096 Q4_K, N=1
    assert synth.algorithmic_bytes(synth.Q4_K, 4096, 4096, 1) == 9_469_952
    layer = sum(synth.algorithmic_bytes(t, M, K, 1) for _, t, M, K in synth.LLAMA32_3B_LAYER)
    assert layer == 64_139_264


def rms_norm_golden_input(n: int) -> np.ndarray:
    """The reference's RMS_NORM golden input: x[i] = ((i * 7) % 31) * 0.05 - 0.7
    (tests/jsep-rms-norm-golden.test.ts:129), as f32."""
    i = np.arange(n)
    return (((i * 7) % 31) * 0.05 - 0.7).astype(np.float32)


@pytest.mark.parametrize("cols,eps", [(2048, 1e-5), (64, 1e-6)])
def test_rms_norm_matches_reference_golden(cols, eps):
    """The reference's two RMS_NORM golden cases (1 x 2048, eps 1e-5; 1 x 64,
    eps 1e-6; tests/jsep-rms-norm-golden.test.ts:182-188), against its CPU
    reference written out as a per-element loop in f64 (cpuRmsNorm, :64-86),
    at its tolerance 1e-4 (max abs)."""
    x = rms_norm_golden_input(cols)
    sum_sq = 0.0
    for v in x.tolist():
        sum_sq += v * v
    inv = 1.0 / float(np.sqrt(sum_sq / cols + eps))
    ref = np.array([v * inv for v in x.tolist()], dtype=np.float32)
    got = O.rms_norm_f64(x[None, :], eps)[0]
    assert np.max(np.abs(got - ref)) < 1e-4
    # rows are independent, and the gain multiplies after the norm
    two = np.stack([x, 3.0 * x])
    g = np.linspace(0.5, 1.5, cols)
    out = O.rms_norm_f64(two, eps, g)
    assert np.allclose(out[0], O.rms_norm_f64(x, eps) * g)
    assert np.allclose(out[1], O.rms_norm_f64(3.0 * x, eps) * g)


def test_glu_restatements():
    """SwiGLU: silu(g) * u with silu(0) = 0 and silu(g) -> g for large g.
    GELU (ggml's f16-table form): the clamps at +-10, exact f16 values
    elsewhere, and the tanh form within f16 rounding."""
    g = np.array([-50.0, -10.0, -9.99, -1.0, 0.0, 0.5, 3.0, 9.99, 10.0, 40.0], dtype=np.float32)
    u = np.linspace(-2.0, 2.0, g.size).astype(np.float32)
    s = O.swiglu_f64(g, u)
    assert s[4] == 0.0 and abs(s[-1] - 40.0 * u[-1]) < 1e-9 and abs(s[0]) < 1e-15
    gd = g.astype(np.float64)
    assert np.allclose(s, gd / (1.0 + np.exp(-gd)) * u)
    e = O.gelu_ggml(g)
    assert e[0] == 0.0 and e[1] == 0.0 and e[8] == 10.0 and e[9] == 40.0
    inner = e[2:8]
    assert np.array_equal(inner, inner.astype(np.float16).astype(np.float64))  # f16 values
    f = gd[2:8]
    exact = 0.5 * f * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * f * (1.0 + 0.044715 * f * f)))
    assert np.allclose(inner, exact, rtol=2e-3, atol=1e-3)
    assert np.allclose(O.geglu_f64(g, u), e * u)
