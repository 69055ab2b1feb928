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
                                            ("q4_0", O.TYPE_Q4_0, 32)])
def test_dequant_matches_gguf(golden, name, qtype, be):
    z = golden("gguf_blocks.npz")
    raw = z[f"{name}_raw"]
    ref = z[f"{name}_dequant"]
    got = O.dequantize(qtype, raw.reshape(-1), raw.shape[0] * be)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), name


@pytest.mark.parametrize("qtype", [O.TYPE_Q4_K, O.TYPE_Q6_K, O.TYPE_Q8_0, O.TYPE_Q5_K, O.TYPE_Q4_0])
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
