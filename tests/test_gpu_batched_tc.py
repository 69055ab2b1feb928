"""The tcgen05 small-batch GEMM (Q4_K, Q5_K and Q8_0 weights, several
sequences decoding together, N = 5..64, and N = 3-4 where the streaming
kernel cannot take the shape): both error metrics of the path (max-normalized
and per-element, 1e-3) against a float64 matmul of the device-dequantized
weights, on N(0,1) activations and on outlier channels; shapes with partial
row tiles, split K and K not a multiple of 1024. Weights of at most 4096 x 4096
below 16 vectors route to the mma.sync GEMM instead; the shapes above that
size (5000 x 4352, 4200 x 4608: partial row tiles, K = 17 and 18 blocks) keep
those N on this kernel. Q8_0 goes in as two exact f16 weight planes (d q
rounded to f16, and the remainder) and takes this kernel above 16 vectors
(the integer mma.sync GEMM below); a test drives its scales through the f16
subnormal range and up to 2^8. Q6_K (rows a multiple of 16 bytes: K a
multiple of 2048) goes in as two planes of sc (q - 32), which reaches 4096,
with the Q4_K routing (below 4096 x 4096 only above 16 vectors); a test sets
its int8 scales to the extremes -128 and 127. IQ4_XS (K a multiple of 512)
takes the same two planes for (ls - 32) level, up to 4064 in magnitude,
above 16 vectors. Above 32 vectors the two-plane types run their two vector
groups in one CTA (N = 33, 40, 64 here, with and without split K)."""
from __future__ import annotations

import zlib

import numpy as np
import pytest

from oracle import oracle as O
from webllm_b200 import jsep, synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _run(runtime, qtype, M, K, x_np, seed):
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    N = x_np.shape[0]
    w = synth.weights_torch(gen, qtype, M, K, dev)
    x = torch.from_numpy(x_np).to(dev)
    y = torch.full((N, M), float("nan"), device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    k0 = _kernels()
    assert jsep.mul_mat_device(qtype, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N,
                               stream) == jsep.STATUS_OK, jsep.last_error()
    launched = _kernels() - k0
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(qtype, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ x.double().t()).t()
    return y.double().cpu().numpy(), ref.cpu().numpy(), launched


def _kernels():
    c = jsep.WllmCounters()
    jsep.load_library().wllm_get_counters(c)
    return c.kernels_launched


@pytest.mark.parametrize("N", [5, 8, 16, 17, 33, 64])
@pytest.mark.parametrize("qtype,M,K", [(jsep.GGML_TYPE_Q4_K, 4096, 4096), (jsep.GGML_TYPE_Q4_K, 14336, 4096),
                                       (jsep.GGML_TYPE_Q4_K, 4096, 14336), (jsep.GGML_TYPE_Q4_K, 1000, 2304),
                                       (jsep.GGML_TYPE_Q5_K, 4096, 4096), (jsep.GGML_TYPE_Q5_K, 333, 3072),
                                       (jsep.GGML_TYPE_Q4_K, 128, 256), (jsep.GGML_TYPE_Q4_K, 5000, 4352),
                                       (jsep.GGML_TYPE_Q5_K, 4200, 4608), (jsep.GGML_TYPE_Q8_0, 9216, 2304),
                                       (jsep.GGML_TYPE_Q8_0, 2304, 9216), (jsep.GGML_TYPE_Q8_0, 5000, 4352),
                                       (jsep.GGML_TYPE_Q8_0, 128, 256), (jsep.GGML_TYPE_Q6_K, 4096, 14336),
                                       (jsep.GGML_TYPE_Q6_K, 14336, 4096), (jsep.GGML_TYPE_Q6_K, 1000, 2048),
                                       (jsep.GGML_TYPE_Q6_K, 5000, 6144), (jsep.GGML_TYPE_IQ4_XS, 14336, 4096),
                                       (jsep.GGML_TYPE_IQ4_XS, 4096, 14336), (jsep.GGML_TYPE_IQ4_XS, 1000, 2048),
                                       (jsep.GGML_TYPE_IQ4_XS, 4200, 4608)])
def test_batched_tc_both_metrics(runtime, qtype, M, K, N):
    rng = np.random.default_rng(zlib.crc32(repr((qtype, M, K, N)).encode()))
    x = synth.activations(rng, N, K)
    y, r, launched = _run(runtime, qtype, M, K, x, seed=M + K + N)
    assert launched == 2  # the activation pre-pass and the GEMM
    assert np.all(np.isfinite(y))
    a, b = O.rel_error(y, r), O.rel_error_elem(y, r)
    assert a <= TOL and b <= TOL, (a, b)


@pytest.mark.parametrize("value", [100.0, 1000.0, 3e4])
@pytest.mark.parametrize("N", [8, 64])
def test_batched_tc_outlier_channels(runtime, N, value):
    """Outlier channels (the activation split is per element, so they cost
    nothing), up to 3e4 (the f16 range is handled by the per-vector scale)."""
    rng = np.random.default_rng(int(value) + N)
    x = synth.activations_with_outliers(rng, N, 4096, value)
    y, r, _ = _run(runtime, jsep.GGML_TYPE_Q4_K, 12288, 4096, x, seed=N)
    a, b = O.rel_error(y, r), O.rel_error_elem(y, r)
    assert a <= TOL and b <= TOL, (a, b)


def test_batched_tc_tiny_and_huge_activations(runtime):
    """Vectors scaled by 1e-30 and 1e30 and an all-zero vector in one batch:
    each vector has its own power-of-two scale."""
    rng = np.random.default_rng(9)
    x = synth.activations(rng, 8, 2048)
    x[1] *= np.float32(1e-30)
    x[2] *= np.float32(1e30)
    x[3] = 0.0
    y, r, _ = _run(runtime, jsep.GGML_TYPE_Q4_K, 512, 2048, x, seed=9)
    assert np.all(y[3] == 0.0)
    for n in (0, 1, 2, 4):
        a, b = O.rel_error(y[n], r[n]), O.rel_error_elem(y[n], r[n])
        assert a <= TOL and b <= TOL, (n, a, b)


@pytest.mark.parametrize("N", [24, 40])
def test_batched_tc_q8_0_scale_range(runtime, N):
    """Q8_0 blocks whose f16 scale d is subnormal (down to 2^-24), tiny, normal
    or large (up to 2^8), mixed within rows: hi = f16(d q) and lo = d q - hi
    stay exact, so the result meets both metrics whatever d is."""
    import torch

    M, K = 5000, 4352
    rng = np.random.default_rng(77 + N)
    w = synth.weights(rng, jsep.GGML_TYPE_Q8_0, M, K)
    blocks = w.reshape(M, K // 32, 34)
    exps = rng.integers(-24, 9, size=(M, K // 32)).astype(np.float64)
    mant = rng.uniform(1.0, 2.0, size=(M, K // 32))
    d = np.ldexp(mant, exps.astype(np.int64)).astype(np.float16)  # subnormals where 2^e < 2^-14
    blocks[:, :, 0:2] = d.view(np.uint8).reshape(M, K // 32, 2)
    x = synth.activations(rng, N, K)
    dev = torch.device("cuda", 0)
    wt = torch.from_numpy(w).to(dev)
    xt = torch.from_numpy(x).to(dev)
    y = torch.full((N, M), float("nan"), device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    k0 = _kernels()
    assert jsep.mul_mat_device(jsep.GGML_TYPE_Q8_0, wt.data_ptr(), wt.shape[1], xt.data_ptr(), K, y.data_ptr(), M, M,
                               K, N, stream) == jsep.STATUS_OK, jsep.last_error()
    assert _kernels() - k0 == 2
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(jsep.GGML_TYPE_Q8_0, wt.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    r = (wf.double() @ xt.double().t()).t().cpu().numpy()
    yy = y.double().cpu().numpy()
    assert np.all(np.isfinite(yy))
    a, b = O.rel_error(yy, r), O.rel_error_elem(yy, r)
    assert a <= TOL and b <= TOL, (a, b)


@pytest.mark.parametrize("N", [8, 24, 40])
def test_batched_tc_q6_k_extreme_scales(runtime, N):
    """Q6_K sub-block scales of -128 and 127 beside small ones: sc (q - 32)
    then reaches 4096 in magnitude, where f16 holds only even integers, and the
    second weight plane carries the odd remainder."""
    import torch

    M, K = 4096, 6144
    rng = np.random.default_rng(99 + N)
    w = synth.weights(rng, jsep.GGML_TYPE_Q6_K, M, K)
    blocks = w.reshape(M, K // 256, 210)
    choice = rng.integers(0, 3, size=(M, K // 256, 16))
    sc = np.where(choice == 0, -128, np.where(choice == 1, 127, rng.integers(-5, 6, size=choice.shape)))
    blocks[:, :, 192:208] = sc.astype(np.int8).view(np.uint8)
    x = synth.activations(rng, N, K)
    dev = torch.device("cuda", 0)
    wt = torch.from_numpy(w).to(dev)
    xt = torch.from_numpy(x).to(dev)
    y = torch.full((N, M), float("nan"), device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    k0 = _kernels()
    assert jsep.mul_mat_device(jsep.GGML_TYPE_Q6_K, wt.data_ptr(), wt.shape[1], xt.data_ptr(), K, y.data_ptr(), M, M,
                               K, N, stream) == jsep.STATUS_OK, jsep.last_error()
    assert _kernels() - k0 == 2
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(jsep.GGML_TYPE_Q6_K, wt.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    r = (wf.double() @ xt.double().t()).t().cpu().numpy()
    yy = y.double().cpu().numpy()
    assert np.all(np.isfinite(yy))
    a, b = O.rel_error(yy, r), O.rel_error_elem(yy, r)
    assert a <= TOL and b <= TOL, (a, b)
