"""GPU parity tests of the prefill path: Q4_K, Q5_K, Q6_K, Q8_0 and Q4_0 MUL_MAT with
N > 64 vectors runs as a tcgen05 tensor-core GEMM (f16 dequantized weights and
activations, f32 accumulation). Q6_K takes it when its rows are a multiple of
16 bytes (K a multiple of 2048), as the tensor-memory copies need, or an even
number of bytes with M a multiple of the row group that makes a multiple of
16: K = 3072 rows (2520 B) in pairs, K = 3584 (2940 B) in fours, K = 2304
(1890 B) in eights. IQ4_XS rows of 8 mod 16 bytes (an odd number of blocks)
go in pairs.

Bar: max relative error <= 2e-2 (rel = max|y - r| / max|r|) against
 - the oracle's f64 dequant-then-dot (small and ragged shapes), and
 - a plain PyTorch fp32 reference (fp32 matmul of the device-dequantized
   weights, bit-exact with the oracle's dequantization) for the
   Llama-3-8B prefill shapes (N = 512 tokens).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from webllm_b200 import jsep, synth

from test_gpu_mulmat import run_mul_mat

pytestmark = pytest.mark.gpu

PREFILL_TOL = 2e-2


def counters():
    c = jsep.WllmCounters()
    jsep.load_library().wllm_get_counters(c)
    return c


@pytest.mark.parametrize("M,K,N", [
    (128, 256, 128),     # one tile, one block
    (128, 512, 65),      # smallest prefill N, partial vector tile
    (200, 768, 130),     # partial row tile and partial vector tile
    (384, 2048, 256),
])
def test_prefill_matches_oracle(runtime, M, K, N):
    rng = np.random.default_rng(1000 + M + K + N)
    w = synth.weights(rng, O.TYPE_Q4_K, M, K)
    x = synth.activations(rng, N, K)
    k0 = counters().kernels_launched
    y = run_mul_mat(runtime, O.TYPE_Q4_K, w, x)
    assert counters().kernels_launched - k0 == 2, "expected the f16 pre-pass and the tensor-core GEMM"
    r = O.mul_mat_f64(O.TYPE_Q4_K, w, x)
    assert O.rel_error(y, r) <= PREFILL_TOL


def test_prefill_activation_magnitudes(runtime):
    rng = np.random.default_rng(7)
    M, K, N = 256, 1024, 96
    w = synth.weights(rng, O.TYPE_Q4_K, M, K)
    for scale in (1e-3, 30.0):
        x = (synth.activations(rng, N, K) * scale).astype(np.float32)
        y = run_mul_mat(runtime, O.TYPE_Q4_K, w, x)
        r = O.mul_mat_f64(O.TYPE_Q4_K, w, x)
        assert O.rel_error(y, r) <= PREFILL_TOL, scale


@pytest.mark.parametrize("M,K", [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)])
def test_prefill_llama3_8b_shapes_vs_torch_fp32(runtime, M, K):
    import torch

    dev = torch.device("cuda", 0)
    N = 512
    gen = torch.Generator(device=dev)
    gen.manual_seed(M * 7 + K)
    w = synth.weights_torch(gen, O.TYPE_Q4_K, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.empty(N, M, device=dev)
    torch.cuda.synchronize()  # the library runs on its own stream
    stream = jsep.library_stream()
    jsep.mul_mat_device(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N, stream)
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(O.TYPE_Q4_K, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = (x.double() @ wf.double().t()).float()  # [N, M]
    rel = ((y - ref).abs().max() / ref.abs().max()).item()
    assert rel <= PREFILL_TOL, rel


@pytest.mark.parametrize("M,K,N", [(20480, 2048, 300), (14336, 4096, 200)])
def test_prefill_large_grids_vs_torch_fp32(runtime, M, K, N):
    """Grids of more than one wave of CTAs (320 and 224 tiles), with a partial
    vector tile (N = 300 and 200), run twice in a row."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(M + K + N)
    w = synth.weights_torch(gen, O.TYPE_Q4_K, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.empty(N, M, device=dev)
    torch.cuda.synchronize()  # the library runs on its own stream
    stream = jsep.library_stream()
    for _ in range(2):
        jsep.mul_mat_device(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N, stream)
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(O.TYPE_Q4_K, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (x.double() @ wf.double().t()).float()
    rel = ((y - ref).abs().max() / ref.abs().max()).item()
    assert rel <= PREFILL_TOL, rel


@pytest.mark.parametrize("M,K,N", [
    (128, 2048, 128),    # one tile, 8 blocks (block offsets 0, 2, ..., 14 in their 16-byte words)
    (200, 2048, 65),     # partial row tile, smallest prefill N
    (384, 4096, 300),    # partial vector tile
])
def test_prefill_q6k_matches_oracle(runtime, M, K, N):
    rng = np.random.default_rng(2000 + M + K + N)
    w = synth.weights(rng, O.TYPE_Q6_K, M, K)
    x = synth.activations(rng, N, K)
    k0 = counters().kernels_launched
    y = run_mul_mat(runtime, O.TYPE_Q6_K, w, x)
    assert counters().kernels_launched - k0 == 2, "expected the f16 pre-pass and the tensor-core GEMM"
    r = O.mul_mat_f64(O.TYPE_Q6_K, w, x)
    assert O.rel_error(y, r) <= PREFILL_TOL


@pytest.mark.parametrize("M,K,N", [(4096, 14336, 512), (1024, 4096, 512), (3072, 8192, 200), (14336, 4096, 77),
                                   (9216, 2304, 512), (2304, 2304, 300)])
def test_prefill_q6k_shapes_vs_torch_fp32(runtime, M, K, N):
    """Q6_K projections of Q4_K_M models in prefill: Llama-3-8B ffn_down and
    attn_v (512 tokens), Llama-3.2-3B ffn_down, a wide one at a short N, and
    Gemma-2-2B ffn_up and attn_q (1890-byte rows, copied in eights)."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(M * 5 + K + N)
    w = synth.weights_torch(gen, O.TYPE_Q6_K, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.empty(N, M, device=dev)
    torch.cuda.synchronize()  # the library runs on its own stream
    stream = jsep.library_stream()
    k0 = counters().kernels_launched
    jsep.mul_mat_device(O.TYPE_Q6_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N, stream)
    assert counters().kernels_launched - k0 == 2
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(O.TYPE_Q6_K, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (x.double() @ wf.double().t()).float()
    rel = ((y - ref).abs().max() / ref.abs().max()).item()
    assert rel <= PREFILL_TOL, rel


@pytest.mark.parametrize("qtype,M,K,N", [
    (O.TYPE_Q5_K, 128, 256, 65),      # one block, smallest prefill N
    (O.TYPE_Q5_K, 200, 2048, 130),    # partial row and vector tiles
    (O.TYPE_Q8_0, 128, 256, 128),     # one 8-block group
    (O.TYPE_Q8_0, 333, 2304, 300),    # Gemma-2-2B hidden: 9 groups; partial tiles
    (O.TYPE_Q4_0, 128, 256, 65),
    (O.TYPE_Q4_0, 260, 2304, 200),
    (O.TYPE_IQ4_XS, 128, 512, 65),    # two 136-byte blocks: offsets 0 and 8 in their boxes
    (O.TYPE_IQ4_XS, 200, 2048, 130),  # partial tiles
    (O.TYPE_IQ4_XS, 256, 2304, 65),   # 1224-byte rows (8 mod 16): copied in pairs
    (O.TYPE_IQ4_XS, 130, 768, 70),    # 408-byte rows in pairs; partial row tile
])
def test_prefill_other_types_matches_oracle(runtime, qtype, M, K, N):
    rng = np.random.default_rng(3000 + qtype + M + K + N)
    w = synth.weights(rng, qtype, M, K)
    x = synth.activations(rng, N, K)
    k0 = counters().kernels_launched
    y = run_mul_mat(runtime, qtype, w, x)
    assert counters().kernels_launched - k0 == 2, "expected the f16 pre-pass and the tensor-core GEMM"
    assert O.rel_error(y, O.mul_mat_f64(qtype, w, x)) <= PREFILL_TOL


@pytest.mark.parametrize("qtype,M,K,N", [(O.TYPE_Q8_0, 9216, 2304, 512), (O.TYPE_Q8_0, 2304, 9216, 256),
                                         (O.TYPE_Q5_K, 14336, 4096, 512), (O.TYPE_Q5_K, 4096, 14336, 200),
                                         (O.TYPE_Q4_0, 14336, 4096, 512), (O.TYPE_Q4_0, 4096, 14336, 128),
                                         (O.TYPE_IQ4_XS, 14336, 4096, 512), (O.TYPE_IQ4_XS, 4096, 14336, 200),
                                         (O.TYPE_IQ4_XS, 9216, 2304, 512)])
def test_prefill_other_types_shapes_vs_torch_fp32(runtime, qtype, M, K, N):
    """Gemma-2-2B ffn_up / ffn_down (Q8_0) and Llama-3-8B ffn_gate / ffn_down
    (Q5_K, Q4_0) in prefill."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(M * 3 + K + N + qtype)
    w = synth.weights_torch(gen, qtype, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.empty(N, M, device=dev)
    torch.cuda.synchronize()  # the library runs on its own stream
    stream = jsep.library_stream()
    k0 = counters().kernels_launched
    jsep.mul_mat_device(qtype, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N, stream)
    assert counters().kernels_launched - k0 == 2
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(qtype, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (x.double() @ wf.double().t()).float()
    rel = ((y - ref).abs().max() / ref.abs().max()).item()
    assert rel <= PREFILL_TOL, rel


@pytest.mark.parametrize("M,K,N", [
    (1024, 3072, 65),    # Llama-3.2-3B attn_v: 2520-byte rows, copied as pairs
    (1000, 3072, 130),   # partial row tile (M even)
    (3072, 1024, 300),   # 840-byte rows
    (256, 2304, 65),     # Gemma-2-2B hidden: 1890-byte rows, copied in eights
    (1000, 2304, 130),   # partial row tile (M a multiple of 8)
    (520, 3584, 100),    # 2940-byte rows, copied in fours; partial row tile
])
def test_prefill_q6k_row_groups_matches_oracle(runtime, M, K, N):
    rng = np.random.default_rng(4000 + M + K + N)
    w = synth.weights(rng, O.TYPE_Q6_K, M, K)
    x = synth.activations(rng, N, K)
    k0 = counters().kernels_launched
    y = run_mul_mat(runtime, O.TYPE_Q6_K, w, x)
    assert counters().kernels_launched - k0 == 2, "expected the f16 pre-pass and the tensor-core GEMM"
    assert O.rel_error(y, O.mul_mat_f64(O.TYPE_Q6_K, w, x)) <= PREFILL_TOL


@pytest.mark.parametrize("M,K", [(333, 3072), (1002, 2304)])
def test_prefill_q6k_ragged_row_groups_take_the_batched_gemm(runtime, M, K):
    """M not a multiple of the row group (2520-byte rows in pairs, 1890-byte
    rows in eights): the batched GEMM runs it, at the GEMV bar."""
    rng = np.random.default_rng(4100 + M)
    N = 70
    w = synth.weights(rng, O.TYPE_Q6_K, M, K)
    x = synth.activations(rng, N, K)
    y = run_mul_mat(runtime, O.TYPE_Q6_K, w, x)
    assert O.rel_error(y, O.mul_mat_f64(O.TYPE_Q6_K, w, x)) <= 1e-3
