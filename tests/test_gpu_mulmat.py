"""GPU parity tests: the CUDA MUL_MAT through the C ABI against the oracle.

Bar (from the path's contract): dequantization bit-exact; GEMV max relative
error <= 1e-3, rel = max|y - r| / max|r| with r the oracle's f64-accumulated
dequant-then-dot. Cases follow the reference's golden tests
(tests/jsep-matmul-golden.test.ts, smoke-test/p2-v2-spike.src.ts) and add
odd shapes, batches, broadcast, aliasing and error paths.
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest

from oracle import oracle as O
from webllm_b200 import jsep, synth

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3


def upload(rt, arr) -> int:
    a = np.ascontiguousarray(arr)
    h = rt.data_manager.alloc(a.nbytes)
    rt.data_manager.write(h, 0, a)
    return h


def run_mul_mat(rt, qtype, w, x, *, check_status=True):
    """dst = MUL_MAT(w, x) through jsepRunOp-style descriptors; returns (N, M)."""
    M = w.shape[0]
    N, K = x.shape
    h0, h1 = upload(rt, w), upload(rt, x)
    hd = rt.data_manager.alloc(4 * M * N)
    desc = jsep.JsepOpDescriptor(jsep.GGML_OP_MUL_MAT, 2, jsep.meta_for(hd, jsep.GGML_TYPE_F32, (M, N, 1, 1)),
                                 [jsep.meta_for(h0, qtype, (K, M, 1, 1)), jsep.meta_for(h1, jsep.GGML_TYPE_F32, (K, N, 1, 1))])
    st = jsep.dispatch_matmul(rt, desc)
    if check_status:
        assert st == jsep.STATUS_OK, jsep.last_error()
    rt.encoder_batcher.flush()
    out = rt.data_manager.read(hd, 0, 4 * M * N).view(np.float32).reshape(N, M)
    for h in (h0, h1, hd):
        rt.data_manager.free(h)
    return out


def test_q4k_kat(runtime, golden):
    """tests/jsep-matmul-golden.test.ts:521-600 (single Q4_K super-block)."""
    z = golden("q4k_kat.npz")
    got = run_mul_mat(runtime, jsep.GGML_TYPE_Q4_K, z["block"].reshape(1, 144), z["src1"].reshape(1, 256))
    assert abs(float(got[0, 0]) - float(z["dst"][0, 0])) < float(z["tol"])
    r = O.mul_mat_f64(O.TYPE_Q4_K, z["block"].reshape(1, 144), z["src1"].reshape(1, 256))
    assert O.rel_error(got, r) <= GEMV_TOL


def test_q4k_synth_64x2048(runtime, golden):
    """buildSyntheticQ4KMatrix M=64 K=2048 N=6 (p2-v2-spike.src.ts:287-360)."""
    z = golden("q4k_synth_64x2048.npz")
    got = run_mul_mat(runtime, jsep.GGML_TYPE_Q4_K, z["weights"], z["src1"])
    assert O.rel_error(got, z["dst_f64"]) <= GEMV_TOL
    assert np.all(np.isfinite(got))


@pytest.mark.parametrize("qtype,name", [(jsep.GGML_TYPE_Q4_K, "q4_k"), (jsep.GGML_TYPE_Q6_K, "q6_k"),
                                        (jsep.GGML_TYPE_Q8_0, "q8_0"), (jsep.GGML_TYPE_Q5_K, "q5_k"),
                                        (jsep.GGML_TYPE_Q4_0, "q4_0"), (jsep.GGML_TYPE_IQ4_XS, "iq4_xs")])
def test_device_dequant_bit_exact(runtime, golden, qtype, name):
    z = golden("gguf_blocks.npz")
    raw = z[f"{name}_raw"]
    be, _ = jsep.BLOCK_GEOMETRY[qtype]
    n = raw.shape[0] * be
    hs = upload(runtime, raw)
    hd = runtime.data_manager.alloc(4 * n)
    ps, _ = runtime.data_manager.get(hs)
    pd, _ = runtime.data_manager.get(hd)
    jsep.dequantize_device(qtype, ps, pd, n)
    runtime.encoder_batcher.flush()
    got = runtime.data_manager.read(hd, 0, 4 * n).view(np.float32)
    assert np.array_equal(got.view(np.uint32), z[f"{name}_dequant"].view(np.uint32))
    # and against the oracle on synthetic blocks of the bench distribution
    rng = np.random.default_rng(qtype)
    w = synth.weights(rng, qtype, 16, 1024)
    hs2 = upload(runtime, w)
    hd2 = runtime.data_manager.alloc(4 * 16 * 1024)
    jsep.dequantize_device(qtype, runtime.data_manager.get(hs2)[0], runtime.data_manager.get(hd2)[0], 16 * 1024)
    got2 = runtime.data_manager.read(hd2, 0, 4 * 16 * 1024).view(np.float32).reshape(16, 1024)
    ref2 = O.dequantize_matrix(qtype, w, 1024)
    assert np.array_equal(got2.view(np.uint32), ref2.view(np.uint32))
    for h in (hs, hd, hs2, hd2):
        runtime.data_manager.free(h)


SHAPES = [(1, 256, 1), (7, 512, 1), (33, 768, 2), (257, 1024, 3), (64, 2048, 5), (96, 3072, 8), (40, 2304, 13)]


@pytest.mark.parametrize("qtype", [jsep.GGML_TYPE_Q4_K, jsep.GGML_TYPE_Q6_K, jsep.GGML_TYPE_Q8_0,
                                   jsep.GGML_TYPE_Q5_K, jsep.GGML_TYPE_Q4_0, jsep.GGML_TYPE_IQ4_XS])
@pytest.mark.parametrize("M,K,N", SHAPES)
def test_gemv_random_shapes(runtime, qtype, M, K, N):
    be, _ = jsep.BLOCK_GEOMETRY[qtype]
    if K % be:
        pytest.skip("K not a multiple of the block")
    rng = np.random.default_rng(M * 7919 + K * 31 + N + qtype)
    w = synth.weights(rng, qtype, M, K)
    x = synth.activations(rng, N, K)
    got = run_mul_mat(runtime, qtype, w, x)
    r = O.mul_mat_f64(qtype, w, x)
    assert O.rel_error(got, r) <= GEMV_TOL


@pytest.mark.parametrize("name,qtype,M,K", synth.LLAMA32_3B_LAYER)
def test_llama32_3b_layer_shapes(runtime, name, qtype, M, K):
    rng = np.random.default_rng(zlib.crc32(name.encode()))
    w = synth.weights(rng, qtype, M, K)
    x = synth.activations(rng, 1, K)
    got = run_mul_mat(runtime, qtype, w, x)
    assert O.rel_error(got, O.mul_mat_f64(qtype, w, x)) <= GEMV_TOL


@pytest.mark.parametrize("name,qtype,M,K", synth.GEMMA2_2B_SHAPES[:2] + [synth.GEMMA2_2B_SHAPES[3]])
@pytest.mark.parametrize("N", [1, 2])
def test_gemma2_q8_0_shapes(runtime, name, qtype, M, K, N):
    rng = np.random.default_rng(zlib.crc32(name.encode()) + N)
    w = synth.weights(rng, qtype, M, K)
    x = synth.activations(rng, N, K)
    got = run_mul_mat(runtime, qtype, w, x)
    assert O.rel_error(got, O.mul_mat_f64(qtype, w, x)) <= GEMV_TOL


@pytest.mark.parametrize("name,M,K,N", [("ffn_up", 9216, 2304, 8), ("ffn_up", 9216, 2304, 64),
                                         ("ffn_down", 2304, 9216, 16), ("attn_proxy", 2304, 2304, 32),
                                         ("attn_proxy", 2304, 2304, 65), ("ragged", 200, 768, 3)])
def test_q8_0_batched_decode(runtime, name, M, K, N):
    """Several sequences decoding together (Gemma-2-2B Q8_0 shapes, batch up to
    64): the integer tensor-core batched GEMM, split K included, at the GEMV
    bar. One past it (N = 65) is the f16 tcgen05 prefill GEMM, at the prefill
    bar (2e-2)."""
    rng = np.random.default_rng(zlib.crc32(name.encode()) + N)
    w = synth.weights(rng, jsep.GGML_TYPE_Q8_0, M, K)
    x = synth.activations(rng, N, K)
    got = run_mul_mat(runtime, jsep.GGML_TYPE_Q8_0, w, x)
    tol = GEMV_TOL if N <= 64 else 2e-2
    assert O.rel_error(got, O.mul_mat_f64(jsep.GGML_TYPE_Q8_0, w, x)) <= tol


@pytest.mark.parametrize("N", [3, 4, 8, 16, 33, 64])
@pytest.mark.parametrize("qtype,M,K", [(jsep.GGML_TYPE_Q4_K, 4096, 4096), (jsep.GGML_TYPE_Q4_K, 14336, 4096),
                                       (jsep.GGML_TYPE_Q6_K, 4096, 14336), (jsep.GGML_TYPE_Q6_K, 1024, 3072),
                                       (jsep.GGML_TYPE_Q5_K, 4096, 4096), (jsep.GGML_TYPE_Q4_0, 4096, 4096),
                                       (jsep.GGML_TYPE_Q5_K, 1000, 2304), (jsep.GGML_TYPE_Q4_0, 1000, 2304)])
def test_kquant_small_batches_vs_torch_fp64(runtime, qtype, M, K, N):
    """Q4_K / Q5_K / Q6_K / Q4_0 with 3 to 64 vectors (several sequences
    decoding together, short prefill tiles) on the integer tensor-core batched
    GEMM, split K included; Q6_K 1024 x 3072 has 2520-byte rows (8-byte
    aligned), M = 1000 leaves a partial 64-row tile. Against a float64 matmul
    of the device-dequantized weights."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(M + K + N)
    w = synth.weights_torch(gen, qtype, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.empty(N, M, device=dev)
    torch.cuda.synchronize()  # the library runs on its own stream
    stream = jsep.library_stream()
    jsep.mul_mat_device(qtype, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N, stream)
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(qtype, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ x.double().t()).t()
    rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel <= GEMV_TOL, rel


@pytest.mark.parametrize("N", [1, 2])
@pytest.mark.parametrize("qtype,M,K", [(jsep.GGML_TYPE_Q5_K, 4096, 4096), (jsep.GGML_TYPE_Q5_K, 14336, 4096),
                                       (jsep.GGML_TYPE_Q5_K, 4096, 14336), (jsep.GGML_TYPE_Q4_0, 4096, 4096),
                                       (jsep.GGML_TYPE_Q4_0, 3000, 2304), (jsep.GGML_TYPE_Q4_0, 4096, 14336)])
def test_q5k_q4_0_decode_vs_torch_fp64(runtime, qtype, M, K, N):
    """Q5_K / Q4_0 decode (batch 1 and 2) on the streaming integer
    tensor-core GEMV, against a float64 matmul of the device-dequantized
    weights (bit-exact with the oracle's dequantization)."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(qtype * 1000 + M + K + N)
    w = synth.weights_torch(gen, qtype, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.empty(N, M, device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    assert jsep.mul_mat_device(qtype, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N,
                               stream) == jsep.STATUS_OK
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(qtype, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ x.double().t()).t()
    rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel <= GEMV_TOL, rel


FUSED_NORM_GROUPS = {
    # name: (eps, [(type, M), ...], K) -- the ops that read one normed activation
    "llama32_attn_qkv": (1e-5, [(jsep.GGML_TYPE_Q4_K, 3072), (jsep.GGML_TYPE_Q4_K, 1024), (jsep.GGML_TYPE_Q6_K, 1024)], 3072),
    "llama32_ffn_gate_up": (1e-5, [(jsep.GGML_TYPE_Q4_K, 8192), (jsep.GGML_TYPE_Q4_K, 8192)], 3072),
    "qwen3_attn_qkv": (1e-6, [(jsep.GGML_TYPE_Q4_K, 4096), (jsep.GGML_TYPE_Q4_K, 1024), (jsep.GGML_TYPE_Q4_K, 1024)], 4096),
    "gemma2_ffn_up": (1e-6, [(jsep.GGML_TYPE_Q8_0, 9216)], 2304),
    "mixed_types": (1e-5, [(jsep.GGML_TYPE_Q5_K, 640), (jsep.GGML_TYPE_Q4_0, 333)], 8192),
}


@pytest.mark.parametrize("with_gain", [True, False])
@pytest.mark.parametrize("N", [1, 2, 3])
@pytest.mark.parametrize("group", sorted(FUSED_NORM_GROUPS))
def test_fused_rms_norm_vs_torch_fp64(runtime, group, N, with_gain):
    """wllm_mul_mat_rms_norm_batch: the RMS_NORM (times gain) feeding a group
    of projections, fused into the streaming kernel, against float64
    x / sqrt(mean(x^2) + eps) * gain, then a float64 matmul of the
    device-dequantized weights. The activations are left as they were."""
    import torch

    eps, mats, K = FUSED_NORM_GROUPS[group]
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(len(group) * 7 + N + int(with_gain))
    x = 3.0 * torch.randn(N, K, device=dev, generator=gen) + 0.5
    gain = (torch.rand(K, device=dev, generator=gen) * 2.0 - 0.5) if with_gain else None
    x0 = x.clone()
    ws, ys, ops = [], [], []
    for t, M in mats:
        w = synth.weights_torch(gen, t, M, K, dev)
        y = torch.empty(N, M, device=dev)
        ws.append(w)
        ys.append(y)
        ops.append(jsep.MulMatArgs(t, M, K, N, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M))
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    rc = jsep.mul_mat_rms_norm_batch(ops, gain.data_ptr() if with_gain else 0, eps, stream)
    assert rc == jsep.STATUS_OK
    runtime.jsep_sync()
    xn = torch.from_numpy(O.rms_norm_f64(x0.cpu().numpy(), eps, gain.cpu().numpy() if with_gain else None)).to(dev)
    for (t, M), w, y in zip(mats, ws, ys):
        wf = torch.empty(M, K, device=dev)
        jsep.dequantize_device(t, w.data_ptr(), wf.data_ptr(), M * K, stream)
        runtime.jsep_sync()
        ref = (wf.double() @ xn.t()).t()
        rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
        assert rel <= GEMV_TOL, (t, M, rel)
    assert torch.equal(x, x0)


def test_fused_rms_norm_reference_golden_input(runtime):
    """The reference's RMS_NORM golden case 1 x 2048, eps 1e-5
    (tests/jsep-rms-norm-golden.test.ts:129,182-184: x[i] = ((i * 7) % 31) *
    0.05 - 0.7), fused into a Q4_K projection: against the oracle's norm, then
    a float64 matmul of the device-dequantized weights."""
    import torch

    K, M, eps = 2048, 512, 1e-5
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(21)
    i = np.arange(K)
    xh = (((i * 7) % 31) * 0.05 - 0.7).astype(np.float32)[None, :]
    x = torch.from_numpy(xh).to(dev)
    w = synth.weights_torch(gen, jsep.GGML_TYPE_Q4_K, M, K, dev)
    y = torch.empty(1, M, device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    op = jsep.MulMatArgs(jsep.GGML_TYPE_Q4_K, M, K, 1, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M)
    assert jsep.mul_mat_rms_norm_batch([op], 0, eps, stream) == jsep.STATUS_OK
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(jsep.GGML_TYPE_Q4_K, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ torch.from_numpy(O.rms_norm_f64(xh, eps)).to(dev).t()).t()
    rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel <= GEMV_TOL, rel


def test_fused_rms_norm_outside_decode_is_not_implemented(runtime):
    """More vectors than the streaming kernel takes: NOT_IMPLEMENTED, so the
    caller runs RMS_NORM, MUL and MUL_MAT unfused; nothing is written."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)
    M, K, N = 256, 1024, 8
    w = synth.weights_torch(gen, jsep.GGML_TYPE_Q4_K, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.full((N, M), 7.0, device=dev)
    torch.cuda.synchronize()
    op = jsep.MulMatArgs(jsep.GGML_TYPE_Q4_K, M, K, N, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M)
    assert jsep.mul_mat_rms_norm_batch([op], 0, 1e-5, jsep.library_stream()) == jsep.STATUS_NOT_IMPLEMENTED
    runtime.jsep_sync()
    assert bool((y == 7.0).all())


FUSED_GLU_GROUPS = {
    # name: ([(type, M), ...], K) -- the down projections that read one act(gate) * up
    "llama32_ffn_down_q6k": ([(jsep.GGML_TYPE_Q6_K, 3072)], 8192),
    "llama32_ffn_down_q4k": ([(jsep.GGML_TYPE_Q4_K, 3072)], 8192),
    "llama3_8b_ffn_down": ([(jsep.GGML_TYPE_Q4_K, 4096)], 14336),
    "gemma2_ffn_down": ([(jsep.GGML_TYPE_Q8_0, 2304)], 9216),
    "mixed_types": ([(jsep.GGML_TYPE_Q5_K, 640), (jsep.GGML_TYPE_Q4_0, 333)], 4096),
}


def glu_fp64(gate, up, glu):
    """act(gate) * up in float64 from the oracle: silu, or ggml's CPU GELU
    (tanh form with its input and output rounded to f16; 0 at gate <= -10,
    gate at gate >= 10)."""
    import torch

    fn = O.swiglu_f64 if glu == jsep.GLU_SWIGLU else O.geglu_f64
    return torch.from_numpy(fn(gate.cpu().numpy(), up.cpu().numpy())).to(gate.device)


@pytest.mark.parametrize("N", [1, 2, 3])
@pytest.mark.parametrize("glu", [jsep.GLU_SWIGLU, jsep.GLU_GELU])
@pytest.mark.parametrize("group", sorted(FUSED_GLU_GROUPS))
def test_fused_glu_vs_torch_fp64(runtime, group, glu, N):
    """wllm_mul_mat_glu_batch: the GLU between the FFN's gate/up projections
    and its down projection, fused into the streaming kernel, against float64
    act(gate) * up, then a float64 matmul of the device-dequantized weights.
    Gate values past +-10 exercise GELU's two clamps. Three vectors of a
    K above 8192 are outside the streaming kernel: NOT_IMPLEMENTED, nothing
    written. gate and up are left as they were."""
    import torch

    mats, K = FUSED_GLU_GROUPS[group]
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(len(group) * 11 + N + 5 * glu)
    up_stride = K + 64  # up in a wider buffer: its own stride
    gate = 2.5 * torch.randn(N, K, device=dev, generator=gen)
    gate[:, ::97] = 12.0 * torch.sign(torch.randn(N, (K + 96) // 97, device=dev, generator=gen))
    upbuf = torch.randn(N, up_stride, device=dev, generator=gen)
    up = upbuf[:, :K]
    gate0, up0 = gate.clone(), upbuf.clone()
    ws, ys, ops = [], [], []
    for t, M in mats:
        w = synth.weights_torch(gen, t, M, K, dev)
        y = torch.full((N, M), 7.0, device=dev)
        ws.append(w)
        ys.append(y)
        ops.append(jsep.MulMatArgs(t, M, K, N, w.data_ptr(), w.shape[1], gate.data_ptr(), K, y.data_ptr(), M))
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    rc = jsep.mul_mat_glu_batch(ops, up.data_ptr(), up_stride, glu, stream)
    runtime.jsep_sync()
    if N > 2 and K > 8192:
        assert rc == jsep.STATUS_NOT_IMPLEMENTED
        assert all(bool((y == 7.0).all()) for y in ys)
        return
    assert rc == jsep.STATUS_OK
    h = glu_fp64(gate0, up0[:, :K], glu)
    for (t, M), w, y in zip(mats, ws, ys):
        wf = torch.empty(M, K, device=dev)
        jsep.dequantize_device(t, w.data_ptr(), wf.data_ptr(), M * K, stream)
        runtime.jsep_sync()
        ref = (wf.double() @ h.t()).t()
        rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
        assert rel <= GEMV_TOL, (t, M, rel)
    assert torch.equal(gate, gate0) and torch.equal(upbuf, up0)


def test_fused_glu_rejects_bad_arguments(runtime):
    """Ops that read different gates, an unknown kind, a misaligned up, an
    output overlapping the gate, up or gain input: FAILED with a message;
    NOT_IMPLEMENTED beyond 4 vectors. Nothing is written."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    M, K = 256, 1024
    w = synth.weights_torch(gen, jsep.GGML_TYPE_Q4_K, M, K, dev)
    g = torch.randn(8, K, device=dev, generator=gen)
    u = torch.randn(8, K + 4, device=dev, generator=gen)
    y = torch.full((8, M), 7.0, device=dev)
    torch.cuda.synchronize()
    s = jsep.library_stream()

    def op(x_off, n):
        return jsep.MulMatArgs(jsep.GGML_TYPE_Q4_K, M, K, n, w.data_ptr(), w.shape[1], g.data_ptr() + 4 * x_off, K,
                               y.data_ptr(), M)

    assert jsep.mul_mat_glu_batch([op(0, 8)], u.data_ptr(), K, jsep.GLU_SWIGLU, s) == jsep.STATUS_NOT_IMPLEMENTED
    def op_y(y_ptr):
        return jsep.MulMatArgs(jsep.GGML_TYPE_Q4_K, M, K, 1, w.data_ptr(), w.shape[1], g.data_ptr(), K, y_ptr, M)

    for args in (([op(0, 1), op(K, 1)], u.data_ptr(), K, jsep.GLU_SWIGLU),
                 ([op(0, 1)], u.data_ptr(), K, 7),
                 ([op(0, 1)], u.data_ptr() + 4, K, jsep.GLU_GELU),
                 ([op(0, 2)], u.data_ptr(), K + 2, jsep.GLU_GELU),
                 ([op_y(u.data_ptr())], u.data_ptr(), K, jsep.GLU_SWIGLU),   # y inside up
                 ([op_y(g.data_ptr())], u.data_ptr(), K, jsep.GLU_SWIGLU)):  # y inside the gate
        with pytest.raises(jsep.WllmError):
            jsep.mul_mat_glu_batch(*args, stream=s)
    with pytest.raises(jsep.WllmError):  # the gain inside y
        jsep.mul_mat_rms_norm_batch([op(0, 1)], y.data_ptr(), 1e-5, s)
    runtime.jsep_sync()
    assert bool((y == 7.0).all())


@pytest.mark.parametrize("N", [65, 200])
def test_q6k_prefill_sizes_vs_torch_fp64(runtime, N):
    """Q6_K with more than 64 vectors (prefill; several 32-vector tiles) whose
    1890-byte rows are neither a multiple of 16 bytes nor of 8, so the
    tensor-memory copies of the tcgen05 path cannot take them: the batched
    GEMM, at the GEMV bar. 1024 x 2304."""
    import torch

    M, K = 1024, 2304
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(N)
    w = synth.weights_torch(gen, jsep.GGML_TYPE_Q6_K, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.empty(N, M, device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    jsep.mul_mat_device(jsep.GGML_TYPE_Q6_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N,
                        stream)
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(jsep.GGML_TYPE_Q6_K, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ x.double().t()).t()
    rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel <= GEMV_TOL, rel


@pytest.mark.parametrize("qtype,M,K", [(jsep.GGML_TYPE_Q4_K, 4096, 4096), (jsep.GGML_TYPE_Q4_K, 1024, 4096),
                                       (jsep.GGML_TYPE_Q4_K, 12288, 4096), (jsep.GGML_TYPE_Q4_K, 4096, 12288)])
def test_qwen3_8b_layer_shapes_vs_torch_fp64(runtime, qtype, M, K):
    """Qwen3-8B decode (batch 1) layer shapes: q/o, k/v, gate/up, down."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(M * 3 + K)
    w = synth.weights_torch(gen, qtype, M, K, dev)
    x = torch.randn(1, K, device=dev, generator=gen)
    y = torch.empty(1, M, device=dev)
    torch.cuda.synchronize()  # the library runs on its own stream
    stream = jsep.library_stream()
    jsep.mul_mat_device(qtype, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, 1, stream)
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(qtype, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ x.double().t()).t()
    rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel <= GEMV_TOL, rel


def test_qwen3_8b_output_projection_vs_torch_fp64(runtime):
    """The largest decode GEMV of the sweeps: Qwen3-8B's 151936 x 4096 Q6_K output
    projection (510 MB of weights) at N = 1, against a float64 matmul of the
    device-dequantized weights (bit-exact with the oracle's dequantization)."""
    import torch

    dev = torch.device("cuda", 0)
    M, K = 151936, 4096
    gen = torch.Generator(device=dev)
    gen.manual_seed(8)
    w = synth.weights_torch(gen, jsep.GGML_TYPE_Q6_K, M, K, dev)
    x = torch.randn(1, K, device=dev, generator=gen)
    y = torch.empty(1, M, device=dev)
    torch.cuda.synchronize()  # the library runs on its own stream
    stream = jsep.library_stream()
    jsep.mul_mat_device(jsep.GGML_TYPE_Q6_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, 1,
                        stream)
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(jsep.GGML_TYPE_Q6_K, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ x.double().t()).t()
    rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
    assert rel <= GEMV_TOL, rel


PARTIAL_ROUND_LAUNCHES = {
    # more units than SMs, the last round partial: CTAs own different unit counts
    "down_q6k": [(jsep.GGML_TYPE_Q6_K, 3072, 8192)],
    "o_q4k": [(jsep.GGML_TYPE_Q4_K, 3072, 3072)],
    "qkv_mixed": [(jsep.GGML_TYPE_Q4_K, 3072, 3072), (jsep.GGML_TYPE_Q4_K, 1024, 3072), (jsep.GGML_TYPE_Q6_K, 1024, 3072)],
    "q8_0": [(jsep.GGML_TYPE_Q8_0, 2848, 2304)],
    # a long-K op followed by many tiny units of a second op
    "wide_and_tiny": [(jsep.GGML_TYPE_Q4_K, 2528, 16384), (jsep.GGML_TYPE_Q4_K, 640, 256)],
    "ragged_rows": [(jsep.GGML_TYPE_Q6_K, 2371, 4096)],
}


@pytest.mark.parametrize("N", [1, 2, 3, 4])
@pytest.mark.parametrize("case", sorted(PARTIAL_ROUND_LAUNCHES))
def test_partial_round_launches_vs_torch_fp64(runtime, case, N):
    """Grouped decode launches with more 16-row units than SMs and a partial
    last round (mixed types, mixed K, ragged rows): against a float64 matmul
    of the device-dequantized weights, and bit-identical over three launches
    in a row."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(len(case) * 101 + N)
    mats = PARTIAL_ROUND_LAUNCHES[case]
    ws, xs, ys, ops = [], [], [], []
    for t, M, K in mats:
        w = synth.weights_torch(gen, t, M, K, dev)
        x = torch.randn(N, K, device=dev, generator=gen)
        y = torch.empty(N, M, device=dev)
        ws.append(w)
        xs.append(x)
        ys.append(y)
        ops.append(jsep.MulMatArgs(t, M, K, N, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M))
    torch.cuda.synchronize()  # the library runs on its own stream
    stream = jsep.library_stream()
    runs = []
    for _ in range(3):
        jsep.mul_mat_batch(ops, stream)
        runtime.jsep_sync()
        runs.append([y.clone() for y in ys])
    for (t, M, K), w, x, y in zip(mats, ws, xs, runs[0]):
        wf = torch.empty(M, K, device=dev)
        jsep.dequantize_device(t, w.data_ptr(), wf.data_ptr(), M * K, stream)
        runtime.jsep_sync()
        ref = (wf.double() @ x.double().t()).t()
        rel = ((y.double() - ref).abs().max() / ref.abs().max()).item()
        assert rel <= GEMV_TOL, (t, M, K, rel)
    for later in runs[1:]:
        for a, b in zip(runs[0], later):
            assert torch.equal(a, b)


@pytest.mark.parametrize("qtype", [jsep.GGML_TYPE_Q4_K, jsep.GGML_TYPE_Q6_K, jsep.GGML_TYPE_Q8_0])
def test_streaming_edge_shapes(runtime, qtype):
    """Shapes around the streaming kernel's unit/segment boundaries: rows not
    a multiple of the 8-row unit, K spanning several segments, a row count
    far below the SM count and one above it."""
    for M, K in ((1, 256), (9, 4096), (15, 12288), (1000, 2560), (2051, 512)):
        rng = np.random.default_rng(M * 31 + K + qtype)
        w = synth.weights(rng, qtype, M, K)
        for N in (1, 2):
            x = synth.activations(rng, N, K)
            got = run_mul_mat(runtime, qtype, w, x)
            assert O.rel_error(got, O.mul_mat_f64(qtype, w, x)) <= GEMV_TOL, (M, K, N)


@pytest.mark.parametrize("scale", [1e-6, 1.0, 3e5])
def test_activation_magnitudes(runtime, scale):
    """Activations far outside N(0,1), including values beyond the f16 range
    (the tensor-core path rescales each vector by a power of two)."""
    rng = np.random.default_rng(int(scale * 1e6) % 2**31)
    for qtype in (jsep.GGML_TYPE_Q4_K, jsep.GGML_TYPE_Q6_K, jsep.GGML_TYPE_Q8_0):
        w = synth.weights(rng, qtype, 64, 2048)
        for N in (1, 2):
            x = (synth.activations(rng, N, 2048) * scale).astype(np.float32)
            x[0, 5] = 0.0
            got = run_mul_mat(runtime, qtype, w, x)
            assert np.all(np.isfinite(got))
            assert O.rel_error(got, O.mul_mat_f64(qtype, w, x)) <= GEMV_TOL, (qtype, N, scale)


def test_single_gemv_4096(runtime):
    """The 4096x4096 Q4_K single-GEMV workload, batch 1."""
    rng = np.random.default_rng(1)
    w = synth.q4_k_blocks(rng, 4096, 4096)
    x = synth.activations(rng, 1, 4096)
    got = run_mul_mat(runtime, jsep.GGML_TYPE_Q4_K, w, x)
    assert O.rel_error(got, O.mul_mat_f64(O.TYPE_Q4_K, w, x)) <= GEMV_TOL


def test_scaling_by_two_is_exact_and_deterministic(runtime):
    """Size-independent properties at a full layer size: doubling x doubles y
    bit-exactly (power-of-two scaling commutes with every rounding), and two
    runs are bit-identical."""
    rng = np.random.default_rng(5)
    w = synth.q4_k_blocks(rng, 8192, 3072)
    x = synth.activations(rng, 1, 3072)
    a = run_mul_mat(runtime, jsep.GGML_TYPE_Q4_K, w, x)
    b = run_mul_mat(runtime, jsep.GGML_TYPE_Q4_K, w, x)
    c = run_mul_mat(runtime, jsep.GGML_TYPE_Q4_K, w, 2 * x)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal((2 * a).view(np.uint32), c.view(np.uint32))


def test_batched_broadcast_and_strides(runtime):
    """ne2 = 4 activation batches sharing 2 weight batches (r2 = 2, the GQA
    broadcast of matmul.ts:594-611) with padded src1/dst row strides."""
    rng = np.random.default_rng(11)
    qtype, M, K, N, B0, B1 = jsep.GGML_TYPE_Q4_K, 48, 512, 3, 2, 4
    w = synth.weights(rng, qtype, M * B0, K).reshape(B0, M, -1)
    xpad, ypad = K + 8, M + 4
    x = np.zeros((B1, N, xpad), np.float32)
    x[:, :, :K] = rng.standard_normal((B1, N, K), dtype=np.float32)
    h0, h1 = upload(runtime, w), upload(runtime, x)
    hd = runtime.data_manager.alloc(4 * B1 * N * ypad)
    runtime.data_manager.clear(hd, 0, 0, 4 * B1 * N * ypad)
    rb = synth.row_bytes(qtype, K)
    src0 = jsep.JsepTensorMeta(h0, 0, qtype, (K, M, B0, 1), (144, rb, rb * M, rb * M * B0))
    src1 = jsep.JsepTensorMeta(h1, 0, 0, (K, N, B1, 1), (4, 4 * xpad, 4 * xpad * N, 4 * xpad * N * B1))
    dst = jsep.JsepTensorMeta(hd, 0, 0, (M, N, B1, 1), (4, 4 * ypad, 4 * ypad * N, 4 * ypad * N * B1))
    assert jsep.dispatch_matmul(runtime, jsep.JsepOpDescriptor(29, 2, dst, [src0, src1])) == 0, jsep.last_error()
    got = runtime.data_manager.read(hd, 0, 4 * B1 * N * ypad).view(np.float32).reshape(B1, N, ypad)
    for b in range(B1):
        r = O.mul_mat_f64(qtype, w[b // 2], x[b, :, :K])
        assert O.rel_error(got[b, :, :M], r) <= GEMV_TOL
        assert np.all(got[b, :, M:] == 0)


def test_dst_aliases_src1_buffer(runtime):
    """dst and src1 in one buffer: disjoint ranges run in place, overlapping
    ranges take the divert path (matmul.ts:675-958)."""
    rng = np.random.default_rng(12)
    qtype, M, K, N = jsep.GGML_TYPE_Q6_K, 256, 256, 2
    w = synth.weights(rng, qtype, M, K)
    x = synth.activations(rng, N, K)
    r = O.mul_mat_f64(qtype, w, x)
    h0 = upload(runtime, w)
    for dst_off in (4 * N * K, 0):  # disjoint, then overlapping (dst over src1)
        hb = runtime.data_manager.alloc(4 * N * K + 4 * M * N)
        runtime.data_manager.write(hb, 0, x)
        desc = jsep.JsepOpDescriptor(29, 2, jsep.meta_for(hb, 0, (M, N, 1, 1), offset=dst_off),
                                     [jsep.meta_for(h0, qtype, (K, M, 1, 1)), jsep.meta_for(hb, 0, (K, N, 1, 1))])
        assert jsep.dispatch_matmul(runtime, desc) == 0, jsep.last_error()
        got = runtime.data_manager.read(hb, dst_off, 4 * M * N).view(np.float32).reshape(N, M)
        assert O.rel_error(got, r) <= GEMV_TOL, dst_off
        runtime.data_manager.free(hb)
    runtime.data_manager.free(h0)


def test_run_ops_grouped_qkv(runtime):
    """q/k/v of one layer (two Q4_K, one Q6_K) in a single launch."""
    rng = np.random.default_rng(13)
    x = synth.activations(rng, 1, 3072)
    hx = upload(runtime, x)
    specs = [(jsep.GGML_TYPE_Q4_K, 3072), (jsep.GGML_TYPE_Q4_K, 1024), (jsep.GGML_TYPE_Q6_K, 1024)]
    ws, hs, descs = [], [], []
    for qtype, M in specs:
        w = synth.weights(rng, qtype, M, 3072)
        h0, hd = upload(runtime, w), runtime.data_manager.alloc(4 * M)
        ws.append(w)
        hs.append((h0, hd))
        descs.append(jsep.JsepOpDescriptor(29, 2, jsep.meta_for(hd, 0, (M, 1, 1, 1)),
                                           [jsep.meta_for(h0, qtype, (3072, M, 1, 1)), jsep.meta_for(hx, 0, (3072, 1, 1, 1))]))
    k0 = runtime.counters()["kernels_launched"]
    assert runtime.run_ops(descs) == 0, jsep.last_error()
    # one kernel launch for all three
    assert runtime.counters()["kernels_launched"] == k0 + 1
    for (qtype, M), w, (h0, hd) in zip(specs, ws, hs):
        got = runtime.data_manager.read(hd, 0, 4 * M).view(np.float32).reshape(1, M)
        assert O.rel_error(got, O.mul_mat_f64(qtype, w, x)) <= GEMV_TOL


def test_status_codes(runtime):
    """NOT_IMPLEMENTED for other ops/types (caller falls back), FAILED with a
    message for shape, stride, range and handle violations."""
    dm = runtime.data_manager
    h0, h1, hd = dm.alloc(144 * 4), dm.alloc(4 * 256), dm.alloc(16)
    good_src0 = jsep.meta_for(h0, jsep.GGML_TYPE_Q4_K, (256, 4, 1, 1))
    src1 = jsep.meta_for(h1, 0, (256, 1, 1, 1))
    dst = jsep.meta_for(hd, 0, (4, 1, 1, 1))

    def st(desc):
        return jsep.dispatch_matmul(runtime, desc)

    assert st(jsep.JsepOpDescriptor(jsep.GGML_OP_RMS_NORM, 1, dst, [src1])) == jsep.STATUS_NOT_IMPLEMENTED
    f16 = jsep.meta_for(h0, jsep.GGML_TYPE_F16, (256, 1, 1, 1))
    assert st(jsep.JsepOpDescriptor(29, 2, dst, [f16, src1])) == jsep.STATUS_NOT_IMPLEMENTED
    assert st(jsep.JsepOpDescriptor(29, 2, dst, [good_src0, src1])) == jsep.STATUS_OK
    bad_shape = jsep.meta_for(hd, 0, (3, 1, 1, 1))
    assert st(jsep.JsepOpDescriptor(29, 2, bad_shape, [good_src0, src1])) == jsep.STATUS_FAILED
    assert "shape mismatch" in jsep.last_error()
    too_long = jsep.meta_for(h0, jsep.GGML_TYPE_Q4_K, (256, 5, 1, 1))  # 5 rows in a 4-row buffer
    assert st(jsep.JsepOpDescriptor(29, 2, jsep.meta_for(hd, 0, (5, 1, 1, 1)), [too_long, src1])) == jsep.STATUS_FAILED
    assert "past" in jsep.last_error()
    dead = jsep.meta_for(9999, jsep.GGML_TYPE_Q4_K, (256, 4, 1, 1))
    assert st(jsep.JsepOpDescriptor(29, 2, dst, [dead, src1])) == jsep.STATUS_FAILED
    assert "invalid handle" in jsep.last_error()
    bad_src1 = jsep.meta_for(h1, jsep.GGML_TYPE_F16, (256, 1, 1, 1))
    assert st(jsep.JsepOpDescriptor(29, 2, dst, [good_src0, bad_src1])) == jsep.STATUS_FAILED
    one_src = jsep.JsepOpDescriptor(29, 1, dst, [good_src0])
    assert st(one_src) == jsep.STATUS_FAILED
    assert "expected 2 srcs" in jsep.last_error()
    for h in (h0, h1, hd):
        dm.free(h)
    dm.free(h0)  # idempotent
    rt_sync = runtime.lib.wllm_sync()
    assert rt_sync == jsep.STATUS_OK


def test_buffers_roundtrip_clear_and_async_read(runtime):
    dm = runtime.data_manager
    h = dm.alloc(1 << 20)
    data = np.arange(1 << 18, dtype=np.uint32)
    dm.write(h, 0, data)
    assert np.array_equal(dm.read(h, 0, 1 << 20).view(np.uint32), data)
    dm.clear(h, 0xAB, 4096, 100)
    back = dm.read(h, 4096, 100)
    assert np.all(back == 0xAB)
    req = dm.read_async(h, 0, 4096)
    for _ in range(100000):
        if req.poll():
            break
    assert np.array_equal(req.finish().view(np.uint32), data[:1024])
    c = runtime.counters()
    assert c["alloc"] >= 1 and c["write"] >= 1 and c["read"] >= 2
    dm.free(h)


@pytest.mark.parametrize("N", [1, 2, 3, 4])
@pytest.mark.parametrize("M,K", [(4096, 4096), (1024, 4096), (12288, 4096), (4096, 12288), (3072, 3072),
                                 (1000, 2304), (33, 256)])
def test_iq4_xs_decode_vs_torch_fp64(runtime, M, K, N):
    """IQ4_XS (136-byte blocks, non-linear 4-bit levels, 6-bit sub-block
    scales) on the streaming integer tensor-core GEMV (and the general
    kernel where the streaming one does not take the shape: K = 2304 rows
    are 1224 bytes, not 16-byte aligned, so they are copied row by row),
    against a float64 matmul of the device-dequantized weights, both
    metrics."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(23 * 1000 + M + K + N)
    t = jsep.GGML_TYPE_IQ4_XS
    w = synth.weights_torch(gen, t, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.full((N, M), float("nan"), device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    assert jsep.mul_mat_device(t, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N,
                               stream) == jsep.STATUS_OK
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(t, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ x.double().t()).t().cpu().numpy()
    got = y.double().cpu().numpy()
    assert O.rel_error(got, ref) <= GEMV_TOL and O.rel_error_elem(got, ref) <= GEMV_TOL


def test_iq4_xs_through_the_descriptor_seam_vs_oracle(runtime):
    """IQ4_XS through wllm_run_op (the jsepRunOp descriptor), against the
    oracle's f64 dequant-then-dot (pinned to gguf 0.19.0's dequantization)."""
    rng = np.random.default_rng(2300)
    t = jsep.GGML_TYPE_IQ4_XS
    for M, K, N in ((96, 2048, 1), (40, 4096, 2), (17, 1024, 5)):
        w = synth.weights(rng, t, M, K)
        x = synth.activations(rng, N, K)
        got = run_mul_mat(runtime, t, w, x)
        r = O.mul_mat_f64(t, w, x)
        assert O.rel_error(got, r) <= GEMV_TOL and O.rel_error_elem(got, r) <= GEMV_TOL, (M, K, N)


@pytest.mark.parametrize("N", [3, 5, 8, 16, 33, 64])
@pytest.mark.parametrize("M,K", [(4096, 4096), (1000, 2304), (12288, 4096), (4096, 14336), (33, 256)])
def test_iq4_xs_batched_vs_torch_fp64(runtime, M, K, N):
    """IQ4_XS at 3-64 vectors on the integer tensor-core batched GEMM (levels
    as s8 A fragments, ls - 32 per sub-block; K = 2304's 8-byte aligned rows
    through the 16-byte copy window; N = 3 with K = 14336, which the streaming
    kernel leaves to it), against a float64 matmul of the device-dequantized
    weights, both metrics."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(23 * 2000 + M + K + N)
    t = jsep.GGML_TYPE_IQ4_XS
    w = synth.weights_torch(gen, t, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.full((N, M), float("nan"), device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    assert jsep.mul_mat_device(t, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N,
                               stream) == jsep.STATUS_OK
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(t, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    ref = (wf.double() @ x.double().t()).t().cpu().numpy()
    got = y.double().cpu().numpy()
    assert O.rel_error(got, ref) <= GEMV_TOL and O.rel_error_elem(got, ref) <= GEMV_TOL
