"""wllm_mul_mat_prefill_static: the prefill MUL_MAT with its activation
workspace in a fixed 16 MiB device array of the library (no allocation).

Compared bit for bit with wllm_mul_mat (same kernels, runtime-allocated
workspace) on two calls in a row, and checked to refuse a workspace need
above the fixed size. Collected last so that it runs both alone and after
every other GPU test.
"""
from __future__ import annotations

import pytest

from oracle import oracle as O
from webllm_b200 import jsep, synth

pytestmark = pytest.mark.gpu

STATIC_WORKSPACE_BYTES = 16 << 20


def _counters():
    c = jsep.WllmCounters()
    jsep.load_library().wllm_get_counters(c)
    return c


def test_static_prefill_matches_allocating_entry_point(runtime):
    import torch

    dev = torch.device("cuda", 0)
    M, K = 384, 2048
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242)
    w = synth.weights_torch(gen, O.TYPE_Q4_K, M, K, dev)
    stream = jsep.library_stream()
    for N in (256, 96):  # two calls in a row, different N, same workspace
        x = torch.randn(N, K, device=dev, generator=gen)
        y_ref = torch.full((N, M), float("nan"), device=dev)
        y_st = torch.full((N, M), float("nan"), device=dev)
        torch.cuda.synchronize()  # the library runs on its own stream
        jsep.mul_mat_device(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y_ref.data_ptr(), M,
                            M, K, N, stream)
        runtime.jsep_sync()
        k0 = _counters().kernels_launched
        a0 = _counters().alloc
        jsep.mul_mat_prefill_static(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y_st.data_ptr(), M,
                                    M, K, N, stream)
        runtime.jsep_sync()
        assert _counters().kernels_launched - k0 == 2
        assert _counters().alloc == a0
        assert torch.equal(y_st, y_ref), (N, (y_st - y_ref).abs().max().item())


def test_static_prefill_rejects_oversize_and_non_prefill_ops(runtime):
    import torch

    dev = torch.device("cuda", 0)
    M, K = 128, 4096
    N = STATIC_WORKSPACE_BYTES // (2 * K)  # N * K * 2 == 16 MiB: the +256 tail no longer fits
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    w = synth.weights_torch(gen, O.TYPE_Q4_K, M, K, dev)
    x = torch.zeros(N, K, device=dev)
    y = torch.zeros(N, M, device=dev)
    torch.cuda.synchronize()
    with pytest.raises(jsep.WllmError, match="above the fixed"):
        jsep.mul_mat_prefill_static(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M,
                                    M, K, N, 0)
    with pytest.raises(jsep.WllmError, match="only the prefill path"):  # N = 8 is a decode shape
        jsep.mul_mat_prefill_static(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M,
                                    M, K, 8, 0)
    runtime.jsep_sync()  # nothing was launched; the stream is clean


def test_static_prefill_near_the_limit(runtime):
    """N * K * 2 just under the fixed 16 MiB: the partial tiles of a K split
    no longer fit beside the activations, so the static entry point runs
    unsplit while the allocating one may split; both stay within the prefill
    bar of a float64 matmul of the device-dequantized weights, and of each
    other."""
    import torch

    dev = torch.device("cuda", 0)
    M, K = 1024, 4096
    N = (STATIC_WORKSPACE_BYTES - 256) // (2 * K)  # 2047
    assert N * K * 2 + 256 <= STATIC_WORKSPACE_BYTES
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    w = synth.weights_torch(gen, O.TYPE_Q4_K, M, K, dev)
    x = torch.randn(N, K, device=dev, generator=gen)
    y_ref = torch.full((N, M), float("nan"), device=dev)
    y_st = torch.full((N, M), float("nan"), device=dev)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    jsep.mul_mat_device(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y_ref.data_ptr(), M, M, K, N, stream)
    a0 = _counters().alloc
    jsep.mul_mat_prefill_static(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y_st.data_ptr(), M,
                                M, K, N, stream)
    wf = torch.empty(M, K, device=dev)
    jsep.dequantize_device(O.TYPE_Q4_K, w.data_ptr(), wf.data_ptr(), M * K, stream)
    runtime.jsep_sync()
    assert _counters().alloc == a0
    ref = (wf.double() @ x.double().t()).t()
    for y in (y_st, y_ref):
        assert ((y.double() - ref).abs().max() / ref.abs().max()).item() <= 2e-2
    assert ((y_st - y_ref).abs().max() / y_ref.abs().max()).item() <= 2e-2


@pytest.mark.parametrize("qtype,M,K,N", [(O.TYPE_Q6_K, 512, 4096, 128), (O.TYPE_Q8_0, 640, 2304, 100)])
def test_static_prefill_other_types_on_a_caller_stream(runtime, qtype, M, K, N):
    """Q6_K and Q8_0 weights through the static entry point on a stream the
    caller created (not the library's): bit for bit the allocating entry
    point's result on the same stream, twice in a row."""
    import torch

    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(qtype * 7 + N)
    w = synth.weights_torch(gen, qtype, M, K, dev)
    side = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    for rep in range(2):
        x = torch.randn(N, K, device=dev, generator=gen)
        y_ref = torch.full((N, M), float("nan"), device=dev)
        y_st = torch.full((N, M), float("nan"), device=dev)
        torch.cuda.synchronize()
        a0 = _counters().alloc
        jsep.mul_mat_device(qtype, w.data_ptr(), w.shape[1], x.data_ptr(), K, y_ref.data_ptr(), M, M, K, N,
                            side.cuda_stream)
        jsep.mul_mat_prefill_static(qtype, w.data_ptr(), w.shape[1], x.data_ptr(), K, y_st.data_ptr(), M,
                                    M, K, N, side.cuda_stream)
        side.synchronize()
        runtime.jsep_sync()
        assert _counters().alloc == a0
        assert torch.equal(y_st, y_ref), (rep, (y_st - y_ref).abs().max().item())
