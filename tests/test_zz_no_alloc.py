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
