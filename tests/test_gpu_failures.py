"""Failure paths and memory accounting on the device, without faulting a GPU.

- A row-sharded launch whose peer never signals: a world-2 group on ONE GPU
  whose "peer" signal array and gather buffer are local zeroed memory that
  nothing increments. The bounded peer wait runs out (after a short limit set
  with wllm_set_wait_limit), the kernel records an error and still ends,
  wllm_sync returns WLLM_STATUS_FAILED with the message, and the next normal
  launch succeeds with correct results. Nothing hangs or faults: every
  pointer the launch touches is valid local memory.
- The library's byte counters follow the reference's MemoryPool contract
  (src/core/memory-pool.ts:72-112: allocate adds the tensor's bytes, free
  takes them off): bytes_live moves by exactly each buffer's size, freeing is
  idempotent, and bytes_reserved keeps freed blocks for reuse.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from webllm_b200 import jsep, synth

pytestmark = pytest.mark.gpu


def _counters():
    c = jsep.WllmCounters()
    jsep.load_library().wllm_get_counters(c)
    return c


def test_row_sharded_peer_wait_times_out_and_recovers(runtime):
    import torch

    dev = torch.device("cuda", 0)
    M, K = 64, 512
    rng = np.random.default_rng(77)
    w_np = synth.weights(rng, O.TYPE_Q4_K, M, K)
    x_np = synth.activations(rng, 1, K)
    w = torch.from_numpy(w_np).to(dev)
    x = torch.from_numpy(x_np).to(dev)
    y_own = torch.zeros(1, M, device=dev)
    y_fake_peer = torch.zeros(1, M, device=dev)  # where "rank 1" would keep rank 0's rows
    own_sig, _ = jsep.ipc_alloc(4 * jsep.MAX_RANKS)
    fake_peer_sig, _ = jsep.ipc_alloc(4 * jsep.MAX_RANKS)
    state, _ = jsep.ipc_alloc(16)
    torch.cuda.synchronize()
    stream = jsep.library_stream()
    try:
        group = jsep.tp_group(2, 0, [own_sig, fake_peer_sig], state)
        op = jsep.MulMatArgs(O.TYPE_Q4_K, M, K, 1, w.data_ptr(), w.shape[1], x.data_ptr(), K, y_own.data_ptr(), M)
        jsep.set_wait_limit(20000)
        jsep.mul_mat_batch_tp([op], [[y_own.data_ptr(), y_fake_peer.data_ptr()]], group, stream)
        rc = jsep.load_library().wllm_sync()
        assert rc == jsep.STATUS_FAILED
        msg = jsep.last_error()
        assert "gave up waiting" in msg and "code 0x" in msg, msg
        code = int(msg.split("code 0x")[1].split(":")[0], 16)
        assert code & 4, msg  # the peer's signal (bit 2)
    finally:
        jsep.set_wait_limit(0)
    # the context is usable: a normal launch gives correct results
    y = torch.full((1, M), float("nan"), device=dev)
    jsep.mul_mat_device(O.TYPE_Q4_K, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, 1, stream)
    runtime.jsep_sync()
    r = O.mul_mat_f64(O.TYPE_Q4_K, w_np, x_np)
    got = y.cpu().numpy()
    assert O.rel_error(got, r) <= 1e-3 and O.rel_error_elem(got, r) <= 1e-3
    for p in (own_sig, fake_peer_sig, state):
        jsep.ipc_free(p)


def test_memory_pool_accounting(runtime):
    dm = runtime.data_manager
    base = _counters()
    # a "model": tensors of GGUF sizes, uploaded as the reference's loadWeights
    # does (alloc, then write), then the MemoryPool figure is the byte sum
    rng = np.random.default_rng(3)
    tensors = [synth.weights(rng, t, M, K) for t, M, K in
               ((O.TYPE_Q4_K, 96, 1024), (O.TYPE_Q6_K, 33, 2048), (O.TYPE_Q8_0, 7, 4096), (O.TYPE_Q4_K, 4096, 2048))]
    handles = []
    for a in tensors:
        h = dm.alloc(a.nbytes)
        dm.write(h, 0, a)
        handles.append(h)
    c = _counters()
    total = sum(a.nbytes for a in tensors)
    assert c.bytes_live - base.bytes_live == total
    assert c.bytes_reserved - base.bytes_reserved >= 0
    assert c.bytes_reserved >= c.bytes_live
    assert c.alloc - base.alloc == len(tensors) and c.write - base.write == len(tensors)
    # reads and clears leave the accounting alone
    got = dm.read(handles[0], 0, tensors[0].nbytes)
    assert np.array_equal(got, tensors[0].reshape(-1).view(np.uint8))
    dm.clear(handles[1], 0, 0, 64)
    assert _counters().bytes_live == c.bytes_live
    # free takes each tensor's bytes off, once (free is idempotent)
    reserved = _counters().bytes_reserved
    dm.free(handles[0])
    dm.free(handles[0])
    c2 = _counters()
    assert c.bytes_live - c2.bytes_live == tensors[0].nbytes
    assert c2.free - c.free == 1
    assert c2.bytes_reserved == reserved  # the block stays in the free list
    # the same size again reuses the freed block: nothing new is reserved
    h = dm.alloc(tensors[0].nbytes)
    assert _counters().bytes_reserved == reserved
    assert _counters().bytes_live == c.bytes_live
    for hh in handles[1:] + [h]:
        dm.free(hh)
    end = _counters()
    assert end.bytes_live == base.bytes_live
    assert end.bytes_reserved == reserved
