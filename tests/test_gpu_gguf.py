"""A GGUF file's tensors streamed into device memory (gguf.stream_to_buffers
with the real GpuDataManager) land bit-identical and feed MUL_MAT through
the descriptor seam (wllm_run_op), against the oracle. This is the path that
replaces the reference's upload through the wasm heap
(src/inference/ggml-wasm.ts:545-620) followed by the graph's MUL_MAT nodes.
The file is written by the third-party `gguf` package."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from webllm_b200 import gguf as G
from webllm_b200 import jsep, synth

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")

TENSORS = [
    # name, ggml type, M rows, K
    ("blk.0.attn_q.weight", O.TYPE_Q4_K, 512, 2048, "Q4_K"),
    ("blk.0.ffn_down.weight", O.TYPE_Q6_K, 256, 3072, "Q6_K"),
    ("token_embd.weight", O.TYPE_Q8_0, 384, 2304, "Q8_0"),
    ("blk.0.ffn_up.weight", O.TYPE_Q5_K, 128, 1024, "Q5_K"),
    ("blk.0.attn_k.weight", O.TYPE_Q4_0, 96, 4096, "Q4_0"),
]


def _counters():
    c = jsep.WllmCounters()
    jsep.load_library().wllm_get_counters(c)
    return c


def test_gguf_file_to_hbm_feeds_run_op(runtime, tmp_path):
    rng = np.random.default_rng(2026)
    path = tmp_path / "model.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    arrays = {}
    for name, t, M, K, qname in TENSORS:
        a = synth.weights(rng, t, M, K)
        arrays[name] = a
        w.add_tensor(name, a, raw_dtype=getattr(gguf.GGMLQuantizationType, qname))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()

    dm = runtime.data_manager
    before = _counters()
    bufs = G.stream_to_buffers(str(path), dm, chunk_bytes=1 << 20)
    # the MemoryPool figure: bytes_live grows by exactly the tensors' bytes
    assert _counters().bytes_live - before.bytes_live == sum(a.nbytes for a in arrays.values())
    try:
        for name, t, M, K, _ in TENSORS:
            h, info, nbytes = bufs[name]
            assert nbytes == arrays[name].nbytes
            got = dm.read(h, 0, nbytes)
            assert np.array_equal(got, arrays[name].reshape(-1).view(np.uint8)), name
            # MUL_MAT straight from the streamed buffer (N = 1 and N = 3)
            for N in (1, 3):
                x = synth.activations(rng, N, K)
                hx = dm.alloc(x.nbytes)
                dm.write(hx, 0, x)
                hy = dm.alloc(4 * M * N)
                desc = jsep.JsepOpDescriptor(
                    jsep.GGML_OP_MUL_MAT, 2, jsep.meta_for(hy, jsep.GGML_TYPE_F32, (M, N, 1, 1)),
                    [jsep.meta_for(h, t, (K, M, 1, 1)), jsep.meta_for(hx, jsep.GGML_TYPE_F32, (K, N, 1, 1))])
                assert jsep.dispatch_matmul(runtime, desc) == jsep.STATUS_OK, jsep.last_error()
                runtime.encoder_batcher.flush()
                y = dm.read(hy, 0, 4 * M * N).view(np.float32).reshape(N, M)
                r = O.mul_mat_f64(t, arrays[name], x)
                assert O.rel_error(y, r) <= 1e-3 and O.rel_error_elem(y, r) <= 1e-3, (name, N)
                dm.free(hx)
                dm.free(hy)
    finally:
        for h, _, _ in bufs.values():
            dm.free(h)
    assert _counters().bytes_live == before.bytes_live
