"""Row-sharded multi-rank MUL_MAT: shard arithmetic and the all-gather
assembly, run as world_size-2 (and 3) gloo ranks on CPU with the oracle as
each rank's local GEMV (no GPU)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from webllm_b200 import synth
from webllm_b200.tp import TPMulMat, row_shard, shard_bytes, shards_cover


@pytest.mark.parametrize("M,world", [(16, 2), (17, 2), (3072, 8), (1024, 8), (151936, 8), (5, 8), (1, 4)])
def test_row_shards_partition_rows(M, world):
    shards = shards_cover(M, world)
    covered = []
    for s in shards:
        covered.extend(range(s.start, s.start + s.count))
        assert s.count <= s.padded
    assert covered == list(range(M))
    assert all(s.padded == -(-M // world) for s in shards)


def test_row_shard_rejects_bad_requests():
    for args in [(0, 2, 0), (8, 0, 0), (8, 2, 2), (8, 2, -1)]:
        with pytest.raises(ValueError):
            row_shard(*args)


def test_shard_bytes_are_whole_rows():
    rng = np.random.default_rng(0)
    w = synth.weights(rng, O.TYPE_Q4_K, 10, 512)
    rb = synth.row_bytes(O.TYPE_Q4_K, 512)
    s = row_shard(10, 3, 1)
    view = shard_bytes(w.tobytes(), rb, s)
    assert len(view) == s.count * rb
    assert bytes(view) == w.tobytes()[s.start * rb:(s.start + s.count) * rb]


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _rank_main(rank, world, port, qtype, M, K, N, seed, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(seed)  # every rank builds the same full weights and x
        w = synth.weights(rng, qtype, M, K)
        x = synth.activations(rng, N, K)
        rb = synth.row_bytes(qtype, K)
        shard = row_shard(M, world, rank)
        w_local = np.frombuffer(bytes(shard_bytes(w.tobytes(), rb, shard)), dtype=np.uint8).reshape(shard.count, rb)

        def local(xt, y_shard):
            y = O.mul_mat_f64(qtype, w_local, xt.numpy())  # (N, count)
            y_shard[:, :shard.count] = torch.from_numpy(y.astype(np.float32))

        tp = TPMulMat(M, N, world, rank, local, dist.all_gather_into_tensor)
        y = tp.forward(torch.from_numpy(x)).numpy()
        ref = O.mul_mat_f64(qtype, w, x).astype(np.float32)
        out_q.put((rank, float(np.max(np.abs(y - ref))), y.shape))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,qtype,M,K,N", [
    (2, O.TYPE_Q4_K, 48, 512, 1),
    (2, O.TYPE_Q6_K, 33, 256, 2),    # M not divisible by world: padded gather
    (3, O.TYPE_Q8_0, 20, 64, 3),
])
def test_gloo_row_sharded_mul_mat_matches_full(world, qtype, M, K, N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, qtype, M, K, N, 7, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, shape in results:
        assert shape == (N, M)
        assert err == 0.0, f"rank {rank}: gathered output differs from the single-rank result by {err}"
