"""Row-sharded decode with the gather fused into the GEMV (wllm_mul_mat_batch_tp):
each rank computes a row slice of every weight and writes its rows straight
into every rank's gather buffer over NVLink; wllm_tp_wait makes them
complete. Two ranks, one process per GPU; skipped with fewer than 2 GPUs.

Bar: every rank's gathered outputs within 1e-3 (max|y - r| / max|r|) of the
oracle's f64 dequant-then-dot, over three launch groups in a row (the
per-launch signal counters carry over) and with rows that do not divide
evenly between the ranks.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2
TOL = 1e-3


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


class _DevArray:
    """A raw device pointer as a torch tensor (zero copy)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def _rank_main(rank, port, out_q):
    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from webllm_b200 import jsep, synth
    from webllm_b200.tp import row_shard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        rt = jsep.install_jsep_callbacks(rank)
        # three launch groups; rows not divisible by the world size in two ops
        groups = [[(O.TYPE_Q4_K, 48, 512), (O.TYPE_Q6_K, 33, 512)],
                  [(O.TYPE_Q4_K, 17, 768)],
                  [(O.TYPE_Q6_K, 64, 1024), (O.TYPE_Q4_K, 31, 1024)]]
        rng = np.random.default_rng(2024)  # same weights and x on every rank
        plans, total = [], 0
        for mats in groups:
            K = mats[0][2]
            x = synth.activations(rng, 1, K)
            ws = [synth.weights(rng, t, M, K) for t, M, _ in mats]
            pads = [row_shard(M, WORLD, rank).padded for _, M, _ in mats]
            gt = sum(pads)
            plans.append((mats, x, ws, pads, gt, total))
            total += WORLD * gt
        # one peer-mappable gather buffer for every group, a signal array, counters
        g_ptr, g_handle = jsep.ipc_alloc(4 * total)
        s_ptr, s_handle = jsep.ipc_alloc(4 * jsep.MAX_RANKS)
        st_ptr, _ = jsep.ipc_alloc(16)
        handles = [None] * WORLD
        dist.all_gather_object(handles, (g_handle, s_handle))
        gbase = [g_ptr if r == rank else jsep.ipc_open(handles[r][0]) for r in range(WORLD)]
        sig = [s_ptr if r == rank else jsep.ipc_open(handles[r][1]) for r in range(WORLD)]
        group = jsep.tp_group(WORLD, rank, sig, st_ptr)
        keep, launches = [], []
        for mats, x, ws, pads, gt, off0 in plans:
            K = mats[0][2]
            xd = torch.from_numpy(x).to(dev)
            ops, outs = [], []
            for i, ((t, M, _), w) in enumerate(zip(mats, ws)):
                sh = row_shard(M, WORLD, rank)
                rb = synth.row_bytes(t, K)
                wd = torch.from_numpy(np.ascontiguousarray(w[sh.start:sh.start + sh.count])).to(dev)
                keep.append(wd)
                col = off0 + rank * gt + sum(pads[:i])  # this rank's rows of op i in every rank's buffer
                ys = [gbase[r] + 4 * col for r in range(WORLD)]
                ops.append(jsep.MulMatArgs(t, sh.count, K, 1, wd.data_ptr(), rb, xd.data_ptr(), K, ys[rank], sh.count))
                outs.append(ys)
            keep.append(xd)
            launches.append((ops, outs))
        torch.cuda.synchronize()
        for ops, outs in launches:
            jsep.mul_mat_batch_tp(ops, outs, group)
        jsep.tp_wait(group)
        rt.jsep_sync()
        dist.barrier()  # every rank's launches are done before anyone reads or frees
        G = torch.as_tensor(_DevArray(g_ptr, total), device=dev).cpu().numpy()
        worst = 0.0
        for (mats, x, ws, pads, gt, off0) in plans:
            for r in range(WORLD):
                for i, ((t, M, _), w) in enumerate(zip(mats, ws)):
                    sh = row_shard(M, WORLD, r)
                    col = off0 + r * gt + sum(pads[:i])
                    got = G[col:col + sh.count][None, :]
                    ref = O.mul_mat_f64(t, w[sh.start:sh.start + sh.count], x)
                    worst = max(worst, O.rel_error(got, ref))
        dist.barrier()
        for r in range(WORLD):
            if r != rank:
                jsep.ipc_close(gbase[r])
                jsep.ipc_close(sig[r])
        dist.barrier()
        out_q.put((rank, worst))
    finally:
        dist.destroy_process_group()


def test_row_sharded_peer_gather_two_ranks():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, worst in results:
        assert worst <= TOL, f"rank {rank}: gathered rows differ from the oracle by {worst}"
