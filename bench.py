#!/usr/bin/env python
"""Benchmark of the quantized MUL_MAT hot path on B200.

Workload (one step = one decode token through every MUL_MAT of the model):
Qwen3-8B-shaped decode, batch 1: 36 layers x 7 Q4_K GEMVs (hidden 4096, FFN
12288, 32 q / 8 kv heads x 128) plus the 151936 x 4096 Q6_K output
projection, f32 N(0,1) activations, seeded synthetic weights: 4.42 GB of
distinct weights per step, larger than the 126 MB L2, so no L2 flush is
needed. Launch grouping follows the real decode dependencies: {q,k,v} share
one input, {gate,up} another, o and down stand alone: 4 launches per layer and
one for the output projection, replayed as one CUDA graph.

With N GPUs (torchrun, one rank per GPU) every weight is row-sharded across
the ranks. The GEMV kernel's epilogue writes each finished row into every
rank's gather buffer over NVLink (peer stores into CUDA-IPC memory), and each
launch waits, bounded, until every rank's rows of the previous launch have
landed: no collective library call on the data path. Total work is fixed
("strong" scaling). `tp_split` adds the same step without the gather (each
rank's GEMVs alone) so the cost of the exchange shows.

value = algorithmic bytes of the whole step (sum over GEMVs of M*K*bpw +
4*N*K + 4*N*M) / device time (CUDA events, max over ranks).
e2e = the same bytes / the time of a step that also copies that step's
activations host->device from pinned memory and its outputs back.
parity = the step's outputs (layer 0, the last layer and the output
projection, every rank's rows) against a float64 matmul of the
library-dequantized weights (that dequantization is bit-exact with the
reference's), both error metrics of the path.

`--impl reference` times the reference algorithm's CPU path (the f32
dequant-then-dot oracle restatement; the reference's llama.cpp CPU kernels
are not vendored in the reference repository) on a bounded sample of the
same workload with all host threads.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
import zlib

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

import numpy as np  # noqa: E402

METRIC = "quantized MUL_MAT GB/s & % HBM peak (decode); prefill TFLOPS; at 1/2/4/8 GPU"
# model: (workload description, layers, output projection in the step)
WORKLOADS = {
    "qwen3-8b": ("qwen3-8b decode (36 layers x 7 Q4_K GEMVs + 151936x4096 Q6_K output projection, f32 "
                 "activations, batch 1)", 36, True),
    "llama-3.2-3b": ("llama-3.2-3b decode sweep (28 layers x 7 GEMVs, Q4_K/Q6_K x f32, batch 1)", 28, False),
}
_MODEL = "qwen3-8b"
# DRAM bytes (read + write) of one Llama-3.2-3B layer's four GEMV launches
# from an ncu capture; its algorithmic bytes are 64,139,264 per layer.
NCU_DRAM_BYTES_PER_LAYER_LLAMA32 = 64_314_496
# The same for Qwen3-8B: one layer's four launches (algorithmic 108,830,720
# bytes) and the 151936x4096 Q6_K output projection (algorithmic 511,129,088).
NCU_DRAM_BYTES_PER_LAYER_QWEN3 = 108_935_168
NCU_DRAM_BYTES_OUTPUT_QWEN3 = 511_432_448
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--model", choices=sorted(WORKLOADS), default="qwen3-8b",
                    help="decode shapes (default: the row-sharded multi-GPU configuration, also the largest "
                         "that fits one GPU)")
    ap.add_argument("--layers", type=int, default=None, help="layers per step (default: the model's)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU-baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill GEMM measurement")
    ap.add_argument("--no-batched", action="store_true", help="skip the batched Q8_0 decode measurement")
    ap.add_argument("--no-fused-norm", action="store_true", help="skip the fused RMS_NORM and GLU measurements")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip every measurement besides the step (prefill, batched, fused ops, sweeps, single GEMV)")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak():
    """Dense bf16/f16 tensor peak in TFLOP/s: the burst figure (a GEMM timed
    alone) from MEASURED_PEAKS.json, else the fallback."""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        if "bf16_tflops" in d:
            return float(d["bf16_tflops"]), "measured bf16_tflops (burst, cuBLAS)"
    return 1590.0, "fallback (1.59 PFLOP/s burst)"


def fused_norm_measure(dev, layers: int = 12, reps: int = 20):
    """The two normed groups of the Llama-3.2-3B decode layer (attn_norm ->
    q|k|v, ffn_norm -> gate|up), `layers` distinct layers replayed as one
    CUDA graph, three ways: the plain GEMVs (activations already normed),
    RMS_NORM * gain fused into the GEMVs (wllm_mul_mat_rms_norm_batch), and
    the norm and gain as separate ops (torch) before the plain GEMVs. Returns
    the JSON object (µs per layer)."""
    import torch

    from webllm_b200 import jsep, synth

    L = {n: (n, t, M, K) for n, t, M, K in synth.LLAMA32_3B_LAYER}
    groups = [[L["attn_q"], L["attn_k"], L["attn_v"]], [L["ffn_gate"], L["ffn_up"]]]
    eps, K = 1e-5, 3072
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    keep, plan = [], []
    for li in range(layers):
        for mats in groups:
            x = torch.randn(1, K, device=dev, generator=gen)
            xn = torch.empty_like(x)
            g = torch.rand(K, device=dev, generator=gen) + 0.5
            out = torch.empty(1, sum(M for _, _, M, _ in mats), device=dev)
            ops_x, ops_n, off = [], [], 0
            for (_, t, M, _) in mats:
                w = synth.weights_torch(gen, t, M, K, dev)
                keep.append(w)
                ops_x.append(jsep.MulMatArgs(t, M, K, 1, w.data_ptr(), w.shape[1], x.data_ptr(), K, out.data_ptr() + 4 * off, M))
                ops_n.append(jsep.MulMatArgs(t, M, K, 1, w.data_ptr(), w.shape[1], xn.data_ptr(), K, out.data_ptr() + 4 * off, M))
                off += M
            keep += [x, xn, g, out]
            plan.append((x, xn, g, ops_x, ops_n))

    def plain(sp):
        for (_, _, _, ops_x, _) in plan:
            jsep.mul_mat_batch(ops_x, sp)

    def fused(sp):
        for (_, _, g, ops_x, _) in plan:
            if jsep.mul_mat_rms_norm_batch(ops_x, g.data_ptr(), eps, sp) != jsep.STATUS_OK:
                raise RuntimeError("fused RMS_NORM not taken")

    def separate(sp):
        for (x, xn, g, _, ops_n) in plan:
            torch.mul(x * torch.rsqrt(x.pow(2).mean(dim=1, keepdim=True) + eps), g, out=xn)
            jsep.mul_mat_batch(ops_n, sp)

    res = graph_times_us((("plain_gemv", plain), ("fused_norm_gemv", fused), ("separate_norm_then_gemv", separate)),
                         layers, reps)
    return {"workload": "llama-3.2-3b decode, attn_norm -> q|k|v and ffn_norm -> gate|up per layer, batch 1",
            "unit": "us per layer", **res,
            "note": "separate = torch RMS_NORM * gain kernels, then the plain GEMVs; fused = one launch per group"}


def graph_times_us(fns, layers: int, reps: int) -> dict:
    """Each fn(stream) recorded as one CUDA graph on torch's current stream,
    3 untimed replays, then `reps` replays between CUDA events: µs per layer."""
    import torch

    res = {}
    for name, fn in fns:
        fn(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn(torch.cuda.current_stream().cuda_stream)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(reps):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
        res[name] = round(ev0.elapsed_time(ev1) * 1e3 / (reps * layers), 2)
        del graph
    return res


def fused_glu_measure(dev, layers: int = 12, reps: int = 20):
    """The Llama-3.2-3B decode layer's down projection (Q6_K 3072 x 8192) fed
    by silu(gate) * up, `layers` distinct layers replayed as one CUDA graph,
    three ways: the plain GEMV (its input already computed), the GLU fused into
    the GEMV (wllm_mul_mat_glu_batch), and the GLU as separate ops (torch)
    before the plain GEMV. Returns the JSON object (µs per layer)."""
    import torch

    from webllm_b200 import jsep, synth

    _, t, M, K = {n: (n, t, M, K) for n, t, M, K in synth.LLAMA32_3B_LAYER}["ffn_down"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(6)
    plan = []
    for _ in range(layers):
        g = 2.0 * torch.randn(1, K, device=dev, generator=gen)
        u = torch.randn(1, K, device=dev, generator=gen)
        h = torch.empty_like(g)
        y = torch.empty(1, M, device=dev)
        w = synth.weights_torch(gen, t, M, K, dev)
        op_g = jsep.MulMatArgs(t, M, K, 1, w.data_ptr(), w.shape[1], g.data_ptr(), K, y.data_ptr(), M)
        op_h = jsep.MulMatArgs(t, M, K, 1, w.data_ptr(), w.shape[1], h.data_ptr(), K, y.data_ptr(), M)
        plan.append((g, u, h, y, w, op_g, op_h))

    def plain(sp):
        for p in plan:
            jsep.mul_mat_batch([p[6]], sp)

    def fused(sp):
        for (_, u, _, _, _, op_g, _) in plan:
            if jsep.mul_mat_glu_batch([op_g], u.data_ptr(), K, jsep.GLU_SWIGLU, sp) != jsep.STATUS_OK:
                raise RuntimeError("fused GLU not taken")

    def separate(sp):
        for (g, u, h, _, _, _, op_h) in plan:
            torch.mul(torch.nn.functional.silu(g), u, out=h)
            jsep.mul_mat_batch([op_h], sp)

    res = graph_times_us((("plain_gemv", plain), ("fused_glu_gemv", fused), ("separate_glu_then_gemv", separate)),
                         layers, reps)
    return {"workload": "llama-3.2-3b decode, silu(ffn_gate) * ffn_up -> ffn_down (Q6_K 3072 x 8192), batch 1",
            "unit": "us per layer", **res,
            "note": "separate = torch silu and mul kernels, then the plain GEMV; fused = one launch"}


def prefill_measure(dev, reps: int = 10, warmup: int = 3):
    """Llama-3-8B prefill GEMMs (N = 512 tokens, Q4_K): each MUL_MAT is the
    f16 pre-pass plus the tcgen05 GEMM. Two weight copies per shape (156 MB,
    more than L2) alternate between launches, which are captured in a CUDA
    graph (no host time between them). Returns the JSON object."""
    import torch

    from webllm_b200 import jsep, synth

    N = 512
    stream_ptr = jsep.library_stream()
    gen = torch.Generator(device=dev)

    def graph_us(call) -> float:
        """Mean device time of call(copy, stream) over `reps` launches that
        alternate the two weight copies, replayed from one CUDA graph."""
        for w in range(warmup):
            call(w & 1, stream_ptr)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            cs = torch.cuda.current_stream().cuda_stream
            for r in range(reps):
                call(r & 1, cs)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        e1.synchronize()
        del g
        return e0.elapsed_time(e1) * 1e3 / reps

    shapes, per = [], []
    for name, t, M, K in synth.LLAMA3_8B_PREFILL:
        gen.manual_seed(zlib.crc32(name.encode()))
        ws = [synth.weights_torch(gen, t, M, K, dev) for _ in range(2)]
        x = torch.randn(N, K, device=dev, generator=gen)
        y = torch.empty(N, M, device=dev)
        shapes.append((name, t, M, K, ws, x, y))
    torch.cuda.synchronize()

    for i, (name, t, M, K, ws, x, y) in enumerate(shapes):
        def run(copy: int, s, t=t, M=M, K=K, ws=ws, x=x, y=y):
            jsep.mul_mat_device(t, ws[copy].data_ptr(), ws[copy].shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K,
                                N, s)

        ms = graph_us(run) / 1e3
        per.append({"shape": f"{M}x{K}", "n": N, "us": round(ms * 1e3, 2),
                    "tflops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1)})
    total_flop = sum(2.0 * M * N * K for (_, _, M, K, _, _, _) in shapes)
    total_us = sum(p["us"] for p in per)
    tflops = total_flop / (total_us * 1e-6) / 1e12
    peak, src = measured_tensor_peak()
    # every weight type the prefill GEMM takes, on the ffn_down shape
    M, K = 4096, 14336
    x = torch.randn(N, K, device=dev, generator=gen)
    y = torch.empty(N, M, device=dev)
    per_type = []
    for tname, t in (("q4_k", jsep.GGML_TYPE_Q4_K), ("q5_k", jsep.GGML_TYPE_Q5_K), ("q6_k", jsep.GGML_TYPE_Q6_K),
                     ("q8_0", jsep.GGML_TYPE_Q8_0), ("q4_0", jsep.GGML_TYPE_Q4_0), ("iq4_xs", jsep.GGML_TYPE_IQ4_XS)):
        gen.manual_seed(zlib.crc32(tname.encode()))
        ws = [synth.weights_torch(gen, t, M, K, dev) for _ in range(2)]
        torch.cuda.synchronize()

        def one(copy: int, s, t=t, ws=ws):
            jsep.mul_mat_device(t, ws[copy].data_ptr(), ws[copy].shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N,
                                s)

        ms = graph_us(one) / 1e3
        per_type.append({"type": tname, "shape": f"{M}x{K}", "n": N, "us": round(ms * 1e3, 2),
                         "tflops": round(2.0 * M * N * K / (ms * 1e-3) / 1e12, 1)})
        del ws
    return {"workload": "llama-3-8b prefill GEMMs (Q4_K 4096x4096, 1024x4096, 14336x4096, 4096x14336; 512 tokens)",
            "value": round(tflops, 1), "unit": "TFLOP/s", "dtype": "f16 x f16 -> f32 (tcgen05)",
            "per_shape": per, "per_type": per_type,
            "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(tflops / peak, 4), "peak_source": src,
                         "note": "time includes the f32->f16 activation pre-pass of each MUL_MAT"}}


class DevArray:
    """A raw device pointer (library memory) as a torch tensor, zero copy."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def batched_measure(dev, reps: int = 10, warmup: int = 3):
    """Several sequences decoding together (N = 1 .. 64) on four weights:
    Gemma-2-2B ffn_up (Q8_0 9216x2304), Llama-3-8B ffn_gate (Q4_K 14336x4096)
    and ffn_down (Q6_K 4096x14336), and ffn_gate as IQ4_XS. N = 1, 2 run the
    streaming GEMV; the K-quant shapes at N >= 8 and the Q8_0 and IQ4_XS shapes
    above 16 vectors the tcgen05 small-batch GEMM, those two at N = 8, 16 the
    integer tensor-core (mma.sync) batched GEMM. Distinct weight copies (over 2x the
    L2) rotate between launches so every launch streams its weights from HBM.
    Returns the JSON object: the Q8_0 shape at the top level, the K-quant
    shapes under "kquant"."""
    import torch

    from webllm_b200 import jsep, synth

    gname, gt, gM, gK = synth.GEMMA2_2B_SHAPES[0]
    shapes = [(f"gemma-2-2b {gname}", gt, gM, gK, 24),
              ("llama-3-8b ffn_gate", jsep.GGML_TYPE_Q4_K, 14336, 4096, 8),
              ("llama-3-8b ffn_down", jsep.GGML_TYPE_Q6_K, 4096, 14336, 6),
              ("llama-3-8b ffn_gate", jsep.GGML_TYPE_IQ4_XS, 14336, 4096, 8)]
    stream_ptr = jsep.library_stream()
    hbm, _ = measured_peaks()
    out = []
    for name, t, M, K, copies in shapes:
        gen = torch.Generator(device=dev)
        gen.manual_seed(zlib.crc32(name.encode()))
        ws = [synth.weights_torch(gen, t, M, K, dev) for _ in range(copies)]
        per = []
        for N in (1, 8, 16, 32, 64):
            x = torch.randn(N, K, device=dev, generator=gen)
            y = torch.empty(N, M, device=dev)
            torch.cuda.synchronize()

            def run(i, s):
                w = ws[i % copies]
                jsep.mul_mat_device(t, w.data_ptr(), w.shape[1], x.data_ptr(), K, y.data_ptr(), M, M, K, N, s)

            # one launch per weight copy, captured as one CUDA graph (no host
            # time between launches), replayed `reps` times
            for i in range(warmup):
                run(i, stream_ptr)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                cs = torch.cuda.current_stream().cuda_stream
                for i in range(copies):
                    run(i, cs)
            graph.replay()
            torch.cuda.synchronize()
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            for _ in range(reps):
                graph.replay()
            ev1.record()
            ev1.synchronize()
            del graph
            us = ev0.elapsed_time(ev1) * 1e3 / (reps * copies)
            nbytes = synth.algorithmic_bytes(t, M, K, N)
            per.append({"n": N, "us": round(us, 2), "gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
                        "hbm_frac": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4),
                        "tflops": round(2.0 * M * K * N / (us * 1e-6) / 1e12, 2)})
        del ws
        tname = {jsep.GGML_TYPE_Q8_0: "Q8_0", jsep.GGML_TYPE_Q4_K: "Q4_K", jsep.GGML_TYPE_Q6_K: "Q6_K",
                 jsep.GGML_TYPE_IQ4_XS: "IQ4_XS"}[t]
        out.append({"workload": f"{name} {tname} {M}x{K}, N sequences decoding together", "unit": "GB/s",
                    "per_n": per})
    res = dict(out[0])
    res["kquant"] = out[1:]
    res["note"] = ("N <= 2: streaming GEMV; Q4_K/Q6_K N >= 5 (N >= 16 at 4096x4096 and below), Q8_0/IQ4_XS N > 16: "
                   "tcgen05 small-batch GEMM; Q8_0/IQ4_XS N = 3..16: integer tensor-core batched GEMM (mma.sync); "
                   "activation pre-passes included; launches timed inside a CUDA graph")
    return res


def layer_table(model: str | None = None):
    """The 7 GEMVs of one decode layer: [(name, qtype, M, K)]."""
    from webllm_b200 import synth

    return synth.QWEN3_8B_LAYER if (model or _MODEL) == "qwen3-8b" else synth.LLAMA32_3B_LAYER


def layer_groups(model: str | None = None):
    """[(input K, [(name, qtype, M, K), ...]), ...] for one layer: the launch
    groups that share an input (q|k|v, o, gate|up, down)."""
    L = {n: (n, t, M, K) for n, t, M, K in layer_table(model)}
    return [
        (L["attn_q"][3], [L["attn_q"], L["attn_k"], L["attn_v"]]),
        (L["attn_output"][3], [L["attn_output"]]),
        (L["ffn_gate"][3], [L["ffn_gate"], L["ffn_up"]]),
        (L["ffn_down"][3], [L["ffn_down"]]),
    ]


def step_groups(layers: int, model: str | None = None):
    """Every launch of one step in order: [(layer, group, input K, mats)];
    the output projection (when the model's step has it) is layer `layers`."""
    from webllm_b200 import synth

    model = model or _MODEL
    out = [(li, gi, kin, mats) for li in range(layers) for gi, (kin, mats) in enumerate(layer_groups(model))]
    if WORKLOADS[model][2]:
        out.append((layers, 0, synth.QWEN3_8B_OUTPUT[3], [synth.QWEN3_8B_OUTPUT]))
    return out


def step_bytes(layers: int, model: str | None = None) -> int:
    from webllm_b200 import synth

    return sum(synth.algorithmic_bytes(t, M, K, 1) for _, _, _, mats in step_groups(layers, model)
               for _, t, M, K in mats)


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id  # GPU UUID (robust to CUDA_VISIBLE_DEVICES remapping) or index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="wllm_clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ------------------------------------------------------------------ CPU arms


CPU_DISTINCT_LAYERS = 8  # 0.5-0.9 GB of weights: larger than any host's last-level cache


class CpuWork:
    """The oracle's f32 dequant-then-dot (the reference algorithm's CPU path)
    over the step's GEMVs: 8 distinct synthetic layers cycled so the weights
    stream from DRAM, and the output projection once per `layers` layers so
    the byte mix is the step's."""

    def __init__(self, layers: int):
        from oracle import oracle as O
        from webllm_b200 import synth

        rng = np.random.default_rng(1234)
        self.O = O
        self.layers_per_step = layers
        self.distinct = [[(t, synth.weights(rng, t, M, K), synth.activations(rng, 1, K),
                           synth.algorithmic_bytes(t, M, K, 1)) for _, t, M, K in layer_table()]
                         for _ in range(CPU_DISTINCT_LAYERS)]
        self.output = None
        if WORKLOADS[_MODEL][2]:
            _, t, M, K = synth.QWEN3_8B_OUTPUT
            self.output = (t, synth.weights(rng, t, M, K), synth.activations(rng, 1, K),
                           synth.algorithmic_bytes(t, M, K, 1))
        self.cores = O.max_threads()
        self.done_layers = 0
        self.weight_mb = (sum(m[1].nbytes for L in self.distinct for m in L)
                          + (self.output[1].nbytes if self.output else 0)) / 1e6

    def layer(self) -> int:
        """One layer's 7 GEMVs (and the output projection after every
        `layers` layers); returns the algorithmic bytes done."""
        b = 0
        for t, w, x, nb in self.distinct[self.done_layers % len(self.distinct)]:
            self.O.mul_mat_f32(t, w, x, threads=self.cores)
            b += nb
        self.done_layers += 1
        if self.output is not None and self.done_layers % self.layers_per_step == 0:
            t, w, x, nb = self.output
            self.O.mul_mat_f32(t, w, x, threads=self.cores)
            b += nb
        return b

    def describe(self) -> str:
        out = " + the 151936x4096 Q6_K output projection once per 36 layers" if self.output else ""
        return (f"whole layers of the step (7 GEMVs each){out}, cycling over {len(self.distinct)} distinct "
                f"layers ({self.weight_mb:.0f} MB of weights) so they stream from DRAM; f32 dequant-then-dot "
                f"oracle on {self.cores} threads (the reference's llama.cpp CPU kernels are not vendored in the "
                f"reference repository)")


def cpu_sample(budget_s: float, layers: int):
    """Time the CPU path on whole layers for about `budget_s` seconds after
    one untimed pass over the distinct layers (page-in, thread pool).
    Returns (GB/s, cores, sample description)."""
    work = CpuWork(layers)
    for _ in range(CPU_DISTINCT_LAYERS):
        work.layer()
    done, t0 = 0, time.perf_counter()
    while True:
        done += work.layer()
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    n = work.done_layers - CPU_DISTINCT_LAYERS
    return done / el / 1e9, work.cores, f"{n} layers, {done / 1e9:.1f} GB in {el:.1f} s: " + work.describe()


def run_reference(args, rank: int):
    """The reference arm: the CPU path on this box's host cores, rank 0 only.
    Every step is the same number of whole layers, chosen from an untimed
    pass so that the K timed steps take about --cpu-seconds together (the
    same budget and sample as the GPU arm's cpu_baseline)."""
    if rank != 0:
        return
    work = CpuWork(args.layers)
    t0 = time.perf_counter()
    for _ in range(CPU_DISTINCT_LAYERS):
        work.layer()
    per_layer_s = (time.perf_counter() - t0) / CPU_DISTINCT_LAYERS
    layers_per_step = max(1, math.ceil(args.cpu_seconds / max(1, args.steps) / per_layer_s))
    for _ in range(args.warmup):
        for _ in range(layers_per_step):
            work.layer()
    done, t0 = 0, time.perf_counter()
    for _ in range(args.steps):
        for _ in range(layers_per_step):
            done += work.layer()
    el = time.perf_counter() - t0
    gbs = done / el / 1e9
    sample = f"each step: {layers_per_step} " + work.describe()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOADS[_MODEL][0], "batch": 1, "layers_per_step": layers_per_step,
                   "timed_s": round(el, 2)},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": work.cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm


def weight_seed(li: int, gi: int, mi: int, rank: int) -> int:
    """Seed of rank `rank`'s row shard of launch (li, gi)'s op mi: any rank
    can regenerate any other rank's weights (the parity check does)."""
    return 1_000_000 + 10_000 * li + 100 * gi + 10 * mi + rank


def check_parity(dev, launches, world: int, rank: int, layers: int, stream_ptr: int) -> dict:
    """Both error metrics of the path for the outputs of layer 0, the last
    layer and the output projection, every rank's rows (other ranks' weight
    shards are regenerated from their seeds), against a float64 matmul of the
    library-dequantized weights (bit-exact with the reference's
    dequantization). Row chunks keep the float64 copy small."""
    import torch

    from webllm_b200 import jsep, synth
    from webllm_b200.tp import row_shard

    def rel(y, r):
        mx = r.abs().max()
        a = ((y - r).abs().max() / mx).item()
        sel = r.abs() >= 1e-2 * mx
        b = ((y[sel] - r[sel]).abs() / r[sel].abs()).max().item()
        return a, b

    gen = torch.Generator(device=dev)
    worst_a = worst_b = 0.0
    n_ops = n_rows = 0
    for L in launches:
        if L["li"] not in (0, layers - 1, layers):
            continue
        x = L["x"].double()
        for mi, (name, t, M, K) in enumerate(L["mats"]):
            got_parts, ref_parts = [], []
            for r in range(world):
                sh = row_shard(M, world, r)
                if sh.count == 0:
                    continue
                if r == rank:
                    w = L["w"][mi]
                else:
                    gen.manual_seed(weight_seed(L["li"], L["gi"], mi, r))
                    w = synth.weights_torch(gen, t, sh.count, K, dev)
                col = r * L["gtot"] + L["offs"][mi]
                got_parts.append(L["out"][0, col:col + sh.count].double())
                rb = synth.row_bytes(t, K)
                for r0 in range(0, sh.count, 16384):
                    rows = min(16384, sh.count - r0)
                    # the dequantization runs on the library stream: torch's
                    # stream must be done with the memory it is handed
                    torch.cuda.synchronize()
                    wf = torch.empty(rows, K, device=dev)
                    jsep.dequantize_device(t, w.data_ptr() + r0 * rb, wf.data_ptr(), rows * K, stream_ptr)
                    torch.cuda.ExternalStream(stream_ptr).synchronize()
                    ref_parts.append((wf.double() @ x.t()).t()[0])
                    torch.cuda.synchronize()
                    del wf
            a, b = rel(torch.cat(got_parts), torch.cat(ref_parts))
            worst_a, worst_b = max(worst_a, a), max(worst_b, b)
            n_ops += 1
            n_rows += M
    return {"max_rel": float(f"{worst_a:.3e}"), "max_rel_elem": float(f"{worst_b:.3e}"), "tol": 1e-3,
            "ok": bool(worst_a <= 1e-3 and worst_b <= 1e-3), "ops_checked": n_ops, "rows_checked": n_rows,
            "reference": "float64 matmul of the library-dequantized weights; layer 0, the last layer and the "
                         "output projection, all ranks' rows; max-normalized and per-element (|r| >= 1e-2 max|r|)"}


def run_b200(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    from webllm_b200 import jsep, synth
    from webllm_b200.build_ext import build
    from webllm_b200.tp import row_shard

    build()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    jsep.install_jsep_callbacks(local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    layers = args.layers
    plan = step_groups(layers)
    gen = torch.Generator(device=dev)
    # Row-sharded (world > 1): each launch's rows from every rank land in one
    # gathered buffer per rank, [world][launch rows]. The GEMV writes this
    # rank's rows into every rank's buffer over NVLink (peer memory opened
    # with CUDA IPC); one bounded wait at the end of the step completes them.
    gtot = [sum(row_shard(M, world, rank).padded for (_, _, M, _) in mats) for *_, mats in plan]
    gather_floats = sum(world * g for g in gtot)
    tp = gview = None
    if world > 1:
        g_ptr, g_handle = jsep.ipc_alloc(4 * gather_floats)
        s_ptr, s_handle = jsep.ipc_alloc(4 * jsep.MAX_RANKS)
        st_ptr, _ = jsep.ipc_alloc(16)
        handles = [None] * world
        dist.all_gather_object(handles, (g_handle, s_handle))
        gbase = [g_ptr if r == rank else jsep.ipc_open(handles[r][0]) for r in range(world)]
        sigs = [s_ptr if r == rank else jsep.ipc_open(handles[r][1]) for r in range(world)]
        tp = jsep.tp_group(world, rank, sigs, st_ptr)
        gview = torch.as_tensor(DevArray(g_ptr, gather_floats), device=dev)
    # ---- resident weights (row shard of every matrix), inputs, outputs.
    # Every launch's activations are a slice of one buffer, and at one GPU
    # every launch's outputs too, so the end-to-end step moves each with one copy.
    x_all = torch.empty(sum(kin for _, _, kin, _ in plan), device=dev)
    y_all = torch.zeros(sum(gtot), device=dev) if world == 1 else None
    x_pos = y_pos = g_pos = 0
    launches = []
    for idx, (li, gi, kin, mats) in enumerate(plan):
        x = x_all[x_pos:x_pos + kin].view(1, kin)
        x_pos += kin
        x.copy_(torch.randn(1, kin, device=dev, generator=gen.manual_seed(10_000 * li + 10 * gi)))
        pads = [row_shard(M, world, rank).padded for (_, _, M, _) in mats]
        offs = [sum(pads[:i]) for i in range(len(pads))]
        if world > 1:
            out = gview[g_pos:g_pos + world * gtot[idx]].view(1, -1)  # the launch's gathered rows
        else:
            out = y_all[y_pos:y_pos + gtot[idx]].view(1, -1)
            y_pos += gtot[idx]
        gops, gouts, ws = [], [], []
        for mi, (name, t, M, K) in enumerate(mats):
            # this rank's contiguous row shard; every rank reserves `padded` rows
            Mr = row_shard(M, world, rank).count
            gen.manual_seed(weight_seed(li, gi, mi, rank))
            w = synth.weights_torch(gen, t, Mr, K, dev)
            ws.append(w)
            col = rank * gtot[idx] + offs[mi]  # float offset of this rank's rows in the launch's rows
            gops.append(jsep.MulMatArgs(t, Mr, K, 1, w.data_ptr(), synth.row_bytes(t, K), x.data_ptr(), K,
                                        out.data_ptr() + 4 * col, Mr))
            if world > 1:
                gouts.append([gbase[r] + 4 * (g_pos + col) for r in range(world)])
        launches.append({"li": li, "gi": gi, "mats": mats, "x": x, "out": out, "ops": gops, "outs": gouts,
                         "w": ws, "gtot": gtot[idx], "offs": offs})
        g_pos += world * gtot[idx]
    torch.cuda.synchronize()
    launches_per_step = len(launches) + (1 if world > 1 else 0)

    def step(stream_ptr: int):
        for L in launches:
            if world > 1:
                jsep.mul_mat_batch_tp(L["ops"], L["outs"], tp, stream_ptr)
            else:
                jsep.mul_mat_batch(L["ops"], stream_ptr)
        if world > 1:
            jsep.tp_wait(tp, stream_ptr)

    def gemv_only(stream_ptr: int):
        # each rank's row-shard GEMVs with no gather and no cross-rank wait
        for L in launches:
            jsep.mul_mat_batch(L["ops"], stream_ptr)

    def capture(fn):
        s = torch.cuda.current_stream()
        for _ in range(max(1, args.warmup)):
            fn(s.cuda_stream)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn(torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        for _ in range(args.warmup):
            g.replay()
        torch.cuda.synchronize()
        return g

    graph = capture(step)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def time_graph(g) -> float:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / args.steps

    # ---- timed region: device-resident inputs
    uuid = getattr(torch.cuda.get_device_properties(dev), "uuid", None)
    gpu_id = f"GPU-{uuid}" if uuid is not None and not str(uuid).startswith("GPU-") else (str(uuid) if uuid else str(local_rank))
    with ClockSampler(gpu_id) as clocks:
        dev_ms = time_graph(graph)
    clk = clocks.summary()

    # ---- parity of the step's outputs (rank 0 checks every rank's rows)
    parity = None
    if rank == 0:
        parity = check_parity(dev, launches, world, rank, layers, jsep.library_stream())
    barrier()

    # ---- the same step without the exchange (row-shard GEMVs alone)
    tp_split = None
    total_bytes = step_bytes(layers)
    if world > 1:
        g2 = capture(gemv_only)
        only_ms = time_graph(g2)
        del g2
        tp_split = {"gemv_only": {"ms_per_step": round(only_ms, 4),
                                  "aggregate_gbs": round(total_bytes / (only_ms * 1e-3) / 1e9, 2),
                                  "per_gpu_gbs": round(total_bytes / world / (only_ms * 1e-3) / 1e9, 2)},
                    "with_gather": {"ms_per_step": round(dev_ms, 4),
                                    "aggregate_gbs": round(total_bytes / (dev_ms * 1e-3) / 1e9, 2),
                                    "per_gpu_gbs": round(total_bytes / world / (dev_ms * 1e-3) / 1e9, 2)},
                    "note": "gemv_only: each rank's row-shard GEMVs, no peer writes, no cross-rank wait "
                            "(outputs incomplete); with_gather: the fused NVLink gather and its per-launch wait"}

    # ---- e2e: pinned host activations in, outputs out, every step: one copy
    # of all the step's activations, one of all its outputs (at N > 1 the
    # gathered rows of all ranks); the host activations are the same on every rank
    x_host = torch.randn(x_all.numel(), generator=torch.Generator().manual_seed(7)).pin_memory()
    outs = y_all if world == 1 else gview
    y_host = torch.empty(outs.numel()).pin_memory()
    h2d = x_host.numel() * 4
    d2h = y_host.numel() * 4 if rank == 0 else 0

    def e2e_step():
        x_all.copy_(x_host, non_blocking=True)
        graph.replay()
        if rank == 0:
            y_host.copy_(outs, non_blocking=True)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    ev0.record()
    for _ in range(args.steps):
        e2e_step()
    ev1.record()
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    e2e_ms = max_over_ranks(max(ev0.elapsed_time(ev1) / args.steps, wall_ms))
    barrier()

    # ---- extras at one GPU: the C-ABI e2e, prefill, batched, fused ops, sweeps
    extras = {}
    if world == 1 and not args.no_extras:
        del launches, graph  # free the step's weights
        torch.cuda.empty_cache()
        extras["e2e_c_abi"] = jsep_path_e2e(args, layers)
        extras["single_gemv"] = single_gemv_measure(dev)
        extras["llama32_sweep"] = sweep_measure(dev, "llama-3.2-3b", args)
        if not args.no_prefill:
            extras["prefill"] = prefill_measure(dev)
        if not args.no_fused_norm:
            extras["fused_norm"] = fused_norm_measure(dev)
            extras["fused_glu"] = fused_glu_measure(dev)
        if not args.no_batched:
            extras["batched"] = batched_measure(dev)

    gbs = total_bytes / (dev_ms * 1e-3) / 1e9
    peak, peak_src = measured_peaks()
    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            v, cores, sample = cpu_sample(args.cpu_seconds, layers)
            cpu = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}
        traffic = None
        if world == 1 and _MODEL == "llama-3.2-3b":
            traffic = NCU_DRAM_BYTES_PER_LAYER_LLAMA32 * layers
        elif world == 1 and _MODEL == "qwen3-8b":
            traffic = NCU_DRAM_BYTES_PER_LAYER_QWEN3 * layers + (NCU_DRAM_BYTES_OUTPUT_QWEN3 if WORKLOADS[_MODEL][2] else 0)
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dev_ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOADS[_MODEL][0], "layers": layers, "batch": 1, "bytes_per_step": total_bytes,
                       "l2": f"inputs larger than L2 ({total_bytes / 1e9:.2f} GB of distinct weights per step), no flush",
                       "parallelism": f"tp{world} row-sharded" + (" + NVLink peer-write gather fused into the GEMV"
                                                                      if world > 1 else ""),
                       "launch": f"{len(plan)} grouped launches per step (4 per layer"
                                 + (" + the output projection" if WORKLOADS[_MODEL][2] else "")
                                 + "), one CUDA graph per step"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "traffic": traffic,
                         "traffic_note": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the step's GEMV launches",
                         "peak_source": f"{peak_src} hbm_gbs (burst copy)",
                         "note": "achieved = step algorithmic bytes / step device time over all launches of the GEMV kernel"
                                 + (" (includes the fused gather and its per-launch waits)" if world > 1 else "")},
            "parity": parity,
            "cpu_baseline": cpu,
            "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                    "path": "pinned host activations -> HBM, graph replay, outputs -> pinned host"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        if tp_split is not None:
            line["tp_split"] = tp_split
        line.update(extras)
    if world > 1:
        del graph
        torch.cuda.synchronize()
        dist.barrier()  # no rank still writes into another's memory
        for r in range(world):
            if r != rank:
                jsep.ipc_close(gbase[r])
                jsep.ipc_close(sigs[r])
        dist.barrier()  # every mapping closed before the owners free
        for ptr in (g_ptr, s_ptr, st_ptr):
            jsep.ipc_free(ptr)
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


def sweep_measure(dev, model: str, args, reps: int = 20) -> dict:
    """A whole decode sweep of `model` at one GPU (the step's grouped launches,
    one CUDA graph): GB/s and the HBM fraction."""
    import torch

    from webllm_b200 import jsep, synth

    layers = WORKLOADS[model][1]
    plan = step_groups(layers, model)
    gen = torch.Generator(device=dev)
    keep, calls = [], []
    for li, gi, kin, mats in plan:
        x = torch.randn(1, kin, device=dev, generator=gen.manual_seed(10_000 * li + 10 * gi))
        out = torch.empty(1, sum(M for _, _, M, _ in mats), device=dev)
        ops, off = [], 0
        for mi, (name, t, M, K) in enumerate(mats):
            gen.manual_seed(weight_seed(li, gi, mi, 0))
            w = synth.weights_torch(gen, t, M, K, dev)
            keep.append(w)
            ops.append(jsep.MulMatArgs(t, M, K, 1, w.data_ptr(), synth.row_bytes(t, K), x.data_ptr(), K,
                                       out.data_ptr() + 4 * off, M))
            off += M
        keep += [x, out]
        calls.append(ops)

    def fn(sp):
        for ops in calls:
            jsep.mul_mat_batch(ops, sp)

    us = graph_times_us((("step", fn),), 1, reps)["step"]
    nbytes = step_bytes(layers, model)
    peak, _ = measured_peaks()
    gbs = nbytes / (us * 1e-6) / 1e9
    del keep
    return {"workload": WORKLOADS[model][0], "us_per_step": us, "gbs": round(gbs, 2),
            "hbm_frac": round(gbs / peak, 4), "launches_per_step": len(plan)}


def single_gemv_measure(dev, reps: int = 20) -> dict:
    """One Q4_K 4096 x 4096 decode GEMV (9.44 MB of weights, batch 1): 54
    distinct weight copies (510 MB, over 4x the 126 MB L2) rotated in one CUDA
    graph, so every launch streams its weights from HBM."""
    import torch

    from webllm_b200 import jsep, synth

    t, M, K, copies = jsep.GGML_TYPE_Q4_K, 4096, 4096, 54
    gen = torch.Generator(device=dev)
    gen.manual_seed(4096)
    ws = [synth.weights_torch(gen, t, M, K, dev) for _ in range(copies)]
    xs = [torch.randn(1, K, device=dev, generator=gen) for _ in range(copies)]
    ys = [torch.empty(1, M, device=dev) for _ in range(copies)]
    ops = [[jsep.MulMatArgs(t, M, K, 1, w.data_ptr(), synth.row_bytes(t, K), x.data_ptr(), K, y.data_ptr(), M)]
           for w, x, y in zip(ws, xs, ys)]

    def fn(sp):
        for o in ops:
            jsep.mul_mat_batch(o, sp)

    us = graph_times_us((("gemv", fn),), copies, reps)["gemv"]
    nbytes = synth.algorithmic_bytes(t, M, K, 1)
    peak, _ = measured_peaks()
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"workload": "single Q4_K 4096x4096 decode GEMV, batch 1 (54 distinct weight copies rotated, 510 MB)",
            "us": us, "gbs": round(gbs, 2), "hbm_frac": round(gbs / peak, 4), "bytes": nbytes}


def jsep_path_e2e(args, layers: int):
    """Same step through the reference-facing seam: descriptors + handles,
    pageable host activations written with wllm_write, one recorded graph of
    the step's wllm_run_ops calls, outputs read back with wllm_read."""
    from webllm_b200 import jsep, synth

    rt = jsep.install_jsep_callbacks(jsep._runtime.device if jsep._runtime else 0)
    dm = rt.data_manager
    plan = step_groups(layers)
    rng = np.random.default_rng(99)
    # one buffer per weight; one buffer for all inputs, one for all outputs
    x_off, y_off = 0, 0
    layout = []
    for li, gi, kin, mats in plan:
        ys = []
        for (name, t, M, K) in mats:
            ys.append(y_off)
            y_off += 4 * M
        layout.append((x_off, kin, mats, ys))
        x_off += 4 * kin
    hx, hy = dm.alloc(x_off), dm.alloc(y_off)
    wh, descs = [], []
    for xo, kin, mats, ys in layout:
        gdescs = []
        for (name, t, M, K), yo in zip(mats, ys):
            w = synth.weights(rng, t, M, K)
            h = dm.alloc(w.nbytes)
            dm.write(h, 0, w)
            wh.append(h)
            gdescs.append(jsep.JsepOpDescriptor(
                29, 2, jsep.meta_for(hy, 0, (M, 1, 1, 1), offset=yo),
                [jsep.meta_for(h, t, (K, M, 1, 1)), jsep.meta_for(hx, 0, (K, 1, 1, 1), offset=xo)]))
        descs.append(gdescs)
    x_host = rng.standard_normal(x_off // 4, dtype=np.float32)
    y_host = np.empty(y_off // 4, dtype=np.float32)

    def record():
        for g in descs:
            st = rt.run_ops(g)
            if st != jsep.STATUS_OK:
                raise RuntimeError(f"run_ops: {st} {jsep.last_error()}")

    dm.write(hx, 0, x_host)
    record()  # eager once (sizes any scratch), then record the graph
    rt.jsep_sync()
    jsep.Graph.begin()
    record()
    g = jsep.Graph.end()

    def step():
        dm.write(hx, 0, x_host)
        g.launch()
        y_host[:] = dm.read(hy, 0, y_off).view(np.float32)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    ms = (time.perf_counter() - t0) * 1e3 / args.steps
    g.destroy()
    for h in wh + [hx, hy]:
        dm.free(h)
    return {"value": round(step_bytes(layers) / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": x_off, "d2h_bytes_per_step": y_off,
            "path": f"wllm_write(pageable host) -> wllm_graph_launch({len(plan)} recorded "
                    "wllm_run_ops) -> wllm_read"}


def main():
    global _MODEL
    args = parse_args()
    _MODEL = args.model
    if args.layers is None:
        args.layers = WORKLOADS[_MODEL][1]
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world != args.gpus and rank == 0:
        print(f"[bench] note: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
