"""ctypes wrapper around the C oracle (TEST INFRASTRUCTURE ONLY).

The oracle restates the reference's quantized MUL_MAT on the CPU (see
quant_ref.h for the reference files it follows). Only tests/, the smoke
check and bench.py's CPU-baseline leg use this module; the product library
never imports it.

Layout conventions follow ggml MUL_MAT (src/inference/jsep/ops/matmul.ts:10-17):
weights are M rows of `row_bytes` bytes; activations are N vectors of K f32;
the result is returned as an (N, M) array, i.e. dst[m + M*n].
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_quant.so")
_lock = threading.Lock()
_lib = None

TYPE_F32 = 0
TYPE_Q4_0 = 2
TYPE_Q8_0 = 8
TYPE_Q4_K = 12
TYPE_Q5_K = 13
TYPE_Q6_K = 14
TYPE_IQ4_XS = 23


def build(force: bool = False) -> str:
    """Compile liboracle_quant.so with the committed Makefile."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "quant_ref.c"))
    ):
        subprocess.run(["make", "-s", "-B" if force else "-s", "-C", _HERE, "liboracle_quant.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            build()
            L = ctypes.CDLL(_LIB_PATH)
            i32, i64, vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p
            L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
            L.oracle_f16_to_f32.restype = ctypes.c_float
            L.oracle_block_elems.argtypes = [i32]
            L.oracle_block_elems.restype = i32
            L.oracle_block_bytes.argtypes = [i32]
            L.oracle_block_bytes.restype = i32
            L.oracle_dequantize_row.argtypes = [i32, vp, vp, i64]
            L.oracle_dequantize_row.restype = i32
            L.oracle_mul_mat_f64.argtypes = [i32, vp, i64, vp, i64, vp, i32, i32, i32]
            L.oracle_mul_mat_f64.restype = i32
            L.oracle_mul_mat_f32.argtypes = [i32, vp, i64, vp, i64, vp, i64, i32, i32, i32, i32]
            L.oracle_mul_mat_f32.restype = i32
            L.oracle_max_threads.argtypes = []
            L.oracle_max_threads.restype = i32
            _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def block_elems(qtype: int) -> int:
    return int(lib().oracle_block_elems(qtype))


def block_bytes(qtype: int) -> int:
    return int(lib().oracle_block_bytes(qtype))


def f16_to_f32(bits: int) -> float:
    return float(lib().oracle_f16_to_f32(bits))


def dequantize(qtype: int, data: np.ndarray, k: int) -> np.ndarray:
    """Dequantize k elements stored as raw block bytes (uint8)."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(k, dtype=np.float32)
    rc = lib().oracle_dequantize_row(qtype, _ptr(data), _ptr(out), k)
    if rc != 0:
        raise ValueError(f"oracle_dequantize_row failed ({rc})")
    return out


def dequantize_matrix(qtype: int, w: np.ndarray, K: int) -> np.ndarray:
    """(M, row_bytes) uint8 -> (M, K) float32."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    M = w.shape[0]
    out = np.empty((M, K), dtype=np.float32)
    for m in range(M):
        rc = lib().oracle_dequantize_row(qtype, _ptr(w[m]), _ptr(out[m]), K)
        if rc != 0:
            raise ValueError(f"oracle_dequantize_row failed ({rc})")
    return out


def mul_mat_f64(qtype: int, w: np.ndarray, x: np.ndarray) -> np.ndarray:
    """w: (M, row_bytes) uint8; x: (N, K) float32 -> (N, M) float64."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, row_bytes = w.shape
    N, K = x.shape
    out = np.empty((N, M), dtype=np.float64)
    rc = lib().oracle_mul_mat_f64(qtype, _ptr(w), row_bytes, _ptr(x), K, _ptr(out), M, K, N)
    if rc != 0:
        raise ValueError(f"oracle_mul_mat_f64 failed ({rc})")
    return out


def mul_mat_f32(qtype: int, w: np.ndarray, x: np.ndarray, threads: int | None = None) -> np.ndarray:
    """f32 dequant-then-dot (the timed CPU baseline). -> (N, M) float32."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, row_bytes = w.shape
    N, K = x.shape
    out = np.empty((N, M), dtype=np.float32)
    t = max_threads() if threads is None else int(threads)
    rc = lib().oracle_mul_mat_f32(qtype, _ptr(w), row_bytes, _ptr(x), K, _ptr(out), M, M, K, N, t)
    if rc != 0:
        raise ValueError(f"oracle_mul_mat_f32 failed ({rc})")
    return out


def max_threads() -> int:
    """Host cores this process may run on (the CPU affinity set). Not the
    OpenMP default, which launchers such as torchrun cap with
    OMP_NUM_THREADS=1; mul_mat_f32 passes its thread count explicitly."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return int(lib().oracle_max_threads())


def rel_error(y: np.ndarray, r: np.ndarray) -> float:
    """max_i |y_i - r_i| / max_i |r_i| (r accumulated in f64)."""
    r = np.asarray(r, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    denom = float(np.max(np.abs(r))) if r.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(y - r))) if r.size else 0.0
    return float(np.max(np.abs(y - r)) / denom)


def rel_error_elem(y: np.ndarray, r: np.ndarray, floor: float = 1e-2) -> float:
    """Per-element relative error max_i |y_i - r_i| / |r_i| over the elements
    with |r_i| >= floor * max|r| (r accumulated in f64): the second of the
    path's two GEMV error metrics, which a max-normalized figure can hide
    when a few large outputs dominate."""
    r = np.asarray(r, dtype=np.float64)
    y = np.asarray(y, dtype=np.float64)
    if not r.size:
        return 0.0
    mx = float(np.max(np.abs(r)))
    if mx == 0.0:
        return float(np.max(np.abs(y - r)))
    sel = np.abs(r) >= floor * mx
    return float(np.max(np.abs(y[sel] - r[sel]) / np.abs(r[sel])))


# ---- the activation-side ops fused into the GEMV (float64 restatements) ----


def rms_norm_f64(x: np.ndarray, eps: float, gain: np.ndarray | None = None) -> np.ndarray:
    """RMS_NORM per vector (last axis), then the gain MUL when given:
    x / sqrt(mean(x^2) + eps) * gain, in float64.

    Follows src/inference/jsep/ops/rms-norm.ts:14-15,61-67 (the op) and the
    CPU reference of tests/jsep-rms-norm-golden.test.ts:64-86 (cpuRmsNorm:
    sum of squares over the row, 1 / sqrt(sum / cols + eps), times x); the
    gain is the separate MUL of src/inference/model-inference.ts:2281,2478-2481.
    """
    xd = np.asarray(x, dtype=np.float64)
    y = xd * (1.0 / np.sqrt((xd * xd).mean(axis=-1, keepdims=True) + eps))
    if gain is not None:
        y = y * np.asarray(gain, dtype=np.float64)
    return y


def swiglu_f64(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """silu(gate) * up in float64: gate / (1 + e^-gate) * up, the SwiGLU the
    reference applies between the FFN's gate/up and down projections
    (src/inference/model-inference.ts:2484-2489, op_swiglu_split of
    src/wasm/webgpu-bridge.cpp:272-275; ggml's scalar CPU form)."""
    g = np.asarray(gate, dtype=np.float64)
    with np.errstate(over="ignore"):
        return g / (1.0 + np.exp(-g)) * np.asarray(up, dtype=np.float64)


def gelu_ggml(gate: np.ndarray) -> np.ndarray:
    """GELU as ggml's CPU backend computes it with its f16 table: the input
    rounded to f16, the tanh form 0.5 f (1 + tanh(sqrt(2/pi) f (1 + 0.044715
    f^2))), the result rounded to f16; 0 at gate <= -10 and gate itself at
    gate >= 10. Returned as float64 (src/inference/model-inference.ts:
    2486-2487, Gemma's GELU(gate) before the MUL by up)."""
    g = np.asarray(gate, dtype=np.float32)
    f = g.astype(np.float16).astype(np.float64)
    t = (0.5 * f * (1.0 + np.tanh(0.7978845608028654 * f * (1.0 + 0.044715 * f * f)))).astype(np.float16)
    return np.where(g <= -10.0, 0.0, np.where(g >= 10.0, g.astype(np.float64), t.astype(np.float64)))


def geglu_f64(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """gelu_ggml(gate) * up in float64 (the Gemma FFN's MUL)."""
    return gelu_ggml(gate) * np.asarray(up, dtype=np.float64)
