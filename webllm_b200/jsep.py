"""Host-side mirror of webllm's JSEP op-plugin interface over libwllm_mulmat.

The reference's host is TypeScript: `installJsepCallbacks(module, device)`
(src/inference/jsep/index.ts:129-395) installs seven callbacks, buffers are
handled by `GpuDataManager` (src/inference/jsep/gpu-data-manager.ts), and
MUL_MAT nodes arrive as descriptor words decoded by `readDescriptor` and run
by `dispatchMatmul` (src/inference/jsep/ops/matmul.ts:150-181,555-1000).
This module keeps those names, argument meanings and status codes, and
calls the C ABI (include/wllm_mulmat.h) through ctypes. There is no
fallback: if the CUDA library is missing or cannot bind a GPU, the calls
raise.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

STATUS_OK = 0
STATUS_NOT_IMPLEMENTED = 1
STATUS_FAILED = -1

GGML_OP_RMS_NORM = 25
GGML_OP_MUL_MAT = 29
GGML_OP_SET_ROWS = 42

GLU_SWIGLU = 1  # silu(gate) * up
GLU_GELU = 2  # gelu(gate) * up (tanh form, f16-rounded like ggml's CPU GELU)

GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q4_0 = 2
GGML_TYPE_Q8_0 = 8
GGML_TYPE_Q4_K = 12
GGML_TYPE_Q5_K = 13
GGML_TYPE_Q6_K = 14
GGML_TYPE_IQ4_XS = 23

TENSOR_BLOCK_I32 = 19

# (elements per block, bytes per block): src/models/gguf-parser.ts:273-294
BLOCK_GEOMETRY = {
    GGML_TYPE_F32: (1, 4),
    GGML_TYPE_F16: (1, 2),
    GGML_TYPE_Q4_0: (32, 18),
    GGML_TYPE_Q8_0: (32, 34),
    GGML_TYPE_Q4_K: (256, 144),
    GGML_TYPE_Q5_K: (256, 176),
    GGML_TYPE_IQ4_XS: (256, 136),
    GGML_TYPE_Q6_K: (256, 210),
}

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG_DIR, "libwllm_mulmat.so")

# Names every build of the library exports (declared in include/wllm_mulmat.h).
EXPORTED_SYMBOLS = (
    "wllm_init", "wllm_shutdown", "wllm_alloc", "wllm_free", "wllm_write", "wllm_read",
    "wllm_read_async_begin", "wllm_read_async_poll", "wllm_read_async_finish", "wllm_read_async_cancel",
    "wllm_clear", "wllm_run_op", "wllm_run_ops", "wllm_sync", "wllm_last_error", "wllm_get_counters",
    "wllm_buffer_device_ptr", "wllm_mul_mat", "wllm_mul_mat_batch", "wllm_mul_mat_rms_norm_batch",
    "wllm_mul_mat_glu_batch",
    "wllm_get_stream",
    "wllm_graph_begin", "wllm_graph_end", "wllm_graph_launch", "wllm_graph_destroy",
    "wllm_dequantize", "wllm_version", "wllm_mul_mat_prefill_static",
    "wllm_ipc_alloc", "wllm_ipc_open", "wllm_ipc_close", "wllm_ipc_free", "wllm_mul_mat_batch_tp", "wllm_tp_wait", "wllm_set_wait_limit",
)

MAX_RANKS = 8
IPC_HANDLE_BYTES = 64


class MulMatArgs(ctypes.Structure):
    """wllm_mulmat_args (include/wllm_mulmat.h)."""
    _fields_ = [("src0_type", ctypes.c_int32), ("M", ctypes.c_int32), ("K", ctypes.c_int32),
                ("N", ctypes.c_int32), ("w", ctypes.c_void_p), ("w_row_bytes", ctypes.c_int64),
                ("x", ctypes.c_void_p), ("x_stride", ctypes.c_int64), ("y", ctypes.c_void_p),
                ("y_stride", ctypes.c_int64)]


class TpGroup(ctypes.Structure):
    """wllm_tp_group (include/wllm_mulmat.h)."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("sig", ctypes.c_void_p * MAX_RANKS), ("state", ctypes.c_void_p)]


class TpOutputs(ctypes.Structure):
    """wllm_tp_outputs (include/wllm_mulmat.h)."""
    _fields_ = [("y_rank", ctypes.c_void_p * MAX_RANKS)]


class WllmCounters(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "alloc", "free", "write", "read", "clear", "run_op", "sync",
        "kernels_launched", "bytes_live", "bytes_reserved")]


_lib = None


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    """dlopen the C-ABI library and declare its signatures (no GPU needed)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m webllm_b200.build_ext`")
    L = ctypes.CDLL(path)
    i32, i64, u64, vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_void_p
    P = ctypes.POINTER
    sig = {
        "wllm_init": ([i32], i32),
        "wllm_shutdown": ([], i32),
        "wllm_alloc": ([u64, P(i32)], i32),
        "wllm_free": ([i32], i32),
        "wllm_write": ([i32, u64, vp, u64], i32),
        "wllm_read": ([i32, u64, vp, u64], i32),
        "wllm_read_async_begin": ([i32, u64, u64, P(i32)], i32),
        "wllm_read_async_poll": ([i32], i32),
        "wllm_read_async_finish": ([i32, vp, u64], i32),
        "wllm_read_async_cancel": ([i32], i32),
        "wllm_clear": ([i32, i32, u64, u64], i32),
        "wllm_run_op": ([vp, i32, vp, i32], i32),
        "wllm_run_ops": ([vp, vp, i32], i32),
        "wllm_sync": ([], i32),
        "wllm_last_error": ([ctypes.c_char_p, i32], i32),
        "wllm_get_counters": ([P(WllmCounters)], i32),
        "wllm_buffer_device_ptr": ([i32, P(vp), P(u64)], i32),
        "wllm_mul_mat": ([i32, vp, i64, vp, i64, vp, i64, i32, i32, i32, vp], i32),
        "wllm_mul_mat_prefill_static": ([i32, vp, i64, vp, i64, vp, i64, i32, i32, i32, vp], i32),
        "wllm_dequantize": ([i32, vp, vp, i64, vp], i32),
        "wllm_mul_mat_batch": ([P(MulMatArgs), i32, vp], i32),
        "wllm_mul_mat_rms_norm_batch": ([P(MulMatArgs), i32, vp, ctypes.c_float, vp], i32),
        "wllm_mul_mat_glu_batch": ([P(MulMatArgs), i32, vp, i64, i32, vp], i32),
        "wllm_ipc_alloc": ([u64, P(vp), vp], i32),
        "wllm_ipc_open": ([vp, P(vp)], i32),
        "wllm_ipc_close": ([vp], i32),
        "wllm_ipc_free": ([vp], i32),
        "wllm_mul_mat_batch_tp": ([P(MulMatArgs), P(TpOutputs), i32, P(TpGroup), vp], i32),
        "wllm_tp_wait": ([P(TpGroup), vp], i32),
        "wllm_set_wait_limit": ([ctypes.c_uint32], i32),
        "wllm_get_stream": ([P(vp)], i32),
        "wllm_graph_begin": ([], i32),
        "wllm_graph_end": ([P(i32)], i32),
        "wllm_graph_launch": ([i32], i32),
        "wllm_graph_destroy": ([i32], i32),
        "wllm_version": ([], ctypes.c_char_p),
    }
    for name, (argtypes, restype) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = argtypes
        fn.restype = restype
    _lib = L
    return L


def last_error() -> str:
    L = load_library()
    buf = ctypes.create_string_buffer(1024)
    L.wllm_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


class WllmError(RuntimeError):
    pass


def _check(rc: int, what: str) -> int:
    if rc == STATUS_FAILED:
        raise WllmError(f"{what}: {last_error()}")
    return rc


# ---------------------------------------------------------------- descriptors


@dataclass
class JsepTensorMeta:
    """One 19-word tensor block (matmul.ts:67-80)."""
    buf_handle: int
    offset: int
    type: int
    ne: tuple = (1, 1, 1, 1)
    nb: tuple = (0, 0, 0, 0)


@dataclass
class JsepOpDescriptor:
    op: int
    n_src: int
    dst: JsepTensorMeta
    srcs: list = field(default_factory=list)


def _split64(v: int) -> tuple[int, int]:
    v &= (1 << 64) - 1
    lo, hi = v & 0xFFFFFFFF, v >> 32
    to_i32 = lambda u: u - (1 << 32) if u >= (1 << 31) else u  # noqa: E731
    return to_i32(lo), to_i32(hi)


def _block_words(t: JsepTensorMeta) -> list[int]:
    ne = [_split64(int(v)) for v in t.ne]
    nb = [_split64(int(v)) for v in t.nb]
    off = int(t.offset) & 0xFFFFFFFF
    off = off - (1 << 32) if off >= (1 << 31) else off
    return ([int(t.buf_handle), off, int(t.type)] + [lo for lo, _ in ne] + [hi for _, hi in ne]
            + [lo for lo, _ in nb] + [hi for _, hi in nb])


def pack_descriptor(desc: JsepOpDescriptor) -> np.ndarray:
    """Descriptor words as the C++ backend packs them (matmul.ts:22-41)."""
    words = [int(desc.op), int(desc.n_src)] + _block_words(desc.dst)
    for s in desc.srcs:
        words += _block_words(s)
    return np.asarray(words, dtype=np.int32)


def read_descriptor(words: Sequence[int], byte_offset: int = 0) -> JsepOpDescriptor:
    """Decode descriptor words (matmul.ts:150-181), including the hi halves."""
    w = np.asarray(words, dtype=np.int32).view(np.uint32).astype(np.uint64)
    base = byte_offset >> 2

    def block(slot: int) -> JsepTensorMeta:
        o = base + slot
        ne = tuple(int(w[o + 3 + i] | (w[o + 7 + i] << np.uint64(32))) for i in range(4))
        nb = tuple(int(w[o + 11 + i] | (w[o + 15 + i] << np.uint64(32))) for i in range(4))
        return JsepTensorMeta(int(np.int32(np.uint32(w[o]))), int(w[o + 1]), int(np.int32(np.uint32(w[o + 2]))), ne, nb)

    op = int(np.int32(np.uint32(w[base])))
    n_src = int(np.int32(np.uint32(w[base + 1])))
    dst = block(2)
    srcs = [block(2 + TENSOR_BLOCK_I32 * (1 + i)) for i in range(n_src)]
    return JsepOpDescriptor(op, n_src, dst, srcs)


def make_meta(handle: int, type_: int, ne: Sequence[int], bytes_per_elem: int, elems_per_block: int,
              offset: int = 0) -> JsepTensorMeta:
    """Row-contiguous tensor meta (tests/jsep-matmul-golden.test.ts:274-296)."""
    nb0 = bytes_per_elem
    nb1 = (ne[0] // elems_per_block) * bytes_per_elem
    nb2 = nb1 * ne[1]
    nb3 = nb2 * ne[2]
    return JsepTensorMeta(handle, offset, type_, tuple(int(v) for v in ne), (nb0, nb1, nb2, nb3))


def meta_for(handle: int, type_: int, ne: Sequence[int], offset: int = 0) -> JsepTensorMeta:
    be, bb = BLOCK_GEOMETRY[type_]
    return make_meta(handle, type_, ne, bb, be, offset)


# ---------------------------------------------------------------- runtime


class GpuDataManager:
    """Handle -> HBM buffer map (gpu-data-manager.ts:55-205), in libwllm_mulmat."""

    def __init__(self, lib: ctypes.CDLL):
        self._L = lib
        self._live: set[int] = set()

    def alloc(self, size: int) -> int:
        if size <= 0:
            raise ValueError(f"GpuDataManager.alloc: invalid size {size}")
        h = ctypes.c_int32(0)
        _check(self._L.wllm_alloc(int(size), ctypes.byref(h)), "GpuDataManager.alloc")
        self._live.add(h.value)
        return h.value

    def free(self, handle: int) -> None:
        self._L.wllm_free(int(handle))
        self._live.discard(handle)

    def get(self, handle: int) -> tuple[int, int]:
        """(device address, size)."""
        p, n = ctypes.c_void_p(0), ctypes.c_uint64(0)
        _check(self._L.wllm_buffer_device_ptr(int(handle), ctypes.byref(p), ctypes.byref(n)),
               "GpuDataManager.get")
        return int(p.value or 0), int(n.value)

    def write(self, handle: int, offset: int, data) -> None:
        a = np.ascontiguousarray(data)
        _check(self._L.wllm_write(int(handle), int(offset), a.ctypes.data, a.nbytes), "GpuDataManager.write")

    def read(self, handle: int, offset: int, size: int) -> np.ndarray:
        out = np.empty(int(size), dtype=np.uint8)
        _check(self._L.wllm_read(int(handle), int(offset), out.ctypes.data, out.nbytes), "GpuDataManager.read")
        return out

    def read_async(self, handle: int, offset: int, size: int):
        """begin/poll/finish readback (webgpu-bridge.cpp:353-370)."""
        req = ctypes.c_int32(0)
        _check(self._L.wllm_read_async_begin(int(handle), int(offset), int(size), ctypes.byref(req)),
               "read_async_begin")
        return AsyncRead(self._L, req.value, int(size))

    def clear(self, handle: int, value: int, offset: int, size: int) -> None:
        _check(self._L.wllm_clear(int(handle), int(value), int(offset), int(size)), "GpuDataManager.clear")

    def live_handle_count(self) -> int:
        return len(self._live)

    def destroy(self) -> None:
        for h in list(self._live):
            self.free(h)


class AsyncRead:
    def __init__(self, lib, request: int, size: int):
        self._L, self.request, self.size = lib, request, size

    def poll(self) -> bool:
        return _check(self._L.wllm_read_async_poll(self.request), "read_async_poll") == 1

    def finish(self) -> np.ndarray:
        out = np.empty(self.size, dtype=np.uint8)
        _check(self._L.wllm_read_async_finish(self.request, out.ctypes.data, self.size), "read_async_finish")
        return out

    def cancel(self) -> None:
        self._L.wllm_read_async_cancel(self.request)


class CommandEncoderBatcher:
    """The WebGPU batcher's flush becomes a stream synchronisation."""

    def __init__(self, lib):
        self._L = lib

    def flush(self) -> None:
        _check(self._L.wllm_sync(), "flush")


@dataclass
class JsepRuntime:
    device: int
    data_manager: GpuDataManager
    encoder_batcher: CommandEncoderBatcher
    lib: ctypes.CDLL

    def counters(self) -> dict:
        c = WllmCounters()
        _check(self.lib.wllm_get_counters(ctypes.byref(c)), "get_counters")
        return {n: int(getattr(c, n)) for n, _ in WllmCounters._fields_}

    # the seven callbacks (jsep/index.ts:163-305)
    def jsep_alloc(self, size: int) -> int:
        return self.data_manager.alloc(size)

    def jsep_free(self, handle: int) -> None:
        self.data_manager.free(handle)

    def jsep_write(self, handle: int, offset: int, data) -> None:
        self.data_manager.write(handle, offset, data)

    def jsep_read(self, handle: int, offset: int, size: int) -> np.ndarray:
        return self.data_manager.read(handle, offset, size)

    def jsep_clear(self, handle: int, value: int, offset: int, size: int) -> None:
        self.data_manager.clear(handle, value, offset, size)

    def jsep_run_op(self, words: np.ndarray, op_params: bytes = b"") -> int:
        w = np.ascontiguousarray(words, dtype=np.int32)
        pp = ctypes.c_char_p(op_params) if op_params else None
        return int(self.lib.wllm_run_op(w.ctypes.data, int(w.size), pp, len(op_params)))

    def jsep_sync(self) -> None:
        self.encoder_batcher.flush()

    def run_ops(self, descs: Sequence[JsepOpDescriptor]) -> int:
        """Independent MUL_MAT nodes in one launch (wllm_run_ops)."""
        packed = [pack_descriptor(d) for d in descs]
        ptrs = (ctypes.c_void_p * len(packed))(*[p.ctypes.data for p in packed])
        words = (ctypes.c_int32 * len(packed))(*[p.size for p in packed])
        return int(self.lib.wllm_run_ops(ptrs, words, len(packed)))

    def destroy(self) -> None:
        self.data_manager.destroy()


_runtime: JsepRuntime | None = None


def install_jsep_callbacks(device: int = 0) -> JsepRuntime:
    """Bind libwllm_mulmat to `device` (installJsepCallbacks, jsep/index.ts:129)."""
    global _runtime
    L = load_library()
    _check(L.wllm_init(int(device)), "wllm_init")
    if _runtime is None or _runtime.device != device:
        _runtime = JsepRuntime(device, GpuDataManager(L), CommandEncoderBatcher(L), L)
    return _runtime


def destroy_jsep_callbacks() -> None:
    global _runtime
    if _runtime is not None:
        _runtime.destroy()
    load_library().wllm_shutdown()
    _runtime = None


def dispatch_matmul(ctx: JsepRuntime, desc: JsepOpDescriptor) -> int:
    """dispatchMatmul(ctx, desc) (matmul.ts:555): 0 ok, 1 not implemented, -1 failed."""
    return ctx.jsep_run_op(pack_descriptor(desc))


def mul_mat_device(src0_type: int, w_ptr: int, w_row_bytes: int, x_ptr: int, x_stride: int,
                   y_ptr: int, y_stride: int, M: int, K: int, N: int, stream: int = 0) -> int:
    """Device-pointer MUL_MAT (wllm_mul_mat) on `stream` (0 = library stream)."""
    L = load_library()
    rc = L.wllm_mul_mat(int(src0_type), int(w_ptr), int(w_row_bytes), int(x_ptr), int(x_stride),
                        int(y_ptr), int(y_stride), int(M), int(K), int(N), int(stream) or None)
    return _check(rc, "wllm_mul_mat")


def mul_mat_prefill_static(src0_type: int, w_ptr: int, w_row_bytes: int, x_ptr: int, x_stride: int,
                           y_ptr: int, y_stride: int, M: int, K: int, N: int, stream: int = 0) -> int:
    """Prefill MUL_MAT with the library's fixed device workspace
    (wllm_mul_mat_prefill_static): allocates nothing; N * K * 2 + 256 bytes
    must fit in 16 MiB; overlapping calls race on the one workspace."""
    L = load_library()
    rc = L.wllm_mul_mat_prefill_static(int(src0_type), int(w_ptr), int(w_row_bytes), int(x_ptr), int(x_stride),
                                       int(y_ptr), int(y_stride), int(M), int(K), int(N), int(stream) or None)
    return _check(rc, "wllm_mul_mat_prefill_static")


def mul_mat_batch(ops: Sequence[MulMatArgs], stream: int = 0) -> int:
    """Independent device-pointer MUL_MATs in one launch (wllm_mul_mat_batch)."""
    L = load_library()
    arr = (MulMatArgs * len(ops))(*ops)
    return _check(L.wllm_mul_mat_batch(arr, len(ops), int(stream) or None), "wllm_mul_mat_batch")


def mul_mat_rms_norm_batch(ops: Sequence[MulMatArgs], gain_ptr: int, eps: float, stream: int = 0) -> int:
    """MUL_MATs of RMS_NORM(x) * gain with the norm fused into the kernel
    (wllm_mul_mat_rms_norm_batch): STATUS_OK, or STATUS_NOT_IMPLEMENTED outside
    the decode regime (the caller then runs the ops unfused)."""
    L = load_library()
    arr = (MulMatArgs * len(ops))(*ops)
    return _check(L.wllm_mul_mat_rms_norm_batch(arr, len(ops), int(gain_ptr) or None, float(eps),
                                                int(stream) or None), "wllm_mul_mat_rms_norm_batch")


def mul_mat_glu_batch(ops: Sequence[MulMatArgs], up_ptr: int, up_stride: int, glu: int, stream: int = 0) -> int:
    """MUL_MATs of act(gate) * up with the GLU fused into the kernel
    (wllm_mul_mat_glu_batch; the ops' x is the gate, up_stride is in floats):
    STATUS_OK, or STATUS_NOT_IMPLEMENTED outside the decode regime (the caller
    then runs the ops unfused)."""
    L = load_library()
    arr = (MulMatArgs * len(ops))(*ops)
    return _check(L.wllm_mul_mat_glu_batch(arr, len(ops), int(up_ptr) or None, int(up_stride), int(glu),
                                           int(stream) or None), "wllm_mul_mat_glu_batch")


def ipc_alloc(size: int) -> tuple[int, bytes]:
    """Peer-mappable zeroed device memory: (device pointer, 64-byte IPC handle)."""
    p = ctypes.c_void_p(0)
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(load_library().wllm_ipc_alloc(int(size), ctypes.byref(p), h), "wllm_ipc_alloc")
    return int(p.value), h.raw


def ipc_open(handle: bytes) -> int:
    """Maps another process's wllm_ipc_alloc memory; returns its device pointer here."""
    p = ctypes.c_void_p(0)
    buf = ctypes.create_string_buffer(bytes(handle), IPC_HANDLE_BYTES)
    _check(load_library().wllm_ipc_open(buf, ctypes.byref(p)), "wllm_ipc_open")
    return int(p.value)


def ipc_close(ptr: int) -> None:
    _check(load_library().wllm_ipc_close(int(ptr)), "wllm_ipc_close")


def ipc_free(ptr: int) -> None:
    _check(load_library().wllm_ipc_free(int(ptr)), "wllm_ipc_free")


def tp_group(world: int, rank: int, sig_ptrs: Sequence[int], state_ptr: int) -> TpGroup:
    g = TpGroup()
    g.world, g.rank = int(world), int(rank)
    for r, p in enumerate(sig_ptrs):
        g.sig[r] = int(p)
    g.state = int(state_ptr)
    return g


def mul_mat_batch_tp(ops: Sequence[MulMatArgs], outs: Sequence[Sequence[int]], group: TpGroup, stream: int = 0) -> int:
    """Row-sharded MUL_MATs: op i's rows also go to outs[i][r] on every other rank r
    (wllm_mul_mat_batch_tp)."""
    arr = (MulMatArgs * len(ops))(*ops)
    oa = (TpOutputs * len(ops))()
    for i, ys in enumerate(outs):
        for r, p in enumerate(ys):
            oa[i].y_rank[r] = int(p)
    return _check(load_library().wllm_mul_mat_batch_tp(arr, oa, len(ops), ctypes.byref(group), int(stream) or None),
                  "wllm_mul_mat_batch_tp")


def tp_wait(group: TpGroup, stream: int = 0) -> int:
    """Waits (on the stream, bounded) for every peer's rows of the last row-sharded launch."""
    return _check(load_library().wllm_tp_wait(ctypes.byref(group), int(stream) or None), "wllm_tp_wait")


def set_wait_limit(polls: int) -> None:
    """Polls before a device-side wait of the decode kernels gives up (0: the
    default); a wait that gives up fails the next sync instead of hanging."""
    _check(load_library().wllm_set_wait_limit(int(polls)), "wllm_set_wait_limit")


def library_stream() -> int:
    """The library's cudaStream_t (wrap with torch.cuda.ExternalStream)."""
    p = ctypes.c_void_p(0)
    _check(load_library().wllm_get_stream(ctypes.byref(p)), "wllm_get_stream")
    return int(p.value or 0)


class Graph:
    """run_op sequence recorded once and replayed (wllm_graph_*)."""

    def __init__(self, graph_id: int):
        self.id = graph_id

    @staticmethod
    def begin() -> None:
        _check(load_library().wllm_graph_begin(), "wllm_graph_begin")

    @classmethod
    def end(cls) -> "Graph":
        g = ctypes.c_int32(0)
        _check(load_library().wllm_graph_end(ctypes.byref(g)), "wllm_graph_end")
        return cls(g.value)

    def launch(self) -> None:
        _check(load_library().wllm_graph_launch(self.id), "wllm_graph_launch")

    def destroy(self) -> None:
        load_library().wllm_graph_destroy(self.id)


def dequantize_device(qtype: int, src_ptr: int, dst_ptr: int, n: int, stream: int = 0) -> None:
    L = load_library()
    _check(L.wllm_dequantize(int(qtype), int(src_ptr), int(dst_ptr), int(n), int(stream) or None),
           "wllm_dequantize")
