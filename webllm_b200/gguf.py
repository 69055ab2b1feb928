"""GGUF files: the header parser, and streaming of tensor data into library
buffers (device memory) straight from the file.

The parser mirrors the reference's GgufParser (src/models/gguf-parser.ts:
19-66 `parse`, 144-294 the readers; constants src/models/gguf-types.ts:2-24):
same fields, the same alignment rule (`general.alignment` when it is a
number, UINT64/INT64 included since the reference converts those with
Number(); otherwise 32) and the same errors (bad magic, a version other than
3, an unknown value type). `total_data_size` is, as in the reference's
calculateTotalDataSize, elements x bytes per element, fractional when a
tensor is not whole blocks; only streaming such a tensor raises. One
deliberate difference: an alignment <= 0 raises ValueError here, where the
reference would compute a NaN or infinite data offset.

`stream_to_buffers` replaces the reference's upload path, which copies each
tensor through a 4 MiB scratch buffer in the wasm heap
(src/inference/ggml-wasm.ts:545-620, `uploadRangeChunked`): the file is
memory-mapped and every tensor's bytes go to `wllm_write` in large chunks
from the mapping itself, with no intermediate copy. Tensors keep the GGUF
block layout the kernels read, so there is no repacking.
"""
from __future__ import annotations

import math
import mmap
import struct
import traceback
from dataclasses import dataclass, field
from fractions import Fraction

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian
GGUF_VERSION = 3
GGUF_DEFAULT_ALIGNMENT = 32

# value types (src/models/gguf-types.ts:11-24)
UINT8, INT8, UINT16, INT16, UINT32, INT32, FLOAT32, BOOL, STRING, ARRAY, UINT64, INT64, FLOAT64 = range(13)
_SCALARS = {UINT8: "<B", INT8: "<b", UINT16: "<H", INT16: "<h", UINT32: "<I", INT32: "<i", FLOAT32: "<f",
            UINT64: "<Q", INT64: "<q", FLOAT64: "<d"}

# bytes per element of each ggml type (the reference's ggmlTypeSize,
# src/models/gguf-parser.ts:274-294; unknown types count 4 bytes there too).
# IQ4_XS (23, 136 bytes per 256 elements) is added: the reference's table has
# no I-quant and would count it at 4 bytes per element, too much to stream.
TYPE_SIZE = {0: Fraction(4), 1: Fraction(2), 2: Fraction(18, 32), 3: Fraction(20, 32), 6: Fraction(22, 32),
             7: Fraction(24, 32), 8: Fraction(34, 32), 9: Fraction(36, 32), 10: Fraction(84, 256),
             11: Fraction(110, 256), 12: Fraction(144, 256), 13: Fraction(176, 256), 14: Fraction(210, 256),
             15: Fraction(292, 256), 23: Fraction(136, 256), 26: Fraction(4), 30: Fraction(2)}


@dataclass
class GgufTensorInfo:
    name: str
    n_dimensions: int
    dimensions: list[int]
    type: int
    offset: int  # bytes from the start of the data section


@dataclass
class GgufContext:
    magic: int
    version: int
    tensor_count: int
    metadata_kv_count: int
    metadata: dict = field(default_factory=dict)  # key -> (value type, value)
    tensors: list[GgufTensorInfo] = field(default_factory=list)
    alignment: int = GGUF_DEFAULT_ALIGNMENT
    data_offset: int = 0
    total_data_size: int = 0


class _Reader:
    def __init__(self, buf):
        self.buf = buf
        self.pos = 0

    def scalar(self, fmt: str):
        (v,) = struct.unpack_from(fmt, self.buf, self.pos)
        self.pos += struct.calcsize(fmt)
        return v

    def string(self) -> str:
        n = self.scalar("<Q")
        s = bytes(self.buf[self.pos:self.pos + n]).decode("utf-8")
        self.pos += n
        return s

    def value(self, vtype: int):
        if vtype in _SCALARS:
            return self.scalar(_SCALARS[vtype])
        if vtype == BOOL:
            return self.scalar("<B") != 0
        if vtype == STRING:
            return self.string()
        if vtype == ARRAY:
            etype = self.scalar("<I")
            count = self.scalar("<Q")
            return [self.value(etype) for _ in range(count)]
        raise ValueError(f"Unknown GGUF value type: {vtype}")


def _elements(t: GgufTensorInfo) -> int:
    n = 1
    for d in t.dimensions:
        n *= int(d)
    return n


def tensor_nbytes(t: GgufTensorInfo) -> int:
    """Bytes of a tensor's data: elements x the type's bytes per element
    (ValueError when that is not whole blocks)."""
    n = _elements(t)
    size = n * TYPE_SIZE.get(t.type, Fraction(4))
    if size.denominator != 1:
        raise ValueError(f"tensor {t.name}: {n} elements are not whole blocks of type {t.type}")
    return int(size)


def parse(data) -> GgufContext:
    """Header, metadata, tensor infos, alignment and data offset of a GGUF
    image (bytes, memoryview, mmap or uint8 array)."""
    r = _Reader(memoryview(data).cast("B") if not isinstance(data, mmap.mmap) else data)
    magic = r.scalar("<I")
    version = r.scalar("<I")
    ctx = GgufContext(magic, version, r.scalar("<Q"), r.scalar("<Q"))
    if magic != GGUF_MAGIC:
        raise ValueError(f"Invalid GGUF magic: expected 0x{GGUF_MAGIC:x}, got 0x{magic:x}")
    if version != GGUF_VERSION:
        raise ValueError(f"Unsupported GGUF version: {version}, expected {GGUF_VERSION}")
    for _ in range(ctx.metadata_kv_count):
        key = r.string()
        vtype = r.scalar("<I")
        ctx.metadata[key] = (vtype, r.value(vtype))
    for _ in range(ctx.tensor_count):
        name = r.string()
        nd = r.scalar("<I")
        dims = [r.scalar("<Q") for _ in range(nd)]
        ttype = r.scalar("<I")
        ctx.tensors.append(GgufTensorInfo(name, nd, dims, ttype, r.scalar("<Q")))
    align = ctx.metadata.get("general.alignment")
    if align is not None and isinstance(align[1], (int, float)) and not isinstance(align[1], bool):
        if not align[1] > 0:
            raise ValueError(f"Invalid GGUF alignment: {align[1]}")
        ctx.alignment = align[1]
    ctx.data_offset = math.ceil(r.pos / ctx.alignment) * ctx.alignment
    total = max((t.offset + _elements(t) * TYPE_SIZE.get(t.type, Fraction(4)) for t in ctx.tensors), default=0)
    ctx.total_data_size = int(total) if Fraction(total).denominator == 1 else float(total)
    return ctx


def stream_to_buffers(path: str, data_manager, chunk_bytes: int = 64 << 20, names=None) -> dict:
    """Allocate one library buffer per tensor (all, or those in `names`) and
    write its bytes from the memory-mapped file in chunks of `chunk_bytes`.
    `data_manager` has the GpuDataManager interface (alloc(size) -> handle,
    write(handle, offset, uint8 array), free(handle)). Returns {name:
    (handle, info, nbytes)}; the caller frees the handles. If any tensor
    fails, the handles already allocated are freed and the error is raised
    once the mapping is closed (its traceback is attached as a note: frames
    kept alive by it would hold views of the mapping and stop it closing)."""
    if chunk_bytes <= 0:
        raise ValueError("chunk_bytes must be positive")
    out = {}
    pending = None
    with open(path, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        try:
            base = np.frombuffer(mm, dtype=np.uint8)
            view = None
            ctx = parse(mm)
            for t in ctx.tensors:
                if names is not None and t.name not in names:
                    continue
                nbytes = tensor_nbytes(t)
                start = ctx.data_offset + t.offset
                if start + nbytes > base.size:
                    raise ValueError(f"tensor {t.name}: data runs past the end of the file")
                h = data_manager.alloc(max(nbytes, 1))
                out[t.name] = (h, t, nbytes)
                for off in range(0, nbytes, chunk_bytes):
                    n = min(chunk_bytes, nbytes - off)
                    view = base[start + off:start + off + n]
                    data_manager.write(h, off, view)
                    del view
        except BaseException as e:  # noqa: BLE001 - re-raised below, after the mapping closes
            for h, _, _ in out.values():
                data_manager.free(h)
            out = {}
            pending = e
            pending.add_note("".join(traceback.format_exception(e)))
            pending.__traceback__ = None
            del e
        finally:
            base = view = None  # the mapping closes only once no array refers to it
            mm.close()
    if pending is not None:
        raise pending
    return out
