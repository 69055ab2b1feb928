"""GGUF parsing and streaming into library buffers (CPU: the writes go to a
fake data manager). Files are written by the third-party `gguf` package and
read back with its own reader as the check; the parser mirrors the
reference's GgufParser (src/models/gguf-parser.ts)."""
from __future__ import annotations

import struct

import numpy as np
import pytest

from webllm_b200 import gguf as G
from webllm_b200 import synth

gguf = pytest.importorskip("gguf")


class FakeDataManager:
    def __init__(self):
        self.bufs, self.writes = {}, 0

    def alloc(self, size):
        h = len(self.bufs) + 1
        self.bufs[h] = np.zeros(size, np.uint8)
        return h

    def write(self, h, off, data):
        a = np.ascontiguousarray(data)
        self.bufs[h][off:off + a.nbytes] = a.view(np.uint8).reshape(-1)
        self.writes += 1


def write_model(path):
    rng = np.random.default_rng(11)
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_uint32("llama.block_count", 2)
    w.add_float32("llama.attention.layer_norm_rms_epsilon", 1e-5)
    w.add_bool("test.flag", True)
    w.add_array("test.ints", [1, 2, 3])
    w.add_string("test.name", "synthetic")
    tensors = {
        "blk.0.attn_q.weight": (synth.weights(rng, 12, 64, 512), gguf.GGMLQuantizationType.Q4_K, (64, 512)),
        "blk.0.ffn_down.weight": (synth.weights(rng, 14, 32, 1024), gguf.GGMLQuantizationType.Q6_K, (32, 1024)),
        "blk.0.attn_v.weight": (synth.weights(rng, 8, 16, 256), gguf.GGMLQuantizationType.Q8_0, (16, 256)),
        "output_norm.weight": (rng.standard_normal(512).astype(np.float32), None, None),
    }
    for name, (arr, qt, shape) in tensors.items():
        if qt is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=qt)  # the byte shape: rows x row bytes
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


def test_parse_matches_gguf_reader(tmp_path):
    path = tmp_path / "m.gguf"
    write_model(path)
    ctx = G.parse(path.read_bytes())
    rd = gguf.GGUFReader(str(path))
    assert (ctx.magic, ctx.version, ctx.tensor_count) == (G.GGUF_MAGIC, 3, len(rd.tensors))
    assert ctx.metadata["llama.block_count"] == (G.UINT32, 2)
    assert ctx.metadata["test.flag"] == (G.BOOL, True)
    assert ctx.metadata["test.ints"][1] == [1, 2, 3]
    assert ctx.metadata["test.name"] == (G.STRING, "synthetic")
    assert abs(ctx.metadata["llama.attention.layer_norm_rms_epsilon"][1] - 1e-5) < 1e-12
    assert ctx.alignment == 32 and ctx.data_offset % 32 == 0
    by_name = {t.name: t for t in rd.tensors}
    for t in ctx.tensors:
        r = by_name[t.name]
        assert t.type == int(r.tensor_type)
        assert t.dimensions == [int(d) for d in r.shape]
        assert ctx.data_offset + t.offset == int(r.data_offset)
        assert G.tensor_nbytes(t) == int(r.n_bytes)


@pytest.mark.parametrize("chunk", [100, 64 << 20])
def test_stream_to_buffers_bytes(tmp_path, chunk):
    """Every tensor's bytes land in its buffer unchanged, in chunks of `chunk`;
    `names` selects tensors."""
    path = tmp_path / "m.gguf"
    tensors = write_model(path)
    dm = FakeDataManager()
    got = G.stream_to_buffers(str(path), dm, chunk_bytes=chunk)
    assert set(got) == set(tensors)
    for name, (arr, _, _) in tensors.items():
        h, info, nbytes = got[name]
        assert nbytes == arr.nbytes
        assert np.array_equal(dm.bufs[h][:nbytes], np.ascontiguousarray(arr).view(np.uint8).reshape(-1))
    expect = sum(-(-a.nbytes // chunk) for a, _, _ in tensors.values())
    assert dm.writes == expect
    dm2 = FakeDataManager()
    only = G.stream_to_buffers(str(path), dm2, names={"blk.0.attn_v.weight"})
    assert list(only) == ["blk.0.attn_v.weight"] and len(dm2.bufs) == 1


def test_parse_errors():
    """The reference's three errors: magic, version, unknown value type."""
    def header(magic=G.GGUF_MAGIC, version=3, nt=0, nkv=0):
        return struct.pack("<IIQQ", magic, version, nt, nkv)
    with pytest.raises(ValueError, match="magic"):
        G.parse(header(magic=0x12345678))
    with pytest.raises(ValueError, match="version"):
        G.parse(header(version=2))
    key = b"k"
    bad = header(nkv=1) + struct.pack("<Q", len(key)) + key + struct.pack("<I", 99)
    with pytest.raises(ValueError, match="value type"):
        G.parse(bad)
    # an explicit general.alignment moves the data offset
    k = b"general.alignment"
    ok = header(nkv=1) + struct.pack("<Q", len(k)) + k + struct.pack("<II", G.UINT32, 64)
    ctx = G.parse(ok)
    assert ctx.alignment == 64 and ctx.data_offset == 64 and ctx.total_data_size == 0


def test_alignment_and_fractional_sizes():
    """UINT64 alignment is honoured (the reference converts it with Number());
    an alignment <= 0 is a clear error; a tensor that is not whole blocks
    parses with a fractional total size, as the reference computes it."""
    def header(nt=0, nkv=0):
        return struct.pack("<IIQQ", G.GGUF_MAGIC, 3, nt, nkv)
    k = b"general.alignment"
    kv = lambda vt, fmt, v: struct.pack("<Q", len(k)) + k + struct.pack("<I", vt) + struct.pack(fmt, v)  # noqa: E731
    assert G.parse(header(nkv=1) + kv(G.UINT64, "<Q", 128)).alignment == 128
    with pytest.raises(ValueError, match="alignment"):
        G.parse(header(nkv=1) + kv(G.UINT32, "<I", 0))
    name = b"t"
    info = struct.pack("<Q", len(name)) + name + struct.pack("<I", 1) + struct.pack("<Q", 100) + \
        struct.pack("<I", 12) + struct.pack("<Q", 0)  # 100 Q4_K elements: not a whole block
    ctx = G.parse(header(nt=1) + info)
    assert ctx.total_data_size == pytest.approx(100 * 144 / 256)
    with pytest.raises(ValueError, match="whole blocks"):
        G.tensor_nbytes(ctx.tensors[0])


class FailingDataManager(FakeDataManager):
    """Fails the write of the second tensor; records frees."""

    def __init__(self):
        super().__init__()
        self.freed = []

    def write(self, h, off, data):
        if h == 2:
            raise RuntimeError("device write failed")
        super().write(h, off, data)

    def free(self, h):
        self.freed.append(h)


def test_stream_to_buffers_failure_frees_and_keeps_the_error(tmp_path):
    """A failing tensor frees the handles already allocated and raises the
    original error (the memory map still closes cleanly)."""
    path = tmp_path / "m.gguf"
    write_model(path)
    dm = FailingDataManager()
    with pytest.raises(RuntimeError, match="device write failed"):
        G.stream_to_buffers(str(path), dm, chunk_bytes=100)
    assert sorted(dm.freed) == [1, 2]
