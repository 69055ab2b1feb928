"""C-ABI checks that need no GPU: the library loads, exports every symbol
include/wllm_mulmat.h declares, rejects calls before init, and the
descriptor words round-trip like readDescriptor (matmul.ts:150-181)."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from webllm_b200 import jsep
from webllm_b200.build_ext import LIB_PATH, build

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols() -> set[str]:
    names = set()
    for fn in os.listdir(os.path.join(REPO, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(REPO, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(wllm_[a-z0-9_]+)\s*\(", src))
    return names


@pytest.fixture(scope="module")
def lib():
    build()
    return jsep.load_library()


def test_library_exports_every_declared_symbol(lib):
    declared = declared_symbols()
    assert declared, "no declarations found"
    cdll = ctypes.CDLL(LIB_PATH)
    missing = [n for n in sorted(declared) if not hasattr(cdll, n)]
    assert not missing, missing
    assert set(jsep.EXPORTED_SYMBOLS) <= declared


def test_version_string(lib):
    assert b"sm_100a" in lib.wllm_version()


def test_calls_before_init_fail_cleanly(lib):
    h = ctypes.c_int32(123)
    assert lib.wllm_alloc(1024, ctypes.byref(h)) == jsep.STATUS_FAILED
    assert h.value == 0
    assert "wllm_init" in jsep.last_error()
    assert lib.wllm_sync() == jsep.STATUS_FAILED
    # free of an unknown handle is a no-op (gpu-data-manager.ts:105-116)
    assert lib.wllm_free(77) == jsep.STATUS_OK


def test_run_op_before_init_fails(lib):
    d = jsep.JsepOpDescriptor(jsep.GGML_OP_MUL_MAT, 2, jsep.meta_for(1, 0, (4, 1, 1, 1)),
                              [jsep.meta_for(2, jsep.GGML_TYPE_Q4_K, (256, 4, 1, 1)),
                               jsep.meta_for(3, 0, (256, 1, 1, 1))])
    w = jsep.pack_descriptor(d)
    assert lib.wllm_run_op(w.ctypes.data, w.size, None, 0) == jsep.STATUS_FAILED


def test_descriptor_roundtrip_with_64bit_halves():
    big = 10 * (151936 * 4096 * 210 // 256)  # a batch stride past 2^32 bytes
    d = jsep.JsepOpDescriptor(
        jsep.GGML_OP_MUL_MAT, 2,
        jsep.JsepTensorMeta(3, 256, 0, (151936, 1, 1, 1), (4, 151936 * 4, 151936 * 4, 151936 * 4)),
        [jsep.JsepTensorMeta(1, 0, jsep.GGML_TYPE_Q6_K, (4096, 151936, 1, 1), (210, 3360, big, big)),
         jsep.JsepTensorMeta(2, 4096, 0, (4096, 1, 1, 1), (4, 16384, 16384, 16384))])
    w = jsep.pack_descriptor(d)
    assert w.dtype == np.int32 and w.size == 2 + 3 * jsep.TENSOR_BLOCK_I32
    back = jsep.read_descriptor(w)
    assert back.op == d.op and back.n_src == 2
    assert back.dst == d.dst and back.srcs == d.srcs
    assert back.srcs[0].nb[2] == big > 2**32


def test_make_meta_strides():
    # tests/jsep-matmul-golden.test.ts:274-296: nb1 = ne0/blk * blockBytes
    m = jsep.make_meta(5, jsep.GGML_TYPE_Q4_K, (2048, 64, 1, 1), 144, 256)
    assert m.nb == (144, 8 * 144, 8 * 144 * 64, 8 * 144 * 64)
    m = jsep.meta_for(5, jsep.GGML_TYPE_Q8_0, (2304, 9216, 1, 1))
    assert m.nb[1] == 72 * 34
