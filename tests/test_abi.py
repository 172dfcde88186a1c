"""The C ABI without a GPU: liblq.so loads, exports every function include/lq.h declares, and rejects
bad arguments with LQ_E_* codes before touching a device. CPU only."""

import ctypes
import os
import re

import pytest

from locals_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "lq.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int|unsigned int|const char\*)\s+(lq_\w+)\s*\(", src, re.M)))


def test_library_loads():
    L = _lib.lib()
    assert L.lq_version() >= 100


def test_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "the ctypes table and the header disagree"


def test_strerror_names():
    L = _lib.lib()
    assert L.lq_strerror(_lib.LQ_E_SHAPE) == b"unsupported shape"
    assert L.lq_strerror(999) == b"unknown"


def test_null_pointers_rejected():
    L = _lib.lib()
    rc = L.lq_qmm(None, None, None, None, None, 1, 64, 512, 4, 64, _lib.BF16, None, None)
    assert rc == _lib.LQ_E_ARG


@pytest.mark.parametrize("bits,group,dtype,code", [
    (3, 64, _lib.BF16, _lib.LQ_E_UNSUPPORTED),
    (4, 32, _lib.BF16, _lib.LQ_E_UNSUPPORTED),
    (4, 64, _lib.F32, _lib.LQ_E_UNSUPPORTED),
])
def test_unsupported_formats_rejected(bits, group, dtype, code):
    L = _lib.lib()
    fake = ctypes.c_void_p(4096)  # never dereferenced: argument checks come first
    rc = L.lq_qmm(fake, fake, fake, fake, fake, 1, 64, 512, bits, group, dtype, None, None)
    assert rc == code


def test_bad_shapes_rejected():
    L = _lib.lib()
    fake = ctypes.c_void_p(4096)
    assert L.lq_qmm(fake, fake, fake, fake, fake, 0, 64, 512, 4, 64, _lib.BF16, None, None) == _lib.LQ_E_SHAPE
    assert L.lq_qmm(fake, fake, fake, fake, fake, 1, 64, 100, 4, 64, _lib.BF16, None, None) == _lib.LQ_E_SHAPE


def test_misaligned_rejected():
    L = _lib.lib()
    ok, bad = ctypes.c_void_p(4096), ctypes.c_void_p(4098)
    assert L.lq_qmm(bad, ok, ok, ok, ok, 1, 64, 512, 4, 64, _lib.BF16, None, None) == _lib.LQ_E_ALIGN


def test_routing_args_rejected():
    L = _lib.lib()
    fake = ctypes.c_void_p(4096)
    assert L.lq_route_topk(fake, 4, 64, 4, 2, fake, fake, None) == _lib.LQ_E_ARG
    assert L.lq_route_topk(fake, 4, 2048, 4, 0, fake, fake, None) == _lib.LQ_E_SHAPE
    assert L.lq_moe_group(None, 4, 64, fake, fake, fake, fake, None, None) == _lib.LQ_E_ARG
