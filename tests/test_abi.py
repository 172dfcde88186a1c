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
    return sorted(set(re.findall(r"^(?:int|unsigned int|size_t|const char\*)\s+(lq_\w+)\s*\(", src, re.M)))


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


def test_supported_and_candidates():
    # host-only: the family predicates and the tuner's candidate list, no GPU needed
    from locals_b200 import kernels
    from locals_b200._lib import lib

    L = lib()
    # (family, M, N, K, bits, group, dtype) -> expected
    assert L.lq_supported(1, 16, 6144, 2560, 4, 64, 1) == 1   # qmv: 4-bit K % 256 == 0
    assert L.lq_supported(1, 16, 6144, 2496, 4, 64, 1) == 0   # 4-bit K not a multiple of 256
    assert L.lq_supported(3, 16, 6144, 2560, 4, 64, 1) == 1   # tcv: K % 128 == 0
    assert L.lq_supported(3, 16, 6144, 2496, 4, 64, 1) == 0
    assert L.lq_supported(2, 2048, 14336, 4096, 4, 64, 1) == 1  # tc
    assert L.lq_supported(0, 16, 6144, 2560, 4, 32, 1) == 0   # group 32 is not built
    assert L.lq_supported(0, 16, 6144, 2560, 3, 64, 1) == 0   # 3-bit is not built
    assert L.lq_supported(0, 16, 6144, 2560, 4, 64, 2) == 0   # fp32 activations are not built
    assert L.lq_supported(4, 16, 6144, 2560, 4, 64, 1) == 1   # qmvg: 4-bit, M <= 16, K % 256 == 0
    assert L.lq_supported(4, 17, 6144, 2560, 4, 64, 1) == 0
    assert L.lq_supported(4, 16, 6144, 2560, 8, 64, 1) == 0
    assert L.lq_supported(5, 16, 6144, 2560, 4, 64, 1) == 1   # qmvq: as qmvg
    assert L.lq_supported(5, 17, 6144, 2560, 4, 64, 1) == 0
    assert L.lq_supported(7, 16, 6144, 2560, 4, 64, 1) == 0   # unknown family
    dec = kernels.candidates(16, 2560, 6144, 4)
    assert dec[0] == ("qmv", 0, 0, 0, 0) and ("tcv", 0, 0, 0, 0) in dec and ("tcv", 0, 0, 0, 1) in dec
    assert ("qmvg", 0, 0) in dec and ("qmvg", 4, 0) in dec
    assert ("qmvq", 0, 0, 0, 0) in dec and ("qmvq", 4, 0, 0, 2) in dec
    assert all(c[0] in ("qmv", "qmvg", "qmvq", "tcv") for c in dec)
    assert all(c[0] not in ("qmvg", "qmvq") for c in kernels.candidates(32, 2560, 6144, 4))
    pre = kernels.candidates(2048, 4096, 14336, 4)
    assert ("tc", 0) in pre and ("tc", 256) in pre and ("tcv", 256, 1, 0, 0) in pre
    assert ("dense",) in pre and ("dense", 224) in pre  # the reference's dequantize + dense GEMM path
    assert all(c[0] != "dense" for c in kernels.candidates(64, 4096, 14336, 4))  # decode sizes: never
    assert all(c[0] != "dense" for c in kernels.candidates(2048, 16384, 16384, 4))  # past DENSE_MAX weights
    assert L.lq_list_configs(16, 6144, 2560, 4, 64, 1, None, 0) == len(dec)
    assert kernels.candidates(16, 2496, 6144, 4) == [] or all(c[0] != "tcv" for c in kernels.candidates(16, 2496, 6144, 4))
    assert kernels.supported("tc", 2048, 4096, 14336) and not kernels.supported("qmv", 16, 2496, 6144)
