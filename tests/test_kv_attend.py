"""8-bit KV decode attention on the CPU: the oracle against a known answer and against an independent numpy
statement of the reference test's own formulation (attention over the unpacked keys and values with a mask from
start and the sinks, tests/test_flint.py:277-299), and the C ABI's argument checks (no GPU needed)."""

import ctypes

import numpy as np
import pytest

from locals_b200 import _lib
from oracle import oracle as O


def _pack8(codes: np.ndarray) -> np.ndarray:
    """uint8 codes (..., D) -> uint32 words (..., D/4), low byte first."""
    return np.ascontiguousarray(codes.astype(np.uint8)).view(np.uint32)


def _cache(rng, B, KVH, cap, HD, spread):
    codes = rng.integers(0, 256, (B, KVH, cap, HD), dtype=np.uint8)
    s = O.round_to((spread * rng.random((B, KVH, cap, HD // 64)) / 255 + 1e-3).astype(np.float32), "bfloat16")
    b = O.round_to((-spread * rng.random((B, KVH, cap, HD // 64))).astype(np.float32), "bfloat16")
    return codes, s, b


def _numpy_attend(q, kc, ks, kb, vc, vs, vb, n, sinks, scale, start):
    """Attention over the dequantized keys and values (float32 s * q + b, as qkv.py:50-53) with the sink as one
    more logit carrying no value, in float64."""
    B, H, HD = q.shape
    KVH = kc.shape[1]
    G = H // KVH
    k = (kc.astype(np.float32) * np.repeat(ks, 64, axis=-1) + np.repeat(kb, 64, axis=-1)).astype(np.float64)
    v = (vc.astype(np.float32) * np.repeat(vs, 64, axis=-1) + np.repeat(vb, 64, axis=-1)).astype(np.float64)
    out = np.zeros((B, H, HD))
    for b in range(B):
        lo = max(int(start[b]), 0) if start is not None else 0
        for h in range(H):
            kh = h // G
            sc = scale * (k[b, kh, lo:n] @ q[b, h].astype(np.float64))
            logits = np.concatenate([sc, [sinks[h]]]) if sinks is not None else sc
            if logits.size == 0:
                continue
            p = np.exp(logits - logits.max())
            out[b, h] = (p[:sc.size] @ v[b, kh, lo:n]) / p.sum()
    return out


def test_kv_attend_known_answer():
    HD = 64
    q = np.full((1, 1, HD), 1.0 / HD, np.float32)
    kc = np.zeros((1, 1, 2, HD), np.uint8)
    kc[0, 0, 0] = 1  # key 0 = ones, key 1 = zeros -> scores (1, 0)
    vc = np.zeros((1, 1, 2, HD), np.uint8)
    vc[0, 0, 0] = 2  # value 0 = twos, value 1 = zeros
    one = np.ones((1, 1, 2, 1), np.float32)
    zero = np.zeros((1, 1, 2, 1), np.float32)
    out = O.kv_attend(q, (_pack8(kc), one, zero), (_pack8(vc), one, zero), 2, np.zeros(1, np.float32), 1.0)
    e = np.exp(-1.0)
    assert np.allclose(out, 2.0 / (1.0 + e + e), rtol=1e-6, atol=0)
    # no sink, only key 1 (start = 1): softmax of one key is its value
    out = O.kv_attend(q, (_pack8(kc), one, zero), (_pack8(vc), one, zero), 2, None, 1.0, np.array([1], np.int32))
    assert np.array_equal(out, np.zeros_like(out))
    # nothing attended and no sink: 0
    out = O.kv_attend(q, (_pack8(kc), one, zero), (_pack8(vc), one, zero), 0, None, 1.0)
    assert np.array_equal(out, np.zeros_like(out))


@pytest.mark.parametrize("H,KVH", [(32, 4), (4, 2)])
@pytest.mark.parametrize("B,n,cap,pads", [(1, 1, 256, [0]), (1, 13, 256, [0]), (1, 700, 768, [0]),
                                          (3, 300, 512, [0, 37, 300])])
def test_kv_attend_oracle_is_attention_over_unpacked_keys(H, KVH, B, n, cap, pads):
    rng = np.random.default_rng(B * 1000 + n)
    HD = 128
    q = O.round_to(rng.standard_normal((B, H, HD)).astype(np.float32), "bfloat16")
    kc, ks, kb = _cache(rng, B, KVH, cap, HD, 8.0)
    vc, vs, vb = _cache(rng, B, KVH, cap, HD, 4.0)
    sinks = O.round_to((2 * rng.standard_normal(H)).astype(np.float32), "bfloat16")
    start = np.array(pads, np.int32)
    got = O.kv_attend(q, (_pack8(kc), ks, kb), (_pack8(vc), vs, vb), n, sinks, 0.0884, start)
    ref = _numpy_attend(q, kc, ks, kb, vc, vs, vb, n, sinks, 0.0884, start)
    assert np.max(np.abs(got - ref)) <= 1e-5 * (1 + np.abs(ref).max())


def test_kv_attend_abi_rejects_bad_arguments():
    L = _lib.lib()
    fake = ctypes.c_void_p(4096)  # never dereferenced: argument checks come first

    def rc(B=1, H=32, KVH=4, n=10, cap=256, hd=128, dtype=_lib.BF16, q=fake):
        return L.lq_kv_attend(q, fake, fake, fake, fake, fake, fake, None, n, None, 0.1, B, H, KVH, cap, hd, dtype,
                              None, 0, fake, None)

    assert rc(q=None) == _lib.LQ_E_ARG
    assert rc(dtype=_lib.F32) == _lib.LQ_E_UNSUPPORTED
    assert rc(hd=64) == _lib.LQ_E_SHAPE
    assert rc(H=64, KVH=2) == _lib.LQ_E_SHAPE  # 32 query heads a kv head
    assert rc(H=30, KVH=4) == _lib.LQ_E_SHAPE
    assert rc(n=257) == _lib.LQ_E_SHAPE
    assert rc(n=-1) == _lib.LQ_E_SHAPE
    assert rc(B=65536) == _lib.LQ_E_SHAPE  # B is the attend kernel's grid z (at most 65535)
    assert rc(H=65536 * 2, KVH=65536) == _lib.LQ_E_SHAPE  # KVH is its grid y


def test_kv_attend_noalloc_abi_rejects_bad_arguments():
    L = _lib.lib()
    fake = ctypes.c_void_p(4096)

    def rc(B=1, H=32, KVH=4, n=10, cap=256, hd=128, dtype=_lib.BF16, q=fake):
        return L.lq_kv_attend_noalloc(q, fake, fake, fake, fake, fake, fake, None, n, None, 0.1, B, H, KVH, cap, hd,
                                      dtype, fake, None)

    assert rc(q=None) == _lib.LQ_E_ARG
    assert rc(dtype=_lib.F32) == _lib.LQ_E_UNSUPPORTED
    assert rc(B=65536) == _lib.LQ_E_SHAPE
    assert rc(n=257) == _lib.LQ_E_SHAPE
