"""The CPU oracle against the golden vectors (tests/golden/golden.json) and against properties of the
format. CPU only."""

import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


def test_pack_order_4bit():
    g = GOLD["pack4"]
    words = np.array([g["words"]], dtype=np.uint32)
    assert words[0, 0] == 0x87654321
    assert O.unpack(words, 16, 4)[0].tolist() == g["codes"]


def test_pack_order_8bit():
    g = GOLD["pack8"]
    words = np.array([g["words"]], dtype=np.uint32)
    assert O.unpack(words, 8, 8)[0].tolist() == g["codes"]


@pytest.mark.parametrize("name", sorted(GOLD["quantize"]))
def test_quantize_known_answers(name):
    g = GOLD["quantize"][name]
    w = np.array([g["w"]], dtype=np.float32)
    wq, s, b = O.quantize(w, 64, g["bits"], "float32")
    assert O.unpack(wq, 64, g["bits"])[0].tolist() == g["codes"]
    assert s[0, 0] == np.float32(g["scale"]) and b[0, 0] == np.float32(g["bias"])


@pytest.mark.parametrize("bits", [4, 8])
def test_qmm_golden(bits):
    g = GOLD[f"qmm_b{bits}"]
    x = np.array(g["x"], dtype=np.float32)
    wq = np.array(g["words"], dtype=np.uint32)
    y = O.qmm(x, wq, np.array(g["scales"], np.float32), np.array(g["biases"], np.float32), 64, bits)
    ref = np.array(g["y"], dtype=np.float32)
    # same float32 factoring; only the association order inside a group may differ
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))


@pytest.mark.parametrize("mode", ["softmax", "sigmoid"])
def test_topk_golden(mode):
    g = GOLD[f"topk_{mode}"]
    logits = np.array([[math.nan if v is None else v for v in r] for r in g["logits"]], dtype=np.float32)
    inds, w = O.topk(logits, g["k"], mode)
    assert inds.tolist() == g["inds"]
    np.testing.assert_allclose(w, np.array(g["weights"], np.float32), rtol=1e-6, atol=1e-7)


def test_group_golden():
    g = GOLD["group"]
    order, starts, experts, nseg = O.group(np.array(g["inds"], np.uint32), g["E"])
    assert order.tolist() == g["order"]
    assert starts[: nseg + 1].tolist() == g["starts"]
    assert experts[:nseg].tolist() == g["experts"]


@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_roundtrip_error_bound(bits):
    rng = np.random.default_rng(bits)
    w = rng.standard_normal((16, 512)).astype(np.float32) * 0.02
    wq, s, b = O.quantize(w, 64, bits, "float32")
    deq = O.dequantize(wq, s, b, 64, bits)
    codes = O.unpack(wq, 512, bits)
    step = np.repeat(np.abs(s), 64, axis=1)
    err = np.abs(deq - w)
    # codes strictly inside the range are within half a step; the edge made exact can shrink the
    # step so the opposite extreme clips, still within 1.5 steps
    inside = (codes > 0) & (codes < (1 << bits) - 1)
    assert np.all(err[inside] <= 0.5 * step[inside] * (1 + 1e-4) + 1e-7)
    assert np.all(err <= 1.5 * step + 1e-7)


def test_qmm_matches_dequant_matmul():
    rng = np.random.default_rng(7)
    x = rng.standard_normal((5, 256)).astype(np.float32)
    wq, s, b = O.quantize(rng.standard_normal((9, 256)).astype(np.float32) * 0.02, 64, 4, "bfloat16")
    y = O.qmm(x, wq, s, b)
    ref = x.astype(np.float64) @ O.dequantize(wq, s, b).astype(np.float64).T
    assert np.max(np.abs(y - ref)) <= 1e-5 * np.max(np.abs(ref))


def test_group_properties():
    rng = np.random.default_rng(3)
    inds = rng.integers(0, 64, 4 * 37).astype(np.uint32)
    order, starts, experts, nseg = O.group(inds, 64)
    assert sorted(order.tolist()) == list(range(inds.size))
    for s in range(nseg):
        seg = order[starts[s]:starts[s + 1]]
        assert np.all(inds[seg] == experts[s]) and np.all(np.diff(seg) > 0)
    assert np.all(np.diff(experts[:nseg]) > 0)


def test_bf16_rounding_ties_to_even():
    # 1 + 2^-8 is halfway between bf16 1.0 and 1 + 2^-7: ties to even -> 1.0
    assert O.round_to(np.array([1.0 + 2**-8], np.float32), "bfloat16")[0] == 1.0
    assert O.round_to(np.array([1.0 + 3 * 2**-8], np.float32), "bfloat16")[0] == 1.0 + 2**-6
    v = np.float32(65520.0)
    assert np.isinf(O.round_to(np.array([v]), "float16")[0])
    sub = np.float32(3 * 2**-25)  # fp16 subnormal halfway: ties to even
    assert O.round_to(np.array([sub]), "float16")[0] == np.float32(2 * 2**-24)
