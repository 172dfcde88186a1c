"""The steps either side of the projections, on the CPU: the oracle's residual add + RMS norm and MoE
combine + norm (known answers), row packing's indices and the padding rule (no GPU needed)."""

import numpy as np

from oracle import oracle as O


def test_add_rms_known_answer():
    # x + r = [3, 4] -> mean square 12.5 -> n = h / sqrt(12.5) * w exactly representable inputs
    x = np.array([[1.0, 2.0]], np.float32)
    r = np.array([[2.0, 2.0]], np.float32)
    w = np.array([1.0, 2.0], np.float32)
    h, n = O.add_rms(x, r, w, 0.0, "bfloat16")
    assert np.array_equal(h, [[3.0, 4.0]])
    inv = 1.0 / np.sqrt(np.float32(12.5))
    ref = [O.round_to(np.float32(1.0) * O.round_to(np.float32(3.0 * inv), "bfloat16"), "bfloat16"),
           O.round_to(np.float32(2.0) * O.round_to(np.float32(4.0 * inv), "bfloat16"), "bfloat16")]
    assert np.allclose(n[0], np.array(ref, np.float32).ravel(), rtol=0, atol=0)


def test_add_rms_matches_float64_within_rounding():
    rng = np.random.default_rng(0)
    x = O.round_to(rng.standard_normal((4, 2560)).astype(np.float32), "bfloat16")
    r = O.round_to(rng.standard_normal((4, 2560)).astype(np.float32), "bfloat16")
    w = O.round_to((1 + 0.1 * rng.standard_normal(2560)).astype(np.float32), "bfloat16")
    h, n = O.add_rms(x, r, w, 1e-6, "bfloat16")
    assert np.array_equal(h, O.round_to(x + r, "bfloat16"))
    h64 = h.astype(np.float64)
    ref = h64 / np.sqrt((h64 ** 2).mean(axis=1, keepdims=True) + 1e-6) * w
    assert np.max(np.abs(n - ref) / (np.abs(ref) + 1e-3)) < 2 ** -6


def test_combine_norm_is_combine_plus_add_rms():
    rng = np.random.default_rng(1)
    T, k, D = 3, 4, 256
    ys = O.round_to(rng.standard_normal((T * k, D)).astype(np.float32), "bfloat16")
    wt = rng.random((T, k)).astype(np.float32)
    res = O.round_to(rng.standard_normal((T, D)).astype(np.float32), "bfloat16")
    nw = O.round_to((1 + 0.1 * rng.standard_normal(D)).astype(np.float32), "bfloat16")
    y, n = O.combine_norm(ys, wt, res, nw, 1e-5, "bfloat16")
    c = O.round_to(O.combine(ys, wt), "bfloat16")
    h, n2 = O.add_rms(res, c, nw, 1e-5, "bfloat16")  # res + c adds in the same order as res + combine
    assert np.array_equal(y, h) and np.array_equal(n, n2)
    sh = O.round_to(rng.standard_normal((T, D)).astype(np.float32), "bfloat16")
    y2, _ = O.combine_norm(ys, wt, res, nw, 1e-5, "bfloat16", shared=sh)
    assert np.array_equal(y2, O.round_to(res + O.round_to(c + sh, "bfloat16"), "bfloat16"))


def test_packed_rows_indices_and_padding_rule(monkeypatch):
    import torch

    from locals_b200 import kernels, tune

    p = kernels.packed_rows(3, 4, [2, 0, 4], device="cpu")
    B, L, idx, R = p.ctx
    assert (B, L, R) == (3, 4, 6) and idx.tolist() == [0, 1, 8, 9, 10, 11]
    # padding: 12 rows pad to 16 when the tuner timed 16 rows >= 7% faster (locals/kernels.py:764-794)
    monkeypatch.setattr(tune, "_LOADED", True)
    monkeypatch.setattr(tune, "_TIMES", {tune._key(4096, 2560, 12, torch.bfloat16, 4): 10.0,
                                         tune._key(4096, 2560, 16, torch.bfloat16, 4): 9.0,
                                         tune._key(4096, 2560, 14, torch.bfloat16, 4): 9.5})
    assert kernels.pad_rows(4096, 2560, 12, torch.bfloat16) == 16
    assert kernels.pad_rows(4096, 2560, 5, torch.bfloat16) == 5        # outside 8..16: never
    monkeypatch.setenv("LOCALS_PAD_ROWS", "0")
    assert kernels.pad_rows(4096, 2560, 12, torch.bfloat16) == 12
