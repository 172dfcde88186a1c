"""The tuner on the GPU (the analogue of the reference's _time_shape / _tune_prefill, locals/kernels.py:649-740,
872-898): every candidate of a shape passes the correctness gate or is dropped, the fastest is recorded, persisted to
the JSON cache and read back by lookup; the recorded choice computes the same result as the oracle. Covers a decode
shape (qmv / qmvg / tcv candidates) and a prefill shape (tc, tcv and the dense dequantize + GEMM path)."""

import json

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, act, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(4, 768, 2560), (512, 448, 1024)])
def test_choose_records_a_correct_candidate(cuda, tmp_path, monkeypatch, M, N, K):
    import torch
    from locals_b200 import kernels, tune

    monkeypatch.setenv("LQ_TUNE_CACHE", str(tmp_path / "tune.json"))
    monkeypatch.setattr(tune, "_LOADED", True)
    monkeypatch.setattr(tune, "_CHOICE", {})
    monkeypatch.setattr(tune, "_TIMES", {})
    monkeypatch.setattr(tune, "_CRASHED", {})
    monkeypatch.setattr(tune, "_STALE", set())
    rng = np.random.default_rng(M + N)
    wq, s, b = qweights(rng, N, K, 4, "bfloat16")
    x = act(rng, M, K, "bfloat16")
    tw, ts, tb = to_torch(wq, s, b, "bfloat16", cuda)
    xt = x_torch(x, "bfloat16", cuda)
    best = tune.choose(xt, tw, ts, tb, bits=4, reps=3, l2_bytes=16 << 20, persist=True)
    # a challenger only when 10% faster than the library's own choice ("auto")
    assert best == tune.AUTO or best in kernels.candidates(M, K, N, 4, torch.bfloat16)
    assert tune.lookup(N, K, M, torch.bfloat16) == best
    data = json.loads((tmp_path / "tune.json").read_text())
    key = tune._key(N, K, M, torch.bfloat16, 4)
    assert tuple(data[key]) == best and key in data["__times__"] and data["__lib__"] == tune.lib_version()
    assert not list(tmp_path.glob("*.tuning-*"))  # the crash marker is gone after the timing
    y = kernels.quantized_matmul(xt, tw, ts, tb, choice=best)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    ref = O.round_to(O.qmm(x, wq, s, b), "bfloat16")
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL
