"""Per-shape kernel choice with a JSON cache (the analogue of the reference's tuner,
locals/kernels.py:594-740 and its cache handling 254-486).

``choose(...)`` times every candidate of a shape on weight copies whose total exceeds the L2 cache
(the reference times over >= 64 MB of copies for the same reason, locals/kernels.py:687-699), keeps
only candidates whose output matches the auto choice within 0.05 * (1 + max|ref|) (the reference's
correctness gate, locals/kernels.py:675-686), and stores the fastest under the key
``NxKxM[xdtype]`` (locals/kernels.py:606). The cache file is merged and replaced atomically.
``lookup`` is the hot-path read: a dict hit, no I/O.
"""

from __future__ import annotations

import json
import os
import tempfile
import threading
from typing import Optional

import torch

_LOCK = threading.RLock()
_CHOICE: dict = {}
_TIMES: dict = {}  # key -> ms per call of the chosen candidate (the cache's "__times__", as the reference keeps)
_LOADED = False


def cache_path() -> str:
    return os.environ.get("LQ_TUNE_CACHE") or os.path.join(os.path.expanduser("~"), ".cache", "locals_b200",
                                                          "tune_sm100.json")


def _key(N: int, K: int, M: int, dtype: torch.dtype, bits: int) -> str:
    dt = str(dtype).split(".")[-1]
    return f"{N}x{K}x{M}" + ("" if dt == "float16" else f"x{dt}") + ("" if bits == 4 else f"xb{bits}")


def _load() -> None:
    global _LOADED
    with _LOCK:
        if _LOADED:
            return
        _LOADED = True
        try:
            with open(cache_path()) as f:
                data = json.load(f)
        except (OSError, ValueError):
            return
        for k, v in data.items():
            if isinstance(v, list) and v and isinstance(v[0], str):
                _CHOICE[k] = tuple(v)
        times = data.get("__times__")
        if isinstance(times, dict):
            _TIMES.update({k: float(v) for k, v in times.items() if isinstance(v, (int, float))})


def lookup(N: int, K: int, M: int, dtype: torch.dtype, bits: int = 4) -> Optional[tuple]:
    if not _LOADED:
        _load()
    return _CHOICE.get(_key(N, K, M, dtype, bits))


def best_time(N: int, K: int, M: int, dtype: torch.dtype, bits: int = 4) -> Optional[float]:
    """ms per call of the tuned choice for this shape, if the tuner has timed it (pad_rows reads it)."""
    if not _LOADED:
        _load()
    return _TIMES.get(_key(N, K, M, dtype, bits))


def save() -> None:
    """Merge this process's choices into the cache file (atomic replace)."""
    with _LOCK:
        path = cache_path()
        os.makedirs(os.path.dirname(path), exist_ok=True)
        try:
            with open(path) as f:
                data = json.load(f)
        except (OSError, ValueError):
            data = {}
        data.update({k: list(v) for k, v in _CHOICE.items()})
        times = data.get("__times__") if isinstance(data.get("__times__"), dict) else {}
        times.update(_TIMES)
        data["__times__"] = times
        fd, tmp = tempfile.mkstemp(dir=os.path.dirname(path), suffix=".tmp")
        try:
            with os.fdopen(fd, "w") as f:
                json.dump(data, f, indent=1, sort_keys=True)
                f.flush()
                os.fsync(f.fileno())
            os.replace(tmp, path)
        except BaseException:
            try:
                os.unlink(tmp)
            except OSError:
                pass
            raise


def set_choice(N: int, K: int, M: int, dtype: torch.dtype, bits: int, choice: tuple) -> None:
    with _LOCK:
        _CHOICE[_key(N, K, M, dtype, bits)] = tuple(choice)


def choose(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int = 4,
           group_size: int = 64, reps: int = 20, l2_bytes: int = 256 << 20, persist: bool = False) -> tuple:
    """Time the candidates of this shape and record the fastest correct one."""
    from . import kernels

    M, K = x.shape[0], x.shape[-1]
    N = w.shape[0]
    ref = kernels.quantized_matmul(x, w, scales, biases, group_size=group_size, bits=bits).float()
    tol = 0.05 * (1.0 + float(ref.abs().max()))
    nbytes = w.numel() * 4 + scales.numel() * 2 * 2
    ncopy = max(1, min(32, l2_bytes // max(nbytes, 1)))
    copies = [(w.clone(), scales.clone(), biases.clone()) for _ in range(ncopy)]
    best, best_t = None, float("inf")
    for c in kernels.candidates(M, K, N, bits, x.dtype):
        try:
            got = kernels.quantized_matmul(x, w, scales, biases, group_size=group_size, bits=bits, choice=c).float()
        except kernels._lib.LQError:
            continue
        if not float((got - ref).abs().max()) <= tol:
            continue
        f = kernels.launch(c, M, K, N, x.dtype, bits, group_size)
        for cp in copies:
            f(x, *cp)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps * ncopy):
            f(x, *copies[i % ncopy])
        e1.record()
        e1.synchronize()
        t = e0.elapsed_time(e1) / (reps * ncopy)
        if t < best_t:
            best, best_t = c, t
    if best is None:
        raise RuntimeError("no candidate kernel passed the correctness gate")
    set_choice(N, K, M, x.dtype, bits, best)
    with _LOCK:
        _TIMES[_key(N, K, M, x.dtype, bits)] = best_t
    if persist:
        save()
    return best
