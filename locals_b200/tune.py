"""Per-shape kernel choice with a crash-safe JSON cache (the analogue of the reference's tuner,
locals/kernels.py:594-740, and its cache handling, locals/kernels.py:178-486).

``choose(...)`` times every candidate of a shape on weight copies whose total exceeds the L2 cache
(the reference times over >= 64 MB of copies for the same reason, locals/kernels.py:687-699), keeps
only candidates whose output matches the library's own choice within 0.05 * (1 + max|ref|) (the
reference's correctness gate, locals/kernels.py:675-686), and records a challenger only when it beats
the library's own choice by 10% (the reference's margin over MLX, locals/kernels.py:734). Calls are
timed chained: back to back on one stream inside a CUDA graph, each call's grid waiting on the one
before, as a model's layers wait on each other (locals/kernels.py:703-718). The choice is stored under
the key ``NxKxM[xdtype][xbBITS]`` (locals/kernels.py:606). ``lookup`` is the hot-path read: a dict hit,
no I/O.

Crash safety, as the reference's cache has it:
  * while a shape is timed, a marker file ``<cache>.tuning-<pid>`` names it; a process that dies there
    leaves the marker, and the next load counts the shape in ``__crashed__``; a shape that stopped a
    process twice is pinned to the library's own choice ("auto",) and never timed again
    (locals/kernels.py:403-434,624-646). ``stop_timing`` (SIGTERM) removes the marker first, so a stop is
    not a crash (locals/kernels.py:368-378);
  * every save merges with the file as it is now under an ``flock`` and replaces it atomically (fsync'd
    temporary, rename), so two processes tuning at once keep each other's results (locals/kernels.py:
    439-486); temporaries a killed save left are removed after ten minutes (locals/kernels.py:392-400);
  * a cache that does not parse (a write cut short) is set aside as ``<cache>.bad``, not silently
    replaced (locals/kernels.py:254-280);
  * the cache records the kernel library's version (``__lib__``, the hash of the sources liblq.so was
    built from); choices timed under another version are ``__stale__``: still used, and timed again by
    ``retime_stale`` or the next ``choose`` (locals/kernels.py:178-197);
  * processes working on the GPU touch a heartbeat file once a second (``mark_busy``); an idle tuner
    leaves its shapes while another process is busy (``others_busy``, locals/kernels.py:301-365).
"""

from __future__ import annotations

import atexit
import fcntl
import glob
import json
import os
import re
import signal
import sys
import tempfile
import threading
import time
from typing import Callable, Optional

import torch

_LOCK = threading.RLock()
_CHOICE: dict = {}   # key -> choice tuple
_TIMES: dict = {}    # key -> ms per call of the chosen candidate (the cache's "__times__")
_CRASHED: dict = {}  # key -> processes that died while timing it (the cache's "__crashed__")
_STALE: set = set()  # keys timed under another library version (the cache's "__stale__")
_LOADED = False

AUTO = ("auto",)     # the library's own choice (lq_qmm with LQ_FAM_AUTO)
MARGIN = 0.9         # a challenger must run in under 90% of the library's own choice's time
_SHAPE_KEY = re.compile(r"\d+x\d+x\d+(x[a-z0-9]+)*")


def cache_path() -> str:
    return os.environ.get("LQ_TUNE_CACHE") or os.path.join(os.path.expanduser("~"), ".cache", "locals_b200",
                                                          "tune_sm100.json")


def _key(N: int, K: int, M: int, dtype: torch.dtype, bits: int) -> str:
    dt = str(dtype).split(".")[-1]
    return f"{N}x{K}x{M}" + ("" if dt == "float16" else f"x{dt}") + ("" if bits == 4 else f"xb{bits}")


def lib_version() -> str:
    """The kernel library's version for the cache: the hash of the sources liblq.so was built from (recorded
    beside it by the build), else its size and modification time."""
    from . import _lib

    try:
        with open(_lib.LIB_PATH + ".srchash") as f:
            return f.read().strip()[:16]
    except OSError:
        pass
    try:
        st = os.stat(_lib.LIB_PATH)
        return f"{st.st_size:x}-{int(st.st_mtime):x}"
    except OSError:
        return "unknown"


# ---- reading and writing the cache ------------------------------------------------------------------

def _read(path: str) -> dict:
    with open(path) as f:
        data = json.load(f)
    if not isinstance(data, dict):
        raise ValueError("the tuning cache is not a JSON object")
    return data


def _from_file(data: dict) -> tuple:
    """(choices, times, crashed, stale) held in a cache file's dict."""
    choices = {k: tuple(v) for k, v in data.items()
               if not k.startswith("__") and isinstance(v, list) and v and isinstance(v[0], str)}
    t = data.get("__times__")
    times = {k: float(v) for k, v in t.items() if isinstance(v, (int, float))} if isinstance(t, dict) else {}
    c = data.get("__crashed__")
    crashed = {k: int(v) for k, v in c.items() if isinstance(v, int)} if isinstance(c, dict) else {}
    s = data.get("__stale__")
    stale = {k for k in s if isinstance(k, str)} if isinstance(s, list) else set()
    return choices, times, crashed, stale


def _to_file() -> dict:
    data = {k: list(v) for k, v in _CHOICE.items()}
    data["__times__"] = dict(_TIMES)
    if _CRASHED:
        data["__crashed__"] = dict(_CRASHED)
    data["__stale__"] = sorted(_STALE)
    data["__lib__"] = lib_version()
    return data


def _load() -> None:
    """Read the cache once: set a file that does not parse aside, mark choices of another library version
    stale, count the shapes dead processes were timing, drop temporaries of killed saves."""
    global _LOADED
    with _LOCK:
        if _LOADED:
            return
        _LOADED = True
        path = cache_path()
        user = None
        if os.path.exists(path):
            try:
                user = _read(path)
            except (OSError, ValueError):
                try:
                    os.replace(path, path + ".bad")  # (a write cut short: kept for a look, not overwritten)
                except OSError:
                    pass
        changed = False
        if user is not None:
            choices, times, crashed, stale = _from_file(user)
            _CHOICE.update(choices)
            _TIMES.update(times)
            _CRASHED.update(crashed)
            _STALE.update(stale)
            was, now = user.get("__lib__"), lib_version()
            if was != now:
                # a cache from before versions were recorded gets one; choices of another build are stale
                if was is not None:
                    _STALE.update(k for k in _CHOICE if _SHAPE_KEY.fullmatch(k))
                changed = True
        changed = _crashed_shapes() or changed
        _drop_old_temps()
        if changed:
            try:
                save()
            except OSError:
                pass


def lookup(N: int, K: int, M: int, dtype: torch.dtype, bits: int = 4) -> Optional[tuple]:
    """The recorded choice for this shape (stale ones included: they are used until timed again)."""
    if not _LOADED:
        _load()
    return _CHOICE.get(_key(N, K, M, dtype, bits))


def best_time(N: int, K: int, M: int, dtype: torch.dtype, bits: int = 4) -> Optional[float]:
    """ms per call of the tuned choice for this shape, if the tuner has timed it (pad_rows reads it)."""
    if not _LOADED:
        _load()
    return _TIMES.get(_key(N, K, M, dtype, bits))


def stale_keys() -> list:
    """Shapes whose choice was timed under another build of the kernel library."""
    if not _LOADED:
        _load()
    return sorted(_STALE)


def crash_count(key: str) -> int:
    if not _LOADED:
        _load()
    return _CRASHED.get(key, 0)


def _merge(mine: dict, theirs: dict) -> dict:
    """Two caches as one: ``mine`` wins a key both have; the timings and crash counts are merged entry by
    entry; a shape stays stale only if both call it stale (a process that timed it again took it off)."""
    out = dict(theirs)
    for k, v in mine.items():
        w = out.get(k)
        if k == "__crashed__" and isinstance(w, dict):
            out[k] = {kk: max(int(w.get(kk, 0)), int(vv)) for kk, vv in {**w, **v}.items()}
        elif isinstance(v, dict) and isinstance(w, dict):
            out[k] = {**w, **v}
        elif k == "__stale__" and isinstance(w, list):
            out[k] = [x for x in w if x in v]
        else:
            out[k] = v
    return out


def save() -> None:
    """Merge this process's cache with the file as it is now, under an exclusive flock, and replace the file
    atomically (an fsync'd temporary renamed over it); this process then uses the other's keys too."""
    with _LOCK:
        path = cache_path()
        d = os.path.dirname(path) or "."
        os.makedirs(d, exist_ok=True)
        with open(path + ".lock", "w") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            try:
                theirs = _read(path) if os.path.exists(path) else {}
            except (OSError, ValueError):
                theirs = {}  # (a file that does not parse: ours replaces it)
            data = _merge(_to_file(), theirs)
            choices, times, crashed, stale = _from_file(data)
            for k, v in choices.items():
                _CHOICE.setdefault(k, v)
            for k, v in times.items():
                _TIMES.setdefault(k, v)
            _CRASHED.update(crashed)
            _STALE.intersection_update(stale)
            fd, tmp = tempfile.mkstemp(dir=d, prefix=".tune-", suffix=".json")
            try:
                with os.fdopen(fd, "w") as f:
                    json.dump(data, f, indent=1, sort_keys=True)
                    f.flush()
                    os.fsync(f.fileno())  # (renamed after a power cut, an unsynced file could come back empty)
                os.replace(tmp, path)
            except BaseException:
                try:
                    os.unlink(tmp)
                except OSError:
                    pass
                raise


def set_choice(N: int, K: int, M: int, dtype: torch.dtype, bits: int, choice: tuple) -> None:
    with _LOCK:
        key = _key(N, K, M, dtype, bits)
        _CHOICE[key] = tuple(choice)
        _STALE.discard(key)


# ---- crash markers -------------------------------------------------------------------------------

_MARKER_LOCK = threading.Lock()
_STOPPING = False


def _marker(pid: int) -> str:
    return f"{cache_path()}.tuning-{pid}"


def _alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except OSError:  # (another user's process)
        return True
    return True


def _crashed_shapes() -> bool:
    """Shapes dead processes were timing (their marker files are left: a kernel fault that kills the process
    runs no cleanup). Each counts in ``__crashed__``; a shape that stopped a process twice keeps the library's
    own choice (it would be timed again, and stop the process again, at every start); one death (a kill, a power
    cut) only times it again. Whether anything changed."""
    changed = False
    for m in glob.glob(glob.escape(cache_path()) + ".tuning-*"):
        try:
            pid = int(m.rsplit("-", 1)[1])
            with open(m) as f:
                key = f.read().strip()
        except (ValueError, OSError):
            continue
        if pid == os.getpid() or _alive(pid):
            continue
        try:
            os.unlink(m)
        except OSError:
            continue  # (another process took it)
        if not key:
            continue
        _CRASHED[key] = _CRASHED.get(key, 0) + 1
        changed = True
        if _CRASHED[key] >= 2:
            _CHOICE[key] = AUTO
            _STALE.discard(key)
            print(f"locals_b200: timing the kernels of shape {key} stopped a process twice; that shape keeps the "
                  f"library's own kernel choice", file=sys.stderr, flush=True)
    return changed


def _drop_old_temps() -> None:
    """Temporaries that killed saves left (a save takes well under a second: one ten minutes old is no live save)."""
    d = os.path.dirname(cache_path()) or "."
    for t in glob.glob(os.path.join(glob.escape(d), ".tune-*.json")):
        try:
            if time.time() - os.path.getmtime(t) > 600:
                os.unlink(t)
        except OSError:
            pass


def stop_timing() -> None:
    """This process is being stopped (SIGTERM): its marker goes and no new one is written, so the shape it was
    timing does not count as one that crashed."""
    global _STOPPING
    with _MARKER_LOCK:
        _STOPPING = True
        try:
            os.unlink(_marker(os.getpid()))
        except OSError:
            pass


def install_sigterm_handler() -> None:
    """On SIGTERM: stop_timing, then die by SIGTERM as before (the previous handler, or the default action)."""
    prev = signal.getsignal(signal.SIGTERM)

    def on_term(signum, frame):
        stop_timing()
        if callable(prev):
            prev(signum, frame)
            return
        signal.signal(signal.SIGTERM, signal.SIG_DFL)
        os.kill(os.getpid(), signal.SIGTERM)

    signal.signal(signal.SIGTERM, on_term)


def _tune_shape(key: str, fn: Callable[[], tuple]) -> tuple:
    """fn() (the timing of one shape) with the shape named in this process's marker file while it runs."""
    marker = _marker(os.getpid())
    with _MARKER_LOCK:
        try:
            if _STOPPING:
                raise OSError
            os.makedirs(os.path.dirname(marker) or ".", exist_ok=True)
            with open(marker, "w") as f:
                f.write(key)
                f.flush()
                os.fsync(f.fileno())
        except OSError:
            marker = None
    mark_busy(now=True)
    try:
        return fn()
    finally:
        if marker:
            try:
                os.unlink(marker)
            except OSError:
                pass


# ---- GPU-busy heartbeat between processes --------------------------------------------------------

_BUSY_AT = 0.0


def _busy_dir() -> str:
    return os.environ.get("LQ_BUSY_DIR") or os.path.join(tempfile.gettempdir(), "locals_b200-gpu")


def _busy_file(pid: int) -> str:
    return os.path.join(_busy_dir(), f"busy-{pid}")


def mark_busy(now: bool = False) -> None:
    """This process works on the GPU: its heartbeat file is touched (at most once a second unless ``now``)."""
    global _BUSY_AT
    t = time.time()
    if not now and t - _BUSY_AT < 1.0:
        return
    _BUSY_AT = t
    path = _busy_file(os.getpid())
    try:
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "a"):
            pass
        os.utime(path, None)
    except OSError:
        pass


def others_busy(window: float = 3.0) -> bool:
    """Whether another live process marked the GPU busy in the last ``window`` seconds (a dead one's file goes)."""
    t = time.time()
    for f in glob.glob(os.path.join(glob.escape(_busy_dir()), "busy-*")):
        try:
            pid = int(f.rsplit("-", 1)[1])
        except ValueError:
            continue
        if pid == os.getpid():
            continue
        if not _alive(pid):
            try:
                os.unlink(f)
            except OSError:
                pass
            continue
        try:
            if t - os.path.getmtime(f) < window:
                return True
        except OSError:
            pass
    return False


def _drop_busy() -> None:
    try:
        os.unlink(_busy_file(os.getpid()))
    except OSError:
        pass


atexit.register(_drop_busy)


# ---- timing ----------------------------------------------------------------------------------------

def _chain_ms(calls: Callable[[], None], n: int, rounds: int = 3) -> float:
    """ms per call of ``calls()`` (n calls back to back on one stream), captured once in a CUDA graph and
    replayed: each call's grid waits on the one before, as in a model's step; best of ``rounds`` replays."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        calls()  # (warm: kernel attributes are set outside the capture)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            calls()
        g.replay()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(rounds):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1) / n)
    del g
    return best


def pick(times: dict) -> tuple:
    """The recorded choice from candidate times (ms): the fastest challenger if it beats the library's own choice
    by the margin, else the library's own choice (locals/kernels.py:731-736)."""
    base = times.get(AUTO, float("inf"))
    challengers = {c: t for c, t in times.items() if c != AUTO}
    if not challengers:
        return AUTO
    best = min(challengers, key=challengers.get)
    return best if challengers[best] < MARGIN * base else AUTO


def _time_shape(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int,
                group_size: int, reps: int, l2_bytes: int) -> tuple:
    """(choice, ms): every candidate gated against the library's own choice, timed chained over weight copies."""
    from . import kernels

    M, K = x.shape[0], x.shape[-1]
    N = w.shape[0]
    ref = kernels.quantized_matmul(x, w, scales, biases, group_size=group_size, bits=bits).float()
    tol = 0.05 * (1.0 + float(ref.abs().max()))
    nbytes = w.numel() * 4 + scales.numel() * 2 * 2
    ncopy = max(1, min(32, l2_bytes // max(nbytes, 1)))
    copies = [(w.clone(), scales.clone(), biases.clone()) for _ in range(ncopy)]
    ok = [AUTO]
    for c in kernels.candidates(M, K, N, bits, x.dtype):
        try:
            got = kernels.quantized_matmul(x, w, scales, biases, group_size=group_size, bits=bits, choice=c).float()
        except kernels._lib.LQError:
            continue
        if float((got - ref).abs().max()) <= tol:  # (a NaN fails too)
            ok.append(c)
    times = {}
    n = reps * ncopy
    for c in ok:
        f = kernels.launch(c, M, K, N, x.dtype, bits, group_size)

        def calls(f=f):
            for i in range(n):
                f(x, *copies[i % ncopy])

        times[c] = _chain_ms(calls, n)
    del copies
    choice = pick(times)
    return choice, times[choice]


def choose(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int = 4,
           group_size: int = 64, reps: int = 20, l2_bytes: int = 256 << 20, persist: bool = False) -> tuple:
    """Time the candidates of this shape and record the choice (a shape that stopped a process twice keeps the
    library's own choice untimed)."""
    if not _LOADED:
        _load()
    M, K = x.shape[0], x.shape[-1]
    N = w.shape[0]
    key = _key(N, K, M, x.dtype, bits)
    if _CRASHED.get(key, 0) >= 2:
        set_choice(N, K, M, x.dtype, bits, AUTO)
        return AUTO
    choice, ms = _tune_shape(key, lambda: _time_shape(x, w, scales, biases, bits, group_size, reps, l2_bytes))
    set_choice(N, K, M, x.dtype, bits, choice)
    with _LOCK:
        _TIMES[key] = ms
    if persist:
        save()
    return choice


def retime_stale(make_inputs: Callable[[str], Optional[tuple]], persist: bool = True,
                 skip_if_busy: bool = True) -> list:
    """Time again the stale shapes ``make_inputs(key)`` gives inputs for ((x, w, scales, biases, bits) or None).
    Leaves them for later while another process marks the GPU busy. Returns the keys timed."""
    done = []
    for key in stale_keys():
        if skip_if_busy and others_busy():
            break
        inp = make_inputs(key)
        if inp is None:
            continue
        x, w, s, b, bits = inp
        choose(x, w, s, b, bits=bits, persist=persist)
        done.append(key)
    return done
