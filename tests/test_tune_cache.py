"""The tuner's cache and crash safety on the CPU (the reference's tests/test_tune_cache.py,
tests/test_kernel_patching.py:55-65 and tests/test_background_tune.py:129-160 restated for locals_b200.tune):
merged saves, crash markers and the pin after two deaths, a SIGTERM that is not a crash, temporaries of killed
saves, a cut-short cache set aside, stale choices after a library rebuild, the 10% margin rule and the GPU-busy
heartbeat. Failures are made on the host (dead child processes, a signal); nothing here touches a GPU."""

import json
import os
import signal
import subprocess
import sys
import time

import pytest
import torch

from locals_b200 import tune

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture
def cache(tmp_path, monkeypatch):
    path = tmp_path / "tune.json"
    monkeypatch.setenv("LQ_TUNE_CACHE", str(path))
    monkeypatch.setenv("LQ_BUSY_DIR", str(tmp_path / "busy"))
    monkeypatch.setattr(tune, "_LOADED", False)
    monkeypatch.setattr(tune, "_CHOICE", {})
    monkeypatch.setattr(tune, "_TIMES", {})
    monkeypatch.setattr(tune, "_CRASHED", {})
    monkeypatch.setattr(tune, "_STALE", set())
    monkeypatch.setattr(tune, "_STOPPING", False)
    monkeypatch.setattr(tune, "lib_version", lambda: "v2")
    return path


def _dead_pid():
    p = subprocess.Popen(["true"])
    p.wait()
    return p.pid


def _args(M=8, N=2560, K=4096):
    x = torch.zeros((M, K), dtype=torch.bfloat16)
    w = torch.zeros((N, K // 8), dtype=torch.int32)
    s = torch.zeros((N, K // 64), dtype=torch.bfloat16)
    return x, w, s, s


def test_a_save_keeps_what_another_process_wrote(cache):
    tune._load()
    tune._CHOICE["2560x4096x8xbfloat16"] = ("qmvg", 2, 0)
    tune._TIMES["2560x4096x8xbfloat16"] = 0.010
    cache.write_text(json.dumps({"9216x2560x8xbfloat16": ["qmv", 1, 2, 1, 0],
                                 "__times__": {"9216x2560x8xbfloat16": 0.020}, "__lib__": "v2"}))  # another process
    tune.save()
    data = json.loads(cache.read_text())
    assert data["2560x4096x8xbfloat16"] == ["qmvg", 2, 0] and data["9216x2560x8xbfloat16"] == ["qmv", 1, 2, 1, 0]
    assert set(data["__times__"]) == {"2560x4096x8xbfloat16", "9216x2560x8xbfloat16"}
    assert tune.lookup(9216, 2560, 8, torch.bfloat16) == ("qmv", 1, 2, 1, 0)  # the other's results are used now


def test_the_marker_names_the_shape_while_it_is_timed(cache, monkeypatch):
    seen = []

    def timing(*a):
        seen.append(open(tune._marker(os.getpid())).read())
        return ("qmvg", 0, 0), 0.01

    monkeypatch.setattr(tune, "_time_shape", timing)
    assert tune.choose(*_args()) == ("qmvg", 0, 0)
    assert seen == ["2560x4096x8xbfloat16"] and not os.path.exists(tune._marker(os.getpid()))


def test_a_shape_that_stops_the_process_twice_keeps_the_library_choice(cache, monkeypatch):
    key = "2560x4096x8xbfloat16"
    pid = _dead_pid()
    for deaths in (1, 2):
        monkeypatch.setattr(tune, "_LOADED", False)
        monkeypatch.setattr(tune, "_CRASHED", {})
        monkeypatch.setattr(tune, "_CHOICE", {})
        (cache.parent / f"tune.json.tuning-{pid}").write_text(key)
        tune._load()
        assert tune.crash_count(key) == deaths and not list(cache.parent.glob("*.tuning-*"))
        assert (tune.lookup(2560, 4096, 8, torch.bfloat16) == tune.AUTO) == (deaths == 2)
    data = json.loads(cache.read_text())
    assert data[key] == ["auto"] and data["__crashed__"] == {key: 2}
    # pinned: never timed again
    monkeypatch.setattr(tune, "_time_shape", lambda *a: pytest.fail("a pinned shape was timed"))
    assert tune.choose(*_args()) == tune.AUTO
    # a process still timing: its marker is left alone
    monkeypatch.setattr(tune, "_LOADED", False)
    live = cache.parent / f"tune.json.tuning-{os.getppid()}"
    live.write_text("9216x2560x8xbfloat16")
    tune._load()
    assert tune.crash_count("9216x2560x8xbfloat16") == 0 and live.exists()


def test_a_stop_while_a_shape_is_timed_is_not_a_crash(tmp_path):
    child = (
        "import threading, time\n"
        "from locals_b200 import tune\n"
        "tune.install_sigterm_handler()\n"
        "tune._time_shape = lambda *a: time.sleep(60)\n"
        "threading.Thread(target=tune._tune_shape, args=('8x64x1', lambda: tune._time_shape()), daemon=True).start()\n"
        "time.sleep(0.5)\n"
        "print('timing', flush=True)\n"
        "time.sleep(60)\n")
    env = dict(os.environ, LQ_TUNE_CACHE=str(tmp_path / "tune.json"), LQ_BUSY_DIR=str(tmp_path / "busy"),
               PYTHONPATH=ROOT)
    p = subprocess.Popen([sys.executable, "-c", child], env=env, stdout=subprocess.PIPE, text=True)
    try:
        assert p.stdout.readline().strip() == "timing"
        assert (tmp_path / f"tune.json.tuning-{p.pid}").exists()
        p.send_signal(signal.SIGTERM)
        assert p.wait(timeout=60) == -signal.SIGTERM
        assert not list(tmp_path.glob("*.tuning-*"))
    finally:
        p.kill()


def test_a_process_killed_while_timing_leaves_its_marker(tmp_path, monkeypatch):
    """SIGKILL runs no cleanup: the marker stays and the next load counts the shape once."""
    child = (
        "import time\n"
        "from locals_b200 import tune\n"
        "tune._tune_shape('8x64x1', lambda: (print('timing', flush=True), time.sleep(60)))\n")
    env = dict(os.environ, LQ_TUNE_CACHE=str(tmp_path / "tune.json"), LQ_BUSY_DIR=str(tmp_path / "busy"),
               PYTHONPATH=ROOT)
    p = subprocess.Popen([sys.executable, "-c", child], env=env, stdout=subprocess.PIPE, text=True)
    try:
        assert p.stdout.readline().strip() == "timing"
        p.kill()
        p.wait(timeout=30)
    finally:
        p.kill()
    assert (tmp_path / f"tune.json.tuning-{p.pid}").exists()
    monkeypatch.setenv("LQ_TUNE_CACHE", str(tmp_path / "tune.json"))
    monkeypatch.setattr(tune, "_LOADED", False)
    monkeypatch.setattr(tune, "_CRASHED", {})
    monkeypatch.setattr(tune, "_CHOICE", {})
    monkeypatch.setattr(tune, "lib_version", lambda: "v2")
    tune._load()
    assert tune.crash_count("8x64x1") == 1 and "8x64x1" not in tune._CHOICE


def test_a_save_a_killed_process_left_is_removed(cache):
    old, new = cache.parent / ".tune-old.json", cache.parent / ".tune-new.json"
    old.write_text("{}")
    new.write_text("{}")  # (another process saving right now)
    os.utime(old, (time.time() - 3600, time.time() - 3600))
    tune._load()
    assert not old.exists() and new.exists()


def test_a_cut_short_tuning_cache_is_set_aside(cache):
    cache.write_text('{"1x64x2": ["qmv", 1, 1, 1, 0], "2x64')
    assert tune.lookup(1, 64, 2, torch.float16) is None
    assert (cache.parent / "tune.json.bad").exists()
    tune.set_choice(3, 64, 2, torch.float16, 4, ("qmv", 1, 1, 1, 0))
    tune.save()
    data = json.loads(cache.read_text())
    assert data["3x64x2"] == ["qmv", 1, 1, 1, 0] and "1x64x2" not in data and data["__lib__"] == "v2"


def test_choices_timed_under_another_build_are_stale_until_timed_again(cache, monkeypatch):
    key = "2560x4096x8xbfloat16"
    cache.write_text(json.dumps({key: ["qmv", 1, 2, 1, 0], "__times__": {key: 0.02}, "__lib__": "v1"}))
    assert tune.lookup(2560, 4096, 8, torch.bfloat16) == ("qmv", 1, 2, 1, 0)  # still used
    assert tune.stale_keys() == [key]
    data = json.loads(cache.read_text())
    assert data["__lib__"] == "v2" and data["__stale__"] == [key]
    monkeypatch.setattr(tune, "_time_shape", lambda *a: (("qmvg", 0, 0), 0.01))
    inputs = {key: (*_args(), 4)}
    assert tune.retime_stale(inputs.get) == [key]
    assert tune.stale_keys() == [] and json.loads(cache.read_text())["__stale__"] == []
    assert tune.lookup(2560, 4096, 8, torch.bfloat16) == ("qmvg", 0, 0)


def test_a_cache_from_before_versions_gets_one_and_nothing_is_stale(cache):
    cache.write_text(json.dumps({"1024x512x1": ["qmv", 1, 1, 1, 0]}))
    tune._load()
    assert tune.stale_keys() == [] and json.loads(cache.read_text())["__lib__"] == "v2"


def test_a_challenger_must_beat_the_library_choice_by_ten_percent():
    a, b = ("qmvg", 2, 0), ("qmv", 1, 2, 1, 0)
    assert tune.pick({tune.AUTO: 10.0, a: 9.5, b: 9.2}) == tune.AUTO
    assert tune.pick({tune.AUTO: 10.0, a: 8.9, b: 9.2}) == a
    assert tune.pick({tune.AUTO: 10.0}) == tune.AUTO
    assert tune.pick({a: 1.0}) == a  # (no library time: any challenger)


def test_merge_keeps_both_processes_crash_counts_and_shared_stale_keys():
    mine = {"a": ["qmv"], "__crashed__": {"x": 1}, "__stale__": ["s1", "s2"], "__times__": {"a": 1.0}}
    theirs = {"b": ["tcv"], "__crashed__": {"x": 2, "y": 1}, "__stale__": ["s2", "s3"], "__times__": {"b": 2.0}}
    out = tune._merge(mine, theirs)
    assert out["a"] == ["qmv"] and out["b"] == ["tcv"]
    assert out["__crashed__"] == {"x": 2, "y": 1} and out["__stale__"] == ["s2"]
    assert out["__times__"] == {"a": 1.0, "b": 2.0}


def test_an_idle_tuner_leaves_its_shapes_while_another_process_is_busy(cache, monkeypatch):
    busy = cache.parent / "busy"
    busy.mkdir()
    dead = busy / f"busy-{_dead_pid()}"
    dead.write_text("")
    assert not tune.others_busy() and not dead.exists()  # a dead process's heartbeat goes
    other = busy / f"busy-{os.getppid()}"
    other.write_text("")
    assert tune.others_busy()
    key = "2560x4096x8xbfloat16"
    cache.write_text(json.dumps({key: ["qmv", 1, 2, 1, 0], "__lib__": "v1"}))
    monkeypatch.setattr(tune, "_time_shape", lambda *a: (("qmvg", 0, 0), 0.01))
    inputs = {key: (*_args(), 4)}
    assert tune.retime_stale(inputs.get) == [] and tune.stale_keys() == [key]  # left for later, not dropped
    os.utime(other, (time.time() - 10, time.time() - 10))
    assert not tune.others_busy()
    assert tune.retime_stale(inputs.get) == [key]
    tune.mark_busy(now=True)
    assert (busy / f"busy-{os.getpid()}").exists()
