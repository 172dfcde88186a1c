"""Build liblq.so (all CUDA kernels + the C ABI) for sm_100a, in-tree.

    python -m locals_b200.build            # or build() from __graft_entry__
    python -m locals_b200.build --force    # recompile every translation unit
    python -m locals_b200.build -v         # with ptxas register / spill / shared-memory reports

Each csrc/*.cu file is its own translation unit (compiled in parallel into csrc/../_build/*.o, then linked with the
static CUDA runtime). The library is rebuilt whenever the hash of its sources, headers and flags differs from the
one recorded beside it (liblq.so.srchash) -- never on file times alone, so a library left over from other sources
cannot stand in for a compile of these.
"""

from __future__ import annotations

import concurrent.futures
import glob
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "liblq.so")
HASH = LIB + ".srchash"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
HEADER = os.path.join(HERE, "..", "include", "lq.h")

FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def _units():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [HEADER])


def _digest(paths, extra=""):
    h = hashlib.sha256(extra.encode())
    for p in paths:
        h.update(os.path.basename(p).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def source_hash() -> str:
    """Hash of every source and header and of the compiler flags."""
    return _digest(_units() + _headers(), " ".join(FLAGS))


def up_to_date() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(HASH):
        return False
    with open(HASH) as f:
        return f.read().strip() == source_hash()


def _local_includes(path, seen=None):
    """The project headers a source includes, directly or through other project headers."""
    seen = set() if seen is None else seen
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line.startswith("#include \""):
                inc = os.path.normpath(os.path.join(os.path.dirname(path), line.split('"')[1]))
                if inc not in seen and os.path.exists(inc):
                    seen.add(inc)
                    _local_includes(inc, seen)
    return seen


def _compile(unit, verbose):
    """One translation unit -> _build/<name>.o (skipped when the hash of it, its headers and the flags matches)."""
    name = os.path.splitext(os.path.basename(unit))[0]
    obj = os.path.join(OBJ, name + ".o")
    tag = obj + ".hash"
    want = _digest([unit] + sorted(_local_includes(unit)), " ".join(FLAGS) + (" -v" if verbose else ""))
    if os.path.exists(obj) and os.path.exists(tag):
        with open(tag) as f:
            if f.read().strip() == want:
                return obj, ""
    cmd = [NVCC, *FLAGS, "-c", "-o", obj + ".tmp", unit]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(unit)}:\n{r.stdout}\n{r.stderr}")
    os.replace(obj + ".tmp", obj)
    with open(tag, "w") as f:
        f.write(want)
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not verbose and up_to_date():
        return LIB
    os.makedirs(OBJ, exist_ok=True)
    if force:
        for t in glob.glob(os.path.join(OBJ, "*.hash")):
            os.remove(t)
    units = _units()
    workers = max(1, min(len(units), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(workers) as ex:
        results = list(ex.map(lambda u: _compile(u, verbose), units))
    if verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static", "-o", LIB + ".tmp",
           *[o for o, _ in results]]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    with open(HASH, "w") as f:
        f.write(source_hash())
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
