"""Build the in-tree CUDA library ``treeattn_b200/lib/libtreeattn_b200.so`` for sm_100a.

    python -m treeattn_b200.build [--force]

Plain ``nvcc -shared``: the library exposes only the C ABI of ``include/treeattn_b200.h``
and does not link against torch, so it builds in seconds and loads from any host language.
"""

from __future__ import annotations

import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libtreeattn_b200.so")
HEADER = os.path.join(ROOT, "include", "treeattn_b200.h")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _digest() -> str:
    h = hashlib.sha256()
    for f in sources() + [HEADER] + sorted(
            os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cuh")):
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _includes(path: str, seen: set[str]) -> None:
    """The csrc headers `path` includes, transitively."""
    with open(path) as fh:
        for line in fh:
            line = line.strip()
            if line.startswith("#include \""):
                name = line.split('"')[1]
                inc = os.path.normpath(os.path.join(os.path.dirname(path), name))
                if os.path.exists(inc) and inc not in seen:
                    seen.add(inc)
                    _includes(inc, seen)


def _object_digest(src: str) -> str:
    """Digest of one translation unit: its source, the headers it includes and the flags."""
    deps: set[str] = set()
    _includes(src, deps)
    h = hashlib.sha256()
    for f in [src] + sorted(deps):
        with open(f, "rb") as fh:
            h.update(fh.read())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every csrc/*.cu into one shared library (skipped when up to date).

    Object files are kept in lib/obj/ with the digest of their translation unit, so a change
    recompiles only the sources that see it."""
    os.makedirs(LIBDIR, exist_ok=True)
    objdir = os.path.join(LIBDIR, "obj")
    os.makedirs(objdir, exist_ok=True)
    stamp = LIB + ".sha256"
    digest = _digest()
    if not force and os.path.exists(LIB) and os.path.exists(stamp):
        with open(stamp) as fh:
            if fh.read().strip() == digest:
                return LIB
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        odig = _object_digest(src)
        objs.append(obj)
        if not force and os.path.exists(obj) and os.path.exists(obj + ".sha256"):
            with open(obj + ".sha256") as fh:
                if fh.read().strip() == odig:
                    continue
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT), src, obj, odig))
    for proc, src, obj, odig in procs:
        out, _ = proc.communicate()
        text = out.decode(errors="replace")
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{text}")
        if verbose and text.strip():
            print(text, file=sys.stderr)
        with open(obj + ".sha256", "w") as fh:
            fh.write(odig)
    tmp = LIB + ".tmp"
    link = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    with open(stamp, "w") as fh:
        fh.write(digest)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
