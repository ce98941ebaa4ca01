"""Build ``libsf_engine.so`` (the engine's C ABI) in-tree with nvcc.

Every CUDA translation unit is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); nvcc cross-compiles without a
GPU.  Objects go to ``_build/`` at the repository root, the shared library
next to this file, where ``scaffolding_b200._lib`` loads it.

    python -m scaffolding_b200.build [--verbose-ptxas]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libsf_engine.so")

SOURCES = ["runtime.cu", "engine.cu", "attention.cu", "norm.cu", "noalloc.cu", "peer.cu",
           "comm.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _flags(verbose_ptxas: bool) -> list[str]:
    f = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", *ARCH, f"-I{os.path.join(ROOT, 'include')}"]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _local_includes(path: str, seen: set[str]) -> None:
    """Add `path` and, recursively, the files it #includes with quotes."""
    path = os.path.normpath(path)
    if path in seen or not os.path.exists(path):
        return
    seen.add(path)
    with open(path, errors="replace") as fh:
        for line in fh:
            line = line.strip()
            if line.startswith("#include") and '"' in line:
                name = line.split('"')[1]
                _local_includes(os.path.join(os.path.dirname(path), name), seen)


def _digest(paths: list[str], flags: list[str]) -> str:
    h = hashlib.sha256(" ".join(flags).encode())
    for p in sorted(paths):
        h.update(p.encode())
        with open(p, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def _tu_digest(src: str, flags: list[str]) -> str:
    deps: set[str] = set()
    _local_includes(os.path.join(CSRC, src), deps)
    return _digest(sorted(deps), flags)


def build(verbose_ptxas: bool = False, force: bool = False, quiet: bool = False) -> str:
    """Compile the translation units whose sources (or local headers) changed
    and relink the engine; return the library path."""
    nvcc = _nvcc()
    flags = _flags(verbose_ptxas)
    digests = {src: _tu_digest(src, flags) for src in SOURCES}
    digest = _digest([], flags + [digests[s] for s in SOURCES])
    stamp = LIB + ".sha256"
    if not force and os.path.exists(LIB) and os.path.exists(stamp):
        with open(stamp) as fh:
            if fh.read().strip() == digest:
                return LIB
    os.makedirs(BUILD, exist_ok=True)

    def compile_one(src: str) -> tuple[str, str]:
        obj = os.path.join(BUILD, src + ".o")
        ostamp = obj + ".sha256"
        if not force and not verbose_ptxas and os.path.exists(obj) and os.path.exists(ostamp):
            with open(ostamp) as fh:
                if fh.read().strip() == digests[src]:
                    return obj, ""
        cmd = [nvcc, *flags, "-c", os.path.join(CSRC, src), "-o", obj]
        if src.endswith(".cpp"):
            cmd = [nvcc, "-std=c++17", "-O3", "-Xcompiler", "-fPIC", *ARCH,
                   f"-I{os.path.join(ROOT, 'include')}", "-x", "cu", "-c",
                   os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        with open(ostamp, "w") as fh:
            fh.write(digests[src])
        return obj, r.stderr

    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    for _, log in results:
        if log.strip() and (verbose_ptxas or not quiet):
            sys.stderr.write(log)
    tmp = LIB + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *[o for o, _ in results], "-lcudart", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    with open(stamp, "w") as fh:
        fh.write(digest)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose_ptxas=a.verbose_ptxas, force=a.force))


if __name__ == "__main__":
    main()
