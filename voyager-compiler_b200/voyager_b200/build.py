"""Build ``libvoyager_b200.so`` in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` and ``csrc/*.cpp`` file is compiled to an object under
``_build/`` (in parallel, skipped when up to date) and linked into
``voyager_b200/libvoyager_b200.so``.  The CUDA runtime is linked statically,
so the library needs only the driver at run time.  No fast-math: the
numerics rely on IEEE division and round-to-nearest-even.
"""

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
PROJ = os.path.dirname(PKG)
ROOT = os.path.dirname(PROJ)
CSRC = os.path.join(PROJ, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
OUT = os.path.join(PKG, "libvoyager_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off",
          f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    out = []
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cpp")):
            out.append(os.path.join(CSRC, f))
    return out


def _headers_mtime():
    ts = [os.path.getmtime(os.path.join(INCLUDE, f)) for f in os.listdir(INCLUDE)]
    ts += [os.path.getmtime(os.path.join(CSRC, f)) for f in os.listdir(CSRC)
           if f.endswith((".cuh", ".h", ".hpp", ".inc"))]
    return max(ts) if ts else 0.0


def _compile(src: str, verbose: bool, extra) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if (os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(src)
            and os.path.getmtime(obj) >= _headers_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *COMMON, *extra, "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd[1:1] = ["-x", "c++"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, extra=()) -> str:
    """Compile and link; returns the path of the shared object."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max(1, min(len(srcs), os.cpu_count() or 4))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, list(extra)), srcs))
    newest = max(os.path.getmtime(o) for o in objs)
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= newest:
        return OUT
    cmd = [nvcc(), *ARCH, "-shared", "-o", OUT + ".tmp", *objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose=True))
