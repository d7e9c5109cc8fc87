"""Build ``libsilogic_b200.so`` (all CUDA kernels + the C ABI) for sm_100a, in-tree.

    python -m silogic_b200.build [--force] [-j N]

Each ``csrc/*.cu`` is compiled to ``_build/*.o`` with nvcc (only when the source,
a header, or the flags changed), then linked into ``silogic_b200/libsilogic_b200.so``.
No torch headers are involved: the library is a plain C ABI (``include/silogic_b200.h``).
"""
import argparse
import concurrent.futures as cf
import glob
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libsilogic_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", INCLUDE, "-I", CSRC]


def _nvcc():
    for c in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _includes(path, seen):
    """Local headers a source includes, transitively."""
    import re
    with open(path) as f:
        for name in re.findall(r'#include\s+"([^"]+)"', f.read()):
            for d in (os.path.dirname(path), CSRC, INCLUDE):
                q = os.path.join(d, name)
                if os.path.exists(q) and q not in seen:
                    seen.add(q)
                    _includes(q, seen)
                    break
    return seen


def _deps_digest(src):
    h = hashlib.sha1(" ".join(ARCH + FLAGS).encode())
    for p in sorted(_includes(src, set())):
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def _compile(src, force, digest, extra):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    stamp = obj + ".stamp"
    with open(src, "rb") as f:
        key = hashlib.sha1(f.read() + digest.encode() + " ".join(extra).encode()).hexdigest()
    if not force and os.path.exists(obj) and os.path.exists(stamp) and open(stamp).read() == key:
        return obj, None
    cmd = [_nvcc()] + ARCH + FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    with open(stamp, "w") as f:
        f.write(key)
    return obj, None


def build(force=False, jobs=8, verbose=False, extra=()):
    """Compile and link; returns the path of the shared library."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    extra = list(extra)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        res = list(ex.map(lambda s: _compile(s, force, _deps_digest(s), extra), srcs))
    errs = [e for _, e in res if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in res]
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [_nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/spill usage")
    a = ap.parse_args()
    try:
        build(a.force or a.ptxas_v, a.j, True, ["-Xptxas", "-v"] if a.ptxas_v else [])
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
