"""
Build recipe of the product library: every CUDA source in ragrt_b200/csrc compiled for
sm_100a into ragrt_b200/libragrt_b200.so (in-tree, so it travels with the repository
snapshot).  Exposes the C ABI declared in include/ragrt_b200.h.

    python -m ragrt_b200.build [--force] [-j N]
"""
import argparse
import concurrent.futures as cf
import glob
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libragrt_b200.so")
OBJ_DIR = os.path.join(REPO, "_build", "obj")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills", "-I" + os.path.join(REPO, "include")]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers_digest():
    h = hashlib.sha256()
    for f in sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(REPO, "include", "*.h"))):
        h.update(open(f, "rb").read())
    return h.hexdigest()[:16]


def _compile(src, force, verbose):
    os.makedirs(OBJ_DIR, exist_ok=True)
    h = hashlib.sha256(open(src, "rb").read() + _headers_digest().encode() + " ".join(FLAGS + ARCH).encode())
    obj = os.path.join(OBJ_DIR, os.path.basename(src) + "." + h.hexdigest()[:16] + ".o")
    if force or not os.path.exists(obj):
        cmd = [NVCC] + ARCH + FLAGS + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, file=sys.stderr)
    return obj


def build(force=False, jobs=None, verbose=False):
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), srcs))
    # Objects are cached by content, so a source put back to an earlier state reuses an older
    # object: relink whenever the set of objects differs from the one the library was linked from.
    stamp = os.path.join(OBJ_DIR, "libragrt_b200.objs")
    linked = open(stamp).read() if os.path.exists(stamp) else ""
    want = "\n".join(os.path.basename(o) for o in objs)
    if force or not os.path.exists(LIB) or linked != want:
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        with open(stamp, "w") as f:
            f.write(want)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))
