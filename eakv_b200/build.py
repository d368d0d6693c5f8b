"""Build recipe of libeakv_b200.so (sm_100a), in-tree.

    python -m eakv_b200.build            # compile what changed
    python -m eakv_b200.build --force    # recompile everything

Each csrc/*.cu is compiled by nvcc for sm_100a only (-gencode
arch=compute_100a,code=sm_100a) into _build/, then linked into
eakv_b200/libeakv_b200.so with the CUDA runtime linked statically, so the
library carries no dependency on a particular libcudart.so; NCCL is
resolved at run time (split.cu), so it is no link dependency either. The kernels
whose results must equal the reference bit for bit (quantize, the two-call
attention API, file I/O) are compiled with -fmad=false on top of the
explicit round-to-nearest intrinsics they already use.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libeakv_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-Wall",
          "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]
EXACT = {"quantize.cu", "attention.cu", "io.cu"}


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA library cannot be built")


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime():
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max(os.path.getmtime(p) for p in paths)


def _compile(src, force, extra):
    obj = os.path.join(BUILD, src[:-3] + ".o")
    srcp = os.path.join(CSRC, src)
    if (not force and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(srcp), _headers_mtime())):
        return obj, None
    flags = list(COMMON) + list(extra)
    if src in EXACT:
        flags.append("-fmad=false")
    cmd = [nvcc()] + ARCH + flags + ["-c", srcp, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, (" ".join(cmd) + "\n" + r.stdout + r.stderr)
    return obj, None


def build(force=False, verbose=False, extra=()):
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, force, extra), srcs))
    errors = [e for _, e in results if e]
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    objs = [o for o, _ in results]
    if (force or not os.path.exists(LIB)
            or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs + ["-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    if verbose:
        print(LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    if args.ptxas_info:
        os.makedirs(BUILD, exist_ok=True)
        for s in _sources():
            flags = list(COMMON) + extra + (["-fmad=false"] if s in EXACT else [])
            cmd = [nvcc()] + ARCH + flags + ["-c", os.path.join(CSRC, s), "-o", os.devnull]
            r = subprocess.run(cmd, capture_output=True, text=True)
            sys.stdout.write(r.stdout + r.stderr)
        return 0
    build(force=args.force, verbose=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
