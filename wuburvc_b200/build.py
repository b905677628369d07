"""Build recipe for the native library (nvcc, sm_100a).

``python -m wuburvc_b200.build`` compiles every CUDA / C++ source under ``csrc/`` into
``wuburvc_b200/libwuburvc_b200.so`` (in-tree, so it travels with the repository).
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libwuburvc_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> str:
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + [
        os.path.join(HERE, "..", "include", "wuburvc_b200.h")]
    if not force and not _stale(LIB, deps):
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        objs.append(obj)
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-x", "cu",
               "-I" + CSRC, "-I" + os.path.join(HERE, "..", "include"), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = False
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed = True
            sys.stderr.write(out.decode())
        elif verbose and out:
            sys.stderr.write(out.decode())
    if failed:
        raise RuntimeError("nvcc failed")
    cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    return LIB


SHIM_SRC = os.path.join(HERE, "shim", "wubu_train_b200.c")
SHIM_LIB = os.path.join(HERE, "shim", "libwubu_train_b200.so")


def build_shim(ref_src: str, ref_lib: str) -> str:
    """The drop-in shim compiled against the reference's own headers (``ref_src``) into a shared
    object that resolves this library and the reference's host objects (``ref_lib``) at load time
    through relative run paths, so it travels with the repository."""
    ref_dir = os.path.dirname(os.path.abspath(ref_lib))
    rel_ref = os.path.relpath(ref_dir, os.path.dirname(SHIM_LIB))
    cmd = ["gcc", "-std=gnu11", "-shared", "-fPIC", "-O2", "-I" + ref_src, "-I" + os.path.join(HERE, "..", "include"),
           SHIM_SRC, "-o", SHIM_LIB, "-L" + HERE, "-l:libwuburvc_b200.so", "-L" + ref_dir,
           "-l:" + os.path.basename(ref_lib), "-lm", "-Wl,--no-undefined", "-Wl,-rpath,$ORIGIN/..",
           "-Wl,-rpath,$ORIGIN/" + rel_ref]
    subprocess.check_call(cmd)
    return SHIM_LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
