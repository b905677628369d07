"""The drop-in shim (wuburvc_b200/shim/wubu_train_b200.c), the file a maintainer adds to the reference
tree in place of src/wubu_train_cuda.cu, checked on the CPU:

* it compiles against the reference's own src/wubu_train.h / src/wubu_rvc_real.h and links, with no
  undefined symbol, against the reference's host objects (oracle/_ref, built from src/wubu_train.c)
  and this library;
* the reference's own CUDA A/B program, src/test_train_cuda.c, compiles unmodified and links against
  the shim with no undefined symbol (its model-file loader replaced by oracle/ref_model_stub.c);
* every entry point returns -1 on NULL arguments before touching a GPU (src/wubu_train_cuda.cu:801).
The compile checks need the reference sources (WUBU_REFERENCE, else the default in oracle/Makefile)."""
import ctypes
import os
import subprocess

import pytest

from oracle.refpath import reference_root

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = reference_root()
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libwubu_ref.so")
OUR_LIB = os.path.join(ROOT, "wuburvc_b200", "libwuburvc_b200.so")
SHIM_SRC = os.path.join(ROOT, "wuburvc_b200", "shim", "wubu_train_b200.c")
SHIM_LIB = os.path.join(ROOT, "wuburvc_b200", "shim", "libwubu_train_b200.so")

needs_ref = pytest.mark.skipif(not (REF and os.path.exists(REF_LIB)), reason="reference sources / oracle/_ref absent")


def build_shim(out):
    cmd = ["gcc", "-std=gnu11", "-shared", "-fPIC", "-O2", "-Wall", "-Werror=implicit-function-declaration",
           "-I" + os.path.join(REF, "src"), "-I" + os.path.join(ROOT, "include"), SHIM_SRC, "-o", str(out),
           "-L" + os.path.dirname(OUR_LIB), "-l:libwuburvc_b200.so", "-L" + os.path.dirname(REF_LIB),
           "-l:libwubu_ref.so", "-lm", "-Wl,--no-undefined"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return r


@needs_ref
def test_shim_builds_against_reference_headers_and_links(tmp_path):
    r = build_shim(tmp_path / "libwubu_train_b200.so")
    assert "warning" not in r.stderr, r.stderr


@needs_ref
def test_reference_ab_program_links_against_the_shim(tmp_path):
    """src/test_train_cuda.c (the reference's CPU-vs-CUDA A/B of wubu_train_forward_cuda,
    wubu_train_backward_cuda and wubu_train_step_cuda) builds unmodified against the shim."""
    shim = tmp_path / "libwubu_train_b200.so"
    build_shim(shim)
    exe = tmp_path / "test_train_cuda"
    cmd = ["gcc", "-std=gnu11", "-O2", "-w", "-I" + os.path.join(REF, "src"),
           os.path.join(REF, "src", "test_train_cuda.c"), os.path.join(ROOT, "oracle", "ref_model_stub.c"),
           "-o", str(exe), "-L" + str(tmp_path), "-l:libwubu_train_b200.so", "-L" + os.path.dirname(REF_LIB),
           "-l:libwubu_ref.so", "-L" + os.path.dirname(OUR_LIB), "-l:libwuburvc_b200.so", "-lm",
           "-Wl,--no-undefined"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert exe.exists()


@pytest.mark.skipif(not os.path.exists(SHIM_LIB), reason="shim not built")
def test_shim_entry_points_reject_null_arguments_without_a_gpu():
    shim = ctypes.CDLL(SHIM_LIB)
    vp, ip = ctypes.c_void_p, ctypes.c_int
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.cast(buf, vp)
    shim.wubu_train_forward_cuda.argtypes = [vp, vp, ip, vp, ip, vp]
    shim.wubu_train_backward_cuda.argtypes = [vp, vp, vp, vp, vp]
    shim.wubu_train_step_cuda.argtypes = [vp, vp, vp, vp, ip, vp, ip, vp, ip]
    shim.wubu_generator_nsf_cuda.argtypes = [vp, vp, ip, ip, vp, vp, vp, ip, ip, ip]
    shim.wubu_train_cache_alloc_cuda.restype = vp
    shim.wubu_train_cache_free_cuda.argtypes = [vp]
    cache = shim.wubu_train_cache_alloc_cuda()
    assert cache
    assert shim.wubu_train_forward_cuda(None, p, 4, p, 1600, cache) == -1
    assert shim.wubu_train_forward_cuda(p, p, 4, p, 1600, None) == -1
    assert shim.wubu_train_backward_cuda(p, cache, p, None, p) == -1
    # a backward without a forward in this cache
    assert shim.wubu_train_backward_cuda(p, cache, p, p, p) == -1
    assert shim.wubu_train_step_cuda(p, p, None, p, 4, p, 1600, None, 1) == -1
    assert shim.wubu_generator_nsf_cuda(p, p, 4, 192, None, None, p, 1600, 0, 0) == -1
    shim.wubu_train_cache_free_cuda(cache)
    shim.wubu_train_cache_free_cuda(None)
