"""The drop-in shim (wuburvc_b200/shim/wubu_train_b200.c) that a maintainer adds to the reference tree
in place of src/wubu_train_cuda.cu: it must compile against the reference's own src/wubu_train.h and
link, with no undefined symbol, against the reference's host objects (oracle/_ref, built from
src/wubu_train.c) and this library.  Needs the reference sources, so it runs where they are."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SRC = os.path.join(os.environ.get("WUBU_REFERENCE", "/root/reference"), "src")
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libwubu_ref.so")
OUR_LIB = os.path.join(ROOT, "wuburvc_b200", "libwuburvc_b200.so")


@pytest.mark.skipif(not (os.path.exists(os.path.join(REF_SRC, "wubu_train.h")) and os.path.exists(REF_LIB)),
                    reason="reference sources / oracle/_ref not present")
def test_shim_builds_against_reference_header_and_links(tmp_path):
    out = tmp_path / "libwubu_train_b200.so"
    cmd = ["gcc", "-std=gnu11", "-shared", "-fPIC", "-O2", "-Wall", "-Werror=implicit-function-declaration",
           "-I" + REF_SRC, "-I" + os.path.join(ROOT, "include"),
           os.path.join(ROOT, "wuburvc_b200", "shim", "wubu_train_b200.c"), "-o", str(out),
           "-L" + os.path.dirname(OUR_LIB), "-l:libwuburvc_b200.so", "-L" + os.path.dirname(REF_LIB),
           "-l:libwubu_ref.so", "-lm", "-Wl,--no-undefined"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert out.exists()


def test_integration_notes_show_the_committed_shim():
    import re

    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    block = re.search(r"```c\n(/\* wubu_train_b200\.c.*?)```", doc, re.S).group(1)
    assert block == open(os.path.join(ROOT, "wuburvc_b200", "shim", "wubu_train_b200.c")).read()
