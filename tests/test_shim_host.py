"""CPU: include/jieyu_b200_shim.hpp (the reference's operator and generate
entry points under their own names) compiles against the reference's real
headers and structs, and its misuse paths throw as the reference's do; the
shim test driver builds and links against libjieyu_b200.so. No device work."""
import ctypes as C
import os
import subprocess

import pytest

import _shim

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _ref_tree():
    ref = os.environ.get("JIEYU_REF_TREE") or os.path.join(os.path.dirname(ROOT), "reference")
    return ref if os.path.isdir(os.path.join(ref, "libs")) else None


@pytest.mark.skipif(_ref_tree() is None, reason="the reference source tree is not on this machine")
def test_shim_compiles_with_the_reference_headers(tmp_path):
    ref = _ref_tree()
    exe = str(tmp_path / "shim_ref_compile")
    r = subprocess.run(["g++", "-std=c++17", "-O0", "-fopenmp", "-w", "-I", ref, "-I", os.path.join(ref, "libs"),
                        "-I", os.path.join(ROOT, "include"), os.path.join(HERE, "shim", "shim_ref_compile.cpp"),
                        "-L", _shim.LIBDIR, "-ljieyu_b200", f"-Wl,-rpath,{_shim.LIBDIR}", "-o", exe],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "13 of 13" in run.stdout


def test_shim_driver_builds_and_reports_misuse(tmp_path):
    lib = _shim.build(str(tmp_path))
    assert lib.shim_rmsnorm(None, None, None, 4, C.c_float(1e-5)) == -1
    assert b"rmsnorm" in lib.shim_last_error()
    assert lib.shim_matmul_q(None, None, None, 1, 1, 32, 3) == -1
    assert lib.shim_silu(None, None, 4) == -1
    # prompt_len <= 0 returns 0 before anything is bound (generate.h:25)
    out = (C.c_int * 4)()
    assert lib.shim_generate(None, out, 0, None, 0, 4, 0.0, 1.0, 0, out) == 0
