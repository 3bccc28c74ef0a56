"""Builds the shim test driver (tests/shim/shim_check.cpp) against
include/jieyu_b200_shim.hpp into a scratch shared library and binds it."""
import ctypes as C
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIBDIR = os.path.join(ROOT, "jieyu_b200")

_P, _I, _F = C.c_void_p, C.c_int, C.c_float
SIGS = {
    "shim_last_error": (C.c_char_p, []),
    "shim_matmul_q": (_I, [_P, _P, _P, _I, _I, _I, _I]),
    "shim_matmul": (_I, [_I, _I, _I, _P, _P, _P]),
    "shim_matmul_w": (_I, [_P, _P, _I, _I, _I, _I, _P, _P]),
    "shim_rmsnorm": (_I, [_P, _P, _P, _I, _F]),
    "shim_rope_pos": (_I, [_P, _I, _I, _I, _I, _P, _P]),
    "shim_kv_pack_q8": (_I, [_P, _P, _P, _I, _I, _I]),
    "shim_attention_q8": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I]),
    "shim_silu": (_I, [_P, _P, _I]),
    "shim_ffn": (_I, [_P, _P, _P, _P, _P, _I, _I, _I]),
    "shim_generate": (_I, [_P, _P, _I, _P, _I, _I, _F, _F, _I, _P]),
    "shim_generate_cached": (_I, [_P, _P, _I, _I, _P, _I, _P, _P, _P, _P, _P]),
    "shim_release": (None, []),
}


def build(out_dir: str) -> C.CDLL:
    so = os.path.join(out_dir, "libshimcheck.so")
    subprocess.run(["g++", "-std=c++17", "-O1", "-fPIC", "-shared", "-Wall", "-Werror",
                    "-I", os.path.join(ROOT, "include"), os.path.join(HERE, "shim", "shim_check.cpp"),
                    "-L", LIBDIR, "-ljieyu_b200", f"-Wl,-rpath,{LIBDIR}", "-o", so],
                   check=True, capture_output=True, text=True)
    lib = C.CDLL(so)
    for name, (res, args) in SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib
