"""TEST INFRASTRUCTURE ONLY — ctypes access to the CPU checkers.

  liboracle.so      plain-C restatement of the reference path (oracle/jy_oracle.c)
  _ref/libjyref.so  the reference's own headers compiled in place (oracle/ref_harness.cpp)

Used by tests/, __graft_entry__.smoke() and bench.py's CPU baseline as the
checker; the product library never calls into it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libjyref.so")

_P, _I, _F = C.c_void_p, C.c_int, C.c_float


def _sig(lib, prefix: str):
    s = {
        "matmul_q8": (None, [_P, _P, _P, _I, _I, _I]),
        "matmul_qk": (None, [_P, _P, _P, _I, _I, _I, _I]),
        "matmul_f32": (None, [_I, _I, _I, _P, _P, _P]),
        "matmul_f16": (None, [_P, _P, _P, _I, _I, _I]),
        "rmsnorm": (None, [_P, _P, _P, _I, _F]),
        "rope_table": (None, [_I, _I, _F, _P, _P]),
        "rope_pos": (None, [_P, _I, _I, _I, _I, _P, _P]),
        "kv_pack_q8": (None, [_P, _P, _P, _I, _I, _I]),
        "attention_q8": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I]),
        "silu": (None, [_P, _P, _I]),
        "cache_create": (_P, [_I, _I, _I, _I]),
        "cache_free": (None, [_P]),
        "cache_read": (None, [_P, _I, _I, _P, _P, _P, _P]),
        "cache_write": (None, [_P, _I, _I, _P, _P, _P, _P]),
        "forward_logits": (_I, [_P, _P, _P, _I, _I, _P, _P]),
    }
    for name, (res, args) in s.items():
        fn = getattr(lib, prefix + name)
        fn.restype, fn.argtypes = res, args


def build() -> None:
    """Builds liboracle.so (and _ref/ when the reference tree is present)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)


class _Checker:
    prefix = ""

    def __init__(self, path: str):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run `make -C {HERE}`")
        self.lib = C.CDLL(path)
        _sig(self.lib, self.prefix)

    def __getattr__(self, name):
        return getattr(self.lib, self.prefix + name)


class Oracle(_Checker):
    """The C restatement."""
    prefix = "jyo_"

    def __init__(self, threads: int = 0):
        super().__init__(ORACLE_SO)
        self.lib.jyo_set_threads.argtypes = [_I]
        self.lib.jyo_generate.restype = _I
        self.lib.jyo_generate.argtypes = [_P, _P, _I, _P, _I, _I, _F, _P, _F]
        self.lib.jyo_sample.restype = _I
        self.lib.jyo_sample.argtypes = [_P, _I, _F, _F, _P, _I, _I, C.POINTER(C.c_uint)]
        if threads:
            self.lib.jyo_set_threads(threads)

    def generate(self, desc, prompt, max_new, eos=None, temperature=0.0, rep=1.0, max_seq=None):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros((max_seq or 1 << 16) + 1, dtype=np.int32)
        e = np.ascontiguousarray(eos if eos else [0], dtype=np.int32)
        n = self.lib.jyo_generate(C.byref(desc), prompt.ctypes.data, len(prompt), e.ctypes.data,
                                  len(eos) if eos else 0, max_new, temperature, out.ctypes.data, rep)
        if n < 0:
            raise RuntimeError("oracle generate failed")
        return out[:n].copy()


class Reference(_Checker):
    """The reference's own code (compiled from its sources into _ref/)."""
    prefix = "jyref_"

    def __init__(self, isa: str = "fma", threads: int = 0):
        super().__init__(REF_SO)
        self.lib.jyref_init.argtypes = [C.c_char_p, _I]
        self.lib.jyref_threads.restype = _I
        self.lib.jyref_generate.restype = _I
        self.lib.jyref_generate.argtypes = [_P, _P, _I, _P, _I, _I, _F, _P, _F, _P]
        self.lib.jyref_last_error.restype = C.c_char_p
        self.lib.jyref_decode_steps.restype = _I
        self.lib.jyref_decode_steps.argtypes = [_P, _P, _I, _I, _I, _P, _P]
        self.lib.jyref_init(isa.encode(), threads)

    def generate(self, desc, prompt, max_new, eos=None, temperature=0.0, rep=1.0, max_seq=None,
                 times=None):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros((max_seq or 1 << 16) + 1, dtype=np.int32)
        e = np.ascontiguousarray(eos if eos else [0], dtype=np.int32)
        t = np.zeros(3, dtype=np.float64)
        n = self.lib.jyref_generate(C.byref(desc), prompt.ctypes.data, len(prompt), e.ctypes.data,
                                    len(eos) if eos else 0, max_new, temperature, out.ctypes.data,
                                    rep, t.ctypes.data)
        if n < 0:
            raise RuntimeError(self.lib.jyref_last_error().decode())
        if times is not None:
            times[:] = t
        return out[:n].copy()


    def decode_steps(self, desc, cache, start_pos: int, first_id: int, n: int):
        """n greedy steps of generate_cached's body from a cache holding
        [0, start_pos); returns (new ids, seconds per step)."""
        out = np.zeros(n, np.int32)
        t = np.zeros(n, np.float64)
        r = self.lib.jyref_decode_steps(C.byref(desc), cache, start_pos, first_id, n, out.ctypes.data, t.ctypes.data)
        if r < 0:
            raise RuntimeError(self.lib.jyref_last_error().decode())
        return out, t


def reference_available() -> bool:
    return os.path.exists(REF_SO)
