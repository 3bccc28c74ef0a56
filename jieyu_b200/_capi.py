"""ctypes binding of libjieyu_b200.so (the C ABIs declared in include/jieyu_b200.h
and include/jieyu.h).

The library is the product: every compute call below runs a CUDA kernel of
that library. There is no fallback; if the shared object is missing the import
raises with the build command.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libjieyu_b200.so")

JYC_OK = 0
JYC_ERR_ARG = -1
JYC_ERR_CUDA = -2
JYC_ERR_KV_OOM = -3
JYC_ERR_UNSUPPORTED = -4
JYC_ERR_NOMEM = -5
JYC_Q4K, JYC_Q5K, JYC_Q6K, JYC_Q8_0 = 0, 1, 2, 3  # qmat block types (matmul_q.h:15)


class JycError(RuntimeError):
    """A C-ABI call returned a negative status (message from jyc_last_error)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


class WMat(C.Structure):
    """Layout of jyc_wmat == the reference's WMat (libs/date_libs/wmat.h:32-44)."""

    _fields_ = [("f", C.c_void_p), ("h", C.c_void_p), ("q", C.c_void_p), ("qt", C.c_uint8)]


class LayerWeights(C.Structure):
    """Layout of jyc_layer_weights == LayerWeights (libs/date_libs/date.h:75-88)."""

    _fields_ = [
        ("rms1_weight", C.c_void_p),
        ("Wq", WMat), ("Wk", WMat), ("Wv", WMat), ("Wo", WMat),
        ("bq", C.c_void_p), ("bk", C.c_void_p), ("bv", C.c_void_p),
        ("rms2_weight", C.c_void_p),
        ("W1", WMat), ("W2", WMat), ("W3", WMat),
    ]


class ModelDesc(C.Structure):
    _fields_ = [
        ("layers", C.POINTER(LayerWeights)),
        ("num_layers", C.c_int),
        ("embed", WMat),
        ("lm_head", WMat),
        ("final_rms_weight", C.c_void_p),
        ("cos_table", C.c_void_p),
        ("sin_table", C.c_void_p),
        ("max_seq", C.c_int),
        ("vocab_size", C.c_int),
        ("hidden", C.c_int),
        ("num_heads", C.c_int),
        ("num_kv_heads", C.c_int),
        ("head_dim", C.c_int),
        ("intermediate", C.c_int),
        ("embed_rows", C.c_int),
        ("vocab_offset", C.c_int),
    ]


TOKEN_CB = C.CFUNCTYPE(C.c_int, C.c_int, C.c_void_p)

# (name, restype, argtypes) of every exported entry point.
_P, _I, _F, _U64, _SZ = C.c_void_p, C.c_int, C.c_float, C.c_uint64, C.c_size_t
SIGNATURES = [
    ("jyc_version", C.c_char_p, []),
    ("jyc_last_error", C.c_char_p, []),
    ("jyc_kernel_launches", C.c_longlong, []),
    ("jyc_rope_table", _I, [_I, _I, _F, _P, _P]),
    ("jyc_synth_f32", _I, [_U64, _U64, _F, _P, _SZ]),
    ("jyc_synth_q8_0", _I, [_U64, _U64, _F, _P, _SZ, _SZ]),
    ("jyc_synth_ids", _I, [_U64, _U64, _I, _P, _SZ]),
    ("jyc_quantize_q8_0", _I, [_P, _P, _SZ, _SZ]),
    ("jyc_q8_repack", _I, [_P, _I, _I, _P, _P, _P]),
    ("jyc_matmul_q8", _I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    ("jyc_matmul_qk", _I, [_P, _P, _P, _I, _I, _I, _I, _P]),
    ("jyc_matmul_f32", _I, [_P, _P, _P, _I, _I, _I, _P]),
    ("jyc_f32_transpose", _I, [_P, _P, _I, _I, _P]),
    ("jyc_matmul_f16", _I, [_P, _P, _P, _I, _I, _I, _P]),
    ("jyc_f16_transpose", _I, [_P, _P, _I, _I, _P]),
    ("jyc_rmsnorm", _I, [_P, _P, _P, _I, _I, _F, _P]),
    ("jyc_rope_pos", _I, [_P, _I, _I, _I, _I, _P, _P, _P]),
    ("jyc_kv_pack_q8", _I, [_P, _P, _P, _I, _I, _I, _P]),
    ("jyc_attention_q8", _I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P]),
    ("jyc_attention_q8_noalloc", _I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P]),
    ("jyc_silu", _I, [_P, _P, _I, _P]),
    ("jyc_host_matmul_q", _I, [_P, _P, _P, _I, _I, _I, _I]),
    ("jyc_host_matmul_f32", _I, [_I, _I, _I, _P, _P, _P]),
    ("jyc_host_matmul_f16", _I, [_P, _P, _P, _I, _I, _I]),
    ("jyc_host_matmul_w", _I, [_P, _I, _I, _I, _P, _P]),
    ("jyc_host_rmsnorm", _I, [_P, _P, _P, _I, _F]),
    ("jyc_host_rope_pos", _I, [_P, _I, _I, _I, _I, _P, _P]),
    ("jyc_host_kv_pack_q8", _I, [_P, _P, _P, _I, _I, _I]),
    ("jyc_host_attention_q8", _I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _I]),
    ("jyc_host_silu", _I, [_P, _P, _I]),
    ("jyc_host_ffn", _I, [_P, _P, _P, _P, _P, _I, _I, _I]),
    ("jyc_argmax", _I, [_P, _I, _P, _P]),
    ("jyc_sample", _I, [_P, _I, C.c_float, C.c_float, _P, _I, _I, _P, _P, _P]),
    ("jyc_model_create", _P, [C.POINTER(ModelDesc)]),
    ("jyc_model_free", None, [_P]),
    ("jyc_model_weight_bytes_per_token", C.c_double, [_P]),
    ("jyc_model_kv_bytes_per_token", C.c_double, [_P, _I]),
    ("jyc_generate", _I, [_P, _P, _I, _P, _I, _I, _F, _P, _F, TOKEN_CB, _P]),
    ("jyc_forward_logits", _I, [_P, _P, _I, _I, _P, _P]),
    ("jyc_model_read_kv", _I, [_P, _I, _I, _P, _P, _P, _P]),
    ("jyc_model_write_kv", _I, [_P, _I, _I, _P, _P, _P, _P]),
    ("jyc_prefill_device", _I, [_P, _P, _I, _P]),
    ("jyc_decode_device", _I, [_P, _I, _P]),
    ("jyc_model_rewind", _I, [_P, _I, _P]),
    ("jyc_model_kernels_per_step", _I, [_P]),
    ("jyc_model_profile_decode", _I, [_P, _I, _P, _P, _P, _P]),
    ("jyc_model_decode_path", _I, [_P]),
    ("jyc_model_decode_window", _I, [_P, _I, _I, _P]),
    ("jyc_model_tp_open", _I, [_P, _I, _I, _P]),
    ("jyc_model_tp_connect", _I, [_P, _P]),
    ("jyc_model_partials", _I, [_P, C.POINTER(_P), C.POINTER(_I), C.POINTER(_P), C.POINTER(_I)]),
    ("jyc_model_prefill_window", _I, [_P, _I, _I, _I, _I, _P]),
    ("jyc_model_prefill_partial", _I, [_P, C.POINTER(_P), C.POINTER(_I)]),
    ("jyc_device_error", _I, [_I]),
    ("jyc_model_trace_points", _I, [_P]),
    ("jyc_model_trace_decode", _I, [_P, _P, _P, _I]),
    ("jyc_model_tokens_device", _P, [_P]),
    ("jyc_model_length", _I, [_P, _P]),
    ("jyc_batch_create", _P, [_P, _I]),
    ("jyc_batch_free", None, [_P]),
    ("jyc_batch_prefill", _I, [_P, _I, _P, _I]),
    ("jyc_batch_decode", _I, [_P, _I, _P]),
    ("jyc_batch_rewind", _I, [_P, _I, _P]),
    ("jyc_batch_tokens", _I, [_P, _I, _P, _I]),
    ("jyc_batch_path", _I, [_P]),
    ("jyc_batch_kernels_per_step", _I, [_P]),
    ("jyc_batch_kv_bytes_per_step", C.c_double, [_P, _I]),
    # text C ABI (include/jieyu.h)
    ("jieyu_load", _P, [C.c_char_p, _I]),
    ("jieyu_free", None, [_P]),
    ("jieyu_last_error", C.c_char_p, [_P]),
    ("jieyu_version", C.c_char_p, []),
    ("jieyu_context_length", _I, [_P]),
    ("jieyu_model_dir", C.c_char_p, [_P]),
    ("jieyu_generate", _I, [_P, C.c_char_p, _P, _I, _I, C.c_float, C.c_float]),
    ("jieyu_generate_jsonl", _I, [_P, C.c_char_p, C.c_char_p, C.c_char_p, _P, _I, _I, C.c_float, C.c_float]),
    ("jyt_tok_load", _P, [C.c_char_p, C.c_char_p]),
    ("jyt_tok_free", None, [_P]),
    ("jyt_tok_encode", _I, [_P, C.c_char_p, _I, _P, _I]),
    ("jyt_tok_decode", _I, [_P, _P, _I, _P, _I]),
    ("jyt_tok_add_special", _I, [_P, C.c_char_p, _I]),
    ("jyt_tok_info", _I, [_P, _P]),
    ("jyt_model_dir_probe", _I, [C.c_char_p, _I, _P, _P, _I]),
]

_lib = None


def load() -> C.CDLL:
    """Loads the library once; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C {os.path.join(_HERE, 'csrc')}` "
            "(or __graft_entry__.build()); the B200 path has no fallback")
    lib = C.CDLL(LIB_PATH)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    return load().jyc_last_error().decode("utf-8", "replace")


def check(code: int) -> int:
    """Raises JycError for a negative status; returns the value otherwise."""
    if code < 0:
        raise JycError(code, last_error())
    return code
