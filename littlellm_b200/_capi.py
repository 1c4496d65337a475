"""ctypes binding of ``libkllm_b200.so`` (the C ABI in ``include/kllm_b200.h``).

The library is loaded at import time from the package directory. There is no
fallback: if the library has not been built, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH  # noqa: F401  (re-exported)

F32, F16, I32, I8 = 0, 1, 2, 3

OK = 0
ERR_INVALID_ARG = -1
ERR_SHAPE = -2
ERR_DTYPE = -3
ERR_ALIGN = -4
ERR_RANGE = -5
ERR_CAPACITY = -6
ERR_CUDA = -7
ERR_IO = -8
ERR_FORMAT = -9

FLAG_BAD_TOKEN = 1
FLAG_BAD_POSITION = 2
FLAG_BAD_SLOT = 4
FLAG_BAD_SEQ_END = 8
FLAG_TIMEOUT = 16

PARAM_IDS = 7680  # host ids carried per launch by kllm_b200_embedding_host_ids

OP_EMBEDDING, OP_INPUT_NORM, OP_QKV_ROPE, OP_POST_NORM, OP_SWIGLU, OP_FINAL_NORM, OP_SELECT = (
    1, 2, 4, 8, 16, 32, 64)
OP_ATTENTION = 128
OP_GEMM = 256
OP_CHAIN = 0x7f  # the seven ops of op_mask 0
OP_FORWARD = OP_CHAIN | OP_ATTENTION | OP_GEMM  # the whole forward step


class KllmError(RuntimeError):
    """A non-zero status from the C ABI, with the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status


class LayerBuffers(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "q", "k", "v", "q_bias", "k_bias", "v_bias", "attn_out", "ffn_out", "gate", "up",
        "input_norm_w", "post_norm_w", "attn_norm_out", "ffn_norm_out", "swiglu_out",
        "k_cache", "v_cache", "attn_ctx")]


class LayerWeights(ctypes.Structure):
    _fields_ = [(name, ctypes.c_void_p) for name in (
        "wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "o_bias", "gate_bias", "up_bias", "down_bias")]


class Chain(ctypes.Structure):
    _fields_ = [
        ("n_tokens", ctypes.c_int64), ("hidden", ctypes.c_int64), ("n_heads", ctypes.c_int64),
        ("n_kv_heads", ctypes.c_int64), ("head_dim", ctypes.c_int64),
        ("intermediate", ctypes.c_int64), ("vocab", ctypes.c_int64),
        ("n_layers", ctypes.c_int64), ("n_slots", ctypes.c_int64), ("max_seq", ctypes.c_int64),
        ("n_seqs", ctypes.c_int64), ("seq_len", ctypes.c_int64),
        ("eps", ctypes.c_float), ("theta", ctypes.c_float),
        ("weight_dtype", ctypes.c_int), ("use_pdl", ctypes.c_int), ("op_mask", ctypes.c_int),
        ("embed_table", ctypes.c_void_p), ("ids", ctypes.c_void_p),
        ("positions", ctypes.c_void_p), ("slots", ctypes.c_void_p),
        ("seq_ends", ctypes.c_void_p), ("residual", ctypes.c_void_p),
        ("final_norm_w", ctypes.c_void_p), ("final_norm_out", ctypes.c_void_p),
        ("last_rows", ctypes.c_void_p), ("layers", ctypes.POINTER(LayerBuffers)),
        ("err_flags", ctypes.c_void_p),
        ("attn_workspace", ctypes.c_void_p), ("attn_workspace_bytes", ctypes.c_int64),
        ("weights", ctypes.POINTER(LayerWeights)), ("lm_head", ctypes.c_void_p), ("logits", ctypes.c_void_p),
    ]


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_int = ctypes.c_int
_f32 = ctypes.c_float

# name -> argtypes; every entry returns int unless listed in _RESTYPES.
SIGNATURES = {
    "kllm_b200_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "kllm_b200_status_string": [_int],
    "kllm_b200_version": [],
    "kllm_b200_set_pdl": [_int],
    "kllm_b200_embedding": [_vp, _i64, _i64, _int, _vp, _i64, _vp, _int, _vp, _vp],
    "kllm_b200_embedding_host_ids": [_vp, _i64, _i64, _int, _vp, _i64, _vp, _int, _vp, _vp],
    "kllm_b200_embedding_rms_norm": [_vp, _i64, _i64, _vp, _i64, _vp, _int, _f32, _vp, _vp, _vp, _vp],
    "kllm_b200_rms_norm": [_vp, _vp, _vp, _i64, _i64, _f32, _int, _int, _vp],
    "kllm_b200_add_inplace": [_vp, _vp, _i64, _int, _int, _vp],
    "kllm_b200_add_bias_inplace": [_vp, _vp, _i64, _i64, _int, _int, _vp],
    "kllm_b200_select_last_row": [_vp, _i64, _i64, _vp, _int, _vp],
    "kllm_b200_silu_mul": [_vp, _vp, _vp, _i64, _int, _vp],
    "kllm_b200_rope_inplace": [_vp, _i64, _i64, _i64, _i32, _f32, _int, _vp],
    "kllm_b200_copy_kv_to_cache": [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _i32, _int, _int, _vp],
    "kllm_b200_dequantize_int8": [_vp, _vp, _vp, _i64, _int, _vp],
    "kllm_b200_dequantize_int8_batched": [ctypes.POINTER(_vp), ctypes.POINTER(_vp), ctypes.POINTER(_vp),
                                          ctypes.POINTER(_i64), _int, _int, _vp],
    "kllm_b200_add_rms_norm": [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _int, _int, _vp],
    "kllm_b200_qkv_bias_rope_kv_append": [_vp, _vp, _vp, _vp, _vp, _vp, _int, _vp, _vp, _i64, _i64,
                                          _i64, _i64, _f32, _vp, _vp, _i64, _i64, _vp, _vp],
    "kllm_b200_select_last_rows": [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _int, _vp, _vp],
    "kllm_b200_dequantize_int8_rne": [_vp, _vp, _vp, _i64, _vp, _vp],
    "kllm_b200_attention_workspace_bytes": [_i64, _i64, _i64, _i64, _i64, _vp],
    "kllm_b200_attention_head_major": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
                                       _i64, _int, _vp, _i64, _vp, _vp],
    "kllm_b200_chain_run": [ctypes.POINTER(Chain), ctypes.POINTER(ctypes.c_int), _vp],
    "kllm_b200_dequantize_int8_host_static": [_vp, _f32, _vp, _i64, _int, _vp],
    "kllm_b200_linear": [_vp, _vp, _vp, _int, _vp, _i64, _i64, _i64, _vp, _vp],
    "kllm_b200_linear_swiglu": [_vp, _vp, _vp, _vp, _vp, _int, _vp, _i64, _i64, _i64, _vp, _vp],
    "kllm_b200_qkv_linear_rope_kv_append": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _vp, _vp, _i64, _i64, _i64,
                                            _i64, _i64, _f32, _vp, _vp, _vp, _i64, _i64, _vp, _vp],
    # argtypes of the .kllm entry points use the structures in loader.py
    "kllm_b200_kllm_read_index": None,
    "kllm_b200_kllm_load": None,
}
_RESTYPES = {
    "kllm_b200_last_error": ctypes.c_size_t,
    "kllm_b200_status_string": ctypes.c_char_p,
}


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m littlellm_b200.build` "
            "(the CUDA path has no fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        if argtypes is not None:
            fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    return lib


lib = _load()


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib.kllm_b200_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != OK:
        raise KllmError(status, last_error())
