"""Python bindings of the CPU checkers (test infrastructure only).

Only the tests, ``__graft_entry__.smoke()`` and the CPU-baseline / reference
legs of ``bench.py`` import this module, and only as the checker. The CUDA
product in ``littlellm_b200`` never imports it.

Two libraries are wrapped:

* ``Oracle`` -> ``oracle/liboracle.so``: the C restatement of the reference
  CPU operators (``kllm_oracle.c``; each function cites the reference
  file:line it follows).
* ``Reference`` -> ``oracle/_ref/libkllm_ref.so``: the reference's own CPU
  operators compiled from its sources by ``oracle/Makefile`` and exposed by
  ``ref_capi.cpp``. It is optional (absent when the reference tree was not
  available at build time).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libkllm_ref.so")

F32, F16, I32, I8 = 0, 1, 2, 3

_c_f32p = ctypes.POINTER(ctypes.c_float)
_c_u16p = ctypes.POINTER(ctypes.c_uint16)
_c_i32p = ctypes.POINTER(ctypes.c_int32)
_c_i8p = ctypes.POINTER(ctypes.c_int8)
_c_i64 = ctypes.c_int64


def reference_dir() -> str:
    """The reference source tree the Makefile compiles: $KLLM_REFERENCE_SRC,
    else the read-only checkout of this build machine."""
    return os.environ.get("KLLM_REFERENCE_SRC", "/root/reference")


def reference_sources_present() -> bool:
    """Whether the reference source tree the Makefile compiles is here (it is
    not on machines that only run the prebuilt checkers)."""
    return os.path.isfile(os.path.join(reference_dir(), "include", "kllm", "op", "ops.h"))


def make(*targets: str) -> None:
    """Runs oracle/Makefile for `targets`, with REF set when the reference
    sources are present."""
    cmd = ["make", "-C", HERE, "-s"]
    if reference_sources_present():
        cmd.append(f"REF={reference_dir()}")
    subprocess.run(cmd + list(targets), check=True)


def build(force: bool = False) -> None:
    """Runs oracle/Makefile (C restatement, plus the compiled reference when
    its source tree is present)."""
    if force or not os.path.exists(ORACLE_SO) or reference_sources_present():
        make()


def _ptr(a: np.ndarray | None, ctype):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctype)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Oracle:
    """fp32 restatement of the reference CPU ops (``kllm_oracle.c``)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        self.lib = lib = ctypes.CDLL(path)
        lib.kllm_oracle_float_to_half.restype = ctypes.c_uint16
        lib.kllm_oracle_float_to_half.argtypes = [ctypes.c_float]
        lib.kllm_oracle_half_to_float.restype = ctypes.c_float
        lib.kllm_oracle_half_to_float.argtypes = [ctypes.c_uint16]
        lib.kllm_oracle_float_to_half_array.argtypes = [_c_f32p, _c_u16p, _c_i64]
        lib.kllm_oracle_half_to_float_array.argtypes = [_c_u16p, _c_f32p, _c_i64]
        lib.kllm_oracle_embedding.restype = ctypes.c_int
        lib.kllm_oracle_embedding.argtypes = [_c_f32p, _c_i64, _c_i64, _c_i32p, _c_i64, _c_f32p,
                                              ctypes.POINTER(ctypes.c_int64)]
        lib.kllm_oracle_rms_norm.argtypes = [_c_f32p, _c_f32p, _c_f32p, _c_i64, _c_i64,
                                             ctypes.c_float]
        lib.kllm_oracle_add_inplace.argtypes = [_c_f32p, _c_f32p, _c_i64]
        lib.kllm_oracle_add_bias_inplace.argtypes = [_c_f32p, _c_f32p, _c_i64, _c_i64]
        lib.kllm_oracle_select_last_row.argtypes = [_c_f32p, _c_i64, _c_i64, _c_f32p]
        lib.kllm_oracle_silu_mul.argtypes = [_c_f32p, _c_f32p, _c_f32p, _c_i64]
        lib.kllm_oracle_rope_inplace.argtypes = [_c_f32p, _c_i64, _c_i64, _c_i64,
                                                 ctypes.c_int32, ctypes.c_float]
        lib.kllm_oracle_copy_kv_to_cache.restype = ctypes.c_int
        lib.kllm_oracle_copy_kv_to_cache.argtypes = [_c_f32p, _c_f32p, _c_i64, _c_i64, _c_i64,
                                                     _c_f32p, _c_f32p, _c_i64, ctypes.c_int32]
        lib.kllm_oracle_dequantize_int8_f32.argtypes = [_c_i8p, _c_i64, ctypes.c_float, _c_f32p]
        lib.kllm_oracle_dequantize_int8_f16.argtypes = [_c_i8p, _c_i64, ctypes.c_float, _c_u16p]
        lib.kllm_oracle_add_rms_norm.argtypes = [_c_f32p, _c_f32p, _c_f32p, _c_f32p, _c_i64,
                                                 _c_i64, ctypes.c_float]
        lib.kllm_oracle_qkv_bias_rope_kv_append.restype = ctypes.c_int64
        lib.kllm_oracle_qkv_bias_rope_kv_append.argtypes = [
            _c_f32p, _c_f32p, _c_f32p, _c_f32p, _c_f32p, _c_f32p, _c_i32p, _c_i32p, _c_i64,
            _c_i64, _c_i64, _c_i64, ctypes.c_float, _c_f32p, _c_f32p, _c_i64, _c_i64]
        lib.kllm_oracle_select_last_rows.restype = ctypes.c_int
        lib.kllm_oracle_select_last_rows.argtypes = [_c_f32p, _c_i64, _c_i64, _c_i32p, _c_i64,
                                                     _c_i64, _c_f32p]
        lib.kllm_oracle_matmul.argtypes = [_c_f32p, _c_f32p, _c_f32p, _c_i64, _c_i64, _c_i64]
        lib.kllm_oracle_attention.argtypes = [_c_f32p, _c_f32p, _c_f32p, _c_f32p, _c_i64,
                                              ctypes.c_int32, _c_i64, _c_i64, _c_i64]
        lib.kllm_oracle_attention_head_major.restype = ctypes.c_int64
        lib.kllm_oracle_attention_head_major.argtypes = [
            _c_f32p, _c_f32p, _c_f32p, _c_f32p, _c_i32p, _c_i32p, _c_i64, _c_i64, _c_i64, _c_i64,
            _c_i64, _c_i64]

    # -- fp16 conversion ----------------------------------------------------
    def float_to_half_bits(self, x) -> np.ndarray:
        x = _f32(x)
        out = np.empty(x.shape, dtype=np.uint16)
        self.lib.kllm_oracle_float_to_half_array(_ptr(x, _c_f32p), _ptr(out, _c_u16p), x.size)
        return out

    def half_bits_to_float(self, h) -> np.ndarray:
        h = np.ascontiguousarray(h, dtype=np.uint16)
        out = np.empty(h.shape, dtype=np.float32)
        self.lib.kllm_oracle_half_to_float_array(_ptr(h, _c_u16p), _ptr(out, _c_f32p), h.size)
        return out

    # -- operators (fp32, return new arrays; inputs untouched) --------------
    def embedding(self, table, ids) -> np.ndarray:
        table = _f32(table)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros((ids.size, table.shape[1]), dtype=np.float32)
        bad = ctypes.c_int64(-1)
        rc = self.lib.kllm_oracle_embedding(_ptr(table, _c_f32p), table.shape[0], table.shape[1],
                                            _ptr(ids, _c_i32p), ids.size, _ptr(out, _c_f32p),
                                            ctypes.byref(bad))
        if rc != 0:
            raise ValueError(f"token id out of vocabulary range at index {bad.value}")
        return out

    def rms_norm(self, x, w, eps: float) -> np.ndarray:
        x, w = _f32(x), _f32(w)
        out = np.empty_like(x)
        self.lib.kllm_oracle_rms_norm(_ptr(x, _c_f32p), _ptr(w, _c_f32p), _ptr(out, _c_f32p),
                                      x.shape[0], x.shape[1], eps)
        return out

    def add(self, x, y) -> np.ndarray:
        x = _f32(x).copy()
        y = _f32(y)
        self.lib.kllm_oracle_add_inplace(_ptr(x, _c_f32p), _ptr(y, _c_f32p), x.size)
        return x

    def add_bias(self, x, bias) -> np.ndarray:
        x = _f32(x).copy()
        b = None if bias is None else _f32(bias)
        self.lib.kllm_oracle_add_bias_inplace(_ptr(x, _c_f32p), _ptr(b, _c_f32p), x.shape[0],
                                              x.shape[1])
        return x

    def select_last_row(self, x) -> np.ndarray:
        x = _f32(x)
        out = np.empty((1, x.shape[1]), dtype=np.float32)
        self.lib.kllm_oracle_select_last_row(_ptr(x, _c_f32p), x.shape[0], x.shape[1],
                                             _ptr(out, _c_f32p))
        return out

    def matmul(self, a, b) -> np.ndarray:
        """a [m, k] times b [n, k] transposed, fp32 (cpu_matmul)."""
        a, b = _f32(a), _f32(b)
        if a.shape[1] != b.shape[1]:
            raise ValueError("matmul shape mismatch")
        out = np.empty((a.shape[0], b.shape[0]), dtype=np.float32)
        self.lib.kllm_oracle_matmul(_ptr(a, _c_f32p), _ptr(b, _c_f32p), _ptr(out, _c_f32p), a.shape[0],
                                    b.shape[0], a.shape[1])
        return out

    def linear(self, x, w, bias=None) -> np.ndarray:
        """linear() of src/model/llama.cpp:12-24 in fp32: matmul, then
        add_bias_inplace."""
        out = self.matmul(x, w)
        if bias is not None:
            out = self.add_bias(out, bias)
        return out

    def silu_mul(self, g, u) -> np.ndarray:
        g, u = _f32(g), _f32(u)
        out = np.empty_like(g)
        self.lib.kllm_oracle_silu_mul(_ptr(g, _c_f32p), _ptr(u, _c_f32p), _ptr(out, _c_f32p),
                                      g.size)
        return out

    def rope(self, x, past_len: int, theta: float) -> np.ndarray:
        x = _f32(x).copy()
        self.lib.kllm_oracle_rope_inplace(_ptr(x, _c_f32p), x.shape[0], x.shape[1], x.shape[2],
                                          past_len, theta)
        return x

    def copy_kv_to_cache(self, k, v, k_cache, v_cache, past_len: int):
        k, v = _f32(k), _f32(v)
        kc, vc = _f32(k_cache).copy(), _f32(v_cache).copy()
        rc = self.lib.kllm_oracle_copy_kv_to_cache(
            _ptr(k, _c_f32p), _ptr(v, _c_f32p), k.shape[0], k.shape[1], k.shape[2],
            _ptr(kc, _c_f32p), _ptr(vc, _c_f32p), kc.shape[0], past_len)
        if rc != 0:
            raise ValueError("KV cache capacity exceeded")
        return kc, vc

    def dequantize_int8_f32(self, q, scale: float) -> np.ndarray:
        q = np.ascontiguousarray(q, dtype=np.int8)
        out = np.empty(q.shape, dtype=np.float32)
        self.lib.kllm_oracle_dequantize_int8_f32(_ptr(q, _c_i8p), q.size, scale,
                                                 _ptr(out, _c_f32p))
        return out

    def dequantize_int8_f16_bits(self, q, scale: float) -> np.ndarray:
        q = np.ascontiguousarray(q, dtype=np.int8)
        out = np.empty(q.shape, dtype=np.uint16)
        self.lib.kllm_oracle_dequantize_int8_f16(_ptr(q, _c_i8p), q.size, scale,
                                                 _ptr(out, _c_u16p))
        return out

    def add_rms_norm(self, residual, delta, w, eps: float):
        r = _f32(residual).copy()
        d = None if delta is None else _f32(delta)
        w = _f32(w)
        out = np.empty_like(r)
        self.lib.kllm_oracle_add_rms_norm(_ptr(r, _c_f32p), _ptr(d, _c_f32p), _ptr(w, _c_f32p),
                                          _ptr(out, _c_f32p), r.shape[0], r.shape[1], eps)
        return r, out

    def qkv_bias_rope_kv_append(self, q, k, v, bq, bk, bv, positions, slots, theta: float,
                                k_cache, v_cache):
        """q [T, Hq, D], k/v [T, Hkv, D], caches [n_slots, Hkv, max_seq, D].
        Returns (q_rotated, k_cache, v_cache, n_skipped)."""
        q = _f32(q).copy()
        k, v = _f32(k), _f32(v)
        bq = None if bq is None else _f32(bq)
        bk = None if bk is None else _f32(bk)
        bv = None if bv is None else _f32(bv)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        slo = np.ascontiguousarray(slots, dtype=np.int32)
        kc, vc = _f32(k_cache).copy(), _f32(v_cache).copy()
        T, Hq, D = q.shape
        Hkv = k.shape[1]
        skipped = self.lib.kllm_oracle_qkv_bias_rope_kv_append(
            _ptr(q, _c_f32p), _ptr(k, _c_f32p), _ptr(v, _c_f32p), _ptr(bq, _c_f32p),
            _ptr(bk, _c_f32p), _ptr(bv, _c_f32p), _ptr(pos, _c_i32p), _ptr(slo, _c_i32p), T, Hq,
            Hkv, D, theta, _ptr(kc, _c_f32p), _ptr(vc, _c_f32p), kc.shape[0], kc.shape[2])
        if skipped < 0:
            raise ValueError("kv row too wide for the oracle")
        return q, kc, vc, int(skipped)

    def select_last_rows(self, x, seq_ends=None, seq_len: int = 0, n_seqs: int = 0):
        x = _f32(x)
        ends = None if seq_ends is None else np.ascontiguousarray(seq_ends, dtype=np.int32)
        if ends is not None:
            n_seqs = ends.size
        out = np.empty((n_seqs, x.shape[1]), dtype=np.float32)
        rc = self.lib.kllm_oracle_select_last_rows(_ptr(x, _c_f32p), x.shape[0], x.shape[1],
                                                   _ptr(ends, _c_i32p), seq_len, n_seqs,
                                                   _ptr(out, _c_f32p))
        return out, rc

    def forward(self, p: dict, fp16_storage: bool = True):
        """LlamaRunner::forward (src/model/llama.cpp:78-184) composed of this
        module's operators, for a batch of sequences with per-token positions
        and slots over head-major caches [n_slots, Hkv, max_seq, D].

        `p` holds numpy arrays: table, ids, positions, slots, final_norm_w,
        lm_head, and `layers`, a list of dicts with input_norm_w, post_norm_w,
        q_bias, k_bias, v_bias (or None), wq, wk, wv, wo, w_gate, w_up, w_down
        ([out, in]) and the layer's k_cache, v_cache before the step; plus the
        shape scalars n_heads, n_kv_heads, head_dim, eps, theta, seq_len,
        n_seqs. With fp16_storage every op output (and the cache) is rounded
        to fp16, the storage points of the fp16 device path. Returns
        (last rows, logits, [(k_cache, v_cache) per layer])."""
        rnd = (lambda a: np.asarray(a, np.float32).astype(np.float16).astype(np.float32)) if fp16_storage \
            else (lambda a: np.asarray(a, np.float32))
        Hq, Hkv, D = p["n_heads"], p["n_kv_heads"], p["head_dim"]
        pos = np.ascontiguousarray(p["positions"], np.int32)
        slots = np.ascontiguousarray(p["slots"], np.int32)
        T = pos.size
        x = self.embedding(p["table"], p["ids"])
        d = None
        caches = []
        for L in p["layers"]:
            if d is not None:
                x = rnd(x + d)                                            # add_inplace(ffn_out, x)
            h = rnd(self.rms_norm(x, L["input_norm_w"], p["eps"]))
            q = rnd(self.matmul(h, L["wq"]))
            k = rnd(self.matmul(h, L["wk"]))
            v = rnd(self.matmul(h, L["wv"]))
            q, kc, vc, bad = self.qkv_bias_rope_kv_append(
                q.reshape(T, Hq, D), k.reshape(T, Hkv, D), v.reshape(T, Hkv, D), L["q_bias"], L["k_bias"],
                L["v_bias"], pos, slots, p["theta"], L["k_cache"], L["v_cache"])
            if bad:
                raise ValueError(f"{bad} tokens with an out-of-range position or slot")
            q, kc, vc = rnd(q), rnd(kc), rnd(vc)
            caches.append((kc, vc))
            ctx, bad = self.attention_head_major(q, kc, vc, pos, slots)
            a = rnd(self.matmul(rnd(ctx).reshape(T, Hq * D), L["wo"]))
            x = rnd(x + a)                                                # add_inplace(attn_out, x)
            h2 = rnd(self.rms_norm(x, L["post_norm_w"], p["eps"]))
            s = rnd(self.silu_mul(rnd(self.matmul(h2, L["w_gate"])), rnd(self.matmul(h2, L["w_up"]))))
            d = rnd(self.matmul(s, L["w_down"]))
        x = rnd(x + d)
        normed = rnd(self.rms_norm(x, p["final_norm_w"], p["eps"]))
        last, rc = self.select_last_rows(normed, seq_len=p["seq_len"], n_seqs=p["n_seqs"])
        if rc != 0:
            raise ValueError("select_last_rows: bad sequence end")
        return last, self.matmul(last, p["lm_head"]), caches

    def attention(self, q, k_cache, v_cache, past_len: int, n_kv_heads: int) -> np.ndarray:
        """q [seq, Hq, D]; caches [max_seq, Hkv, D] (the reference layout)."""
        q, kc, vc = _f32(q), _f32(k_cache), _f32(v_cache)
        out = np.empty_like(q)
        self.lib.kllm_oracle_attention(_ptr(q, _c_f32p), _ptr(kc, _c_f32p), _ptr(vc, _c_f32p),
                                       _ptr(out, _c_f32p), q.shape[0], past_len, q.shape[1],
                                       n_kv_heads, q.shape[2])
        return out

    def attention_head_major(self, q, k_cache, v_cache, positions, slots):
        """q [T, Hq, D]; caches [n_slots, Hkv, max_seq, D]. Returns (out, n_invalid)."""
        q, kc, vc = _f32(q), _f32(k_cache), _f32(v_cache)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        slo = np.ascontiguousarray(slots, dtype=np.int32)
        out = np.empty_like(q)
        bad = self.lib.kllm_oracle_attention_head_major(
            _ptr(q, _c_f32p), _ptr(kc, _c_f32p), _ptr(vc, _c_f32p), _ptr(out, _c_f32p),
            _ptr(pos, _c_i32p), _ptr(slo, _c_i32p), q.shape[0], q.shape[1], kc.shape[1], q.shape[2],
            kc.shape[0], kc.shape[2])
        if bad < 0:
            raise MemoryError("oracle attention: allocation failed")
        return out, int(bad)


class Reference:
    """The reference's compiled CPU operators (``oracle/_ref/libkllm_ref.so``).

    Buffers are passed as raw bytes of the given DType (F32 = 0, F16 = 1;
    fp16 arrays are np.float16 whose bits the reference reads as float16_t).
    """

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = lib = ctypes.CDLL(path)
        vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        lib.kref_last_error.restype = ctypes.c_char_p
        lib.kref_float_to_half.restype = ctypes.c_uint16
        lib.kref_float_to_half.argtypes = [ctypes.c_float]
        lib.kref_half_to_float.restype = ctypes.c_float
        lib.kref_half_to_float.argtypes = [ctypes.c_uint16]
        lib.kref_float_to_half_array.argtypes = [vp, vp, i64]
        lib.kref_embedding.argtypes = [vp, i64, i64, i32, vp, i64, vp]
        lib.kref_rms_norm.argtypes = [vp, vp, vp, i64, i64, ctypes.c_float, i32, i32]
        lib.kref_add_inplace.argtypes = [vp, vp, i64, i32]
        lib.kref_add_bias_inplace.argtypes = [vp, vp, i64, i64, i32]
        lib.kref_select_last_row.argtypes = [vp, i64, i64, vp, i32]
        lib.kref_silu_mul.argtypes = [vp, vp, vp, i64, i32]
        lib.kref_matmul.argtypes = [vp, vp, vp, i64, i64, i64, i32]
        lib.kref_rope_inplace.argtypes = [vp, i64, i64, i64, i32, ctypes.c_float, i32]
        lib.kref_copy_kv_to_cache.argtypes = [vp, vp, i64, i64, i64, vp, vp, i64, i32, i32]
        lib.kref_attention.argtypes = [vp, vp, vp, vp, i64, i64, i32, i32, i32, i32, i32]
        lib.kref_dequantize_int8.argtypes = [vp, i64, ctypes.c_float, vp]
        lib.kref_dequantize_int8_f16.argtypes = [vp, i64, ctypes.c_float, vp]
        lib.kref_runner_create.restype = vp
        lib.kref_runner_create.argtypes = [ctypes.c_char_p, i32]
        lib.kref_runner_destroy.argtypes = [vp]
        lib.kref_runner_forward.argtypes = [vp, vp, i32, i32, vp, i64]
        lib.kref_table_create.restype = vp
        lib.kref_table_create.argtypes = [i64, i64, ctypes.c_uint64]
        lib.kref_table_destroy.argtypes = [vp]
        lib.kref_chain_create.restype = vp
        lib.kref_chain_create.argtypes = [vp, i32, i32, i32, i32, i32, i32, ctypes.c_float,
                                          ctypes.c_float, ctypes.c_uint64]
        lib.kref_chain_destroy.argtypes = [vp]
        lib.kref_chain_run.restype = i32
        lib.kref_chain_run.argtypes = [vp, i32]
        lib.kref_weights_load.restype = vp
        lib.kref_weights_load.argtypes = [ctypes.c_char_p]
        lib.kref_weights_free.argtypes = [vp]
        lib.kref_weights_get.restype = i64
        lib.kref_weights_get.argtypes = [vp, ctypes.c_char_p, vp, i64]
        lib.kref_weights_dtype.restype = i32
        lib.kref_weights_dtype.argtypes = [vp, ctypes.c_char_p]

    def _check(self, rc: int) -> None:
        if rc != 0:
            raise RuntimeError(self.lib.kref_last_error().decode())

    @staticmethod
    def _buf(a, dtype: int) -> np.ndarray:
        return np.ascontiguousarray(a, dtype=np.float32 if dtype == F32 else np.float16)

    @staticmethod
    def _vp(a):
        return None if a is None else ctypes.c_void_p(a.ctypes.data)

    def float_to_half_bits(self, x) -> np.ndarray:
        x = _f32(x)
        out = np.empty(x.shape, dtype=np.uint16)
        self.lib.kref_float_to_half_array(self._vp(x), self._vp(out), x.size)
        return out

    def embedding(self, table, ids, dtype: int = F32):
        table = self._buf(table, dtype)
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros((ids.size, table.shape[1]), dtype=table.dtype)
        self._check(self.lib.kref_embedding(self._vp(table), table.shape[0], table.shape[1],
                                            dtype, self._vp(ids), ids.size, self._vp(out)))
        return out

    def rms_norm(self, x, w, eps: float, dtype: int = F32, w_dtype: int | None = None):
        w_dtype = dtype if w_dtype is None else w_dtype
        x, w = self._buf(x, dtype), self._buf(w, w_dtype)
        out = np.empty_like(x)
        self._check(self.lib.kref_rms_norm(self._vp(x), self._vp(w), self._vp(out), x.shape[0],
                                           x.shape[1], eps, dtype, w_dtype))
        return out

    def add(self, x, y, dtype: int = F32):
        x = self._buf(x, dtype).copy()
        y = self._buf(y, dtype)
        self._check(self.lib.kref_add_inplace(self._vp(x), self._vp(y), x.size, dtype))
        return x

    def add_bias(self, x, bias, dtype: int = F32):
        x = self._buf(x, dtype).copy()
        b = None if bias is None else self._buf(bias, dtype)
        self._check(self.lib.kref_add_bias_inplace(self._vp(x), self._vp(b), x.shape[0],
                                                   x.shape[1], dtype))
        return x

    def select_last_row(self, x, dtype: int = F32):
        x = self._buf(x, dtype)
        out = np.empty((1, x.shape[1]), dtype=x.dtype)
        self._check(self.lib.kref_select_last_row(self._vp(x), x.shape[0], x.shape[1],
                                                  self._vp(out), dtype))
        return out

    def matmul(self, a, b, dtype: int = F32):
        """kllm::op::matmul: a [m, k] times b [n, k] transposed."""
        a, b = self._buf(a, dtype), self._buf(b, dtype)
        out = np.empty((a.shape[0], b.shape[0]), dtype=a.dtype)
        self._check(self.lib.kref_matmul(self._vp(a), self._vp(b), self._vp(out), a.shape[0], b.shape[0],
                                         a.shape[1], dtype))
        return out

    def silu_mul(self, g, u, dtype: int = F32):
        g, u = self._buf(g, dtype), self._buf(u, dtype)
        out = np.empty_like(g)
        self._check(self.lib.kref_silu_mul(self._vp(g), self._vp(u), self._vp(out), g.size,
                                           dtype))
        return out

    def rope(self, x, past_len: int, theta: float, dtype: int = F32):
        x = self._buf(x, dtype).copy()
        self._check(self.lib.kref_rope_inplace(self._vp(x), x.shape[0], x.shape[1], x.shape[2],
                                               past_len, theta, dtype))
        return x

    def copy_kv_to_cache(self, k, v, k_cache, v_cache, past_len: int, dtype: int = F32):
        k, v = self._buf(k, dtype), self._buf(v, dtype)
        kc, vc = self._buf(k_cache, dtype).copy(), self._buf(v_cache, dtype).copy()
        self._check(self.lib.kref_copy_kv_to_cache(
            self._vp(k), self._vp(v), k.shape[0], k.shape[1], k.shape[2], self._vp(kc),
            self._vp(vc), kc.shape[0], past_len, dtype))
        return kc, vc

    def attention(self, q, k_cache, v_cache, past_len: int, n_kv_heads: int, dtype: int = F32):
        """kllm::op::attention: q [seq, Hq, D]; caches [max_seq, Hkv, D]."""
        q, kc, vc = self._buf(q, dtype), self._buf(k_cache, dtype), self._buf(v_cache, dtype)
        out = np.empty_like(q)
        self._check(self.lib.kref_attention(self._vp(q), self._vp(kc), self._vp(vc), self._vp(out),
                                            q.shape[0], kc.shape[0], past_len, q.shape[1], n_kv_heads,
                                            q.shape[2], dtype))
        return out

    def dequantize_int8_f32(self, q, scale: float):
        q = np.ascontiguousarray(q, dtype=np.int8)
        out = np.empty(q.shape, dtype=np.float32)
        self._check(self.lib.kref_dequantize_int8(self._vp(q), q.size, scale, self._vp(out)))
        return out

    def dequantize_int8_f16_bits(self, q, scale: float):
        q = np.ascontiguousarray(q, dtype=np.int8)
        out = np.empty(q.shape, dtype=np.uint16)
        self.lib.kref_dequantize_int8_f16(self._vp(q), q.size, scale, self._vp(out))
        return out


class ReferenceRunner:
    """The reference's LlamaRunner (src/model/llama.cpp) over a .kllm file on
    the CPU, F32 activations; one KV cache of max_seq positions."""

    def __init__(self, ref: "Reference", path: str, max_seq: int, vocab: int):
        self.lib, self.vocab = ref.lib, vocab
        self.h = self.lib.kref_runner_create(path.encode(), max_seq)
        if not self.h:
            raise RuntimeError(self.lib.kref_last_error().decode())

    def forward(self, ids, past_len: int) -> np.ndarray:
        """LlamaRunner::forward: the last token's logits."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.vocab, dtype=np.float32)
        if self.lib.kref_runner_forward(self.h, ctypes.c_void_p(ids.ctypes.data), ids.size, past_len,
                                        ctypes.c_void_p(out.ctypes.data), self.vocab) != 0:
            raise RuntimeError(self.lib.kref_last_error().decode())
        return out

    def close(self) -> None:
        if self.h:
            self.lib.kref_runner_destroy(self.h)
            self.h = None


class ReferenceWeights:
    """A .kllm file loaded by the reference's own ModelWeights::load on the
    CPU (INT8 records become fp32 float(q) * scale there)."""

    def __init__(self, ref: "Reference", path: str):
        self.lib = ref.lib
        self.h = self.lib.kref_weights_load(path.encode())
        if not self.h:
            raise RuntimeError(self.lib.kref_last_error().decode())

    def get(self, name: str, numel: int) -> np.ndarray:
        out = np.empty(max(numel, 1), dtype=np.float32)
        n = self.lib.kref_weights_get(self.h, name.encode(), ctypes.c_void_p(out.ctypes.data), out.size)
        if n < 0:
            raise KeyError(name)
        return out[:n]

    def dtype(self, name: str) -> int:
        return self.lib.kref_weights_dtype(self.h, name.encode())

    def close(self) -> None:
        if self.h:
            self.lib.kref_weights_free(self.h)
            self.h = None


def reference_available() -> bool:
    return os.path.exists(REF_SO)
