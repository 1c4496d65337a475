"""torch-facing wrappers of the C ABI.

One function per operator of the reference interface
(``include/kllm/op/ops.h:10-35``: embedding, rms_norm, add_bias_inplace,
add_inplace, select_last_row, silu_mul, rope_inplace, copy_kv_to_cache,
dequantize_int8) plus the fused/batched entry points (add_rms_norm,
qkv_bias_rope_kv_append, select_last_rows, attention_head_major, linear,
linear_swiglu). Each takes CUDA tensors, passes
their device pointers to ``libkllm_b200.so`` on the tensor's current stream
and raises ``KllmError`` with the library's message on a non-zero status,
the way the reference throws ``std::runtime_error``.

torch supplies device memory and streams here; all arithmetic happens in the
library's kernels.
"""
from __future__ import annotations

import torch

from . import _capi
from ._capi import F16, F32, I8, I32, KllmError, check, lib

_DTYPES = {torch.float32: F32, torch.float16: F16, torch.int32: I32, torch.int8: I8}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise KllmError(_capi.ERR_DTYPE, f"unsupported tensor dtype {t.dtype}") from None


def _dev(*tensors):
    """Checks that every given tensor is a contiguous CUDA tensor on one device
    and returns that device."""
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise KllmError(_capi.ERR_INVALID_ARG, "expected a CUDA tensor")
        if not t.is_contiguous():
            raise KllmError(_capi.ERR_SHAPE, "expected a contiguous tensor")
        if device is None:
            device = t.device
        elif t.device != device:
            raise KllmError(_capi.ERR_INVALID_ARG, "tensors are on different devices")
    return device


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def set_pdl(enable: bool) -> bool:
    """Launch mode of the individual entry points for this host thread
    (kllm_b200_set_pdl): programmatic dependent launch with the inputs no
    kernel of the library writes read before the dependency wait. Returns the
    previous mode."""
    return bool(lib.kllm_b200_set_pdl(1 if enable else 0))


def embedding(table: torch.Tensor, ids: torch.Tensor, out: torch.Tensor | None = None,
              err_flags: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = table[ids[t]] (reference embedding, ids on the device)."""
    if out is None:
        out = torch.empty((ids.numel(), table.shape[1]), dtype=table.dtype, device=table.device)
    dev = _dev(table, ids, out, err_flags)
    if ids.dtype != torch.int32:
        raise KllmError(_capi.ERR_DTYPE, "ids must be int32")
    with torch.cuda.device(dev):
        check(lib.kllm_b200_embedding(_ptr(table), table.shape[0], table.shape[1], dtype_code(table),
                                      _ptr(ids), ids.numel(), _ptr(out), dtype_code(out),
                                      _ptr(err_flags), _stream(dev)))
    return out


def embedding_host_ids(table: torch.Tensor, ids, out: torch.Tensor | None = None,
                       err_flags: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = table[ids[t]] with the ids in host memory (a sequence of ints,
    as the reference's cuda_embedding takes them); they travel in the kernel
    launches' parameters, no device buffer or blocking copy."""
    import numpy as np
    host = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
    if out is None:
        out = torch.empty((host.size, table.shape[1]), dtype=table.dtype, device=table.device)
    dev = _dev(table, out, err_flags)
    with torch.cuda.device(dev):
        check(lib.kllm_b200_embedding_host_ids(_ptr(table), table.shape[0], table.shape[1], dtype_code(table),
                                               host.ctypes.data, host.size, _ptr(out), dtype_code(out),
                                               _ptr(err_flags), _stream(dev)))
    return out


def embedding_rms_norm(table: torch.Tensor, ids: torch.Tensor, weight: torch.Tensor, eps: float,
                       residual: torch.Tensor | None = None, out: torch.Tensor | None = None,
                       err_flags: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """residual = table[ids] and out = rms_norm(residual) * weight, one launch
    (embedding + layer 0's input norm). Returns (residual, out)."""
    if ids.dtype != torch.int32:
        raise KllmError(_capi.ERR_DTYPE, "ids must be int32")
    if table.dtype != torch.float16:
        raise KllmError(_capi.ERR_DTYPE, "embedding_rms_norm takes an fp16 table")
    shape = (ids.numel(), table.shape[1])
    if residual is None:
        residual = torch.empty(shape, dtype=table.dtype, device=table.device)
    if out is None:
        out = torch.empty(shape, dtype=table.dtype, device=table.device)
    dev = _dev(table, ids, weight, residual, out, err_flags)
    with torch.cuda.device(dev):
        check(lib.kllm_b200_embedding_rms_norm(_ptr(table), table.shape[0], table.shape[1], _ptr(ids), ids.numel(),
                                               _ptr(weight), dtype_code(weight), eps, _ptr(residual), _ptr(out),
                                               _ptr(err_flags), _stream(dev)))
    return residual, out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float,
             out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    dev = _dev(x, weight, out)
    hidden = x.shape[-1]
    with torch.cuda.device(dev):
        check(lib.kllm_b200_rms_norm(_ptr(x), _ptr(weight), _ptr(out), x.numel() // hidden, hidden,
                                     eps, dtype_code(x), dtype_code(weight), _stream(dev)))
    return out


def add_rms_norm(residual: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor,
                 eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """residual += delta (stored, fp16-rounded); returns RMSNorm(residual) * weight."""
    if out is None:
        out = torch.empty_like(residual)
    dev = _dev(residual, delta, weight, out)
    hidden = residual.shape[-1]
    with torch.cuda.device(dev):
        check(lib.kllm_b200_add_rms_norm(_ptr(residual), _ptr(delta), _ptr(weight), _ptr(out),
                                         residual.numel() // hidden, hidden, eps,
                                         dtype_code(residual), dtype_code(weight), _stream(dev)))
    return out


def add_inplace(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    dev = _dev(x, y)
    if x.numel() != y.numel():
        raise KllmError(_capi.ERR_SHAPE, "add shape mismatch")
    with torch.cuda.device(dev):
        check(lib.kllm_b200_add_inplace(_ptr(x), _ptr(y), x.numel(), dtype_code(x), dtype_code(y),
                                        _stream(dev)))
    return x


def add_bias_inplace(x: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    if bias is None:
        return x
    dev = _dev(x, bias)
    cols = x.shape[-1]
    with torch.cuda.device(dev):
        check(lib.kllm_b200_add_bias_inplace(_ptr(x), _ptr(bias), x.numel() // cols, cols,
                                             dtype_code(x), dtype_code(bias), _stream(dev)))
    return x


def select_last_row(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty((1, x.shape[-1]), dtype=x.dtype, device=x.device)
    dev = _dev(x, out)
    cols = x.shape[-1]
    with torch.cuda.device(dev):
        check(lib.kllm_b200_select_last_row(_ptr(x), x.numel() // cols, cols, _ptr(out),
                                            dtype_code(x), _stream(dev)))
    return out


def select_last_rows(x: torch.Tensor, seq_len: int = 0, n_seqs: int | None = None,
                     seq_ends: torch.Tensor | None = None, out: torch.Tensor | None = None,
                     err_flags: torch.Tensor | None = None) -> torch.Tensor:
    cols = x.shape[-1]
    rows = x.numel() // cols
    if seq_ends is not None:
        n_seqs = seq_ends.numel()
    elif n_seqs is None:
        n_seqs = rows // seq_len
    if out is None:
        out = torch.empty((n_seqs, cols), dtype=x.dtype, device=x.device)
    dev = _dev(x, out, seq_ends, err_flags)
    with torch.cuda.device(dev):
        check(lib.kllm_b200_select_last_rows(_ptr(x), rows, cols, _ptr(seq_ends), seq_len, n_seqs,
                                             _ptr(out), dtype_code(x), _ptr(err_flags),
                                             _stream(dev)))
    return out


def attention_workspace_bytes(n_tokens: int, n_heads: int, n_kv_heads: int, head_dim: int,
                              max_seq: int) -> int:
    import ctypes
    n = ctypes.c_int64(0)
    check(lib.kllm_b200_attention_workspace_bytes(n_tokens, n_heads, n_kv_heads, head_dim, max_seq,
                                                  ctypes.addressof(n)))
    return n.value


def attention_head_major(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         positions: torch.Tensor, slots: torch.Tensor, seq_len: int = 1,
                         out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                         err_flags: torch.Tensor | None = None) -> torch.Tensor:
    """Causal attention of q [T, Hq, D] over the head-major cache of one
    layer [n_slots, Hkv, max_seq, D]: token t sees positions 0..positions[t]
    of slot slots[t]. ``workspace=None`` allocates the preferred split
    workspace here, zero-filled (the C entry point itself never allocates; a
    caller-provided workspace must be zeroed once before its first use)."""
    T, Hq, D = q.shape
    n_slots, Hkv, max_seq, _ = k_cache.shape
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        nbytes = attention_workspace_bytes(T, Hq, Hkv, D, max_seq)
        workspace = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=q.device)
    dev = _dev(q, k_cache, v_cache, positions, slots, out, workspace, err_flags)
    if positions.dtype != torch.int32 or slots.dtype != torch.int32:
        raise KllmError(_capi.ERR_DTYPE, "attention: positions and slots must be int32")
    with torch.cuda.device(dev):
        check(lib.kllm_b200_attention_head_major(
            _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(out), _ptr(positions), _ptr(slots), T, seq_len, Hq,
            Hkv, D, n_slots, max_seq, dtype_code(q), _ptr(workspace), workspace.numel(), _ptr(err_flags),
            _stream(dev)))
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(gate)
    dev = _dev(gate, up, out)
    if not (gate.numel() == up.numel() == out.numel()):
        raise KllmError(_capi.ERR_SHAPE, "silu_mul shape mismatch")
    if not (gate.dtype == up.dtype == out.dtype):
        raise KllmError(_capi.ERR_DTYPE, "silu_mul dtype mismatch")
    with torch.cuda.device(dev):
        check(lib.kllm_b200_silu_mul(_ptr(gate), _ptr(up), _ptr(out), gate.numel(),
                                     dtype_code(gate), _stream(dev)))
    return out


def _gemm_checks(x: torch.Tensor, weights, out: torch.Tensor, biases):
    if x.dim() != 2 or any(w.dim() != 2 for w in weights):
        raise KllmError(_capi.ERR_SHAPE, "linear: x and weights must be 2-D")
    if any(t.dtype != torch.float16 for t in (x, out, *weights)):
        raise KllmError(_capi.ERR_DTYPE, "linear: x, weights and out must be float16")
    n, k = weights[0].shape
    if x.shape[1] != k or any(w.shape != (n, k) for w in weights) or out.shape != (x.shape[0], n):
        raise KllmError(_capi.ERR_SHAPE, "linear shape mismatch")
    present = [b for b in biases if b is not None]
    if any(b.numel() != n for b in present):
        raise KllmError(_capi.ERR_SHAPE, "linear: bias length must equal the output columns")
    if len({b.dtype for b in present}) > 1:
        raise KllmError(_capi.ERR_DTYPE, "linear_swiglu: biases must share a dtype")
    return dtype_code(present[0]) if present else F16


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None, err_flags: torch.Tensor | None = None) -> torch.Tensor:
    """out = fp16(fp16(x @ w.T) + bias): the reference linear() (matmul +
    add_bias_inplace) as one tcgen05 GEMM. x [m, k], w [n, k] fp16."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=torch.float16, device=x.device)
    dev = _dev(x, w, bias, out, err_flags)
    bias_dtype = _gemm_checks(x, [w], out, [bias])
    with torch.cuda.device(dev):
        check(lib.kllm_b200_linear(_ptr(x), _ptr(w), _ptr(bias), bias_dtype, _ptr(out), x.shape[0],
                                   w.shape[0], x.shape[1], _ptr(err_flags), _stream(dev)))
    return out


def linear_swiglu(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                  b_gate: torch.Tensor | None = None, b_up: torch.Tensor | None = None,
                  out: torch.Tensor | None = None, err_flags: torch.Tensor | None = None) -> torch.Tensor:
    """out = silu_mul(linear(x, w_gate, b_gate), linear(x, w_up, b_up)) in one
    kernel; w_gate and w_up [n, k] fp16."""
    if out is None:
        out = torch.empty(x.shape[0], w_gate.shape[0], dtype=torch.float16, device=x.device)
    dev = _dev(x, w_gate, w_up, b_gate, b_up, out, err_flags)
    bias_dtype = _gemm_checks(x, [w_gate, w_up], out, [b_gate, b_up])
    with torch.cuda.device(dev):
        check(lib.kllm_b200_linear_swiglu(_ptr(x), _ptr(w_gate), _ptr(w_up), _ptr(b_gate), _ptr(b_up),
                                          bias_dtype, _ptr(out), x.shape[0], w_gate.shape[0], x.shape[1],
                                          _ptr(err_flags), _stream(dev)))
    return out


def qkv_linear_rope_kv_append(x: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor,
                              bq: torch.Tensor | None, bk: torch.Tensor | None, bv: torch.Tensor | None,
                              positions: torch.Tensor, slots: torch.Tensor, theta: float,
                              k_cache: torch.Tensor, v_cache: torch.Tensor, q_out: torch.Tensor | None = None,
                              err_flags: torch.Tensor | None = None) -> torch.Tensor:
    """q = rope(x @ wq.T + bq) into q_out [T, Hq*D]; k = rope(x @ wk.T + bk) and
    v = x @ wv.T + bv appended to the caches [n_slots, Hkv, max_seq, D] (one
    tcgen05 GEMM with the bias + RoPE + KV append in its epilogue)."""
    n_slots, Hkv, max_seq, D = k_cache.shape
    Hq = wq.shape[0] // D
    if q_out is None:
        q_out = torch.empty(x.shape[0], wq.shape[0], dtype=torch.float16, device=x.device)
    dev = _dev(x, wq, wk, wv, bq, bk, bv, positions, slots, k_cache, v_cache, q_out, err_flags)
    bias = next((b for b in (bq, bk, bv) if b is not None), None)
    bias_dtype = dtype_code(bias) if bias is not None else F16
    with torch.cuda.device(dev):
        check(lib.kllm_b200_qkv_linear_rope_kv_append(
            _ptr(x), _ptr(wq), _ptr(wk), _ptr(wv), _ptr(bq), _ptr(bk), _ptr(bv), bias_dtype, _ptr(positions),
            _ptr(slots), x.shape[0], x.shape[1], Hq, Hkv, D, theta, _ptr(q_out), _ptr(k_cache), _ptr(v_cache),
            n_slots, max_seq, _ptr(err_flags), _stream(dev)))
    return q_out


def rope_inplace(x: torch.Tensor, past_len: int, theta: float) -> torch.Tensor:
    """x [seq, heads, head_dim] rotated in place at positions past_len + t."""
    dev = _dev(x)
    seq, heads, head_dim = x.shape
    with torch.cuda.device(dev):
        check(lib.kllm_b200_rope_inplace(_ptr(x), seq, heads, head_dim, past_len, theta,
                                         dtype_code(x), _stream(dev)))
    return x


def copy_kv_to_cache(k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                     v_cache: torch.Tensor, past_len: int) -> None:
    """k/v [seq, kv_heads, head_dim] -> caches [max_seq, kv_heads, head_dim] at past_len."""
    dev = _dev(k, v, k_cache, v_cache)
    seq, kv_heads, head_dim = k.shape
    with torch.cuda.device(dev):
        check(lib.kllm_b200_copy_kv_to_cache(_ptr(k), _ptr(v), seq, kv_heads, head_dim,
                                             _ptr(k_cache), _ptr(v_cache), k_cache.shape[0],
                                             past_len, dtype_code(k), dtype_code(k_cache),
                                             _stream(dev)))


def qkv_bias_rope_kv_append(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            bq: torch.Tensor | None, bk: torch.Tensor | None,
                            bv: torch.Tensor | None, positions: torch.Tensor,
                            slots: torch.Tensor, theta: float, k_cache: torch.Tensor,
                            v_cache: torch.Tensor,
                            err_flags: torch.Tensor | None = None) -> None:
    """q [T, Hq, D] rotated in place; k/v [T, Hkv, D] appended (rotated /
    biased) into caches [n_slots, Hkv, max_seq, D]."""
    dev = _dev(q, k, v, bq, bk, bv, positions, slots, k_cache, v_cache, err_flags)
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    bias = next((b for b in (bq, bk, bv) if b is not None), None)
    bias_dtype = dtype_code(bias) if bias is not None else F16
    with torch.cuda.device(dev):
        check(lib.kllm_b200_qkv_bias_rope_kv_append(
            _ptr(q), _ptr(k), _ptr(v), _ptr(bq), _ptr(bk), _ptr(bv), bias_dtype, _ptr(positions),
            _ptr(slots), T, Hq, Hkv, D, theta, _ptr(k_cache), _ptr(v_cache), k_cache.shape[0],
            k_cache.shape[2], _ptr(err_flags), _stream(dev)))


def dequantize_int8(data: torch.Tensor, scale: torch.Tensor,
                    out_dtype: torch.dtype = torch.float16,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """out = data * scale[0]; fp16 output rounds like the reference weight loader."""
    if out is None:
        out = torch.empty(data.shape, dtype=out_dtype, device=data.device)
    dev = _dev(data, scale, out)
    if data.dtype != torch.int8 or scale.dtype != torch.float32:
        raise KllmError(_capi.ERR_DTYPE, "dequantize_int8 expects int8 data and an fp32 scale")
    with torch.cuda.device(dev):
        check(lib.kllm_b200_dequantize_int8(_ptr(data), _ptr(scale), _ptr(out), data.numel(),
                                            dtype_code(out), _stream(dev)))
    return out


def dequantize_int8_rne(data: torch.Tensor, scale: torch.Tensor, out: torch.Tensor | None = None,
                        mismatches: torch.Tensor | None = None) -> torch.Tensor:
    """out = data * scale[0] in fp16 rounded to nearest even (IEEE), not by
    the reference loader's rounding; when given, ``mismatches`` (a CUDA int64
    tensor of one element) is increased by the number of elements where the
    two roundings differ."""
    if out is None:
        out = torch.empty(data.shape, dtype=torch.float16, device=data.device)
    dev = _dev(data, scale, out, mismatches)
    if data.dtype != torch.int8 or scale.dtype != torch.float32 or out.dtype != torch.float16:
        raise KllmError(_capi.ERR_DTYPE, "dequantize_int8_rne expects int8 data, an fp32 scale and fp16 out")
    if mismatches is not None and (mismatches.dtype != torch.int64 or mismatches.numel() != 1):
        raise KllmError(_capi.ERR_DTYPE, "dequantize_int8_rne: mismatches must be one int64")
    with torch.cuda.device(dev):
        check(lib.kllm_b200_dequantize_int8_rne(_ptr(data), _ptr(scale), _ptr(out), data.numel(), _ptr(mismatches),
                                                _stream(dev)))
    return out


def dequantize_int8_batched(data: list[torch.Tensor], scales: list[torch.Tensor],
                            outs: list[torch.Tensor]) -> list[torch.Tensor]:
    """outs[i] = data[i] * scales[i][0] for every i in one launch (rounding
    as in dequantize_int8 for the outputs' dtype, which must all match)."""
    import ctypes
    n = len(data)
    if not (len(scales) == len(outs) == n):
        raise KllmError(_capi.ERR_SHAPE, "dequantize_int8_batched: list lengths differ")
    if n == 0:
        return outs
    dev = _dev(*data, *scales, *outs)
    out_dtypes = {dtype_code(o) for o in outs}
    if len(out_dtypes) != 1:
        raise KllmError(_capi.ERR_DTYPE, "dequantize_int8_batched: outputs must share one dtype")
    for d, sc, o in zip(data, scales, outs):
        if d.dtype != torch.int8 or sc.dtype != torch.float32 or d.numel() != o.numel():
            raise KllmError(_capi.ERR_DTYPE, "dequantize_int8_batched: int8 data, fp32 scale, matching sizes")
    arr = ctypes.c_void_p * n
    d_arr = arr(*[d.data_ptr() for d in data])
    s_arr = arr(*[sc.data_ptr() for sc in scales])
    o_arr = arr(*[o.data_ptr() for o in outs])
    c_arr = (ctypes.c_int64 * n)(*[d.numel() for d in data])
    with torch.cuda.device(dev):
        check(lib.kllm_b200_dequantize_int8_batched(d_arr, s_arr, o_arr, c_arr, n, out_dtypes.pop(),
                                                    _stream(dev)))
    return outs
