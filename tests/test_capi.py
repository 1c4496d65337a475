"""The C ABI on the CPU: the library loads, exports exactly what
include/kllm_b200.h declares, and rejects bad arguments with the documented
status codes before touching a GPU."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "kllm_b200.h")


@pytest.fixture(scope="module")
def capi():
    from littlellm_b200 import build
    build.build()
    from littlellm_b200 import _capi
    return _capi


def declared_functions() -> set[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(kllm_b200_[a-z0-9_]+)\s*\(", text))


def test_exports_match_header(capi):
    declared = declared_functions()
    assert len(declared) >= 16
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH if hasattr(capi, "LIB_PATH")
                          else capi.lib._name], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line and "kllm_b200_" in line}
    assert declared == exported, (declared ^ exported)
    for name in declared:
        assert hasattr(capi.lib, name)
    assert set(capi.SIGNATURES) == declared


def test_version_and_messages(capi):
    assert capi.lib.kllm_b200_version() >= 100
    assert capi.lib.kllm_b200_status_string(capi.ERR_CAPACITY) == b"KV cache capacity exceeded"
    assert capi.lib.kllm_b200_status_string(12345) == b"unknown status"


def _rc_msg(capi, rc):
    return rc, capi.last_error()


def test_argument_validation_without_gpu(capi):
    lib = capi.lib
    # null pointers
    rc, msg = _rc_msg(capi, lib.kllm_b200_silu_mul(None, None, None, 8, capi.F16, None))
    assert rc == capi.ERR_INVALID_ARG and "null" in msg
    # negative sizes
    assert lib.kllm_b200_add_inplace(1, 1, -1, capi.F16, capi.F16, None) == capi.ERR_INVALID_ARG
    # unsupported dtypes
    assert lib.kllm_b200_rms_norm(16, 16, 16, 4, 8, 1e-6, capi.I8, capi.F16, None) == capi.ERR_DTYPE
    assert lib.kllm_b200_dequantize_int8(16, 16, 16, 8, capi.I32, None) == capi.ERR_DTYPE
    # odd head_dim (the reference: "rope requires an even head_dim")
    rc, msg = _rc_msg(capi, lib.kllm_b200_rope_inplace(16, 2, 2, 7, 0, 1e4, capi.F16, None))
    assert rc == capi.ERR_SHAPE and "even" in msg
    rc = lib.kllm_b200_qkv_bias_rope_kv_append(16, 16, 16, None, None, None, capi.F16, 16, 16, 4, 2, 2, 258,
                                               1e4, 16, 16, 1, 8, None, None)
    assert rc == capi.ERR_SHAPE
    # KV capacity, as the reference CPU path checks it
    rc, msg = _rc_msg(capi, lib.kllm_b200_copy_kv_to_cache(16, 16, 4, 2, 8, 16, 16, 10, 7, capi.F16, capi.F16,
                                                           None))
    assert rc == capi.ERR_CAPACITY and "capacity" in msg
    assert lib.kllm_b200_copy_kv_to_cache(16, 16, 1, 2, 8, 16, 16, 10, -1, capi.F16, capi.F16,
                                          None) == capi.ERR_RANGE
    # select_last_rows with more rows requested than exist
    assert lib.kllm_b200_select_last_rows(16, 10, 8, None, 4, 3, 16, capi.F16, None, None) == capi.ERR_SHAPE
    # chain: null descriptor
    assert lib.kllm_b200_chain_run(None, None, None) == capi.ERR_INVALID_ARG
    # the fused embedding + norm and the host-ids embedding
    rc, msg = _rc_msg(capi, lib.kllm_b200_embedding_rms_norm(16, 10, 8, None, 4, 16, capi.F16, 1e-6, 16, 16,
                                                              None, None))
    assert rc == capi.ERR_INVALID_ARG and "null" in msg
    assert lib.kllm_b200_embedding_rms_norm(16, 10, 8, 16, 4, 16, capi.I8, 1e-6, 16, 16, None,
                                            None) == capi.ERR_DTYPE
    assert lib.kllm_b200_embedding_rms_norm(16, 10, 8, 16, -1, 16, capi.F16, 1e-6, 16, 16, None,
                                            None) == capi.ERR_INVALID_ARG
    assert lib.kllm_b200_embedding_host_ids(16, 10, 8, capi.F16, None, 4, 16, capi.F16, None,
                                            None) == capi.ERR_INVALID_ARG
    assert lib.kllm_b200_embedding_host_ids(16, 10, 8, capi.I32, 16, 4, 16, capi.F16, None,
                                            None) == capi.ERR_DTYPE


def test_empty_inputs_are_noops(capi):
    lib = capi.lib
    assert lib.kllm_b200_silu_mul(None, None, None, 0, capi.F16, None) == capi.OK
    assert lib.kllm_b200_embedding(None, 10, 8, capi.F16, None, 0, None, capi.F16, None, None) == capi.OK
    assert lib.kllm_b200_embedding_host_ids(None, 10, 8, capi.F16, None, 0, None, capi.F16, None, None) == capi.OK
    assert lib.kllm_b200_embedding_rms_norm(None, 10, 8, None, 0, None, capi.F16, 1e-6, None, None, None,
                                            None) == capi.OK
    assert lib.kllm_b200_add_bias_inplace(16, None, 4, 4, capi.F16, capi.F16, None) == capi.OK  # null bias
    assert lib.kllm_b200_dequantize_int8(None, None, None, 0, capi.F16, None) == capi.OK


def test_python_wrappers_refuse_host_tensors(capi):
    import torch

    from littlellm_b200 import ops
    x = torch.zeros(16, dtype=torch.float16)
    with pytest.raises(capi.KllmError) as e:
        ops.silu_mul(x, x)
    assert e.value.status == capi.ERR_INVALID_ARG


def test_last_error_is_per_thread(capi):
    import threading
    lib = capi.lib
    lib.kllm_b200_rope_inplace(16, 2, 2, 7, 0, 1e4, capi.F16, None)
    seen = {}

    def other():
        lib.kllm_b200_silu_mul(None, None, None, 8, capi.F16, None)
        seen["msg"] = capi.last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert "null" in seen["msg"]
    assert "even" in capi.last_error()


def test_chain_struct_layout(capi, tmp_path):
    # the ctypes mirrors of kllm_b200_chain, kllm_b200_layer_buffers and
    # kllm_b200_layer_weights must match the C layout the header declares:
    # compile a probe against include/kllm_b200.h and compare every offset
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    structs = {"kllm_b200_chain": capi.Chain, "kllm_b200_layer_buffers": capi.LayerBuffers,
               "kllm_b200_layer_weights": capi.LayerWeights}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "kllm_b200.h"', 'int main(void) {']
    for cname, cls in structs.items():
        lines.append(f'  printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ['  return 0;', '}']
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "probe"
    subprocess.run([cc, "-std=c11", "-I", os.path.join(root, "include"), str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        cname, fname, value = line.split()
        got[(cname, fname)] = int(value)
    for cname, cls in structs.items():
        assert got[(cname, "sizeof")] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, (cname, fname)


def test_attention_validation_without_gpu(capi):
    """kllm_b200_attention_head_major rejects bad shapes, dtypes and pointers
    on the host, before any CUDA call; the workspace query needs no GPU."""
    lib = capi.lib
    n = ctypes.c_int64(-1)
    assert lib.kllm_b200_attention_workspace_bytes(2048, 14, 2, 64, 4096, ctypes.addressof(n)) == capi.OK
    assert n.value >= 0
    assert lib.kllm_b200_attention_workspace_bytes(0, 14, 2, 64, 4096, ctypes.addressof(n)) == capi.OK
    assert n.value == 0
    assert lib.kllm_b200_attention_workspace_bytes(1, 1, 1, 64, 8, None) == capi.ERR_INVALID_ARG
    p = 16  # any non-null, 16-byte aligned value: nothing is dereferenced before validation fails
    cases = [
        ((p,) * 6 + (1, 1, 2, 2, 96, 1, 8, capi.F16), capi.ERR_SHAPE, "head_dim"),      # head_dim 96
        ((p,) * 6 + (1, 1, 3, 2, 64, 1, 8, capi.F16), capi.ERR_SHAPE, "multiple"),      # 3 heads over 2
        ((p,) * 6 + (1, 1, 40, 2, 64, 1, 8, capi.F16), capi.ERR_SHAPE, "16"),           # 20 per kv head
        ((p,) * 6 + (1, 1, 2, 2, 64, 1, 8, capi.F32), capi.ERR_DTYPE, "dtype"),
        ((None,) * 6 + (4, 1, 2, 2, 64, 1, 8, capi.F16), capi.ERR_INVALID_ARG, "null"),
        ((p + 2,) + (p,) * 5 + (4, 1, 2, 2, 64, 1, 8, capi.F16), capi.ERR_ALIGN, "aligned"),
        ((p,) * 6 + (4, 0, 2, 2, 64, 1, 8, capi.F16), capi.ERR_SHAPE, "seq_len"),
        ((p,) * 6 + (4, 1, 2, 2, 64, 0, 8, capi.F16), capi.ERR_SHAPE, "empty cache"),
    ]
    for args, status, word in cases:
        rc = lib.kllm_b200_attention_head_major(*args, None, 0, None, None)
        assert rc == status, (args, rc, capi.last_error())
        assert word in capi.last_error()
    # nothing to do: no tokens
    assert lib.kllm_b200_attention_head_major(*(None,) * 6, 0, 1, 2, 2, 64, 1, 8, capi.F16, None, 0, None,
                                              None) == capi.OK


def test_chain_attention_needs_context_buffers(capi):
    """KLLM_B200_OP_ATTENTION with a layer lacking attn_ctx is refused before
    any launch."""
    layers = (capi.LayerBuffers * 2)()
    c = capi.Chain()
    c.n_tokens, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim = 4, 64, 2, 2, 64
    c.intermediate, c.vocab, c.n_layers, c.n_slots, c.max_seq, c.n_seqs, c.seq_len = 128, 10, 2, 1, 8, 1, 4
    c.weight_dtype = capi.F16
    c.op_mask = capi.OP_CHAIN | capi.OP_ATTENTION
    c.layers = ctypes.cast(layers, ctypes.POINTER(capi.LayerBuffers))
    assert capi.lib.kllm_b200_chain_run(ctypes.byref(c), None, None) == capi.ERR_INVALID_ARG
    assert "attn_ctx" in capi.last_error()


def test_chain_gemm_needs_attention_and_weights(capi):
    """KLLM_B200_OP_GEMM without the attention op, without weights, or with a
    layer missing a weight is refused before any launch."""
    p = 256
    layers = (capi.LayerBuffers * 2)()
    for L in layers:
        L.attn_ctx = p
    weights = (capi.LayerWeights * 2)()
    c = capi.Chain()
    c.n_tokens, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim = 4, 64, 2, 2, 64
    c.intermediate, c.vocab, c.n_layers, c.n_slots, c.max_seq, c.n_seqs, c.seq_len = 128, 10, 2, 1, 8, 1, 4
    c.weight_dtype = capi.F16
    c.layers = ctypes.cast(layers, ctypes.POINTER(capi.LayerBuffers))
    c.op_mask = capi.OP_CHAIN | capi.OP_GEMM
    assert capi.lib.kllm_b200_chain_run(ctypes.byref(c), None, None) == capi.ERR_INVALID_ARG
    assert "attention" in capi.last_error()
    c.op_mask = capi.OP_FORWARD
    assert capi.lib.kllm_b200_chain_run(ctypes.byref(c), None, None) == capi.ERR_INVALID_ARG
    assert "weights" in capi.last_error()
    c.weights = ctypes.cast(weights, ctypes.POINTER(capi.LayerWeights))
    for W in weights:
        for name in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down"):
            setattr(W, name, p)
    weights[1].w_down = None
    assert capi.lib.kllm_b200_chain_run(ctypes.byref(c), None, None) == capi.ERR_INVALID_ARG
    assert "layer 1" in capi.last_error()


def test_gemm_validation_without_gpu(capi):
    """kllm_b200_linear / kllm_b200_linear_swiglu reject bad sizes, pointers,
    alignment and bias dtypes on the host, before any CUDA call; an empty
    output is a successful no-op."""
    lib = capi.lib
    p = 16  # non-null and 16-byte aligned; nothing is dereferenced before validation fails
    cases = [  # (x, w, bias, bias_dtype, out, m, n, k)
        ((p, p, None, capi.F16, p, -1, 8, 8), capi.ERR_INVALID_ARG, "negative"),
        ((p, p, None, capi.F16, p, 4, 8, 0), capi.ERR_SHAPE, "positive"),
        ((p, p, None, capi.F16, p, 4, 8, 12), capi.ERR_SHAPE, "multiple of 8"),
        ((None, p, None, capi.F16, p, 4, 8, 8), capi.ERR_INVALID_ARG, "null"),
        ((p + 8, p, None, capi.F16, p, 4, 8, 8), capi.ERR_ALIGN, "aligned"),
        ((p, p, p + 2, capi.F16, p, 4, 8, 8), capi.ERR_ALIGN, "bias"),
        ((p, p, p, capi.I32, p, 4, 8, 8), capi.ERR_DTYPE, "bias dtype"),
    ]
    for args, status, word in cases:
        rc = lib.kllm_b200_linear(*args, None, None)
        assert rc == status, (args, rc, capi.last_error())
        assert word in capi.last_error()
    assert lib.kllm_b200_linear(p, p, None, capi.F16, p, 0, 8, 8, None, None) == capi.OK
    assert lib.kllm_b200_linear(p, p, None, capi.F16, p, 4, 0, 8, None, None) == capi.OK
    # the SwiGLU form also needs the up weight
    rc = lib.kllm_b200_linear_swiglu(p, p, None, None, None, capi.F16, p, 4, 8, 8, None, None)
    assert rc == capi.ERR_INVALID_ARG and "null" in capi.last_error()
    rc = lib.kllm_b200_linear_swiglu(p, p, p + 8, None, None, capi.F16, p, 4, 8, 8, None, None)
    assert rc == capi.ERR_ALIGN
    assert lib.kllm_b200_linear_swiglu(p, p, p, None, None, capi.F16, p, 0, 8, 8, None, None) == capi.OK


def test_qkv_rope_linear_validation_without_gpu(capi):
    """kllm_b200_qkv_linear_rope_kv_append rejects bad shapes, pointers and
    alignment before any CUDA call; no tokens is a successful no-op."""
    lib = capi.lib
    p = 16

    def call(x=p, wq=p, n_tokens=4, hidden=64, hq=2, hkv=2, d=64, n_slots=1, max_seq=8, bias=None,
             bias_dtype=capi.F16):
        return lib.kllm_b200_qkv_linear_rope_kv_append(x, wq, p, p, bias, None, None, bias_dtype, p, p, n_tokens,
                                                       hidden, hq, hkv, d, 1e4, p, p, p, n_slots, max_seq, None, None)

    assert call(d=96) == capi.ERR_SHAPE and "head_dim" in capi.last_error()
    assert call(hidden=60) == capi.ERR_SHAPE and "multiple of 8" in capi.last_error()
    assert call(max_seq=0) == capi.ERR_SHAPE and "empty cache" in capi.last_error()
    assert call(hq=0) == capi.ERR_SHAPE
    assert call(x=None) == capi.ERR_INVALID_ARG and "null" in capi.last_error()
    assert call(wq=p + 8) == capi.ERR_ALIGN
    assert call(bias=p, bias_dtype=capi.I8) == capi.ERR_DTYPE
    assert call(n_tokens=-1) == capi.ERR_INVALID_ARG
    assert call(n_tokens=0) == capi.OK


def test_set_pdl_is_per_thread_and_returns_previous(capi):
    import threading
    lib = capi.lib
    assert lib.kllm_b200_set_pdl(1) == 0
    assert lib.kllm_b200_set_pdl(1) == 1
    seen = []
    t = threading.Thread(target=lambda: seen.append(lib.kllm_b200_set_pdl(0)))
    t.start()
    t.join()
    assert seen == [0]  # another thread starts from the default (off)
    assert lib.kllm_b200_set_pdl(0) == 1
