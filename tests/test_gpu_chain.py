"""The native chain executor (kllm_b200_chain_run) against the oracle applied
op by op in the reference's order (src/model/llama.cpp:78-178), with the
residual stream held in fp16 as the reference's CUDA runner holds it."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import assert_tol, bits16, host

pytestmark = pytest.mark.gpu


def f16r(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float32)


def _tiny(decode: bool, shape: str = "tiny"):
    from littlellm_b200.chain import ModelShape, Workload
    shapes = {
        "tiny": ModelShape("tiny", 128, 4, 2, 32, 384, 1000, 3, 1e-6, 1e4),
        # Qwen2.5-0.5B and Llama-2-7B layer shapes, 2 layers, small vocab
        "qwen": ModelShape("qwen-2l", 896, 14, 2, 64, 4864, 2000, 2, 1e-6, 1e6),
        "llama": ModelShape("llama-2l", 4096, 32, 32, 128, 11008, 2000, 2, 1e-5, 1e4),
    }
    m = shapes[shape]
    if decode:
        return Workload(f"{shape}_decode", m, n_seqs=9, seq_len=1, max_seq=64, decode=True)
    return Workload(f"{shape}_prefill", m, n_seqs=3, seq_len=17, max_seq=64, decode=False)


@pytest.mark.parametrize("shape,wdt", [("tiny", "f16"), ("qwen", "f16"), ("llama", "f16"), ("qwen", "f32")])
@pytest.mark.parametrize("decode", [False, True])
@pytest.mark.parametrize("use_pdl", [False, True])
def test_chain_matches_oracle(cuda, oracle, shape, wdt, decode, use_pdl):
    """fp16 activations; norm weights and q/k/v biases in fp16, or fp32 (the
    weight dtype the reference's dispatch also accepts)."""
    from littlellm_b200.chain import ChainRunner
    w = _tiny(decode, shape)
    m = w.model
    r = ChainRunner(w, device=cuda, seed=3, use_pdl=use_pdl,
                    weight_dtype=torch.float32 if wdt == "f32" else torch.float16)
    snap = [{k: host(t) for k, t in L.items()} for L in r.layers]
    table, ids = host(r.table), r.ids.cpu().numpy()
    pos, slots = r.positions.cpu().numpy(), r.slots.cpu().numpy()
    launches = r.run()
    torch.cuda.synchronize()
    # the embedding and layer 0's input norm are one kernel, the final norm writes the last rows
    assert launches == 4 * m.n_layers + 1
    assert int(r.err_flags.item()) == 0

    T, D = w.n_tokens, m.head_dim
    res = oracle.embedding(table, ids)
    for l, L in enumerate(snap):
        if l > 0:
            res = f16r(res + snap[l - 1]["ffn_out"])
        assert_tol(host(r.layers[l]["attn_norm_out"]), oracle.rms_norm(res, L["input_norm_w"], m.eps),
                   what=f"attn_norm {l}")
        zeros = np.zeros((w.n_seqs, m.n_kv_heads, w.max_seq, D), np.float32)
        q_ref, kc_ref, vc_ref, skipped = oracle.qkv_bias_rope_kv_append(
            L["q"].reshape(T, m.n_heads, D), L["k"].reshape(T, m.n_kv_heads, D),
            L["v"].reshape(T, m.n_kv_heads, D), L["q_bias"], L["k_bias"], L["v_bias"], pos, slots,
            m.theta, zeros, zeros)
        assert skipped == 0
        assert_tol(host(r.layers[l]["q"]).reshape(T, m.n_heads, D), q_ref, what=f"q {l}")
        kc, vc = host(r.layers[l]["k_cache"]), host(r.layers[l]["v_cache"])
        assert_tol(kc[slots, :, pos], kc_ref[slots, :, pos], what=f"k cache {l}")
        assert_tol(vc[slots, :, pos], vc_ref[slots, :, pos], what=f"v cache {l}")
        res = f16r(res + L["attn_out"])
        assert_tol(host(r.layers[l]["ffn_norm_out"]), oracle.rms_norm(res, L["post_norm_w"], m.eps),
                   what=f"ffn_norm {l}")
        assert_tol(host(r.layers[l]["swiglu_out"]), oracle.silu_mul(L["gate"], L["up"]), what=f"swiglu {l}")
    res = f16r(res + snap[-1]["ffn_out"])
    # the running residual is bit-exact: fp32 sums of the same fp16 values, rounded to nearest even
    assert np.array_equal(bits16(r.residual), res.astype(np.float16).view(np.uint16))
    final = oracle.rms_norm(res, host(r.final_norm_w), m.eps)
    assert_tol(host(r.final_norm_out), final, what="final norm")
    last = final[w.seq_len - 1::w.seq_len]
    assert np.array_equal(bits16(r.last_rows), bits16(r.final_norm_out)[w.seq_len - 1::w.seq_len])
    assert_tol(host(r.last_rows), last, what="last rows")


def test_chain_graph_replay_equals_eager(cuda):
    """A CUDA graph of the chain (as the benchmark replays it) does the work
    of an eager launch: outputs cleared after capture are rewritten by the
    replay with the eager values."""
    from littlellm_b200.chain import ChainRunner
    w = _tiny(False)
    a = ChainRunner(w, device=cuda, seed=9, use_pdl=True)
    b = ChainRunner(w, device=cuda, seed=9, use_pdl=True)
    a.run()
    s = torch.cuda.Stream(cuda)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        b.run(s)
    torch.cuda.synchronize()
    b.final_norm_out.zero_()
    b.last_rows.zero_()
    for L in b.layers:
        L["swiglu_out"].zero_()
        L["attn_norm_out"].zero_()
    with torch.cuda.stream(s):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(a.final_norm_out, b.final_norm_out)
    assert torch.equal(a.last_rows, b.last_rows)
    assert torch.equal(a.layers[-1]["swiglu_out"], b.layers[-1]["swiglu_out"])
    assert torch.equal(a.layers[1]["attn_norm_out"], b.layers[1]["attn_norm_out"])
    assert torch.equal(a.layers[0]["q"], b.layers[0]["q"])
    del g


def test_chain_op_mask_launches_only_selected_ops(cuda, oracle):
    """op_mask = SwiGLU only: one launch per layer, SwiGLU outputs right,
    the norm outputs untouched (profiling mode of the chain executor)."""
    from littlellm_b200 import _capi
    from littlellm_b200.chain import ChainRunner
    w = _tiny(False, "qwen")
    r = ChainRunner(w, device=cuda, seed=4, use_pdl=True)
    for L in r.layers:
        L["attn_norm_out"].fill_(7.0)
    r.desc.op_mask = _capi.OP_SWIGLU
    n = r.run()
    torch.cuda.synchronize()
    assert n == w.model.n_layers
    for L in r.layers:
        assert bool((L["attn_norm_out"] == 7.0).all())
        assert_tol(host(L["swiglu_out"]), oracle.silu_mul(host(L["gate"]), host(L["up"])))
    r.desc.op_mask = _capi.OP_INPUT_NORM | _capi.OP_POST_NORM
    assert r.run() == 2 * w.model.n_layers


@pytest.mark.parametrize("shape", ["qwen", "llama"])
@pytest.mark.parametrize("decode", [False, True])
def test_chain_with_attention(cuda, oracle, shape, decode):
    """KLLM_B200_OP_ATTENTION in the chain (PDL on): every layer's context
    equals the oracle attention of that layer's rotated q over its cache as
    the step left it (prefill: runs of 17 tokens take the prefill kernel,
    tcgen05 at head_dim 128; decode: single tokens over a filled cache)."""
    from littlellm_b200.chain import ChainRunner
    w = _tiny(decode, shape)
    m = w.model
    r = ChainRunner(w, device=cuda, seed=7, use_pdl=True, attention=True)
    launches = r.run()
    torch.cuda.synchronize()
    assert launches == 5 * m.n_layers + 1
    assert int(r.err_flags.item()) == 0
    pos, slots = r.positions.cpu().numpy(), r.slots.cpu().numpy()
    T, D = w.n_tokens, m.head_dim
    for l, L in enumerate(r.layers):
        want, bad = oracle.attention_head_major(host(L["q"]).reshape(T, m.n_heads, D), host(L["k_cache"]),
                                                host(L["v_cache"]), pos, slots)
        assert bad == 0
        assert_tol(host(L["attn_ctx"]).reshape(T, m.n_heads, D), want, what=f"attention layer {l}")


@pytest.mark.parametrize("decode", [False, True])
def test_final_norm_writes_last_rows(cuda, decode):
    """Final norm + select: one kernel when every sequence has seq_len rows,
    the separate select kernel for a ragged batch (seq_ends); the last rows
    are bit-identical copies of the final norm's rows either way."""
    from littlellm_b200 import _capi
    from littlellm_b200.chain import ChainRunner
    w = _tiny(decode, "qwen")
    r = ChainRunner(w, device=cuda, seed=13, use_pdl=True)
    r.run()  # the whole chain once, so the residual holds a step's value
    r.desc.op_mask = _capi.OP_FINAL_NORM | _capi.OP_SELECT
    assert r.fused_select
    saved = r.residual.clone()  # the final norm adds into the residual: each run starts from this
    r.last_rows.fill_(-7.0)
    assert r.run() == 1
    torch.cuda.synchronize()
    fused = r.last_rows.clone()
    assert np.array_equal(bits16(fused), bits16(r.final_norm_out)[w.seq_len - 1::w.seq_len])
    # ragged form of the same batch: every sequence ends where the uniform one does
    ends = torch.arange(1, w.n_seqs + 1, device=cuda, dtype=torch.int32) * w.seq_len
    r.desc.seq_ends = ends.data_ptr()
    assert not r.fused_select
    r.residual.copy_(saved)
    r.last_rows.fill_(-7.0)
    r.run()
    torch.cuda.synchronize()
    r.desc.seq_ends = None
    assert int(r.err_flags.item()) == 0
    assert torch.equal(r.last_rows, fused)
