"""The layer-op chain at the benchmark's full sizes against the oracle, one
eager step with programmatic dependent launch:

- Qwen2.5-0.5B prefill, 8 x 512 tokens, all 24 layers: every op's output of
  every layer.
- Qwen2.5-0.5B decode, 2048 sequences at positions in [0, 4095) over the full
  [24, 2, 2048, 2, 4096, 64] fp16 cache (103 GB): every op's output of every
  layer and the cache rows each token appends.
- Llama-2-7B prefill, 32 x 512 tokens, all 32 layers: the first and last layers
  op by op, the residual stream bit for bit through every layer.
- INT8 -> fp16 dequant of a whole Llama-2-7B checkpoint (6.74 B values), bit
  for bit.

The oracle runs op by op in the reference's order (src/model/llama.cpp:78-178)
with the residual stream held in fp16, as the reference's CUDA runner holds it.
Tolerance: |gpu - oracle| <= 1e-2 + 1e-2 |oracle| for the fp16 float ops;
the residual stream and the last rows bit-exact."""
from __future__ import annotations

import gc

import numpy as np
import pytest
import torch

from gpu_util import TOL, bits16

pytestmark = pytest.mark.gpu

CHUNK = 1 << 24


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def check(actual, expected, what: str) -> None:
    """The stated tolerance, in float32 and in chunks (arrays of up to 180 M values)."""
    a = np.asarray(actual, np.float32).reshape(-1)
    e = np.asarray(expected, np.float32).reshape(-1)
    assert a.shape == e.shape, (what, a.shape, e.shape)
    for s in range(0, a.size, CHUNK):
        x, y = a[s:s + CHUNK], e[s:s + CHUNK]
        bad = np.abs(x - y) > TOL + TOL * np.abs(y)
        if bad.any():
            i = int(np.argmax(bad))
            raise AssertionError(f"{what}: {int(bad.sum())} values of the chunk at {s} outside tolerance; "
                                 f"first at {s + i}: {x[i]} against {y[i]}")


def f16_add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """fp32 sum of fp16 values, rounded to fp16 (the residual stream's add)."""
    return (a + b).astype(np.float16).astype(np.float32)


def rope_ref(oracle, x: np.ndarray, bias: np.ndarray, positions: np.ndarray, theta: float) -> np.ndarray:
    """x [T, H, D] plus bias, rotated at each row's own position: the fused oracle
    with x in the q role and a one-position cache, so nothing else is produced."""
    T, H, D = x.shape
    kv = np.zeros((T, 1, D), np.float32)
    cache = np.zeros((1, 1, 1, D), np.float32)
    q, _, _, _ = oracle.qkv_bias_rope_kv_append(x, kv, kv, bias, None, None, positions,
                                                np.zeros(T, np.int32), theta, cache, cache)
    return q


@pytest.fixture
def room():
    gc.collect()
    torch.cuda.empty_cache()
    yield
    gc.collect()
    torch.cuda.empty_cache()


def run_step(workload, cuda, keep_q):
    from littlellm_b200.chain import ChainRunner
    r = ChainRunner(workload, device=cuda, seed=5, use_pdl=True)
    q_in = {l: r.layers[l]["q"].clone() for l in keep_q}  # q is rotated in place
    launches = r.run()
    torch.cuda.synchronize()
    assert launches == 4 * r.n_layers + 1
    assert int(r.err_flags.item()) == 0
    return r, q_in


def check_layer(oracle, r, l: int, res_in: np.ndarray, q_in: torch.Tensor) -> np.ndarray:
    """Every op of layer l given the residual entering it; returns the residual
    after the attention add."""
    m, w = r.w.model, r.w
    L = r.layers[l]
    T, D = w.n_tokens, m.head_dim
    pos, slots = r.positions.cpu().numpy(), r.slots.cpu().numpy()
    check(f32(L["attn_norm_out"]), oracle.rms_norm(res_in, f32(L["input_norm_w"]), m.eps), f"attn_norm {l}")
    q_ref = rope_ref(oracle, f32(q_in).reshape(T, m.n_heads, D), f32(L["q_bias"]), pos, m.theta)
    check(f32(L["q"]).reshape(T, m.n_heads, D), q_ref, f"q {l}")
    del q_ref
    k_ref = rope_ref(oracle, f32(L["k"]).reshape(T, m.n_kv_heads, D), f32(L["k_bias"]), pos, m.theta)
    v_ref = f32(L["v"]).reshape(T, m.n_kv_heads, D) + f32(L["v_bias"]).reshape(m.n_kv_heads, D)
    si, pi = r.slots.long(), r.positions.long()
    check(f32(L["k_cache"][si, :, pi]), k_ref, f"k cache rows {l}")
    check(f32(L["v_cache"][si, :, pi]), v_ref, f"v cache rows {l}")
    del k_ref, v_ref
    res_mid = f16_add(res_in, f32(L["attn_out"]))
    check(f32(L["ffn_norm_out"]), oracle.rms_norm(res_mid, f32(L["post_norm_w"]), m.eps), f"ffn_norm {l}")
    check(f32(L["swiglu_out"]), oracle.silu_mul(f32(L["gate"]), f32(L["up"])), f"swiglu {l}")
    return res_mid


def check_end(oracle, r, res: np.ndarray) -> None:
    """The residual after the last layer bit for bit, the final norm, the last rows."""
    w = r.w
    assert np.array_equal(bits16(r.residual), res.astype(np.float16).view(np.uint16))
    check(f32(r.final_norm_out), oracle.rms_norm(res, f32(r.final_norm_w), w.model.eps), "final norm")
    assert np.array_equal(bits16(r.last_rows), bits16(r.final_norm_out)[w.seq_len - 1::w.seq_len])


@pytest.mark.parametrize("name", ["qwen_prefill", "qwen_decode"])
def test_qwen_chain_full_size_every_layer(cuda, oracle, room, name):
    from littlellm_b200.workloads import WORKLOADS
    w = WORKLOADS[name]
    r, q_in = run_step(w, cuda, keep_q=range(w.model.n_layers))
    if w.decode:
        assert r.layers[0]["k_cache"].shape == (2048, 2, 4096, 64)
    res = oracle.embedding(f32(r.table), r.ids.cpu().numpy())
    for l in range(r.n_layers):
        if l > 0:
            res = f16_add(res, f32(r.layers[l - 1]["ffn_out"]))
        res = check_layer(oracle, r, l, res, q_in.pop(l))
    check_end(oracle, r, f16_add(res, f32(r.layers[-1]["ffn_out"])))
    del r, q_in


def test_llama_prefill_full_size(cuda, oracle, room):
    from littlellm_b200.workloads import WORKLOADS
    w = WORKLOADS["llama_prefill"]
    last = w.model.n_layers - 1
    r, q_in = run_step(w, cuda, keep_q=(0, last))
    res = oracle.embedding(f32(r.table), r.ids.cpu().numpy())
    for l in range(r.n_layers):
        if l > 0:
            res = f16_add(res, f32(r.layers[l - 1]["ffn_out"]))
        if l in q_in:
            res = check_layer(oracle, r, l, res, q_in.pop(l))
        else:
            res = f16_add(res, f32(r.layers[l]["attn_out"]))
    check_end(oracle, r, f16_add(res, f32(r.layers[-1]["ffn_out"])))
    del r, q_in


def test_llama_int8_checkpoint_dequant_full_size(cuda, oracle, room):
    """INT8 -> fp16 of every Llama-2-7B linear/embedding tensor (6.74 B values,
    int8 over the whole [-128, 127], one fp32 scale per tensor) in one batched
    launch, bit for bit: each tensor's output equals, element by element, the
    oracle's rounding of its int8 value at that tensor's scale (the oracle run
    on all 256 int8 values per tensor, looked up on the device). The
    per-tensor entry on the largest tensors gives the same bits."""
    from littlellm_b200 import ops
    from littlellm_b200.workloads import LLAMA2_7B_INT8_TENSORS
    gen = torch.Generator(device=cuda)
    gen.manual_seed(11)
    data, scales, outs = [], [], []
    for rows, cols, count in LLAMA2_7B_INT8_TENSORS:
        for _ in range(count):
            data.append(torch.randint(-128, 128, (rows, cols), generator=gen, device=cuda, dtype=torch.int8))
            scales.append(torch.rand((1,), generator=gen, device=cuda) * 9e-3 + 1e-3)
            outs.append(torch.empty((rows, cols), dtype=torch.float16, device=cuda))
    assert sum(d.numel() for d in data) == 6_738_149_376
    ops.dequantize_int8_batched(data, scales, outs)
    torch.cuda.synchronize()
    values = np.arange(-128, 128, dtype=np.int8)
    for i, (d, sc, o) in enumerate(zip(data, scales, outs)):
        lut = torch.from_numpy(oracle.dequantize_int8_f16_bits(values, float(sc.item())).view(np.int16)).to(cuda)
        assert torch.equal(o.view(torch.int16), lut[d.long() + 128]), f"tensor {i} {tuple(d.shape)}"
    for i in (len(data) - 1, 128):  # lm_head 32000 x 4096, a gate/up 11008 x 4096
        single = torch.empty_like(outs[i])
        ops.dequantize_int8(data[i], scales[i], out=single)
        torch.cuda.synchronize()
        assert torch.equal(single.view(torch.int16), outs[i].view(torch.int16)), f"per-tensor {i}"
    del data, scales, outs
