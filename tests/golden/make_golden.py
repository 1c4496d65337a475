"""Generates tests/golden/golden.npz from the reference's own CPU operators.

Runs the compiled reference (oracle/_ref/libkllm_ref.so, built by
oracle/Makefile from the reference sources) on small seeded inputs and
stores inputs + outputs. The fixtures travel with the repository, so tests
on a machine without the reference tree still check against the
reference's results. Activation inputs are rounded to fp16-representable
values first, so the same numbers can be fed to the fp16 CUDA kernels.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import F16, F32, Reference  # noqa: E402

SEED = 0x4B4C4C4D


def f16r(a) -> np.ndarray:
    """fp16-representable float32 copy."""
    return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)


def main(out_path: str = os.path.join(HERE, "golden.npz")) -> None:
    ref = Reference()
    rng = np.random.default_rng(SEED)
    g: dict[str, np.ndarray] = {}

    # embedding (src/op/cpu/embedding.cpp), F32 and F16 tensors
    table = f16r(rng.normal(0, 0.02, (64, 40)))
    ids = rng.integers(0, 64, 16).astype(np.int32)
    g["emb_table"], g["emb_ids"] = table, ids
    g["emb_out"] = ref.embedding(table, ids, F32)
    g["emb_out_f16"] = ref.embedding(table.astype(np.float16), ids, F16).view(np.uint16)

    # rms_norm (src/op/cpu/rms_norm.cpp), two hidden sizes
    for name, (rows, hidden, eps) in {"a": (8, 96, 1e-6), "b": (3, 896, 1e-5)}.items():
        x = f16r(rng.normal(0, 1, (rows, hidden)))
        w = f16r(rng.uniform(0.5, 1.5, hidden))
        g[f"rms_{name}_x"], g[f"rms_{name}_w"] = x, w
        g[f"rms_{name}_eps"] = np.float32(eps)
        g[f"rms_{name}_out"] = ref.rms_norm(x, w, eps, F32)

    # add_inplace then rms_norm (src/model/llama.cpp:135-143)
    r = f16r(rng.normal(0, 1, (6, 128)))
    d = f16r(rng.normal(0, 1, (6, 128)))
    w = f16r(rng.uniform(0.5, 1.5, 128))
    g["addrms_r"], g["addrms_d"], g["addrms_w"] = r, d, w
    r_sum = ref.add(r, d, F32)
    g["addrms_rsum"] = r_sum
    g["addrms_out"] = ref.rms_norm(r_sum, w, 1e-6, F32)

    # add_bias_inplace (src/op/cpu/add.cpp:9-24)
    x = f16r(rng.normal(0, 1, (5, 48)))
    b = f16r(rng.normal(0, 0.02, 48))
    g["bias_x"], g["bias_b"] = x, b
    g["bias_out"] = ref.add_bias(x, b, F32)

    # silu_mul (src/op/cpu/silu.cpp)
    gate = f16r(rng.normal(0, 1, (4, 200)) * 3)
    up = f16r(rng.normal(0, 1, (4, 200)))
    g["silu_g"], g["silu_u"] = gate, up
    g["silu_out"] = ref.silu_mul(gate, up, F32)

    # rope_inplace (src/op/cpu/rope.cpp): small and Qwen-/Llama-like shapes at large positions
    for name, (seq, heads, hd, past, theta) in {
        "a": (6, 3, 16, 37, 1e4), "qwen": (4, 2, 64, 4000, 1e6), "llama": (3, 2, 128, 4090, 1e4),
    }.items():
        x = f16r(rng.normal(0, 1, (seq, heads, hd)))
        g[f"rope_{name}_x"] = x
        g[f"rope_{name}_meta"] = np.array([past, theta], dtype=np.float64)
        g[f"rope_{name}_out"] = ref.rope(x, past, theta, F32)

    # copy_kv_to_cache (src/op/cpu/kv_cache.cpp)
    k = f16r(rng.normal(0, 1, (3, 2, 8)))
    v = f16r(rng.normal(0, 1, (3, 2, 8)))
    kc = f16r(rng.normal(0, 1, (10, 2, 8)))
    vc = f16r(rng.normal(0, 1, (10, 2, 8)))
    g["kv_k"], g["kv_v"], g["kv_kc"], g["kv_vc"] = k, v, kc, vc
    g["kv_kc_out"], g["kv_vc_out"] = ref.copy_kv_to_cache(k, v, kc, vc, 5, F32)

    # fused bias + RoPE + append, composed from the reference ops token by token
    # (one [1, heads, D] call per token with past_len = its position; the
    # per-sequence [S, Hkv, D] cache rows land at [slot, h, pos, :]).
    T, Hq, Hkv, D, S, NS, theta = 6, 4, 2, 16, 12, 3, 1e6
    q = f16r(rng.normal(0, 1, (T, Hq, D)))
    kk = f16r(rng.normal(0, 1, (T, Hkv, D)))
    vv = f16r(rng.normal(0, 1, (T, Hkv, D)))
    bq = f16r(rng.normal(0, 0.02, Hq * D))
    bk = f16r(rng.normal(0, 0.02, Hkv * D))
    bv = f16r(rng.normal(0, 0.02, Hkv * D))
    pos = np.array([0, 11, 3, 7, 7, 1], dtype=np.int32)
    slots = np.array([0, 2, 1, 1, 0, 2], dtype=np.int32)
    q_out = np.empty_like(q)
    kc = np.zeros((NS, Hkv, S, D), np.float32)
    vc = np.zeros((NS, Hkv, S, D), np.float32)
    for t in range(T):
        qt = ref.add_bias(q[t].reshape(1, Hq * D), bq, F32).reshape(1, Hq, D)
        kt = ref.add_bias(kk[t].reshape(1, Hkv * D), bk, F32).reshape(1, Hkv, D)
        vt = ref.add_bias(vv[t].reshape(1, Hkv * D), bv, F32).reshape(1, Hkv, D)
        q_out[t] = ref.rope(qt, int(pos[t]), theta, F32)[0]
        kt = ref.rope(kt, int(pos[t]), theta, F32)
        seq_k = np.ascontiguousarray(kc[slots[t]].transpose(1, 0, 2))  # [S, Hkv, D]
        seq_v = np.ascontiguousarray(vc[slots[t]].transpose(1, 0, 2))
        seq_k, seq_v = ref.copy_kv_to_cache(kt, vt, seq_k, seq_v, int(pos[t]), F32)
        kc[slots[t]] = seq_k.transpose(1, 0, 2)
        vc[slots[t]] = seq_v.transpose(1, 0, 2)
    g.update(qkv_q=q, qkv_k=kk, qkv_v=vv, qkv_bq=bq, qkv_bk=bk, qkv_bv=bv, qkv_pos=pos,
             qkv_slots=slots, qkv_theta=np.float32(theta), qkv_q_out=q_out, qkv_kc_out=kc,
             qkv_vc_out=vc)

    # select_last_row (src/op/cpu/add.cpp:37-49), F32 and F16
    x = f16r(rng.normal(0, 1, (5, 24)))
    g["last_x"] = x
    g["last_out"] = ref.select_last_row(x, F32)
    g["last_out_f16"] = ref.select_last_row(x.astype(np.float16), F16).view(np.uint16)

    # INT8 dequant: fp32 op (src/op/cpu/quantize.cpp:37-48) and the fp16 load
    # path (src/model/weights.cpp:139-148); scales include ones that hit ties
    # and the carry quirk of float_to_half.
    qd = np.arange(-128, 128, dtype=np.int8).repeat(4)
    rng.shuffle(qd)
    g["deq_q"] = qd
    scales = np.array([0.0037, 1e-3, 9.99e-3, 0.5, 2.0 ** -20, 1.0 / 127.0], dtype=np.float32)
    g["deq_scales"] = scales
    g["deq_f32"] = np.stack([ref.dequantize_int8_f32(qd, float(s)) for s in scales])
    g["deq_f16"] = np.stack([ref.dequantize_int8_f16_bits(qd, float(s)) for s in scales])

    # float_to_half on hand-picked values (ties, carry, subnormal, overflow, inf, NaN)
    special = np.array([
        0.0, -0.0, 1.5, 0.12499202, 0.062496, 65504.0, 65519.0, 65520.0, 65536.0, 1e9,
        np.inf, -np.inf, np.nan, 2.0 ** -14, 2.0 ** -24, 2.0 ** -25, 2.0 ** -26, 3.0 * 2.0 ** -26,
        1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, 2.0 - 2.0 ** -12, -(2.0 - 2.0 ** -12), 1e-8,
        0.00049996, 1234.567,
    ], dtype=np.float32)
    extra = rng.uniform(-8, 8, 2000).astype(np.float32)
    vals = np.concatenate([special, extra])
    g["f2h_in"] = vals
    g["f2h_out"] = ref.float_to_half_bits(vals)

    # linear() = matmul + add_bias_inplace (src/model/llama.cpp:12-24) and the
    # MLP's gate/up linears + silu_mul (src/model/llama.cpp:145-158), F32. A
    # separate stream keeps the fixtures above unchanged. k = 72 and 96 are not
    # multiples of the kernel's 64-wide k slices; m and n are partial tiles.
    rng2 = np.random.default_rng(SEED + 1)
    m, n, k = 24, 40, 72
    x = f16r(rng2.normal(0, 1, (m, k)))
    w = f16r(rng2.normal(0, 1, (n, k)) / np.sqrt(k))
    b = f16r(rng2.normal(0, 0.1, n))
    g["mm_x"], g["mm_w"], g["mm_b"] = x, w, b
    g["mm_out"] = ref.matmul(x, w, F32)
    g["lin_out"] = ref.add_bias(g["mm_out"], b, F32)
    m, n, k = 20, 48, 96
    x = f16r(rng2.normal(0, 1, (m, k)))
    wg = f16r(rng2.normal(0, 1, (n, k)) / np.sqrt(k))
    wu = f16r(rng2.normal(0, 1, (n, k)) / np.sqrt(k))
    bg = f16r(rng2.normal(0, 0.1, n))
    bu = f16r(rng2.normal(0, 0.1, n))
    g.update(mlp_x=x, mlp_wg=wg, mlp_wu=wu, mlp_bg=bg, mlp_bu=bu)
    gate = ref.add_bias(ref.matmul(x, wg, F32), bg, F32)
    up = ref.add_bias(ref.matmul(x, wu, F32), bu, F32)
    g["mlp_out"] = ref.silu_mul(gate, up, F32)

    np.savez_compressed(out_path, **g)
    print(f"wrote {out_path}: {len(g)} arrays, {os.path.getsize(out_path)} bytes")


if __name__ == "__main__":
    main()
