"""Writes small random models in LittleLLM's ``.kllm`` format (test helper).

Layout (README.md:274-303 of the reference, read by ModelWeights::load,
src/model/weights.cpp:47-163): magic "KLLM0001", u32 version 1, the model
config (u32 type, i32 vocab/hidden/intermediate/layers/heads/kv_heads/
head_dim/max_seq, f32 eps/theta, u8 tie/qkv_bias/o_bias/mlp_bias), u32 tensor
count, then per tensor: u32 name length, name, u32 dtype (0 f32, 1 f16, 2 i32,
3 i8), u32 ndim, i64 dims, u64 byte count, bytes. INT8 records carry the
int8 data followed by one fp32 per-tensor scale.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np


@dataclass
class TinyConfig:
    model_type: int = 1  # 0 llama, 1 qwen2
    vocab: int = 128
    hidden: int = 64
    intermediate: int = 160
    layers: int = 2
    heads: int = 4
    kv_heads: int = 2
    head_dim: int = 16
    max_seq: int = 64
    eps: float = 1e-6
    theta: float = 1e6
    tie: bool = True
    qkv_bias: bool = True


def _tensor(out, name: str, arr: np.ndarray, dtype: str) -> None:
    enc = name.encode()
    out.write(struct.pack("<I", len(enc)))
    out.write(enc)
    if dtype == "i8":
        a = np.asarray(arr, np.float32)
        scale = np.float32(np.abs(a).max() / 127.0)
        q = np.clip(np.round(a / scale), -127, 127).astype(np.int8)
        data = q.tobytes() + np.array([scale], np.float32).tobytes()
        code = 3
    elif dtype == "f16":
        data = np.asarray(arr, np.float16).tobytes()
        code = 1
    else:
        data = np.asarray(arr, np.float32).tobytes()
        code = 0
    out.write(struct.pack("<II", code, arr.ndim))
    for d in arr.shape:
        out.write(struct.pack("<q", d))
    out.write(struct.pack("<Q", len(data)))
    out.write(data)


def write_model(path: str, cfg: TinyConfig, seed: int = 0, weight_dtype: str = "f32",
                norm_dtype: str = "f32") -> None:
    """Random weights (~N(0, 1/sqrt(fan_in)) for projections, N(0, 0.5) for the
    embedding, U(0.5, 1.5) norms, N(0, 0.02) biases)."""
    rng = np.random.default_rng(seed)
    H, I, D = cfg.hidden, cfg.intermediate, cfg.head_dim
    qd, kvd = cfg.heads * D, cfg.kv_heads * D
    tensors = [("model.embed_tokens.weight", rng.normal(0, 0.5, (cfg.vocab, H)), weight_dtype)]
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        tensors += [
            (p + "input_layernorm.weight", rng.uniform(0.5, 1.5, H), norm_dtype),
            (p + "self_attn.q_proj.weight", rng.normal(0, H ** -0.5, (qd, H)), weight_dtype),
            (p + "self_attn.k_proj.weight", rng.normal(0, H ** -0.5, (kvd, H)), weight_dtype),
            (p + "self_attn.v_proj.weight", rng.normal(0, H ** -0.5, (kvd, H)), weight_dtype),
            (p + "self_attn.o_proj.weight", rng.normal(0, qd ** -0.5, (H, qd)), weight_dtype),
            (p + "post_attention_layernorm.weight", rng.uniform(0.5, 1.5, H), norm_dtype),
            (p + "mlp.gate_proj.weight", rng.normal(0, H ** -0.5, (I, H)), weight_dtype),
            (p + "mlp.up_proj.weight", rng.normal(0, H ** -0.5, (I, H)), weight_dtype),
            (p + "mlp.down_proj.weight", rng.normal(0, I ** -0.5, (H, I)), weight_dtype),
        ]
        if cfg.qkv_bias:
            tensors += [
                (p + "self_attn.q_proj.bias", rng.normal(0, 0.02, qd), norm_dtype),
                (p + "self_attn.k_proj.bias", rng.normal(0, 0.02, kvd), norm_dtype),
                (p + "self_attn.v_proj.bias", rng.normal(0, 0.02, kvd), norm_dtype),
            ]
    tensors.append(("model.norm.weight", rng.uniform(0.5, 1.5, H), norm_dtype))
    if not cfg.tie:
        tensors.append(("lm_head.weight", rng.normal(0, H ** -0.5, (cfg.vocab, H)), weight_dtype))
    with open(path, "wb") as out:
        out.write(b"KLLM0001")
        out.write(struct.pack("<II", 1, cfg.model_type))
        out.write(struct.pack("<8i", cfg.vocab, H, I, cfg.layers, cfg.heads, cfg.kv_heads, D, cfg.max_seq))
        out.write(struct.pack("<ff", cfg.eps, cfg.theta))
        out.write(struct.pack("<BBBB", int(cfg.tie), int(cfg.qkv_bias), 0, 0))
        out.write(struct.pack("<I", len(tensors)))
        for name, arr, dt in tensors:
            _tensor(out, name, np.asarray(arr), dt)
