"""The oracle forward (Oracle.forward: LlamaRunner::forward composed of the
C oracle's operators, head-major caches, per-token positions) pinned
against the reference's own LlamaRunner (src/model/llama.cpp:68-184,
compiled for the CPU) on a tiny random .kllm model: a 12-token prefill, then
two decode steps, F32 activations. The GPU forward test checks the device
path against this oracle."""
from __future__ import annotations

import numpy as np
import pytest

from kllm_model import TinyConfig, write_model


def _params(wts, cfg: TinyConfig, ids, positions, caches, tie: bool) -> dict:
    H, I, D = cfg.hidden, cfg.intermediate, cfg.head_dim
    qd, kvd = cfg.heads * D, cfg.kv_heads * D

    def get(name, shape):
        return wts.get(name, int(np.prod(shape))).reshape(shape)

    layers = []
    for i in range(cfg.layers):
        p = f"model.layers.{i}."
        L = {"input_norm_w": get(p + "input_layernorm.weight", (H,)),
             "post_norm_w": get(p + "post_attention_layernorm.weight", (H,)),
             "wq": get(p + "self_attn.q_proj.weight", (qd, H)), "wk": get(p + "self_attn.k_proj.weight", (kvd, H)),
             "wv": get(p + "self_attn.v_proj.weight", (kvd, H)), "wo": get(p + "self_attn.o_proj.weight", (H, qd)),
             "w_gate": get(p + "mlp.gate_proj.weight", (I, H)), "w_up": get(p + "mlp.up_proj.weight", (I, H)),
             "w_down": get(p + "mlp.down_proj.weight", (H, I)),
             "k_cache": caches[i][0], "v_cache": caches[i][1]}
        for b, n in (("q_bias", qd), ("k_bias", kvd), ("v_bias", kvd)):
            L[b] = get(p + f"self_attn.{b[0]}_proj.bias", (n,)) if cfg.qkv_bias else None
        layers.append(L)
    table = get("model.embed_tokens.weight", (cfg.vocab, H))
    return {"table": table, "ids": np.asarray(ids, np.int32), "positions": np.asarray(positions, np.int32),
            "slots": np.zeros(len(ids), np.int32), "final_norm_w": get("model.norm.weight", (H,)),
            "lm_head": table if tie else get("lm_head.weight", (cfg.vocab, H)), "layers": layers,
            "n_heads": cfg.heads, "n_kv_heads": cfg.kv_heads, "head_dim": D, "eps": cfg.eps,
            "theta": cfg.theta, "seq_len": len(ids), "n_seqs": 1}


@pytest.mark.parametrize("model_type,tie,qkv_bias", [(1, True, True), (0, False, False)])
def test_oracle_forward_matches_reference_runner(oracle, reference, tmp_path, model_type, tie, qkv_bias):
    from oracle.oracle import ReferenceRunner, ReferenceWeights
    cfg = TinyConfig(model_type=model_type, tie=tie, qkv_bias=qkv_bias, theta=1e6 if model_type else 1e4)
    path = str(tmp_path / "tiny.kllm")
    write_model(path, cfg, seed=7)
    runner = ReferenceRunner(reference, path, cfg.max_seq, cfg.vocab)
    wts = ReferenceWeights(reference, path)
    try:
        rng = np.random.default_rng(3)
        prompt = rng.integers(0, cfg.vocab, 12).astype(np.int32)
        shape = (1, cfg.kv_heads, cfg.max_seq, cfg.head_dim)
        caches = [(np.zeros(shape, np.float32), np.zeros(shape, np.float32)) for _ in range(cfg.layers)]
        steps = [(prompt, 0), (np.array([5], np.int32), 12), (np.array([77], np.int32), 13)]
        for ids, past in steps:
            want = runner.forward(ids, past)
            p = _params(wts, cfg, ids, np.arange(past, past + len(ids)), caches, tie)
            _, logits, caches = oracle.forward(p, fp16_storage=False)
            assert logits.shape == (1, cfg.vocab)
            np.testing.assert_allclose(logits[0], want, rtol=1e-5, atol=1e-5)
    finally:
        runner.close()
        wts.close()
