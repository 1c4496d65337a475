"""Algorithmic byte counts of the benchmark's chain step (the denominators of
every HBM fraction it reports), checked against the per-op formulas: every
logical fp16 tensor read once and written once, int32 ids/positions/slots,
norm weights and biases not counted."""
from littlellm_b200.workloads import LLAMA2_7B, QWEN2_5_0_5B, WORKLOADS, Workload, chain_bytes, shard


def test_qwen_prefill_chain_bytes():
    w = WORKLOADS["qwen_prefill"]
    T, H, I, L = 4096, 896, 4864, 24
    qkv = 2 * T * (14 + 2 * 2) * 64 * 2 + 8 * T
    b = chain_bytes(w)
    assert b["embedding"] == 2 * T * H * 2 + 4 * T
    # 2L norms with a delta (4*T*H*2) except layer 0's input norm (2*T*H*2), plus the final norm
    assert b["add_rms_norm"] == (2 * L) * 4 * T * H * 2 + 2 * T * H * 2
    assert b["qkv_bias_rope_kv_append"] == L * qkv == L * 18_907_136
    assert b["silu_mul"] == L * 3 * T * I * 2 == L * 119_537_664
    assert b["select_last_rows"] == 2 * 8 * H * 2
    assert b["total"] == sum(v for k, v in b.items() if k != "total")


def test_fused_embedding_and_select_adjustments():
    w = WORKLOADS["qwen_prefill"]
    T, H = w.n_tokens, w.model.hidden
    plain = chain_bytes(w)
    fused = chain_bytes(w, fused_embedding=True, fused_select=True)
    # the gather + layer 0's norm: table rows read, residual and normed rows written, ids read
    assert fused["embedding"] == 3 * T * H * 2 + 4 * T
    assert fused["add_rms_norm"] == plain["add_rms_norm"] - 2 * T * H * 2
    # the final norm writes the last rows; they are not re-read
    assert fused["select_last_rows"] == w.n_seqs * H * 2
    assert plain["total"] - fused["total"] == T * H * 2 + w.n_seqs * H * 2


def test_llama_and_decode_and_attention_bytes():
    llama = chain_bytes(WORKLOADS["llama_prefill"])
    T = 16384
    assert llama["qkv_bias_rope_kv_append"] == 32 * (2 * T * (32 + 64) * 128 * 2 + 8 * T)
    import numpy as np
    w = Workload("d", QWEN2_5_0_5B, 4, 1, 64, True)
    pos = np.array([0, 5, 63, 10], np.int32)
    b = chain_bytes(w, n_layers=2, positions=pos)
    # decode attention: each token reads its sequence's K and V rows 0..pos
    kv_rows = int((pos + 1).sum())
    assert b["attention"] == 2 * (kv_rows * 2 * 64 * 2 * 2 + 2 * 4 * 14 * 64 * 2)


def test_shard_splits_whole_sequences():
    w = WORKLOADS["llama_prefill_64k"]
    assert shard(w, 3, 8).n_seqs == 16 and shard(w, 3, 8).n_tokens == 8192
    assert shard(WORKLOADS["qwen_decode"], 0, 8).n_seqs == 256
    try:
        shard(WORKLOADS["qwen_prefill"], 0, 3)
    except ValueError:
        pass
    else:
        raise AssertionError("8 sequences must not split over 3 ranks")
    assert LLAMA2_7B.hidden == 4096 and QWEN2_5_0_5B.vocab == 151936
