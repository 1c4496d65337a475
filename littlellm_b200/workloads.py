"""Model shapes, benchmark workloads and their algorithmic byte counts.

Plain data and arithmetic: this module imports neither torch nor the CUDA
library, so code that only needs the shapes (the CPU timing of the
reference's own operators, sharding arithmetic) can use it without mapping
``libkllm_b200.so``.

Model shapes are the ones the benchmark is quoted on: Qwen2.5-0.5B (hidden
896, 14/2 heads x 64, intermediate 4864, vocab 151936, 24 layers, eps 1e-6,
theta 1e6) and Llama-2-7B (4096, 32/32 x 128, 11008, 32000, 32 layers, eps
1e-5, theta 1e4), as LlamaRunner reads them from a .kllm header
(src/model/llama.cpp:26-66).
"""
from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class ModelShape:
    name: str
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    n_layers: int
    eps: float
    theta: float


QWEN2_5_0_5B = ModelShape("qwen2.5-0.5b", 896, 14, 2, 64, 4864, 151936, 24, 1e-6, 1e6)
LLAMA2_7B = ModelShape("llama-2-7b", 4096, 32, 32, 128, 11008, 32000, 32, 1e-5, 1e4)


@dataclass(frozen=True)
class Workload:
    name: str
    model: ModelShape
    n_seqs: int        # sequences in the step (per GPU for weak scaling)
    seq_len: int       # new tokens per sequence in this step
    max_seq: int       # KV cache capacity per sequence
    decode: bool       # decode: one token per sequence at a random position

    @property
    def n_tokens(self) -> int:
        return self.n_seqs * self.seq_len


WORKLOADS = {
    # B=8 x 512 prefill of Qwen2.5-0.5B, cache [24, 2, 8, 2, 4096, 64]
    "qwen_prefill": Workload("qwen_prefill", QWEN2_5_0_5B, 8, 512, 4096, False),
    # B=32 x 512 prefill of Llama-2-7B
    "llama_prefill": Workload("llama_prefill", LLAMA2_7B, 32, 512, 512, False),
    # 2048 sequences x 1 token, positions U[0, 4095), cache [24, 2, 2048, 2, 4096, 64]
    "qwen_decode": Workload("qwen_decode", QWEN2_5_0_5B, 2048, 1, 4096, True),
    # 128 x 512 Llama-2-7B prefill; 16 sequences per GPU at 8 GPUs
    "llama_prefill_64k": Workload("llama_prefill_64k", LLAMA2_7B, 128, 512, 512, False),
}


# The linear and embedding tensors of a Llama-2-7B checkpoint as (rows, cols,
# count): q/k/v/o, gate/up and down of each of the 32 layers, then the
# embedding and lm_head (6.74 B values).
LLAMA2_7B_INT8_TENSORS = ((4096, 4096, 4 * 32), (11008, 4096, 2 * 32), (4096, 11008, 32), (32000, 4096, 2))


def shard(workload: Workload, rank: int, world: int) -> Workload:
    """The slice of a workload one rank runs when sequences are split evenly."""
    if workload.n_seqs % world != 0:
        raise ValueError(f"{workload.n_seqs} sequences do not split over {world} ranks")
    return replace(workload, n_seqs=workload.n_seqs // world)


def chain_bytes(w: Workload, n_layers: int | None = None, positions=None, fused_embedding: bool = False,
                fused_select: bool = False) -> dict:
    """Algorithmic HBM bytes of one chain step: every logical fp16 tensor read
    once and written once; norm weights and biases are negligible and not
    counted; ids/positions/slots are int32. With ``positions`` (host array of
    the step's token positions) the attention of every layer is included:
    each sequence's cached K and V rows 0..position read once (decode: per
    token), q read and the context written.

    With ``fused_embedding`` the embedding gather and layer 0's input norm
    are one op: the gathered rows are written once (the residual) and never
    re-read, so the pair counts T*H*2 (table rows read) + 2*T*H*2 (residual
    and normed rows written) + 4*T, against 2*T*H*2 + 4*T for the gather plus
    2*T*H*2 for the norm when they run apart. With ``fused_select`` the final
    norm writes each sequence's last row as well: those rows are written
    (B*H*2) but not re-read."""
    m, T = w.model, w.n_tokens
    H, I, L = m.hidden, m.intermediate, n_layers or m.n_layers
    qkv_elems = T * (m.n_heads + 2 * m.n_kv_heads) * m.head_dim
    per = {
        "embedding": 2 * T * H * 2 + 4 * T,
        # L post norms + the final norm and layers 1..L-1's input norms add a
        # delta (4*T*H*2 each); layer 0's input norm reads and writes 2*T*H*2
        "add_rms_norm": (L + 1) * 4 * T * H * 2 + (L - 1) * 4 * T * H * 2 + 2 * T * H * 2,
        "qkv_bias_rope_kv_append": L * (2 * qkv_elems * 2 + 8 * T),
        "silu_mul": L * 3 * T * I * 2,
        "select_last_rows": 2 * w.n_seqs * H * 2,
    }
    if fused_embedding:
        # embedding + layer-0 input norm as one op: table rows read, residual
        # and normed rows written, ids read
        per["embedding"] = 3 * T * H * 2 + 4 * T
        per["add_rms_norm"] -= 2 * T * H * 2
    if fused_select:
        per["select_last_rows"] = w.n_seqs * H * 2
    if positions is not None:
        kv_rows = int((positions.astype("int64") + 1).sum()) if w.decode else T
        per["attention"] = L * (kv_rows * m.n_kv_heads * m.head_dim * 2 * 2 + 2 * T * m.n_heads * m.head_dim * 2)
    per["total"] = sum(per.values())
    return per


def silu_bytes_per_launch(w: Workload) -> int:
    return 3 * w.n_tokens * w.model.intermediate * 2
