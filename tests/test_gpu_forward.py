"""The whole forward step (KLLM_B200_OP_GEMM: the chain with its GEMMs, the
analogue of LlamaRunner::forward, src/model/llama.cpp:78-184) against the
oracle forward (Oracle.forward, composed of the C oracle's operators), on a two-layer model
with Qwen-style q/k/v biases: a prefill batch (three 40-token sequences from
position 0) and a decode batch (one token per sequence at positions U[0, 63)
over cache rows from earlier steps). The oracle rounds to fp16 wherever the
GPU path stores fp16 (every op output, the KV cache), so each element of
the last rows and the logits must agree within 1e-2 abs + 1e-2 rel."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import assert_tol

pytestmark = pytest.mark.gpu


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def forward_params(r) -> dict:
    """Runner r's inputs, weights and caches (before the step) as numpy
    arrays for Oracle.forward."""
    m, w = r.w.model, r.w
    layers = []
    for L, W in zip(r.layers, r.weights):
        d = {k: _np(L[k]) for k in ("input_norm_w", "post_norm_w", "q_bias", "k_bias", "v_bias", "k_cache",
                                     "v_cache")}
        d.update({k: _np(t) for k, t in W.items()})
        layers.append(d)
    return {"table": _np(r.table), "ids": _np(r.ids).astype(np.int32), "positions": _np(r.positions),
            "slots": _np(r.slots), "final_norm_w": _np(r.final_norm_w), "lm_head": _np(r.lm_head),
            "layers": layers, "n_heads": m.n_heads, "n_kv_heads": m.n_kv_heads, "head_dim": m.head_dim,
            "eps": m.eps, "theta": m.theta, "seq_len": w.seq_len, "n_seqs": w.n_seqs}


@pytest.mark.parametrize("decode,hidden,inter", [(False, 256, 512), (True, 256, 512), (True, 1024, 2048)])
def test_forward_step_matches_oracle(cuda, oracle, decode, hidden, inter):
    """hidden 1024 with intermediate 2048 makes every GEMM of the decode step
    (q/k/v, o, gate/up + SwiGLU, down) split its k range over a cluster."""
    from littlellm_b200.chain import ChainRunner, ModelShape, Workload
    shape = ModelShape("tiny-2l", hidden, hidden // 64, 2, 64, inter, 512, 2, 1e-6, 1e4)
    w = (Workload("d", shape, n_seqs=6, seq_len=1, max_seq=64, decode=True) if decode
         else Workload("p", shape, n_seqs=3, seq_len=40, max_seq=64, decode=False))
    r = ChainRunner(w, device=cuda, seed=11, use_pdl=True, attention=True, gemm=True)
    params = forward_params(r)
    n = r.run()
    torch.cuda.synchronize()
    # per layer (norm, q/k/v GEMM with RoPE/KV, attention (+ combine), o linear, norm,
    # gate/up+SwiGLU, down linear; layer 0's norm also gathers the embedding) + final norm (which also
    # writes the last rows) + lm_head
    assert n >= shape.n_layers * 7 + 2
    assert int(r.err_flags.item()) == 0
    last, logits, want_caches = oracle.forward(params)
    assert_tol(_np(r.last_rows), last, what="last rows")
    assert_tol(_np(r.logits), logits, what="logits")
    # the caches the step appended to (rotated k, biased v) match too
    for i, (L, (kc, vc)) in enumerate(zip(r.layers, want_caches)):
        assert_tol(_np(L["k_cache"]), kc, what=f"layer {i} k cache")
        assert_tol(_np(L["v_cache"]), vc, what=f"layer {i} v cache")


def test_forward_graph_replay_is_deterministic(cuda):
    """The whole forward captured in one CUDA graph replays to the same logits."""
    from littlellm_b200.chain import ChainRunner, ModelShape, Workload
    shape = ModelShape("tiny-3l", 256, 4, 2, 64, 512, 1000, 3, 1e-6, 1e6)
    r = ChainRunner(Workload("p", shape, n_seqs=4, seq_len=64, max_seq=64, decode=False), device=cuda, seed=5,
                    attention=True, gemm=True)
    stream = torch.cuda.Stream(cuda)
    with torch.cuda.stream(stream):
        r.run(stream)
        stream.synchronize()
        first = r.logits.clone()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            r.run(stream)
        for _ in range(3):
            g.replay()
        stream.synchronize()
    assert torch.equal(first, r.logits)
    assert bool(torch.isfinite(r.logits.float()).all())
    assert int(r.err_flags.item()) == 0


def test_prefill_then_decode_steps_match_oracle(cuda, oracle):
    """A prefill step (three 40-token sequences) followed by two decode steps
    through decode runners that share the prefill runner's weights and KV
    caches: each decode token attends to the cache rows the prefill and the
    earlier decode step wrote, as LlamaRunner::forward does across calls. The
    oracle forward carries its own caches from step to step."""
    from littlellm_b200.chain import ChainRunner, ModelShape, Workload
    shape = ModelShape("tiny-2l", 256, 4, 2, 64, 512, 512, 2, 1e-6, 1e6)
    r = ChainRunner(Workload("p", shape, n_seqs=3, seq_len=40, max_seq=64, decode=False), device=cuda, seed=21,
                    attention=True, gemm=True)
    params = forward_params(r)
    r.run()
    torch.cuda.synchronize()
    last, logits, caches = oracle.forward(params)
    assert_tol(_np(r.logits), logits, what="prefill logits")
    g = torch.Generator(device=cuda).manual_seed(5)
    for step, pos in enumerate((40, 41)):
        ids = torch.randint(0, shape.vocab, (3,), generator=g, device=cuda, dtype=torch.int32)
        d = r.decode_runner(ids, torch.full((3,), pos, dtype=torch.int32, device=cuda))
        d.run()
        torch.cuda.synchronize()
        assert int(d.err_flags.item()) == 0
        p = dict(params, ids=_np(ids).astype(np.int32), positions=np.full(3, pos, np.int32),
                 slots=np.arange(3, dtype=np.int32), seq_len=1, n_seqs=3,
                 layers=[dict(L, k_cache=kc, v_cache=vc) for L, (kc, vc) in zip(params["layers"], caches)])
        _, logits, caches = oracle.forward(p)
        assert_tol(_np(d.logits), logits, what=f"decode step {step} logits")
        for i, (L, (kc, vc)) in enumerate(zip(r.layers, caches)):
            assert_tol(_np(L["k_cache"]), kc, what=f"decode step {step} layer {i} k cache")
