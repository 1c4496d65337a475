"""Individual entry points launched with programmatic dependent launch
(kllm_b200_set_pdl(1)): a sequence of calls in which each reads what the
previous one wrote gives the same bits as with plain launches."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _sequence(ops, seed):
    g = torch.Generator(device="cuda:0")
    g.manual_seed(seed)
    T, H, I, Hq, Hkv, D, V = 1024, 896, 4864, 14, 2, 64, 5000

    def rn(*shape, std=1.0):
        return (torch.randn(shape, generator=g, device="cuda:0") * std).half()

    table, w1, w2 = rn(V, H, std=0.02), rn(H).abs() + 0.5, rn(H).abs() + 0.5
    ids = torch.randint(0, V, (T,), generator=g, device="cuda:0", dtype=torch.int32)
    deltas = [rn(T, H) for _ in range(3)]
    q, k, v = rn(T, Hq, D), rn(T, Hkv, D), rn(T, Hkv, D)
    bq, bk, bv = rn(Hq * D, std=0.02), rn(Hkv * D, std=0.02), rn(Hkv * D, std=0.02)
    gate, up = rn(T, I), rn(T, I)
    pos = (torch.arange(T, device="cuda:0", dtype=torch.int32) % 256)
    slots = torch.arange(T, device="cuda:0", dtype=torch.int32) // 256
    kc = torch.zeros((4, Hkv, 256, D), dtype=torch.float16, device="cuda:0")
    vc = torch.zeros_like(kc)
    res, normed = ops.embedding_rms_norm(table, ids, w1, 1e-6)
    outs = [normed.clone()]
    for i, d in enumerate(deltas):  # each call reads the residual the previous one wrote
        outs.append(ops.add_rms_norm(res, d, w2 if i % 2 else w1, 1e-6).clone())
    ops.qkv_bias_rope_kv_append(q, k, v, bq, bk, bv, pos, slots, 1e6, kc, vc)
    y = ops.silu_mul(gate, up)
    torch.cuda.synchronize()
    return [res, *outs, q, kc, vc, y]


def test_pdl_launches_give_identical_results(ops):
    prev = ops.set_pdl(False)
    try:
        plain = _sequence(ops, 5)
        ops.set_pdl(True)
        chained = _sequence(ops, 5)
    finally:
        ops.set_pdl(prev)
    for a, b in zip(plain, chained):
        assert torch.equal(a, b)
