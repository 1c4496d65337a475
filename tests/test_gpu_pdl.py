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


def test_pdl_entry_points_see_inputs_written_by_the_launch_before(ops):
    """With kllm_b200_set_pdl(1) an entry point reads nothing before its
    dependency wait: a norm weight, q/k/v biases and an embedding table that
    the launch directly before writes (the tail of a 64 M-value INT8 -> fp16
    dequantisation, written late in that kernel) are read as written. Each
    result equals the same call made without PDL after a synchronisation."""
    g = torch.Generator(device="cuda:0")
    g.manual_seed(9)
    T, H, Hq, Hkv, D, V = 512, 896, 14, 2, 64, 1000
    n_fill = 64 << 20

    def produced(n_tail):
        """Launches the dequantisation whose last n_tail values are the input
        under test (zeros until it has run) and returns that view."""
        data = torch.randint(-127, 128, (n_fill + n_tail,), generator=g, device="cuda:0", dtype=torch.int8)
        scale = torch.full((1,), 0.01, device="cuda:0")
        buf = torch.zeros(n_fill + n_tail, dtype=torch.float16, device="cuda:0")
        torch.cuda.synchronize()
        ops.dequantize_int8(data, scale, out=buf)
        return buf[n_fill:]

    x = torch.randn(T, H, generator=g, device="cuda:0").half()
    q0, k0, v0 = (torch.randn(T, h, D, generator=g, device="cuda:0").half() for h in (Hq, Hkv, Hkv))
    pos = torch.arange(T, device="cuda:0", dtype=torch.int32) % 128
    slots = torch.arange(T, device="cuda:0", dtype=torch.int32) // 128
    ids = torch.randint(0, V, (T,), generator=g, device="cuda:0", dtype=torch.int32)
    nb = (Hq + 2 * Hkv) * D

    def rope_buffers():
        kc = torch.zeros((4, Hkv, 128, D), dtype=torch.float16, device="cuda:0")
        return [q0.clone(), kc, torch.zeros_like(kc)]

    def rope(bufs, bias):
        q, kc, vc = bufs
        ops.qkv_bias_rope_kv_append(q, k0, v0, bias[:Hq * D], bias[Hq * D:(Hq + Hkv) * D], bias[(Hq + Hkv) * D:],
                                    pos, slots, 1e6, kc, vc)
        return bufs

    # every buffer exists before each dequantisation, so the call under test is
    # the launch directly after it on the stream
    x1, x2, bufs1, bufs2 = x.clone(), x.clone(), rope_buffers(), rope_buffers()
    prev = ops.set_pdl(True)
    try:
        w = produced(H)
        normed = ops.add_rms_norm(x1, None, w, 1e-6)
        bias = produced(nb)
        roped = rope(bufs1, bias)
        table = produced(V * H).view(V, H)
        res, emb = ops.embedding_rms_norm(table, ids, w, 1e-6)
        torch.cuda.synchronize()
        assert bool((w != 0).any()) and bool((bias != 0).any()) and bool((table != 0).any())
        ops.set_pdl(False)
        assert torch.equal(normed, ops.add_rms_norm(x2, None, w, 1e-6))
        for a, b in zip(roped, rope(bufs2, bias)):
            assert torch.equal(a, b)
        res2, emb2 = ops.embedding_rms_norm(table, ids, w, 1e-6)
        assert torch.equal(res, res2) and torch.equal(emb, emb2)
        assert torch.equal(res, table[ids.long()])
    finally:
        ops.set_pdl(prev)
