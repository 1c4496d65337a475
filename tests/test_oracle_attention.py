"""The attention oracle (scope row f1) pinned before it checks any kernel:
the reference's own known-answer test (tests/test_attention.cpp:7-18), and
bit-identity with the compiled reference kllm::op::attention (CPU, F32) on
seeded inputs; the head-major restatement then equals the reference applied
sequence by sequence to the same cache rows in the reference layout."""
from __future__ import annotations

import numpy as np
import pytest


def test_reference_kat(oracle):
    # one cached key [1, 0] with value [2, 3]; query [1, 0] -> [2, 3]
    kc = np.array([[[1, 0]], [[0, 0]]], np.float32)
    vc = np.array([[[2, 3]], [[0, 0]]], np.float32)
    q = np.array([[[1, 0]]], np.float32)
    assert np.allclose(oracle.attention(q, kc, vc, 0, 1), [[[2, 3]]], atol=1e-6)
    out, bad = oracle.attention_head_major(q, kc.transpose(1, 0, 2)[None], vc.transpose(1, 0, 2)[None],
                                           [0], [0])
    assert bad == 0 and np.allclose(out, [[[2, 3]]], atol=1e-6)


@pytest.mark.parametrize("seq,past,hq,hkv,d", [(5, 0, 4, 2, 8), (3, 9, 14, 2, 64), (1, 40, 2, 2, 128),
                                               (17, 3, 7, 1, 16)])
def test_oracle_matches_reference_bitwise(oracle, reference, seq, past, hq, hkv, d):
    rng = np.random.default_rng(seq * 100 + past)
    max_seq = past + seq + 3
    q = rng.standard_normal((seq, hq, d)).astype(np.float32)
    kc = rng.standard_normal((max_seq, hkv, d)).astype(np.float32)
    vc = rng.standard_normal((max_seq, hkv, d)).astype(np.float32)
    want = reference.attention(q, kc, vc, past, hkv)
    got = oracle.attention(q, kc, vc, past, hkv)
    assert np.array_equal(got, want)


def test_head_major_equals_reference_per_sequence(oracle, reference):
    """Three sequences in slots 2, 0, 1 of a head-major cache: a 6-token
    prefill chunk starting at position 4, a single decode token at position
    11, and a 3-token chunk at 0; each equals kllm::op::attention on that
    slot's rows rearranged to [max_seq, Hkv, D]."""
    rng = np.random.default_rng(7)
    hq, hkv, d, n_slots, max_seq = 6, 2, 32, 3, 16
    kc = rng.standard_normal((n_slots, hkv, max_seq, d)).astype(np.float32)
    vc = rng.standard_normal((n_slots, hkv, max_seq, d)).astype(np.float32)
    runs = [(2, 4, 6), (0, 11, 1), (1, 0, 3)]  # (slot, first position, tokens)
    positions = np.concatenate([np.arange(p, p + n) for _, p, n in runs]).astype(np.int32)
    slots = np.concatenate([np.full(n, s) for s, _, n in runs]).astype(np.int32)
    q = rng.standard_normal((positions.size, hq, d)).astype(np.float32)
    out, bad = oracle.attention_head_major(q, kc, vc, positions, slots)
    assert bad == 0
    row = 0
    for slot, past, n in runs:
        want = reference.attention(q[row:row + n], kc[slot].transpose(1, 0, 2), vc[slot].transpose(1, 0, 2),
                                   past, hkv)
        assert np.array_equal(out[row:row + n], want)
        row += n


def test_head_major_invalid_rows_are_zero(oracle):
    rng = np.random.default_rng(3)
    kc = rng.standard_normal((2, 1, 8, 4)).astype(np.float32)
    q = rng.standard_normal((4, 2, 4)).astype(np.float32)
    out, bad = oracle.attention_head_major(q, kc, kc, [0, 8, -1, 3], [1, 0, 0, 2])
    assert bad == 3
    assert np.all(out[1:] == 0) and np.all(np.isfinite(out[0])) and np.any(out[0] != 0)
