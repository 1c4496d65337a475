"""Attention over the head-major cache (scope row f1) against the oracle
(cpu_attention restated, src/op/cpu/attention.cpp:12-67, pinned to the
compiled reference in test_oracle_attention.py), run in fp32 on the same fp16
inputs. Tolerance: |gpu - oracle| <= 1e-2 + 1e-2 * |oracle|."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import TOL, assert_tol, canary_intact, dev, f16r, host

pytestmark = pytest.mark.gpu


def _cache(rng, n_slots, hkv, max_seq, d):
    k = f16r(rng.standard_normal((n_slots, hkv, max_seq, d)))
    v = f16r(rng.standard_normal((n_slots, hkv, max_seq, d)))
    return k, v


def _run(ops, q, kc, vc, positions, slots, seq_len=1, workspace=None, err=None):
    # seq_len 1 takes the decode kernel; runs of 16 or more tokens the prefill kernel
    return ops.attention_head_major(dev(q), dev(kc), dev(vc), dev(positions, torch.int32), dev(slots, torch.int32),
                                    seq_len=seq_len, workspace=workspace, err_flags=err)


@pytest.mark.parametrize("hq,hkv,d,max_seq,n_tok", [
    (14, 2, 64, 1000, 64),    # Qwen2.5-0.5B heads, ragged max_seq (not a multiple of 128)
    (32, 32, 128, 700, 16),   # Llama-2-7B heads (one query head per kv head)
    (16, 1, 64, 300, 9),      # 16 query heads per kv head (the largest group)
    (8, 2, 128, 4096, 6),     # long cache, positions up to 4095 (several chunks)
])
def test_decode_matches_oracle(cuda, ops, oracle, hq, hkv, d, max_seq, n_tok):
    rng = np.random.default_rng(hq * 1000 + max_seq)
    n_slots = n_tok + 3
    kc, vc = _cache(rng, n_slots, hkv, max_seq, d)
    q = f16r(rng.standard_normal((n_tok, hq, d)))
    positions = rng.integers(0, max_seq, n_tok).astype(np.int32)
    positions[0], positions[-1] = 0, max_seq - 1  # one key; the whole cache
    slots = rng.permutation(n_slots)[:n_tok].astype(np.int32)
    want, bad = oracle.attention_head_major(q, kc, vc, positions, slots)
    assert bad == 0
    got = _run(ops, q, kc, vc, positions, slots)
    torch.cuda.synchronize()
    assert_tol(host(got), want, TOL, "attention decode")
    # a single key: the output is that key's value row exactly
    assert np.array_equal(host(got)[0], vc[slots[0], np.arange(hq) // (hq // hkv), 0])


def test_workspace_size_does_not_change_results(cuda, ops, oracle):
    """No workspace (one chunk per sequence), a small one (coarser split) and
    the preferred one agree with the oracle."""
    rng = np.random.default_rng(17)
    hq, hkv, d, max_seq, n_tok = 14, 2, 64, 2048, 24
    kc, vc = _cache(rng, n_tok, hkv, max_seq, d)
    q = f16r(rng.standard_normal((n_tok, hq, d)))
    positions = rng.integers(0, max_seq, n_tok).astype(np.int32)
    slots = np.arange(n_tok, dtype=np.int32)
    want, _ = oracle.attention_head_major(q, kc, vc, positions, slots)
    full = ops.attention_workspace_bytes(n_tok, hq, hkv, d, max_seq)
    assert full > 0
    from littlellm_b200 import _capi
    args = [dev(q), dev(kc), dev(vc), None, dev(positions, torch.int32), dev(slots, torch.int32)]
    for nbytes in (0, full // 3, full):
        ws = torch.zeros(max(nbytes, 16), dtype=torch.uint8, device=cuda)
        args[3] = out = torch.empty(q.shape, dtype=torch.float16, device=cuda)
        rc = _capi.lib.kllm_b200_attention_head_major(
            *[a.data_ptr() for a in args], n_tok, 1, hq, hkv, d, n_tok, max_seq, _capi.F16,
            ws.data_ptr() if nbytes else None, nbytes, None, torch.cuda.current_stream().cuda_stream)
        assert rc == _capi.OK, _capi.last_error()
        torch.cuda.synchronize()
        assert_tol(host(out), want, TOL, f"workspace {nbytes}")
        if nbytes == full:
            # a second call on the same (now dirty) workspace gives the same result
            first = out.clone()
            rc = _capi.lib.kllm_b200_attention_head_major(
                *[a.data_ptr() for a in args], n_tok, 1, hq, hkv, d, n_tok, max_seq, _capi.F16, ws.data_ptr(),
                nbytes, None, torch.cuda.current_stream().cuda_stream)
            assert rc == _capi.OK
            torch.cuda.synchronize()
            assert torch.equal(out, first)


def test_prefill_runs_match_oracle(cuda, ops, oracle):
    """Three prefill sequences of 37 tokens (positions 0..36) in slots 4, 0,
    2, plus a chunk continuing a sequence at positions 37..73."""
    rng = np.random.default_rng(5)
    hq, hkv, d, max_seq, n_slots, s = 14, 2, 64, 512, 5, 37
    kc, vc = _cache(rng, n_slots, hkv, max_seq, d)
    runs = [(4, 0), (0, 0), (2, 0), (4, s)]
    positions = np.concatenate([np.arange(p, p + s) for _, p in runs]).astype(np.int32)
    slots = np.concatenate([np.full(s, sl) for sl, _ in runs]).astype(np.int32)
    q = f16r(rng.standard_normal((positions.size, hq, d)))
    want, _ = oracle.attention_head_major(q, kc, vc, positions, slots)
    got = _run(ops, q, kc, vc, positions, slots, seq_len=s)
    torch.cuda.synchronize()
    assert_tol(host(got), want, TOL, "attention prefill")


def test_sharp_scores_are_stable(cuda, ops, oracle):
    """Scores spread over +-200 (queries x 25): the running max keeps the
    exponentials finite and the result matches."""
    rng = np.random.default_rng(23)
    hq, hkv, d, max_seq, n_tok = 4, 2, 64, 900, 8
    kc, vc = _cache(rng, n_tok, hkv, max_seq, d)
    q = f16r(25.0 * rng.standard_normal((n_tok, hq, d)))
    positions = rng.integers(100, max_seq, n_tok).astype(np.int32)
    slots = np.arange(n_tok, dtype=np.int32)
    want, _ = oracle.attention_head_major(q, kc, vc, positions, slots)
    got = _run(ops, q, kc, vc, positions, slots)
    torch.cuda.synchronize()
    out = host(got)
    assert np.all(np.isfinite(out))
    assert_tol(out, want, TOL, "sharp scores")


def test_invalid_rows_zero_and_flag(cuda, ops, oracle):
    rng = np.random.default_rng(2)
    hq, hkv, d, max_seq = 4, 2, 64, 256
    kc, vc = _cache(rng, 3, hkv, max_seq, d)
    q = f16r(rng.standard_normal((5, hq, d)))
    positions = np.array([3, max_seq, -1, 10, 200], np.int32)
    slots = np.array([0, 1, 2, 3, -2], np.int32)
    want, bad = oracle.attention_head_major(q, kc, vc, positions, slots)
    assert bad == 4
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    whole = torch.full((5 * hq * d + 64,), -1234.0, dtype=torch.float16, device=cuda)
    out = whole[:5 * hq * d].view(5, hq, d)
    ops.attention_head_major(dev(q), dev(kc), dev(vc), dev(positions, torch.int32), dev(slots, torch.int32),
                             out=out, err_flags=err)
    torch.cuda.synchronize()
    from littlellm_b200 import _capi
    assert int(err.item()) == _capi.FLAG_BAD_POSITION | _capi.FLAG_BAD_SLOT
    assert np.all(host(out)[1:] == 0)
    assert_tol(host(out)[:1], want[:1], TOL, "valid row")
    assert canary_intact(whole, 5 * hq * d)


def test_argument_errors(cuda, ops):
    from littlellm_b200 import _capi
    lib = _capi.lib
    x = torch.zeros(4096, dtype=torch.float16, device=cuda)
    p = x.data_ptr()
    # head_dim 96 is not supported; 3 query heads over 2 kv heads; dtype F32
    assert lib.kllm_b200_attention_head_major(p, p, p, p, p, p, 1, 1, 2, 2, 96, 1, 8, _capi.F16, None, 0, None,
                                              None) == _capi.ERR_SHAPE
    assert lib.kllm_b200_attention_head_major(p, p, p, p, p, p, 1, 1, 3, 2, 64, 1, 8, _capi.F16, None, 0, None,
                                              None) == _capi.ERR_SHAPE
    assert lib.kllm_b200_attention_head_major(p, p, p, p, p, p, 1, 1, 2, 2, 64, 1, 8, _capi.F32, None, 0, None,
                                              None) == _capi.ERR_DTYPE
    assert lib.kllm_b200_attention_head_major(p + 2, p, p, p, p, p, 1, 1, 2, 2, 64, 1, 8, _capi.F16, None, 0,
                                              None, None) == _capi.ERR_ALIGN
    assert lib.kllm_b200_attention_head_major(None, None, None, None, None, None, 0, 1, 2, 2, 64, 1, 8, _capi.F16,
                                              None, 0, None, None) == _capi.OK


@pytest.mark.parametrize("hq,hkv,d,max_seq,seq_len,n_runs,start", [
    (14, 2, 64, 4096, 512, 2, 0),      # Qwen prefill shape
    (32, 32, 128, 512, 200, 3, 0),     # Llama heads, runs not a multiple of 64 tokens
    (8, 2, 128, 2048, 64, 2, 1000),    # a chunk continuing at position 1000
    (4, 4, 64, 300, 16, 5, 7),         # the shortest run the prefill kernel takes
])
def test_prefill_kernel_matches_oracle(cuda, ops, oracle, hq, hkv, d, max_seq, seq_len, n_runs, start):
    rng = np.random.default_rng(seq_len * 7 + hq)
    n_slots = n_runs + 1
    kc, vc = _cache(rng, n_slots, hkv, max_seq, d)
    slot_of_run = rng.permutation(n_slots)[:n_runs]
    positions = np.tile(np.arange(start, start + seq_len), n_runs).astype(np.int32)
    slots = np.repeat(slot_of_run, seq_len).astype(np.int32)
    q = f16r(rng.standard_normal((positions.size, hq, d)))
    want, _ = oracle.attention_head_major(q, kc, vc, positions, slots)
    got = _run(ops, q, kc, vc, positions, slots, seq_len=seq_len)
    per_token = _run(ops, q, kc, vc, positions, slots, seq_len=1)  # the decode kernel on the same rows
    torch.cuda.synchronize()
    assert_tol(host(got), want, TOL, "prefill kernel")
    assert_tol(host(got), host(per_token), TOL, "prefill vs decode kernel")


@pytest.mark.parametrize("d", [64, 128])  # the mma.sync and the tcgen05 prefill kernels
def test_prefill_short_last_run_and_bad_rows(cuda, ops, oracle, d):
    """100 tokens in runs of 40 (the last run has 20); in the second run one
    row names another slot and one an out-of-range position: those rows are
    zero and flagged, the others still match. At head_dim 128 every CTA's
    second 128-row query tile is empty."""
    rng = np.random.default_rng(41)
    hq, hkv, max_seq, seq_len = 6, 2, 256, 40
    kc, vc = _cache(rng, 4, hkv, max_seq, d)
    positions = np.concatenate([np.arange(40), np.arange(40), np.arange(50, 70)]).astype(np.int32)
    slots = np.repeat([2, 0, 3], [40, 40, 20]).astype(np.int32)
    slots[45] = 1
    positions[47] = max_seq + 5
    q = f16r(rng.standard_normal((positions.size, hq, d)))
    want, bad = oracle.attention_head_major(q, kc, vc, positions, slots)
    assert bad == 1  # the oracle attends row 45 to slot 1; the prefill kernel refuses it
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = host(_run(ops, q, kc, vc, positions, slots, seq_len=seq_len, err=err))
    torch.cuda.synchronize()
    from littlellm_b200 import _capi
    assert int(err.item()) == _capi.FLAG_BAD_POSITION | _capi.FLAG_BAD_SLOT
    assert np.all(got[[45, 47]] == 0)
    keep = np.setdiff1d(np.arange(positions.size), [45, 47])
    assert_tol(got[keep], want[keep], TOL, "prefill rows")


def test_prefill_more_items_than_sms(cuda, ops, oracle):
    """head_dim 128 prefill with 12 runs x 2 blocks of 256 tokens x 8 heads =
    192 CTAs (more than one per SM, so SMs take a second CTA that allocates
    the tensor memory the first released), runs at random start positions."""
    rng = np.random.default_rng(61)
    hq, hkv, d, max_seq, seq_len, n_runs = 8, 8, 128, 1024, 512, 12
    kc, vc = _cache(rng, n_runs, hkv, max_seq, d)
    starts = rng.integers(0, max_seq - seq_len, n_runs)
    positions = np.concatenate([np.arange(s0, s0 + seq_len) for s0 in starts]).astype(np.int32)
    slots = np.repeat(rng.permutation(n_runs), seq_len).astype(np.int32)
    q = f16r(rng.standard_normal((positions.size, hq, d)))
    want, _ = oracle.attention_head_major(q, kc, vc, positions, slots)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    got = _run(ops, q, kc, vc, positions, slots, seq_len=seq_len, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert_tol(host(got), want, TOL, "persistent prefill")
