"""The oracle itself: pinned against the reference's own known-answer tests,
against golden vectors produced by the compiled reference, and (when the
compiled reference is present) against the reference on random inputs."""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle.oracle import F16, F32

# ---------------------------------------------------------------------------
# Known-answer tests from the reference's own test files
# ---------------------------------------------------------------------------


def test_kat_embedding(oracle):
    # tests/test_embedding.cpp:7-12
    table = np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    out = oracle.embedding(table, [2, 0])
    np.testing.assert_allclose(out.ravel(), [5, 6, 1, 2], atol=1e-4)


def test_kat_embedding_bad_id(oracle):
    # src/op/cpu/embedding.cpp:22-24 throws on an id outside the vocabulary
    with pytest.raises(ValueError):
        oracle.embedding(np.zeros((3, 2), np.float32), [1, 3])


def test_kat_add_bias(oracle):
    # tests/test_add_bias.cpp:7-12
    out = oracle.add_bias(np.array([[4, 5], [10, 11]], np.float32), np.array([1, -1], np.float32))
    np.testing.assert_allclose(out.ravel(), [5, 4, 11, 10], atol=1e-4)


def test_kat_select_last_row(oracle):
    # tests/test_select_last_row.cpp:7-12
    out = oracle.select_last_row(np.array([[5, 4], [11, 10]], np.float32))
    np.testing.assert_allclose(out.ravel(), [11, 10], atol=1e-4)


def test_kat_rms_norm(oracle):
    # tests/test_rms_norm.cpp:8-15 (eps = 0)
    out = oracle.rms_norm(np.array([[3, 4]], np.float32), np.array([1, 1], np.float32), 0.0)
    s = 1.0 / math.sqrt((9 + 16) / 2)
    np.testing.assert_allclose(out.ravel(), [3 * s, 4 * s], atol=1e-4)


def test_kat_silu(oracle):
    # tests/test_silu.cpp:8-15
    out = oracle.silu_mul(np.array([[0, 1]], np.float32), np.array([[2, 2]], np.float32))
    np.testing.assert_allclose(out.ravel(), [0, 2 / (1 + math.exp(-1))], atol=1e-4)


def test_kat_rope_position_zero(oracle):
    # tests/test_rope.cpp:7-11: position 0 is the identity
    x = np.array([[[1, 2, 3, 4]]], np.float32)
    np.testing.assert_allclose(oracle.rope(x, 0, 10000.0).ravel(), [1, 2, 3, 4], atol=1e-4)


def test_kat_kv_cache(oracle):
    # tests/test_kv_cache.cpp:7-15
    kc, vc = oracle.copy_kv_to_cache(np.array([[[1, 0]]], np.float32), np.array([[[2, 3]]], np.float32),
                                     np.zeros((2, 1, 2), np.float32), np.zeros((2, 1, 2), np.float32), 0)
    np.testing.assert_allclose(kc.ravel(), [1, 0, 0, 0], atol=1e-4)
    np.testing.assert_allclose(vc.ravel(), [2, 3, 0, 0], atol=1e-4)


def test_kat_kv_capacity(oracle):
    # src/op/cpu/kv_cache.cpp:19-21
    with pytest.raises(ValueError):
        oracle.copy_kv_to_cache(np.zeros((2, 1, 2), np.float32), np.zeros((2, 1, 2), np.float32),
                                np.zeros((3, 1, 2), np.float32), np.zeros((3, 1, 2), np.float32), 2)


def test_kat_half_roundtrip(oracle):
    # tests/test_half.cpp:7-11
    h = oracle.float_to_half_bits(np.array([1.5], np.float32))
    assert abs(oracle.half_bits_to_float(h)[0] - 1.5) <= 1e-3


def test_kat_quantize_roundtrip(oracle):
    # tests/test_quantize.cpp:15-51: per-tensor quantize (max/127, round) then
    # dequantize stays within 0.1; the quantize step follows
    # src/op/cpu/quantize.cpp:9-35.
    x = np.array([1, 2, 3, 4, 5, 6, 7, 8, -1, -2, -3, -4, -5, -6, -7, -8], np.float32)
    s = np.float32(np.abs(x).max() / np.float32(127.0))
    q = np.clip(np.round(x * (np.float32(1.0) / s)), -128, 127).astype(np.int8)
    np.testing.assert_allclose(oracle.dequantize_int8_f32(q, float(s)), x, atol=0.1)


# ---------------------------------------------------------------------------
# fp16 rounding of the reference (src/base/half.cpp:38-61)
# ---------------------------------------------------------------------------


def test_float_to_half_quirks(oracle):
    b = oracle.float_to_half_bits
    # ties round away from zero: 1 + 2^-11 is halfway between 1 and 1 + 2^-10
    assert b(np.array([1.0 + 2.0 ** -11], np.float32))[0] == 0x3C01
    # the carry out of the fraction is OR-ed into an odd exponent and lost
    assert b(np.array([0.12499202], np.float32))[0] == 0x2C00
    # exponent >= 31 (overflow, inf, NaN) -> inf; tiny -> signed zero
    assert b(np.array([65536.0], np.float32))[0] == 0x7C00
    assert b(np.array([np.nan], np.float32))[0] == 0x7C00
    assert b(np.array([-(2.0 ** -26)], np.float32))[0] == 0x8000


def test_half_to_float_exhaustive(oracle):
    h = np.arange(65536, dtype=np.uint16)
    f = oracle.half_bits_to_float(h)
    nan = np.isnan(h.view(np.float16))
    assert np.array_equal(f[~nan], h.view(np.float16)[~nan].astype(np.float32))
    # every non-NaN fp16 value survives half -> float -> half unchanged
    assert np.array_equal(oracle.float_to_half_bits(f)[~nan], h[~nan])


# ---------------------------------------------------------------------------
# Oracle vs. golden vectors (produced by the compiled reference)
# ---------------------------------------------------------------------------


def test_golden_float_to_half(oracle, golden):
    assert np.array_equal(oracle.float_to_half_bits(golden["f2h_in"]), golden["f2h_out"])


def test_golden_embedding(oracle, golden):
    assert np.array_equal(oracle.embedding(golden["emb_table"], golden["emb_ids"]), golden["emb_out"])


@pytest.mark.parametrize("name", ["a", "b"])
def test_golden_rms_norm(oracle, golden, name):
    out = oracle.rms_norm(golden[f"rms_{name}_x"], golden[f"rms_{name}_w"], float(golden[f"rms_{name}_eps"]))
    assert np.array_equal(out, golden[f"rms_{name}_out"])


def test_golden_add_rms_norm(oracle, golden):
    r, out = oracle.add_rms_norm(golden["addrms_r"], golden["addrms_d"], golden["addrms_w"], 1e-6)
    assert np.array_equal(r, golden["addrms_rsum"])
    assert np.array_equal(out, golden["addrms_out"])


def test_golden_bias_silu_last(oracle, golden):
    assert np.array_equal(oracle.add_bias(golden["bias_x"], golden["bias_b"]), golden["bias_out"])
    assert np.array_equal(oracle.silu_mul(golden["silu_g"], golden["silu_u"]), golden["silu_out"])
    assert np.array_equal(oracle.select_last_row(golden["last_x"]), golden["last_out"])


@pytest.mark.parametrize("name", ["a", "qwen", "llama"])
def test_golden_rope(oracle, golden, name):
    past, theta = golden[f"rope_{name}_meta"]
    out = oracle.rope(golden[f"rope_{name}_x"], int(past), float(theta))
    assert np.array_equal(out, golden[f"rope_{name}_out"])


def test_golden_kv(oracle, golden):
    kc, vc = oracle.copy_kv_to_cache(golden["kv_k"], golden["kv_v"], golden["kv_kc"], golden["kv_vc"], 5)
    assert np.array_equal(kc, golden["kv_kc_out"]) and np.array_equal(vc, golden["kv_vc_out"])


def test_golden_qkv_fused_composition(oracle, golden):
    g = golden
    kc0 = np.zeros_like(g["qkv_kc_out"])
    q, kc, vc, skipped = oracle.qkv_bias_rope_kv_append(
        g["qkv_q"], g["qkv_k"], g["qkv_v"], g["qkv_bq"], g["qkv_bk"], g["qkv_bv"], g["qkv_pos"],
        g["qkv_slots"], float(g["qkv_theta"]), kc0, kc0)
    assert skipped == 0
    assert np.array_equal(q, g["qkv_q_out"])
    assert np.array_equal(kc, g["qkv_kc_out"]) and np.array_equal(vc, g["qkv_vc_out"])


def test_golden_dequant(oracle, golden):
    for i, s in enumerate(golden["deq_scales"]):
        assert np.array_equal(oracle.dequantize_int8_f32(golden["deq_q"], float(s)), golden["deq_f32"][i])
        assert np.array_equal(oracle.dequantize_int8_f16_bits(golden["deq_q"], float(s)), golden["deq_f16"][i])


# ---------------------------------------------------------------------------
# Oracle vs. the compiled reference on random inputs (skipped without it)
# ---------------------------------------------------------------------------


def test_random_vs_reference(oracle, reference):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((7, 33)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 33).astype(np.float32)
    assert np.array_equal(oracle.rms_norm(x, w, 1e-5), reference.rms_norm(x, w, 1e-5))
    q = rng.standard_normal((5, 3, 10)).astype(np.float32)
    assert np.array_equal(oracle.rope(q, 123, 5e5), reference.rope(q, 123, 5e5))
    g, u = rng.standard_normal(999).astype(np.float32), rng.standard_normal(999).astype(np.float32)
    assert np.array_equal(oracle.silu_mul(g, u), reference.silu_mul(g, u))
    bits = rng.integers(0, 2 ** 32, 200_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    assert np.array_equal(oracle.float_to_half_bits(bits), reference.float_to_half_bits(bits))


def test_reference_f16_copies_are_bit_exact(reference):
    """The reference's CPU ops on F16 tensors round-trip through
    half_to_float/float_to_half, which is exact for every non-NaN fp16 value:
    gathers/copies of fp16 data are bit-exact copies."""
    rng = np.random.default_rng(3)
    table = rng.standard_normal((50, 24)).astype(np.float16)
    ids = rng.integers(0, 50, 9).astype(np.int32)
    out = reference.embedding(table, ids, F16)
    assert np.array_equal(out.view(np.uint16), table[ids].view(np.uint16))
    assert reference.embedding(table.astype(np.float32), ids, F32).dtype == np.float32
