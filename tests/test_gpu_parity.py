"""CUDA kernels vs. the oracle and the reference's golden vectors (small and
medium seeded cases). Copies and the INT8 dequant are bit-exact; fp16 float
ops are within |d| <= 1e-2 + 1e-2 |ref| of the reference's fp32 CPU path."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import assert_tol, bits16, canary_intact, dev, f16r, host, padded

pytestmark = pytest.mark.gpu

F16 = torch.float16
F32 = torch.float32

# ---------------------------------------------------------------------------
# golden vectors (from the compiled reference)
# ---------------------------------------------------------------------------


def test_embedding_golden(ops, golden):
    table, ids = golden["emb_table"], golden["emb_ids"]
    out16 = ops.embedding(dev(table, F16), dev(ids, torch.int32))
    assert np.array_equal(bits16(out16), golden["emb_out_f16"])
    out32 = ops.embedding(dev(table, F32), dev(ids, torch.int32))
    assert np.array_equal(host(out32), golden["emb_out"])


@pytest.mark.parametrize("name", ["a", "b"])
def test_rms_norm_golden(ops, golden, name):
    x, w, eps = golden[f"rms_{name}_x"], golden[f"rms_{name}_w"], float(golden[f"rms_{name}_eps"])
    assert_tol(host(ops.rms_norm(dev(x), dev(w), eps)), golden[f"rms_{name}_out"], what="f16")
    assert_tol(host(ops.rms_norm(dev(x, F32), dev(w, F32), eps)), golden[f"rms_{name}_out"], 1e-5, "f32")
    assert_tol(host(ops.rms_norm(dev(x), dev(w, F32), eps)), golden[f"rms_{name}_out"], what="f16/f32w")


def test_add_rms_norm_golden(ops, golden):
    r, d, w = golden["addrms_r"], golden["addrms_d"], golden["addrms_w"]
    res = dev(r)
    out = ops.add_rms_norm(res, dev(d), dev(w), 1e-6)
    # the stored residual is the fp16 (round-to-nearest-even) sum, as the
    # reference's fp16 add_inplace kernel writes it
    assert np.array_equal(bits16(res), (r + d).astype(np.float16).view(np.uint16))
    assert_tol(host(out), golden["addrms_out"])
    res32 = dev(r, F32)
    out32 = ops.add_rms_norm(res32, dev(d, F32), dev(w, F32), 1e-6)
    assert np.array_equal(host(res32), golden["addrms_rsum"])
    assert_tol(host(out32), golden["addrms_out"], 1e-5)


def test_add_bias_silu_golden(ops, golden):
    x = dev(golden["bias_x"])
    ops.add_bias_inplace(x, dev(golden["bias_b"]))
    assert_tol(host(x), golden["bias_out"])
    x32 = dev(golden["bias_x"], F32)
    ops.add_bias_inplace(x32, dev(golden["bias_b"], F32))
    assert np.array_equal(host(x32), golden["bias_out"])
    out = ops.silu_mul(dev(golden["silu_g"]), dev(golden["silu_u"]))
    assert_tol(host(out), golden["silu_out"])
    out32 = ops.silu_mul(dev(golden["silu_g"], F32), dev(golden["silu_u"], F32))
    assert_tol(host(out32), golden["silu_out"], 1e-5)


@pytest.mark.parametrize("name", ["a", "qwen", "llama"])
def test_rope_golden(ops, golden, name):
    past, theta = golden[f"rope_{name}_meta"]
    x = dev(golden[f"rope_{name}_x"])
    ops.rope_inplace(x, int(past), float(theta))
    assert_tol(host(x), golden[f"rope_{name}_out"])
    x32 = dev(golden[f"rope_{name}_x"], F32)
    ops.rope_inplace(x32, int(past), float(theta))
    assert_tol(host(x32), golden[f"rope_{name}_out"], 1e-4, "f32")


def test_kv_copy_golden(ops, golden):
    kc, vc = dev(golden["kv_kc"]), dev(golden["kv_vc"])
    ops.copy_kv_to_cache(dev(golden["kv_k"]), dev(golden["kv_v"]), kc, vc, 5)
    assert np.array_equal(host(kc), golden["kv_kc_out"]) and np.array_equal(host(vc), golden["kv_vc_out"])
    kc32, vc32 = dev(golden["kv_kc"], F32), dev(golden["kv_vc"], F32)
    ops.copy_kv_to_cache(dev(golden["kv_k"], F32), dev(golden["kv_v"], F32), kc32, vc32, 5)
    assert np.array_equal(host(kc32), golden["kv_kc_out"])


def test_qkv_fused_golden(ops, golden):
    g = golden
    q = dev(g["qkv_q"])
    kc = torch.zeros(g["qkv_kc_out"].shape, dtype=F16, device="cuda:0")
    vc = torch.zeros_like(kc)
    for bias_dtype in (F16, F32):
        q = dev(g["qkv_q"])
        kc.zero_()
        vc.zero_()
        ops.qkv_bias_rope_kv_append(q, dev(g["qkv_k"]), dev(g["qkv_v"]), dev(g["qkv_bq"], bias_dtype),
                                    dev(g["qkv_bk"], bias_dtype), dev(g["qkv_bv"], bias_dtype),
                                    dev(g["qkv_pos"], torch.int32), dev(g["qkv_slots"], torch.int32),
                                    float(g["qkv_theta"]), kc, vc)
        assert_tol(host(q), g["qkv_q_out"], what="q")
        assert_tol(host(kc), g["qkv_kc_out"], what="k cache")
        assert_tol(host(vc), g["qkv_vc_out"], what="v cache")


def test_select_last_row_golden(ops, golden):
    out = ops.select_last_row(dev(golden["last_x"]))
    assert np.array_equal(bits16(out), golden["last_out_f16"])
    out32 = ops.select_last_row(dev(golden["last_x"], F32))
    assert np.array_equal(host(out32), golden["last_out"])


def test_dequant_golden(ops, golden):
    q = dev(golden["deq_q"], torch.int8)
    for i, s in enumerate(golden["deq_scales"]):
        sc = torch.tensor([s], dtype=F32, device="cuda:0")
        assert np.array_equal(bits16(ops.dequantize_int8(q, sc, F16)), golden["deq_f16"][i])
        assert np.array_equal(host(ops.dequantize_int8(q, sc, F32)), golden["deq_f32"][i])


# ---------------------------------------------------------------------------
# seeded medium cases vs. the oracle, fast and generic paths, edge shapes
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("rows,hidden", [(512, 896), (513, 896), (64, 4096), (5, 4096), (33, 2048), (7, 40),
                                         (5, 900), (3, 7), (1, 16384), (2, 17000), (0, 896)])
@pytest.mark.parametrize("with_delta", [True, False])
def test_add_rms_norm_oracle(ops, oracle, rows, hidden, with_delta):
    rng = np.random.default_rng(rows * 7919 + hidden)
    r = f16r(rng.standard_normal((rows, hidden)))
    d = f16r(rng.standard_normal((rows, hidden))) if with_delta else None
    w = f16r(rng.uniform(0.5, 1.5, hidden))
    res = dev(r)
    whole, out = padded(rows * hidden, F16)
    ops.add_rms_norm(res, None if d is None else dev(d), dev(w), 1e-6, out=out.view(rows, hidden))
    r_ref, out_ref = oracle.add_rms_norm(r, d, w, 1e-6)
    if with_delta:
        assert np.array_equal(bits16(res), (r + d).astype(np.float16).view(np.uint16).reshape(rows, hidden))
    else:
        assert np.array_equal(host(res), r)
    assert_tol(host(out).reshape(rows, hidden), out_ref)
    assert canary_intact(whole, rows * hidden)


@pytest.mark.parametrize("n", [4096 * 4864 // 16, 8 * 1000 + 5, 3, 0])
def test_silu_mul_oracle(ops, oracle, n):
    rng = np.random.default_rng(n)
    g = f16r(rng.standard_normal(n) * 4)
    u = f16r(rng.standard_normal(n))
    whole, out = padded(n, F16)
    ops.silu_mul(dev(g), dev(u), out=out)
    assert_tol(host(out), oracle.silu_mul(g, u))
    assert canary_intact(whole, n)


def test_silu_mul_extremes(ops, oracle):
    g = np.array([-65504, -1000, -90, -80, -20, -1e-3, 0, 1e-3, 20, 80, 1000, 30000], np.float32)
    u = np.full_like(g, 2.0)
    out = host(ops.silu_mul(dev(g), dev(u)))
    ref = oracle.silu_mul(g, u)
    finite = np.isfinite(ref) & (np.abs(ref) < 65504)
    assert_tol(out[finite], ref[finite])


@pytest.mark.parametrize("vocab,hidden,n", [(151936, 896, 333), (32000, 4096, 64), (100, 12, 17), (50, 7, 9)])
def test_embedding_oracle(ops, vocab, hidden, n):
    rng = np.random.default_rng(vocab + n)
    table = rng.standard_normal((vocab, hidden)).astype(np.float16)
    ids = rng.integers(0, vocab, n).astype(np.int32)
    ids[:2] = [0, vocab - 1]
    out = ops.embedding(dev(table), dev(ids, torch.int32))
    assert np.array_equal(bits16(out), table[ids].view(np.uint16))


@pytest.mark.parametrize("T,Hq,Hkv,D,theta", [(512, 14, 2, 64, 1e6), (2500, 14, 2, 64, 1e6), (48, 32, 32, 128, 1e4),
                                              (40, 28, 4, 128, 1e6), (33, 32, 8, 128, 5e5),
                                              (37, 4, 2, 16, 1e4), (9, 3, 1, 6, 1e4), (5, 2, 2, 256, 1e6)])
@pytest.mark.parametrize("bias", ["f16", "f32", "none"])
def test_qkv_fused_oracle(ops, oracle, T, Hq, Hkv, D, theta, bias):
    rng = np.random.default_rng(T * 31 + D)
    S, NS = 4096, max(8, -(-T // 64))  # enough slots that positions stay below S
    q = f16r(rng.standard_normal((T, Hq, D)))
    k = f16r(rng.standard_normal((T, Hkv, D)))
    v = f16r(rng.standard_normal((T, Hkv, D)))
    bq, bk, bv = ((f16r(rng.normal(0, 0.02, H * D)) for H in (Hq, Hkv, Hkv)) if bias != "none"
                  else (None, None, None))
    bdt = F32 if bias == "f32" else F16  # fp16-representable values either way
    # distinct (slot, pos) per token so the expected cache does not depend on
    # write order; positions reach S - 1
    slots = (np.arange(T) % NS).astype(np.int32)
    pos = ((np.arange(T) // NS) * 53 + rng.integers(0, 53, T)).astype(np.int32)
    pos[0] = S - 1
    qd = dev(q)
    kc = torch.zeros((NS, Hkv, S, D), dtype=F16, device="cuda:0")
    vc = torch.zeros_like(kc)
    ops.qkv_bias_rope_kv_append(qd, dev(k), dev(v), None if bq is None else dev(bq, bdt),
                                None if bk is None else dev(bk, bdt), None if bv is None else dev(bv, bdt),
                                dev(pos, torch.int32), dev(slots, torch.int32), theta, kc, vc)
    zeros = np.zeros((NS, Hkv, S, D), np.float32)
    q_ref, kc_ref, vc_ref, skipped = oracle.qkv_bias_rope_kv_append(q, k, v, bq, bk, bv, pos, slots, theta,
                                                                     zeros, zeros)
    assert skipped == 0
    assert_tol(host(qd), q_ref, what="q")
    kch, vch = host(kc), host(vc)
    assert_tol(kch[slots, :, pos], kc_ref[slots, :, pos], what="k cache")
    # v rows: the fp16 (RNE) bias sum, bit-exact
    v_exp = (v + (bv.reshape(Hkv, D) if bias != "none" else 0)).astype(np.float16)
    assert np.array_equal(vch[slots, :, pos].astype(np.float16).view(np.uint16), v_exp.view(np.uint16))
    # nothing else of the cache was touched
    mask = np.ones((NS, S), bool)
    mask[slots, pos] = False
    assert not kch.transpose(0, 2, 1, 3)[mask].any() and not vch.transpose(0, 2, 1, 3)[mask].any()


@pytest.mark.parametrize("Hq,Hkv,D", [(14, 2, 64), (32, 32, 128), (4, 2, 64)])
def test_qkv_fused_bad_positions_and_slots(ops, oracle, Hq, Hkv, D):
    """Tokens whose position or slot is outside the cache set the flags and
    write no cache row; q is rotated for every token; the other tokens' rows
    are written as usual."""
    from littlellm_b200 import _capi
    rng = np.random.default_rng(D + Hq)
    T, S, NS, theta = 6, 64, 2, 1e4
    q, k, v = (f16r(rng.standard_normal((T, H, D))) for H in (Hq, Hkv, Hkv))
    pos = np.array([0, -1, 5, S, 7, 3], np.int32)
    slots = np.array([0, 0, NS, 1, -1, 1], np.int32)
    good = np.array([True, False, False, False, False, True])
    qd = dev(q)
    kc = torch.full((NS, Hkv, S, D), 7.0, dtype=F16, device="cuda:0")
    vc = torch.full_like(kc, 7.0)
    flags = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    ops.qkv_bias_rope_kv_append(qd, dev(k), dev(v), None, None, None, dev(pos, torch.int32),
                                dev(slots, torch.int32), theta, kc, vc, flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == _capi.FLAG_BAD_POSITION | _capi.FLAG_BAD_SLOT
    zeros = np.zeros((NS, Hkv, S, D), np.float32)
    q_ref, kc_ref, _, _ = oracle.qkv_bias_rope_kv_append(q[good], k[good], v[good], None, None, None, pos[good],
                                                         slots[good], theta, zeros, zeros)
    assert_tol(host(qd)[good], q_ref, what="q")
    kch, vch = host(kc), host(vc)
    gs, gp = slots[good], pos[good]
    assert_tol(kch[gs, :, gp], kc_ref[gs, :, gp], what="k cache")
    assert np.array_equal(vch[gs, :, gp], v[good])
    mask = np.ones((NS, S), bool)
    mask[gs, gp] = False
    assert (kch.transpose(0, 2, 1, 3)[mask] == 7.0).all() and (vch.transpose(0, 2, 1, 3)[mask] == 7.0).all()


@pytest.mark.parametrize("Hq,Hkv,D", [(14, 2, 64), (32, 32, 128), (28, 4, 128), (32, 8, 128), (4, 2, 64)])
def test_qkv_fused_equals_composed_legacy_ops(ops, Hq, Hkv, D):
    """Fused op == add_bias_inplace x3, rope_inplace x2, then the cache write,
    bit for bit (same rounding points, same rotation arithmetic), for the
    head layouts with a token kernel and one without."""
    rng = np.random.default_rng(11)
    T, S, theta = 64, 512, 1e6
    q, k, v = (f16r(rng.standard_normal((T, H, D))) for H in (Hq, Hkv, Hkv))
    bq, bk, bv = (f16r(rng.normal(0, 0.02, H * D)) for H in (Hq, Hkv, Hkv))
    past = 100
    pos = (past + np.arange(T)).astype(np.int32)
    slots = np.zeros(T, np.int32)
    qf = dev(q)
    kc = torch.zeros((1, Hkv, S, D), dtype=F16, device="cuda:0")
    vc = torch.zeros_like(kc)
    ops.qkv_bias_rope_kv_append(qf, dev(k), dev(v), dev(bq), dev(bk), dev(bv), dev(pos, torch.int32),
                                dev(slots, torch.int32), theta, kc, vc)
    ql, kl, vl = dev(q), dev(k), dev(v)
    ops.add_bias_inplace(ql.view(T, Hq * D), dev(bq))
    ops.add_bias_inplace(kl.view(T, Hkv * D), dev(bk))
    ops.add_bias_inplace(vl.view(T, Hkv * D), dev(bv))
    ops.rope_inplace(ql, past, theta)
    ops.rope_inplace(kl, past, theta)
    kcl = torch.zeros((S, Hkv, D), dtype=F16, device="cuda:0")
    vcl = torch.zeros_like(kcl)
    ops.copy_kv_to_cache(kl, vl, kcl, vcl, 0)
    assert torch.equal(qf, ql)
    assert torch.equal(kc[0, :, past:past + T].transpose(0, 1), kcl[:T])
    assert torch.equal(vc[0, :, past:past + T].transpose(0, 1), vcl[:T])


@pytest.mark.parametrize("n", [11008 * 4096 // 64, 1_000_003, 15, 0])
def test_dequant_oracle(ops, oracle, n):
    rng = np.random.default_rng(n)
    q = rng.integers(-128, 128, n, dtype=np.int8)
    s = np.float32(rng.uniform(1e-3, 1e-2))
    qd = dev(q, torch.int8)
    sc = torch.tensor([s], dtype=F32, device="cuda:0")
    whole, out = padded(n, F16)
    ops.dequantize_int8(qd, sc, F16, out=out)
    assert np.array_equal(bits16(out), oracle.dequantize_int8_f16_bits(q, float(s)))
    assert canary_intact(whole, n)
    assert np.array_equal(host(ops.dequantize_int8(qd, sc, F32)), oracle.dequantize_int8_f32(q, float(s)))


def test_dequant_unaligned(ops, oracle):
    rng = np.random.default_rng(5)
    q = rng.integers(-128, 128, 4099, dtype=np.int8)
    buf = dev(np.concatenate([[0], q]).astype(np.int8), torch.int8)
    qd = buf[1:]  # 1-byte offset: generic path
    sc = torch.tensor([0.0037], dtype=F32, device="cuda:0")
    assert np.array_equal(bits16(ops.dequantize_int8(qd, sc, F16)), oracle.dequantize_int8_f16_bits(q, 0.0037))


def test_select_last_rows(ops):
    rng = np.random.default_rng(2)
    x = rng.standard_normal((8 * 512, 896)).astype(np.float16)
    out = ops.select_last_rows(dev(x), seq_len=512, n_seqs=8)
    assert np.array_equal(bits16(out), x[511::512].view(np.uint16))
    ends = np.array([1, 700, 4096, 2000], np.int32)
    out = ops.select_last_rows(dev(x), seq_ends=dev(ends, torch.int32))
    assert np.array_equal(bits16(out), x[ends - 1].view(np.uint16))


@pytest.mark.parametrize("rows,cols", [(4096, 896), (3, 5)])
def test_add_inplace_and_bias(ops, rows, cols):
    rng = np.random.default_rng(rows)
    a = f16r(rng.standard_normal((rows, cols)))
    b = f16r(rng.standard_normal((rows, cols)))
    x = dev(a)
    ops.add_inplace(x, dev(b))
    assert np.array_equal(bits16(x), (a + b).astype(np.float16).view(np.uint16))
    bias = f16r(rng.standard_normal(cols))
    x = dev(a)
    ops.add_bias_inplace(x, dev(bias))
    assert np.array_equal(bits16(x), (a + bias).astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("out_dtype", [F16, F32])
def test_dequant_batched(ops, oracle, out_dtype):
    """Many tensors in one launch, including empty ones, ragged tails, an
    unaligned tensor (single-tensor fallback) and chunk boundaries."""
    rng = np.random.default_rng(21)
    sizes = [4096 * 4096 // 16, 0, 17, 8192, 8193, 3 * 16384 + 5, 1, 65536 * 3, 1000]
    qs = [rng.integers(-128, 128, n, dtype=np.int8) for n in sizes]
    scales = [np.float32(rng.uniform(1e-3, 1e-2)) for _ in sizes]
    scales[3] = np.float32(0.12499202 / 127)  # a scale that hits the carry quirk for q=127
    data = [dev(q, torch.int8) for q in qs]
    unaligned = dev(np.concatenate([[0], qs[-1]]).astype(np.int8), torch.int8)[1:]
    data[-1] = unaligned
    sc = [torch.tensor([s], dtype=F32, device="cuda:0") for s in scales]
    outs = [torch.empty(n, dtype=out_dtype, device="cuda:0") for n in sizes]
    ops.dequantize_int8_batched(data, sc, outs)
    for q, s, o in zip(qs, scales, outs):
        if out_dtype == F16:
            assert np.array_equal(bits16(o), oracle.dequantize_int8_f16_bits(q, float(s)))
        else:
            assert np.array_equal(host(o), oracle.dequantize_int8_f32(q, float(s)))


def test_dequant_batched_many_tensors(ops, oracle):
    """More tensors than one launch's task table holds (split launches)."""
    rng = np.random.default_rng(22)
    sizes = [int(n) for n in rng.integers(1, 5000, 300)]
    qs = [rng.integers(-128, 128, n, dtype=np.int8) for n in sizes]
    scales = [np.float32(rng.uniform(1e-3, 1e-2)) for _ in sizes]
    data = [dev(q, torch.int8) for q in qs]
    sc = [torch.tensor([s], dtype=F32, device="cuda:0") for s in scales]
    outs = [torch.empty(n, dtype=F16, device="cuda:0") for n in sizes]
    ops.dequantize_int8_batched(data, sc, outs)
    for q, s, o in zip(qs, scales, outs):
        assert np.array_equal(bits16(o), oracle.dequantize_int8_f16_bits(q, float(s)))


@pytest.mark.parametrize("n,offset", [(1_000_003, 0), (70_001, 1)])  # vector path with a ragged tail; unaligned
def test_dequant_rne_and_mismatch_count(cuda, ops, oracle, n, offset):
    """Opt-in IEEE rounding: the fp16 output equals numpy's round-to-nearest-even
    conversion of the same fp32 product, bit for bit, and the count equals the
    number of elements where that differs from the reference loader's
    rounding (ties away from zero, the dropped carry). Two calls add up."""
    rng = np.random.default_rng(n)
    q = rng.integers(-128, 128, n, dtype=np.int8)
    # 0.0061: no disagreement; (1 + 2^-11) * 2^-8 puts 15 of the 256 byte values on exact ties;
    # 0.0062498804 has 6 byte values where the two roundings differ
    for scale in (np.float32(0.0061), np.float32((1 + 2.0 ** -11) * 2.0 ** -8), np.float32(0.006249880418181419)):
        prod = q.astype(np.float32) * scale
        want = prod.astype(np.float16).view(np.uint16)
        ref = oracle.dequantize_int8_f16_bits(q, float(scale))
        expect = int(np.count_nonzero(want != ref))
        qbuf = torch.empty(n + offset, dtype=torch.int8, device=cuda)
        qbuf[offset:] = torch.from_numpy(q).to(cuda)
        obuf = torch.empty(n + offset, dtype=torch.float16, device=cuda)
        count = torch.zeros(1, dtype=torch.int64, device=cuda)
        sc = torch.tensor([scale], dtype=torch.float32, device=cuda)
        for _ in range(2):
            ops.dequantize_int8_rne(qbuf[offset:], sc, out=obuf[offset:], mismatches=count)
        torch.cuda.synchronize()
        got = obuf[offset:].cpu().view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(got, want)
        assert int(count.item()) == 2 * expect
        if scale != np.float32(0.0061):
            assert expect > 0  # the case exercises the count
