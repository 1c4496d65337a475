"""tcgen05 GEMM with fused epilogues (scope row f4) against the oracle:
linear() = matmul + add_bias_inplace and the MLP's gate/up linears +
silu_mul, on the reference's known-answer test, the golden fixtures of the
compiled reference, seeded shapes against the C oracle (ragged m, n and k,
fp16 and fp32 biases), model shapes against a torch fp32 reference, and the
fused SwiGLU against this library's own linear + linear + silu_mul bit for
bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import TOL, assert_tol, bits16, dev, f16r, host

pytestmark = pytest.mark.gpu


def _inputs(rng, m, n, k, n_weights=1):
    x = f16r(rng.standard_normal((m, k)))
    ws = [f16r(rng.standard_normal((n, k)) / np.sqrt(k)) for _ in range(n_weights)]
    return x, ws


def test_reference_kat(cuda, ops):
    # tests/test_matmul.cpp:7-13 and tests/test_ops.cpp:59-68; k is padded from
    # 3 to 8 with zeros (the kernel takes k in multiples of 8), which leaves
    # every dot product unchanged
    a = np.zeros((2, 8), np.float32)
    b = np.zeros((2, 8), np.float32)
    a[:, :3] = [[1, 2, 3], [4, 5, 6]]
    b[:, :3] = [[1, 0, 1], [0, 1, 1]]
    out = ops.linear(dev(a), dev(b))
    assert np.array_equal(host(out), [[4, 5], [10, 11]])
    out = ops.linear(dev(a), dev(b), dev([1, -1]))
    assert np.array_equal(host(out), [[5, 4], [11, 10]])
    out = ops.linear(dev(a), dev(b), dev([1, -1], torch.float32))
    assert np.array_equal(host(out), [[5, 4], [11, 10]])


def test_golden_linear_and_mlp(cuda, ops, golden):
    g = golden
    assert_tol(host(ops.linear(dev(g["mm_x"]), dev(g["mm_w"]))), g["mm_out"], what="matmul")
    assert_tol(host(ops.linear(dev(g["mm_x"]), dev(g["mm_w"]), dev(g["mm_b"]))), g["lin_out"], what="linear")
    out = ops.linear_swiglu(dev(g["mlp_x"]), dev(g["mlp_wg"]), dev(g["mlp_wu"]), dev(g["mlp_bg"]),
                            dev(g["mlp_bu"]))
    assert_tol(host(out), g["mlp_out"], what="linear_swiglu")


@pytest.mark.parametrize("m,n,k", [(1, 256, 64), (128, 256, 64), (130, 300, 136), (256, 512, 896),
                                   (513, 1152, 896), (77, 203, 200)])
@pytest.mark.parametrize("bias", [None, torch.float16, torch.float32])
def test_linear_vs_oracle(cuda, ops, oracle, m, n, k, bias):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    x, (w,) = _inputs(rng, m, n, k)
    b = f16r(rng.normal(0, 0.1, n)) if bias is not None else None
    out = ops.linear(dev(x), dev(w), dev(b, bias) if bias is not None else None)
    want = oracle.linear(x, w, b)
    assert_tol(host(out), want, what=f"linear {m}x{n}x{k}")


@pytest.mark.parametrize("m,n,k", [(5, 128, 64), (300, 640, 896), (129, 203, 136), (1, 4864, 896),
                                   (8, 4864, 896), (64, 1000, 512), (8, 1024, 2048)])
@pytest.mark.parametrize("bias", [None, torch.float16, torch.float32])
def test_swiglu_vs_oracle_and_unfused(cuda, ops, oracle, m, n, k, bias):
    rng = np.random.default_rng(m * 11 + n + k * 5)
    x, (wg, wu) = _inputs(rng, m, n, k, 2)
    bg = f16r(rng.normal(0, 0.1, n)) if bias is not None else None
    bu = f16r(rng.normal(0, 0.1, n)) if bias is not None else None
    tb = (lambda a: dev(a, bias)) if bias is not None else (lambda a: None)
    xd, wgd, wud, bgd, bud = dev(x), dev(wg), dev(wu), tb(bg), tb(bu)
    fused = ops.linear_swiglu(xd, wgd, wud, bgd, bud)
    want = oracle.silu_mul(oracle.linear(x, wg, bg), oracle.linear(x, wu, bu))
    assert_tol(host(fused), want, what=f"linear_swiglu {m}x{n}x{k}")
    # the same values as the separate ops of this library, bit for bit
    unfused = ops.silu_mul(ops.linear(xd, wgd, bgd), ops.linear(xd, wud, bud))
    torch.cuda.synchronize()
    assert np.array_equal(bits16(fused), bits16(unfused))


@pytest.mark.parametrize("what,m,n,k", [
    ("qwen qkv linear", 4096, 1152, 896),
    ("qwen gate/up + silu", 4096, 4864, 896),
    ("llama gate/up + silu", 512, 11008, 4096),
    ("llama down linear", 300, 4096, 11008),
])
def test_model_shapes_vs_torch_fp32(cuda, ops, what, m, n, k):
    g = torch.Generator(device=cuda).manual_seed(m + n + k)
    x = torch.randn(m, k, device=cuda, generator=g).half()
    w = (torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, device=cuda, generator=g) * 0.1).half()
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ref = x.float() @ w.float().T + b.float()
    if "silu" in what:
        w2 = (torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).half()
        b2 = (torch.randn(n, device=cuda, generator=g) * 0.1).half()
        out = ops.linear_swiglu(x, w, w2, b, b2, err_flags=err)
        up = x.float() @ w2.float().T + b2.float()
        ref = ref * torch.sigmoid(ref) * up
    else:
        out = ops.linear(x, w, b, err_flags=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    diff = (out.float() - ref).abs()
    bad = diff > TOL + TOL * ref.abs()
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} outside tolerance, max abs err {float(diff.max()):.3g}"


def test_output_bounds_and_ragged_columns(cuda, ops, oracle):
    """Only out[m, n] is written: rows past m (a partial 128-row tile) and, for
    n not a multiple of 8, the element-wise edge path stay in bounds."""
    rng = np.random.default_rng(3)
    m, n, k = 130, 203, 72
    x, (wg, wu) = _inputs(rng, m, n, k, 2)
    whole = torch.full(((m + 2) * n,), -1234.0, dtype=torch.float16, device=cuda)
    out = whole[: m * n].view(m, n)
    ops.linear(dev(x), dev(wg), out=out)
    torch.cuda.synchronize()
    assert bool((whole[m * n:] == -1234.0).all())
    assert_tol(host(out), oracle.matmul(x, wg), what="ragged linear")
    whole.fill_(-1234.0)
    ops.linear_swiglu(dev(x), dev(wg), dev(wu), out=out)
    torch.cuda.synchronize()
    assert bool((whole[m * n:] == -1234.0).all())
    assert_tol(host(out), oracle.silu_mul(oracle.matmul(x, wg), oracle.matmul(x, wu)), what="ragged swiglu")


def test_repeated_calls_are_deterministic(cuda, ops):
    g = torch.Generator(device=cuda).manual_seed(9)
    x = torch.randn(1000, 896, device=cuda, generator=g).half()
    wg = (torch.randn(4864, 896, device=cuda, generator=g) / 30).half()
    wu = (torch.randn(4864, 896, device=cuda, generator=g) / 30).half()
    first = ops.linear_swiglu(x, wg, wu)
    for _ in range(3):
        again = ops.linear_swiglu(x, wg, wu)
        torch.cuda.synchronize()
        assert torch.equal(first, again)


@pytest.mark.parametrize("m", [1, 8, 32, 64, 100, 128])
@pytest.mark.parametrize("n,k,bias", [
    (896, 4864, torch.float16),   # Qwen2.5-0.5B down projection: clusters of 8 CTAs (m <= 8), 3, 2, none (m > 64)
    (896, 896, None),             # o projection: clusters of 7 (m <= 16), none from m = 32 (short k)
    (203, 2056, torch.float32),   # ragged n (element-wise stores) and k (a partial last k slice): clusters of 4
    (4096, 256, torch.float16),   # many column tiles, no split
])
def test_single_row_tile_vs_torch_fp32(cuda, ops, m, n, k, bias):
    """GEMMs of one row tile (m <= 128: decode batches) load an x box of m
    rows rounded up to 8 into a deeper ring, and with a long k and few
    columns split each tile's k range over a cluster of CTAs whose fp32
    partial sums the leader CTA adds in rank order: against torch fp32,
    deterministic from call to call."""
    g = torch.Generator(device=cuda).manual_seed(m * 1000 + n + k)
    x = torch.randn(m, k, device=cuda, generator=g).half()
    w = (torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, device=cuda, generator=g) * 0.1).to(bias) if bias is not None else None
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    out = ops.linear(x, w, b, err_flags=err)
    again = ops.linear(x, w, b, err_flags=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out, again)
    ref = x.float() @ w.float().T + (b.float() if b is not None else 0)
    diff = (out.float() - ref).abs()
    bad = diff > TOL + TOL * ref.abs()
    assert not bool(bad.any()), f"{m}x{n}x{k}: {int(bad.sum())} outside tolerance, max abs err {float(diff.max()):.3g}"


@pytest.mark.parametrize("what,m,n,k,bias", [
    ("linear, ragged m, n and k", 4100, 4100, 200, torch.float16),
    ("linear, square", 8192, 8192, 256, None),
    ("swiglu, ragged n and k, fp32 bias", 8192, 3000, 136, torch.float32),
    ("linear, 224-wide tiles (n = 896)", 4096, 896, 896, torch.float16),
    ("linear, 224-wide tiles, long k", 300, 896, 4864, None),
    ("linear, 192-wide tiles", 8192, 1152, 256, torch.float32),
    ("swiglu, 192-wide tiles", 2048, 1440, 512, torch.float16),
])
def test_large_tilings_vs_torch_fp32(cuda, ops, what, m, n, k, bias):
    """Problems of many waves (several raster groups of 4096 rows) and the
    192- and 224-wide tilings, with partial row and column tiles and a k tail,
    against torch fp32."""
    g = torch.Generator(device=cuda).manual_seed(m ^ n ^ k)
    x = torch.randn(m, k, device=cuda, generator=g).half()
    w = (torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).half()
    b = (torch.randn(n, device=cuda, generator=g) * 0.1).to(bias) if bias is not None else None
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ref = x.float() @ w.float().T + (b.float() if b is not None else 0)
    if "swiglu" in what:
        w2 = (torch.randn(n, k, device=cuda, generator=g) / k ** 0.5).half()
        b2 = (torch.randn(n, device=cuda, generator=g) * 0.1).to(bias)
        out = ops.linear_swiglu(x, w, w2, b, b2, err_flags=err)
        up = x.float() @ w2.float().T + b2.float()
        ref = ref * torch.sigmoid(ref) * up
        # the fused op equals this library's separate ops bit for bit here too
        unfused = ops.silu_mul(ops.linear(x, w, b), ops.linear(x, w2, b2))
        torch.cuda.synchronize()
        assert torch.equal(out, unfused)
    else:
        out = ops.linear(x, w, b, err_flags=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    diff = (out.float() - ref).abs()
    bad = diff > TOL + TOL * ref.abs()
    assert not bool(bad.any()), f"{what}: {int(bad.sum())} outside tolerance, max abs err {float(diff.max()):.3g}"


@pytest.mark.parametrize("T,hidden,hq,hkv,d,bias", [
    (300, 896, 14, 2, 64, torch.float16),   # Qwen2.5-0.5B heads, fp16 biases
    (130, 512, 8, 8, 128, None),            # Llama-style heads, no bias
    (77, 256, 7, 1, 64, torch.float32),     # odd q heads: the last q tile is half full; fp32 biases
    (8, 896, 14, 2, 64, torch.float16),     # a decode batch of Qwen2.5-0.5B: clusters of 7 CTAs
    (8, 2048, 16, 4, 128, torch.float16),   # a decode batch with k = 2048: split over clusters of 4 CTAs
    (24, 4096, 8, 2, 64, torch.float32),    # k = 4096 split over clusters of 3 (24 rows of partial sums)
    (4096, 512, 16, 16, 128, torch.float16),  # large enough for 256-wide tiles (two heads per tile)
    (4096, 512, 16, 4, 64, None),             # 256-wide tiles of four 64-column heads
])
def test_qkv_rope_fused_equals_separate_ops(cuda, ops, T, hidden, hq, hkv, d, bias):
    """kllm_b200_qkv_linear_rope_kv_append equals linear x3 followed by
    kllm_b200_qkv_bias_rope_kv_append bit for bit: q, both caches (rows not
    written stay as they were) and the error flags, with one token at an
    out-of-range position and one at an out-of-range slot."""
    g = torch.Generator(device=cuda).manual_seed(T * 31 + hidden)
    x = torch.randn(T, hidden, device=cuda, generator=g).half()
    wq, wk, wv = ((torch.randn(h * d, hidden, device=cuda, generator=g) / hidden ** 0.5).half()
                  for h in (hq, hkv, hkv))
    bq, bk, bv = ((torch.randn(h * d, device=cuda, generator=g) * 0.1).to(bias) if bias is not None else None
                  for h in (hq, hkv, hkv))
    n_slots, max_seq, theta = (64 if T > 500 else 5), 96, 1e6
    t = torch.arange(T, device=cuda, dtype=torch.int32)
    slots, positions = t % n_slots, t // n_slots  # distinct (slot, position) per token
    positions[3] = max_seq
    slots[5] = -1
    kc0 = torch.randn(n_slots, hkv, max_seq, d, device=cuda, generator=g).half()
    vc0 = torch.randn(n_slots, hkv, max_seq, d, device=cuda, generator=g).half()

    kc1, vc1, err1 = kc0.clone(), vc0.clone(), torch.zeros(1, dtype=torch.int32, device=cuda)
    q1 = ops.qkv_linear_rope_kv_append(x, wq, wk, wv, bq, bk, bv, positions, slots, theta, kc1, vc1, err_flags=err1)

    kc2, vc2, err2 = kc0.clone(), vc0.clone(), torch.zeros(1, dtype=torch.int32, device=cuda)
    q, k, v = ops.linear(x, wq), ops.linear(x, wk), ops.linear(x, wv)
    ops.qkv_bias_rope_kv_append(q.view(T, hq, d), k.view(T, hkv, d), v.view(T, hkv, d), bq, bk, bv, positions,
                                slots, theta, kc2, vc2, err_flags=err2)
    torch.cuda.synchronize()
    assert torch.equal(q1, q)
    assert torch.equal(kc1, kc2)
    assert torch.equal(vc1, vc2)
    assert int(err1.item()) == int(err2.item()) != 0
