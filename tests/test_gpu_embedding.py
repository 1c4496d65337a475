"""The embedding gather fused with layer 0's input RMSNorm
(kllm_b200_embedding_rms_norm) and the embedding with host-resident ids
(kllm_b200_embedding_host_ids), against the oracle and against the
library's separate entry points.

Bars: the gathered rows (the residual) are bit-exact copies of the table
rows, as the reference's embedding writes them (src/op/cpu/embedding.cpp:9-29);
the normed rows are within |d| <= 1e-2 + 1e-2 |ref| of the oracle's
rms_norm (src/op/cpu/rms_norm.cpp:9-29) of those rows, and bit-identical to
kllm_b200_embedding followed by kllm_b200_rms_norm."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from gpu_util import assert_tol, bits16, host

pytestmark = pytest.mark.gpu

F16 = torch.float16


def _table(vocab, hidden, seed):
    g = torch.Generator(device="cuda:0")
    g.manual_seed(seed)
    return (torch.randn((vocab, hidden), generator=g, device="cuda:0") * 0.02).to(F16)


@pytest.mark.parametrize("hidden,n_tokens,vocab", [
    (896, 4096, 151936),    # Qwen2.5-0.5B prefill (8 x 512)
    (4096, 257, 32000),     # Llama-2-7B rows, ragged count
    (896, 1, 1000),
    (64, 33, 500),          # sub-warp row groups
    (900, 19, 777),         # hidden % 8 != 0: gather + norm as two launches
])
@pytest.mark.parametrize("wdt", [torch.float16, torch.float32])
def test_embedding_rms_norm_matches_oracle_and_unfused(ops, oracle, hidden, n_tokens, vocab, wdt):
    table = _table(vocab, hidden, 11)
    ids = torch.randint(0, vocab, (n_tokens,), device="cuda:0", dtype=torch.int32)
    w = (torch.rand(hidden, device="cuda:0") + 0.5).to(wdt)
    eps = 1e-6
    flags = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    res, out = ops.embedding_rms_norm(table, ids, w, eps, err_flags=flags)
    # unfused: this library's embedding then rms_norm
    res2 = ops.embedding(table, ids)
    out2 = ops.rms_norm(res2, w, eps)
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    ids_h = ids.cpu().numpy()
    assert np.array_equal(bits16(res), bits16(table)[ids_h])
    assert np.array_equal(bits16(out), bits16(out2))
    assert_tol(host(out), oracle.rms_norm(host(res), host(w), eps), what="norm")


def test_embedding_rms_norm_bad_ids_zero_rows_and_flag(ops):
    table = _table(100, 896, 12)
    ids = torch.tensor([3, -1, 99, 100, 5], dtype=torch.int32, device="cuda:0")
    w = torch.ones(896, dtype=F16, device="cuda:0")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    res, out = ops.embedding_rms_norm(table, ids, w, 1e-6, err_flags=flags)
    torch.cuda.synchronize()
    from littlellm_b200 import _capi
    assert int(flags.item()) == _capi.FLAG_BAD_TOKEN
    for row in (1, 3):
        assert bool((res[row] == 0).all()) and bool((out[row] == 0).all())
    for row, i in ((0, 3), (2, 99), (4, 5)):
        assert torch.equal(res[row], table[i])


def test_embedding_rms_norm_pdl_chain_first_layer(cuda, oracle):
    """Through the chain executor (PDL): layer 0's input norm comes from the
    fused kernel, the residual equals the gathered rows until layer 0's post
    norm adds to it."""
    from littlellm_b200 import _capi
    from littlellm_b200.chain import ChainRunner, ModelShape, Workload
    m = ModelShape("q1", 896, 14, 2, 64, 4864, 3000, 1, 1e-6, 1e6)
    r = ChainRunner(Workload("q1", m, 4, 33, 64, False), device=cuda, seed=21, use_pdl=True)
    r.desc.op_mask = _capi.OP_EMBEDDING | _capi.OP_INPUT_NORM
    assert r.run() == 1
    torch.cuda.synchronize()
    ids = r.ids.cpu().numpy()
    assert np.array_equal(bits16(r.residual), bits16(r.table)[ids])
    assert_tol(host(r.layers[0]["attn_norm_out"]),
               oracle.rms_norm(host(r.residual), host(r.layers[0]["input_norm_w"]), m.eps))
    assert int(r.err_flags.item()) == 0


@pytest.mark.parametrize("n_tokens", [1, 100, 7680, 7681, 20000])
def test_embedding_host_ids_bit_exact(ops, n_tokens):
    """Host ids travel in the launches' parameters, 7680 per launch."""
    table = _table(32000, 4096, 13)
    ids = np.random.default_rng(n_tokens).integers(0, 32000, n_tokens).astype(np.int32)
    out = ops.embedding_host_ids(table, ids)
    torch.cuda.synchronize()
    assert np.array_equal(bits16(out), bits16(table)[ids])


def test_embedding_host_ids_generic_paths_and_flags(ops):
    from littlellm_b200 import _capi
    t32 = torch.randn((50, 7), device="cuda:0")           # 28-byte rows: element path, fp32 -> fp16
    ids = [0, 49, 7, 50, -3]
    flags = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    out = torch.full((5, 7), -1234.0, dtype=F16, device="cuda:0")
    ops.embedding_host_ids(t32, ids, out=out, err_flags=flags)
    torch.cuda.synchronize()
    assert int(flags.item()) == _capi.FLAG_BAD_TOKEN
    want = t32.cpu().numpy()[[0, 49, 7]].astype(np.float16)
    assert np.array_equal(bits16(out[:3]), want.view(np.uint16))
    assert bool((out[3:] == 0).all())
    # the ids buffer may be reused at once: the call captured them at launch
    host_ids = np.array([1, 2, 3], np.int32)
    out2 = ops.embedding_host_ids(t32, host_ids)
    host_ids[:] = 0
    torch.cuda.synchronize()
    assert np.array_equal(host(out2), t32.cpu().numpy()[[1, 2, 3]])
