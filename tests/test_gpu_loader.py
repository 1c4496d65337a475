"""Streaming .kllm load with device-side INT8 dequant vs the reference's own
loader (ModelWeights::load): F32/F16 tensors byte-identical, INT8 tensors
equal to the reference's fp16 load result (float(q) * scale through the
reference float_to_half) bit for bit."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from kllm_model import TinyConfig, write_model

pytestmark = pytest.mark.gpu


def _expected(ref_w, oracle, rec):
    from littlellm_b200 import _capi
    name = rec.name.decode()
    vals = ref_w.get(name, rec.numel)  # reference CPU load: F32 values (I8 -> float(q)*scale)
    if rec.dtype == _capi.I8:
        return "bits", oracle.float_to_half_bits(vals)
    return "values", vals


@pytest.mark.parametrize("wdt,ndt,staging", [("f32", "f32", 64 << 20), ("f16", "f16", 64 << 20),
                                             ("i8", "f32", 64 << 20), ("i8", "f16", 64 << 10)])
def test_load_matches_reference_loader(cuda, oracle, reference, tmp_path, wdt, ndt, staging):
    from littlellm_b200 import loader
    from oracle.oracle import ReferenceWeights
    cfg = TinyConfig(vocab=1000, hidden=96, intermediate=320)  # 96K-param embedding: several 32 KB chunks
    path = str(tmp_path / "m.kllm")
    write_model(path, cfg, seed=5, weight_dtype=wdt, norm_dtype=ndt)
    _, tensors = loader.load(path, cuda, staging_bytes=staging)
    torch.cuda.synchronize()
    ref_w = ReferenceWeights(reference, path)
    idx = loader.read_index(path)
    for rec in idx.records:
        t = tensors[rec.name.decode()]
        kind, exp = _expected(ref_w, oracle, rec)
        if kind == "bits":
            got = t.cpu().view(torch.int16).numpy().view(np.uint16).ravel()
            assert np.array_equal(got, exp), rec.name
        else:
            assert np.array_equal(t.float().cpu().numpy().ravel(), exp), rec.name
    ref_w.close()


def test_load_large_int8_tensor_chunked(cuda, oracle, tmp_path):
    """A 12M-value INT8 tensor through 1 MB of staging (many chunks, a ragged
    tail) dequantised bit-exactly."""
    import struct
    from littlellm_b200 import loader
    rng = np.random.default_rng(9)
    n = 12_000_007
    q = rng.integers(-127, 128, n, dtype=np.int8)
    scale = np.float32(0.0061)
    path = str(tmp_path / "big.kllm")
    with open(path, "wb") as f:
        f.write(b"KLLM0001" + struct.pack("<II", 1, 0) + struct.pack("<8i", 1, 1, 1, 1, 1, 1, 2, 1))
        f.write(struct.pack("<ffBBBBI", 1e-5, 1e4, 0, 0, 0, 0, 1))
        name = b"w"
        f.write(struct.pack("<I", len(name)) + name + struct.pack("<II", 3, 1) + struct.pack("<q", n))
        f.write(struct.pack("<Q", n + 4) + q.tobytes() + np.array([scale], np.float32).tobytes())
    _, tensors = loader.load(path, cuda, staging_bytes=1 << 20)
    got = tensors["w"].cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, oracle.dequantize_int8_f16_bits(q, float(scale)))
