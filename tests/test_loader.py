"""The .kllm index reader on the CPU: records, config and the format checks
of the reference loader (ModelWeights::load, src/model/weights.cpp:47-163)."""
from __future__ import annotations

import struct

import numpy as np
import pytest

from kllm_model import TinyConfig, write_model


@pytest.fixture(scope="module")
def loader():
    from littlellm_b200 import build
    build.build()
    from littlellm_b200 import loader as ld
    return ld


@pytest.mark.parametrize("wdt,ndt", [("f32", "f32"), ("f16", "f16"), ("i8", "f32"), ("i8", "f16")])
def test_index_matches_written_model(loader, tmp_path, wdt, ndt):
    from littlellm_b200 import _capi
    cfg = TinyConfig()
    path = str(tmp_path / "m.kllm")
    write_model(path, cfg, seed=2, weight_dtype=wdt, norm_dtype=ndt)
    idx = loader.read_index(path)
    assert idx.config["hidden_size"] == cfg.hidden and idx.config["num_layers"] == cfg.layers
    assert idx.config["model_type"] == cfg.model_type and idx.config["qkv_bias"] == 1
    assert abs(idx.config["rope_theta"] - cfg.theta) < 1
    names = idx.names()
    assert names[0] == "model.embed_tokens.weight" and names[-1] == "model.norm.weight"
    code = {"f32": _capi.F32, "f16": _capi.F16, "i8": _capi.I8}
    emb = idx.records[0]
    assert (emb.dims[0], emb.dims[1]) == (cfg.vocab, cfg.hidden)
    assert emb.dtype == code[wdt]
    assert emb.load_dtype == (_capi.F16 if wdt == "i8" else code[wdt])
    assert emb.nbytes == (emb.numel + 4 if wdt == "i8" else emb.numel * (4 if wdt == "f32" else 2))
    # records tile the file: each starts where the previous one's bytes end (+ its header)
    offs = [r.data_offset for r in idx.records]
    assert offs == sorted(offs)


def _corrupt(path, offset, data):
    with open(path, "r+b") as f:
        f.seek(offset)
        f.write(data)


def test_format_errors(loader, tmp_path, reference):
    from littlellm_b200 import _capi
    from oracle.oracle import ReferenceWeights
    good = str(tmp_path / "good.kllm")
    write_model(good, TinyConfig(), seed=3)
    raw = open(good, "rb").read()
    cases = {}
    cases["magic"] = b"KLLM0002" + raw[8:]
    cases["version"] = raw[:8] + struct.pack("<I", 2) + raw[12:]
    cases["truncated_header"] = raw[:40]
    cases["truncated_data"] = raw[:-7]
    idx = loader.read_index(good)
    # the first record's stored byte count sits 8 bytes before its data
    r0 = idx.records[0]
    bad = bytearray(raw)
    bad[r0.data_offset - 8:r0.data_offset] = struct.pack("<Q", r0.nbytes + 2)
    cases["nbytes"] = bytes(bad)
    for name, blob in cases.items():
        p = str(tmp_path / f"{name}.kllm")
        open(p, "wb").write(blob)
        with pytest.raises(_capi.KllmError) as e:
            loader.read_index(p)
        assert e.value.status == _capi.ERR_FORMAT, name
        # the reference loader rejects the same files
        with pytest.raises(RuntimeError):
            ReferenceWeights(reference, p)
    with pytest.raises(_capi.KllmError) as e:
        loader.read_index(str(tmp_path / "missing.kllm"))
    assert e.value.status == _capi.ERR_IO


def test_load_argument_checks_without_gpu(loader, tmp_path):
    import ctypes

    from littlellm_b200 import _capi
    path = str(tmp_path / "m.kllm")
    write_model(path, TinyConfig(), seed=4, weight_dtype="i8")
    idx = loader.read_index(path)
    n = len(idx.records)
    ptrs = (ctypes.c_void_p * n)(*([16] * n))
    host = np.zeros(1024, np.uint8)
    rc = _capi.lib.kllm_b200_kllm_load(path.encode(), idx.records, n, ptrs, host.ctypes.data, host.nbytes,
                                       None, 0, None)
    assert rc == _capi.ERR_INVALID_ARG and "staging" in _capi.last_error()
