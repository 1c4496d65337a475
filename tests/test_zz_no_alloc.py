"""kllm_b200_dequantize_int8_host_static — INT8 dequant from host memory with
no device allocation — against the entry points that use caller-allocated
device memory: kllm_b200_kllm_load (INT8 records staged in caller-provided
device scratch) and kllm_b200_dequantize_int8 (int8 values already on the
device). Outputs must agree bit for bit, on consecutive calls that reuse the
library's static staging array. Collected last so that it also runs after
every other test in the same process."""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_VALUES = 32 << 20  # the static staging array's size in bytes (one int8 value per byte)


def _host_static(q: np.ndarray, scale: float, out: torch.Tensor, out_dtype: int) -> int:
    from littlellm_b200 import _capi
    stream = torch.cuda.current_stream(out.device).cuda_stream
    return _capi.lib.kllm_b200_dequantize_int8_host_static(q.ctypes.data, scale, out.data_ptr(), q.size,
                                                            out_dtype, stream)


def _write_int8_record(path: str, q: np.ndarray, scale: np.float32) -> None:
    # a .kllm file holding one INT8 tensor "w" of q.size values
    with open(path, "wb") as f:
        f.write(b"KLLM0001" + struct.pack("<II", 1, 0) + struct.pack("<8i", 1, 1, 1, 1, 1, 1, 2, 1))
        f.write(struct.pack("<ffBBBBI", 1e-5, 1e4, 0, 0, 0, 0, 1))
        name = b"w"
        f.write(struct.pack("<I", len(name)) + name + struct.pack("<II", 3, 1) + struct.pack("<q", q.size))
        f.write(struct.pack("<Q", q.size + 4) + q.tobytes() + np.array([scale], np.float32).tobytes())


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def test_two_calls_match_the_allocating_entry_points(cuda, ops, oracle, tmp_path):
    from littlellm_b200 import _capi, loader
    rng = np.random.default_rng(23)

    # call 1: a tensor with a ragged tail vs kllm_b200_kllm_load through 1 MiB of device staging
    q1 = rng.integers(-128, 128, 3_000_017, dtype=np.int8)
    s1 = np.float32(0.0047)
    path = str(tmp_path / "one.kllm")
    _write_int8_record(path, q1, s1)
    _, tensors = loader.load(path, cuda, staging_bytes=1 << 20)
    want1 = _bits(tensors["w"])
    out1 = torch.full((q1.size,), -1234.0, dtype=torch.float16, device=cuda)
    assert _host_static(q1, float(s1), out1, _capi.F16) == _capi.OK, _capi.last_error()

    # call 2, right after it, different values and scale, reusing the same staging:
    # vs kllm_b200_dequantize_int8 on a device copy of the values
    q2 = rng.integers(-128, 128, 1_234_567, dtype=np.int8)
    s2 = np.float32(-0.0913)
    out2 = torch.full((q2.size,), -1234.0, dtype=torch.float16, device=cuda)
    assert _host_static(q2, float(s2), out2, _capi.F16) == _capi.OK, _capi.last_error()
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out1), want1)
    # and directly against the oracle's restatement of the reference loader's rounding
    assert np.array_equal(_bits(out2), oracle.dequantize_int8_f16_bits(q2, float(s2)))
    dev_q2 = torch.from_numpy(q2).to(cuda)
    dev_s2 = torch.tensor([s2], dtype=torch.float32, device=cuda)
    assert np.array_equal(_bits(out2), _bits(ops.dequantize_int8(dev_q2, dev_s2, torch.float16)))

    # F32 output: float(q) * scale, as kllm_b200_dequantize_int8 gives it
    out3 = torch.empty(q2.size, dtype=torch.float32, device=cuda)
    assert _host_static(q2, float(s2), out3, _capi.F32) == _capi.OK, _capi.last_error()
    want3 = ops.dequantize_int8(dev_q2, dev_s2, torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(out3, want3)


def test_capacity_limit(cuda, ops):
    from littlellm_b200 import _capi
    rng = np.random.default_rng(29)
    # exactly the staging size is accepted ...
    q = rng.integers(-128, 128, MAX_VALUES, dtype=np.int8)
    out = torch.empty(MAX_VALUES, dtype=torch.float16, device=cuda)
    assert _host_static(q, 0.25, out, _capi.F16) == _capi.OK, _capi.last_error()
    want = ops.dequantize_int8(torch.from_numpy(q).to(cuda), torch.tensor([0.25], device=cuda), torch.float16)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    # ... one value more is refused before any GPU work, leaving the output untouched
    big = np.zeros(MAX_VALUES + 1, dtype=np.int8)
    out_big = torch.full((MAX_VALUES + 1,), -1234.0, dtype=torch.float16, device=cuda)
    rc = _host_static(big, 1.0, out_big, _capi.F16)
    assert rc == _capi.ERR_CAPACITY
    assert "static staging" in _capi.last_error()
    torch.cuda.synchronize()
    assert bool((out_big == -1234.0).all())


def test_pinned_host_buffer(cuda, ops, oracle):
    """A pinned host buffer gives the same bits as a pageable one."""
    from littlellm_b200 import _capi
    rng = np.random.default_rng(31)
    q = rng.integers(-128, 128, 777_777, dtype=np.int8)
    pinned = torch.empty(q.size, dtype=torch.int8, pin_memory=True)
    pinned.numpy()[:] = q
    out = torch.empty(q.size, dtype=torch.float16, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    rc = _capi.lib.kllm_b200_dequantize_int8_host_static(pinned.data_ptr(), 0.0031, out.data_ptr(), q.size,
                                                          _capi.F16, stream)
    assert rc == _capi.OK, _capi.last_error()
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), oracle.dequantize_int8_f16_bits(q, 0.0031))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs a second GPU")
def test_second_device_after_first(cuda, ops, oracle):
    """The staging address is looked up in each device's own context: a call
    on device 1 after calls on device 0 lands in device 1's array."""
    from littlellm_b200 import _capi
    rng = np.random.default_rng(37)
    q = rng.integers(-128, 128, 500_001, dtype=np.int8)
    want = oracle.dequantize_int8_f16_bits(q, 0.0077)
    for dev in (torch.device("cuda:0"), torch.device("cuda:1"), torch.device("cuda:0")):
        with torch.cuda.device(dev):
            out = torch.empty(q.size, dtype=torch.float16, device=dev)
            assert _host_static(q, 0.0077, out, _capi.F16) == _capi.OK, _capi.last_error()
            torch.cuda.synchronize(dev)
            assert np.array_equal(_bits(out), want), dev
