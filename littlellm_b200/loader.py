"""Loading .kllm weight files onto the GPU through the C ABI.

``read_index`` parses the file's header and record table (host only);
``load`` allocates one device tensor per record (INT8 records become fp16,
as the reference's CUDA loader makes them) and streams the file into them
with ``kllm_b200_kllm_load``, which dequantises INT8 records on the device.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _capi


class KllmConfig(ctypes.Structure):
    _fields_ = [("model_type", ctypes.c_uint32), ("vocab_size", ctypes.c_int32),
                ("hidden_size", ctypes.c_int32), ("intermediate_size", ctypes.c_int32),
                ("num_layers", ctypes.c_int32), ("num_heads", ctypes.c_int32),
                ("num_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("max_seq_len", ctypes.c_int32), ("rms_norm_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float), ("tie_word_embeddings", ctypes.c_uint8),
                ("qkv_bias", ctypes.c_uint8), ("o_bias", ctypes.c_uint8), ("mlp_bias", ctypes.c_uint8)]


class KllmRecord(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 192), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 8), ("numel", ctypes.c_int64), ("data_offset", ctypes.c_uint64),
                ("nbytes", ctypes.c_uint64), ("load_dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("load_bytes", ctypes.c_int64)]


_TORCH = {_capi.F32: torch.float32, _capi.F16: torch.float16, _capi.I32: torch.int32}

_capi.lib.kllm_b200_kllm_read_index.argtypes = [ctypes.c_char_p, ctypes.POINTER(KllmConfig),
                                                ctypes.POINTER(KllmRecord), ctypes.c_int,
                                                ctypes.POINTER(ctypes.c_int)]
_capi.lib.kllm_b200_kllm_load.argtypes = [ctypes.c_char_p, ctypes.POINTER(KllmRecord), ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p, ctypes.c_size_t,
                                          ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]


@dataclass
class Index:
    config: dict
    records: ctypes.Array  # KllmRecord array

    def names(self) -> list[str]:
        return [r.name.decode() for r in self.records]


def read_index(path: str) -> Index:
    n = ctypes.c_int(0)
    cfg = KllmConfig()
    _capi.check(_capi.lib.kllm_b200_kllm_read_index(path.encode(), ctypes.byref(cfg), None, 0, ctypes.byref(n)))
    recs = (KllmRecord * max(n.value, 1))()
    _capi.check(_capi.lib.kllm_b200_kllm_read_index(path.encode(), ctypes.byref(cfg), recs, n.value,
                                                    ctypes.byref(n)))
    config = {name: getattr(cfg, name) for name, _ in KllmConfig._fields_}
    return Index(config, (KllmRecord * n.value).from_buffer(recs) if n.value else recs[:0])


def load(path: str, device: torch.device | str = "cuda:0", staging_bytes: int = 64 << 20,
         index: Index | None = None) -> tuple[dict, dict[str, torch.Tensor]]:
    """Returns (config, {name: device tensor})."""
    device = torch.device(device)
    idx = index or read_index(path)
    recs = idx.records
    tensors = {}
    ptrs = (ctypes.c_void_p * max(len(recs), 1))()
    for i, r in enumerate(recs):
        shape = tuple(r.dims[d] for d in range(r.ndim))
        t = torch.empty(shape, dtype=_TORCH[r.load_dtype], device=device)
        tensors[r.name.decode()] = t
        ptrs[i] = t.data_ptr() if t.numel() else None
    host = torch.empty(staging_bytes, dtype=torch.uint8, pin_memory=True)
    dev = torch.empty(staging_bytes, dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        _capi.check(_capi.lib.kllm_b200_kllm_load(path.encode(), recs, len(recs), ptrs, host.data_ptr(),
                                                  staging_bytes, dev.data_ptr(), staging_bytes,
                                                  stream.cuda_stream))
    return idx.config, tensors
