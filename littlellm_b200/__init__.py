"""littlellm_b200 — B200 (sm_100a) backend for LittleLLM's non-GEMM decoder-layer ops.

The product is ``libkllm_b200.so`` (CUDA kernels + C ABI, ``include/kllm_b200.h``).
This package builds it (``build``), binds it (``_capi``: importing it loads the
library and raises if it is missing — there is no fallback), wraps it for
torch tensors (``ops``) and drives the layer-op chain (``chain``).
"""
import importlib

__all__ = ["build", "ops", "chain", "KllmError"]


def __getattr__(name):
    if name in ("ops", "chain", "_capi", "build"):
        return importlib.import_module(f".{name}", __name__)
    if name == "KllmError":
        return importlib.import_module("._capi", __name__).KllmError
    raise AttributeError(name)
