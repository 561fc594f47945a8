"""miso_b200 — the attention hot path of Qwen3.5-MoE hybrid models, native to B200 (sm_100a).

Four kernel families behind one C ABI (include/miso_cuda.h, library miso_b200/lib/
libmiso_b200.so):
  * GQA full-attention decode (split-K over an fp16 KV cache), single-sequence drop-in and a
    batched stream-K fast path;
  * causal gated GQA prefill;
  * Gated DeltaNet recurrent step (and the fused n-token recurrence);
  * Gated DeltaNet chunked prefill (chunk 64).

This Python package is a thin host layer over that ABI: ctypes bindings (`capi`) and torch-tensor
helpers mirroring the reference engine's host side (`attention`, `deltanet`). Importing it loads
the compiled library; if the library has not been built the import fails — there is no CPU or
PyTorch fallback anywhere in the package.
"""
from . import _capi as capi
from ._capi import MisoError

capi.load()

from . import attention, deltanet  # noqa: E402

__all__ = ["capi", "MisoError", "attention", "deltanet"]
