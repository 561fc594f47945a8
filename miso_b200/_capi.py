"""ctypes mirror of include/miso_cuda.h.

The structures are field-for-field copies of the C header (which in turn is field-for-field the
reference's Params structs), so a caller fills them exactly as the reference engine fills its
Params. All pointer fields are device addresses (ints); `stream` is a cudaStream_t as an int.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

_P = C.c_void_p
_U = C.c_uint
_F = C.c_float


class AttnPrepParams(C.Structure):
    _fields_ = [("qg", _P), ("k", _P), ("v", _P), ("q_norm", _P), ("k_norm", _P),
                ("inv_freq", _P), ("k_cache", _P), ("v_cache", _P), ("q", _P),
                ("pos", _U), ("max_ctx", _U), ("eps", _F)]


class AttnPrepBatchParams(C.Structure):
    _fields_ = [("tok0", AttnPrepParams), ("n", _U), ("proj_stride", _U)]


class AttnSplitParams(C.Structure):
    _fields_ = [("q", _P), ("k_cache", _P), ("v_cache", _P), ("part_m", _P), ("part_l", _P),
                ("part_o", _P), ("len", _U), ("max_ctx", _U), ("n_splits", _U)]


class AttnCombineParams(C.Structure):
    _fields_ = [("part_m", _P), ("part_l", _P), ("part_o", _P), ("qg", _P), ("core", _P),
                ("n_splits", _U)]


class AttnPrefillParams(C.Structure):
    _fields_ = [("q", _P), ("qg", _P), ("k_cache", _P), ("v_cache", _P), ("core", _P),
                ("pos0", _U), ("n", _U), ("max_ctx", _U), ("qg_stride", _U)]


class DeltaNetStepParams(C.Structure):
    _fields_ = [("qkv", _P), ("z", _P), ("a", _P), ("b", _P), ("conv_w", _P), ("conv_in", _P),
                ("conv_out", _P), ("ssm_a", _P), ("dt_bias", _P), ("norm_w", _P),
                ("state", _P), ("out", _P), ("eps", _F)]


class DeltaNetSeqParams(C.Structure):
    _fields_ = [("qkv", _P), ("z", _P), ("a", _P), ("b", _P), ("conv_w", _P), ("conv_in", _P),
                ("conv_out", _P), ("ssm_a", _P), ("dt_bias", _P), ("norm_w", _P),
                ("state", _P), ("out", _P), ("n", _U), ("eps", _F), ("zab_stride", _U),
                ("qkv_stride", _U)]


class DeltaNetConvParams(C.Structure):
    _fields_ = [("qkv", _P), ("a", _P), ("b", _P), ("conv_w", _P), ("conv_in", _P),
                ("conv_out", _P), ("ssm_a", _P), ("dt_bias", _P), ("q", _P), ("k", _P),
                ("v", _P), ("beta", _P), ("log_a", _P), ("n", _U)]


class DeltaNetChunkParams(C.Structure):
    _fields_ = [("q", _P), ("k", _P), ("v", _P), ("beta", _P), ("log_a", _P), ("z", _P),
                ("norm_w", _P), ("state", _P), ("out", _P), ("sk", _P), ("sq", _P),
                ("n", _U), ("eps", _F)]


class AttnDecodeParams(C.Structure):
    _fields_ = [("q", _P), ("qg", _P), ("k_pool", _P), ("v_pool", _P), ("kv_row", _P),
                ("lens", _P), ("core", _P), ("pool_rows", C.c_uint64), ("batch", _U),
                ("qg_stride", _U)]


class AttnPrepBatchedParams(C.Structure):
    _fields_ = [("qg", _P), ("k", _P), ("v", _P), ("q_norm", _P), ("k_norm", _P),
                ("inv_freq", _P), ("k_pool", _P), ("v_pool", _P), ("kv_row", _P),
                ("lens", _P), ("q", _P), ("batch", _U), ("proj_stride", _U), ("eps", _F)]


class AttnPrefillTcParams(C.Structure):
    _fields_ = [("q", _P), ("qg", _P), ("k_cache", _P), ("v_cache", _P), ("core", _P),
                ("pos0", _U), ("n", _U), ("max_ctx", _U), ("qg_stride", _U)]


class DeltaNetStepBatchedParams(C.Structure):
    _fields_ = [("qkv", _P), ("z", _P), ("a", _P), ("b", _P), ("conv_w", _P), ("ssm_a", _P),
                ("dt_bias", _P), ("norm_w", _P), ("conv_in", _P), ("conv_out", _P),
                ("state", _P), ("out", _P), ("batch", _U), ("in_stride", _U), ("eps", _F)]


# name -> (restype, argtypes); every symbol include/miso_cuda.h declares.
SIGNATURES = {
    "miso_attn_n_splits": (_U, [_U, _U]),
    "miso_attn_prefill_items": (_U, [_U]),
    "miso_attn_prep": (C.c_int, [C.POINTER(AttnPrepParams), _P]),
    "miso_attn_prep_batch": (C.c_int, [C.POINTER(AttnPrepBatchParams), _P]),
    "miso_attn_split": (C.c_int, [C.POINTER(AttnSplitParams), _P]),
    "miso_attn_combine": (C.c_int, [C.POINTER(AttnCombineParams), _P]),
    "miso_attn_prefill": (C.c_int, [C.POINTER(AttnPrefillParams), _P]),
    "miso_deltanet_step": (C.c_int, [C.POINTER(DeltaNetStepParams), _P]),
    "miso_deltanet_seq": (C.c_int, [C.POINTER(DeltaNetSeqParams), _P]),
    "miso_deltanet_seq_ckpt": (C.c_int, [C.POINTER(DeltaNetSeqParams), _P, _P, _P]),
    "miso_deltanet_commit": (C.c_int, [_P, _P, C.c_uint, C.c_uint, _P, _P, _P]),
    "miso_deltanet_conv": (C.c_int, [C.POINTER(DeltaNetConvParams), _P]),
    "miso_deltanet_norm": (C.c_int, [C.POINTER(DeltaNetConvParams), _P]),
    "miso_deltanet_chunk": (C.c_int, [C.POINTER(DeltaNetChunkParams), _P]),
    "miso_attn_decode_scratch_bytes": (C.c_size_t, [_U]),
    "miso_attn_decode": (C.c_int, [C.POINTER(AttnDecodeParams), _P, C.c_size_t, _P]),
    "miso_attn_decode_noalloc": (C.c_int, [C.POINTER(AttnDecodeParams), _P]),
    "miso_attn_prep_batched": (C.c_int, [C.POINTER(AttnPrepBatchedParams), _P]),
    "miso_attn_prefill_tc": (C.c_int, [C.POINTER(AttnPrefillTcParams), _P]),
    "miso_deltanet_step_batched": (C.c_int, [C.POINTER(DeltaNetStepBatchedParams), _P]),
    "miso_deltanet_prefill_tc_scratch_bytes": (C.c_size_t, [_U]),
    "miso_deltanet_prefill_tc": (C.c_int, [C.POINTER(DeltaNetSeqParams), _P, C.c_size_t, _P]),
    "miso_deltanet_prefill_tc_front": (C.c_int, [C.POINTER(DeltaNetSeqParams), _P, C.c_size_t,
                                                 _P]),
    "miso_deltanet_prefill_tc_recur": (C.c_int, [C.POINTER(DeltaNetSeqParams), _P, C.c_size_t,
                                                 _P]),
    "miso_deltanet_prefill_tc_chain": (C.c_int, [C.POINTER(DeltaNetSeqParams), _P, C.c_size_t,
                                                 _P]),
    "miso_deltanet_prefill_tc_gate": (C.c_int, [C.POINTER(DeltaNetSeqParams), _P, C.c_size_t,
                                                _P]),
    "miso_attn_prep_batch_f16": (C.c_int, [C.POINTER(AttnPrepBatchParams), _P, _P]),
    "miso_device_status": (C.c_int, [C.c_int, C.POINTER(C.c_int)]),
    "miso_version": (C.c_char_p, []),
}

ERRORS = {-1: "MISO_ERR_INVALID", -2: "MISO_ERR_SCRATCH", -3: "MISO_ERR_NO_DEVICE",
          -4: "MISO_ERR_DRIVER", -5: "MISO_ERR_LIMIT"}


class MisoError(RuntimeError):
    def __init__(self, fn: str, code: int):
        name = ERRORS.get(code, f"cudaError {code}")
        super().__init__(f"{fn} failed: {name} ({code})")
        self.code = code


_lib = None


def load(path: str | None = None) -> C.CDLL:
    """Loads the built library (never builds it). Raises if it is missing: there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or _build.LIB
    if not os.path.exists(path):
        raise ImportError(
            f"miso_b200: CUDA library not built ({path}); run `python miso_b200/build.py`")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(fn: str, code: int) -> None:
    if code != 0:
        raise MisoError(fn, code)
