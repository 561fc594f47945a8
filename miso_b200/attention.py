"""Host side of the attention hot path over torch device tensors.

Mirrors the kernel part of the reference engine's attention mixer (src/engine/attention.hip
:76-148): the same cache layout (AttentionCache, fp16 [2][max_ctx][256] for K and for V), the same
launch sequence (prep -> split -> combine for decode, prep_batch -> prefill for prefill), the same
error behaviour (a full cache raises before anything is launched). The projections around it
(GEMV / GEMM, o_proj) are outside this library. KvPool + decode_batched are the batched fast path.

Tensors are torch CUDA tensors; only their device addresses cross into the library.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _capi as capi

Q_HEADS, KV_HEADS, DIM, ROPE_DIM = 16, 2, 256, 64
MAX_SPLITS = 60  # AttentionScratch::kMaxSplits, src/engine/attention.hpp:46
PROJ = 9216      # AttentionScratch::kProj: [q+gate 8192 | k 512 | v 512]


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream


def rope_inv_freq(base: float = 1.0e7, dim: int = ROPE_DIM) -> np.ndarray:
    """inv_freq[i] = 1 / base^(2i / dim) in fp32 (src/engine/attention.hip:65-69)."""
    i = np.arange(dim // 2, dtype=np.float32)
    return (np.float32(1.0) / np.power(np.float32(base), (2 * i) / np.float32(dim))).astype(
        np.float32)


def n_splits(length: int, max_splits: int = MAX_SPLITS) -> int:
    return int(capi.load().miso_attn_n_splits(length, max_splits))


def prefill_items(n: int) -> int:
    return int(capi.load().miso_attn_prefill_items(n))


class AttentionCache:
    """fp16 KV cache of one layer: k, v [2][max_ctx][256] (src/engine/attention.hpp:35-41)."""

    def __init__(self, max_ctx: int, device="cuda"):
        self.max_ctx = max_ctx
        self.len = 0
        self.k = torch.zeros((KV_HEADS, max_ctx, DIM), dtype=torch.float16, device=device)
        self.v = torch.zeros((KV_HEADS, max_ctx, DIM), dtype=torch.float16, device=device)


class AttentionScratch:
    """Decode scratch (src/engine/attention.hpp:44-54): q, core and split partials."""

    def __init__(self, device="cuda"):
        f = dict(dtype=torch.float32, device=device)
        self.q = torch.empty((Q_HEADS, DIM), **f)
        self.core = torch.empty((Q_HEADS, DIM), **f)
        self.part_m = torch.empty((KV_HEADS * MAX_SPLITS * 8,), **f)
        self.part_l = torch.empty((KV_HEADS * MAX_SPLITS * 8,), **f)
        self.part_o = torch.empty((KV_HEADS * MAX_SPLITS * 8 * DIM,), **f)


def attn_prep(p: capi.AttnPrepParams, stream=None) -> None:
    capi.check("miso_attn_prep", capi.load().miso_attn_prep(C.byref(p), _stream(stream)))


def attn_prep_batch(p: capi.AttnPrepBatchParams, stream=None) -> None:
    capi.check("miso_attn_prep_batch",
               capi.load().miso_attn_prep_batch(C.byref(p), _stream(stream)))


def attn_split(p: capi.AttnSplitParams, stream=None) -> None:
    capi.check("miso_attn_split", capi.load().miso_attn_split(C.byref(p), _stream(stream)))


def attn_combine(p: capi.AttnCombineParams, stream=None) -> None:
    capi.check("miso_attn_combine", capi.load().miso_attn_combine(C.byref(p), _stream(stream)))


def attn_prefill(p: capi.AttnPrefillParams, stream=None) -> None:
    capi.check("miso_attn_prefill", capi.load().miso_attn_prefill(C.byref(p), _stream(stream)))


def attention_decode_core(cache: AttentionCache, sc: AttentionScratch, qg: torch.Tensor,
                          k: torch.Tensor, v: torch.Tensor, q_norm: torch.Tensor,
                          k_norm: torch.Tensor, inv_freq: torch.Tensor, eps: float,
                          stream=None) -> torch.Tensor:
    """One decode token from its projections (qg [16][512], k, v [2][256]): prep at position
    cache.len, ++len, split-K over the cache, gated combine -> sc.core [16][256]
    (the kernel sequence of src/engine/attention.hip:95-110)."""
    if cache.len >= cache.max_ctx:
        raise RuntimeError("attention_decode: KV cache is full")
    prep = capi.AttnPrepParams(_ptr(qg), _ptr(k), _ptr(v), _ptr(q_norm), _ptr(k_norm),
                               _ptr(inv_freq), _ptr(cache.k), _ptr(cache.v), _ptr(sc.q),
                               cache.len, cache.max_ctx, eps)
    attn_prep(prep, stream)
    cache.len += 1
    ns = n_splits(cache.len, MAX_SPLITS)
    attn_split(capi.AttnSplitParams(_ptr(sc.q), _ptr(cache.k), _ptr(cache.v), _ptr(sc.part_m),
                                    _ptr(sc.part_l), _ptr(sc.part_o), cache.len, cache.max_ctx,
                                    ns), stream)
    attn_combine(capi.AttnCombineParams(_ptr(sc.part_m), _ptr(sc.part_l), _ptr(sc.part_o),
                                        _ptr(qg), _ptr(sc.core), ns), stream)
    return sc.core


def attention_prefill_core(cache: AttentionCache, proj: torch.Tensor, n: int,
                           q_norm: torch.Tensor, k_norm: torch.Tensor, inv_freq: torch.Tensor,
                           eps: float, q_buf: torch.Tensor, core: torch.Tensor,
                           stream=None) -> torch.Tensor:
    """n tokens from a [n][9216] projection buffer ([q+gate 8192 | k 512 | v 512] per token):
    prep_batch at positions cache.len.., then causal prefill -> core [n][16][256]
    (src/engine/attention.hip:131-145)."""
    if cache.len + n > cache.max_ctx:
        raise RuntimeError("attention_prefill: KV cache is full")
    base = proj.data_ptr()
    pos0 = cache.len
    tok0 = capi.AttnPrepParams(base, base + 8192 * 4, base + 8704 * 4, _ptr(q_norm),
                               _ptr(k_norm), _ptr(inv_freq), _ptr(cache.k), _ptr(cache.v),
                               _ptr(q_buf), pos0, cache.max_ctx, eps)
    attn_prep_batch(capi.AttnPrepBatchParams(tok0, n, PROJ), stream)
    cache.len += n
    attn_prefill(capi.AttnPrefillParams(_ptr(q_buf), base, _ptr(cache.k), _ptr(cache.v),
                                        _ptr(core), pos0, n, cache.max_ctx, PROJ), stream)
    return core


# ---- batched fast path ------------------------------------------------------------------------


class KvPool:
    """fp16 K and V pools [rows][256] holding `batch` sequences; sequence b, KV head h owns rows
    [kv_row[b][h], kv_row[b][h] + capacity). lens lives on the device (int32) so decode steps can
    be enqueued without host round trips."""

    def __init__(self, batch: int, capacity: int, device="cuda", dtype=torch.float16):
        self.batch, self.capacity = batch, capacity
        self.rows = batch * KV_HEADS * capacity
        self.k = torch.empty((self.rows, DIM), dtype=dtype, device=device)
        self.v = torch.empty((self.rows, DIM), dtype=dtype, device=device)
        rows = (np.arange(batch * KV_HEADS, dtype=np.int64) * capacity).reshape(batch, KV_HEADS)
        self.kv_row = torch.from_numpy(rows).to(device)
        self.lens = torch.zeros((batch,), dtype=torch.int32, device=device)


def decode_scratch(batch: int, device="cuda") -> torch.Tensor:
    """Scratch for decode_batched (any contents: each call zeroes the counters it uses)."""
    n = int(capi.load().miso_attn_decode_scratch_bytes(batch))
    if n == 0:
        raise capi.MisoError("miso_attn_decode_scratch_bytes", -3)
    return torch.zeros((n + 255) // 256 * 256 // 4, dtype=torch.int32, device=device)


def decode_batched(pool: KvPool, q: torch.Tensor, qg: torch.Tensor, core: torch.Tensor,
                   scratch: torch.Tensor, qg_stride: int = Q_HEADS * 2 * DIM,
                   stream=None) -> torch.Tensor:
    """core[b] = softmax(q[b] K_b^T / 16) V_b * sigmoid(gate[b]) for all sequences of the pool."""
    p = capi.AttnDecodeParams(_ptr(q), _ptr(qg), _ptr(pool.k), _ptr(pool.v), _ptr(pool.kv_row),
                              _ptr(pool.lens), _ptr(core), pool.rows, pool.batch, qg_stride)
    capi.check("miso_attn_decode",
               capi.load().miso_attn_decode(C.byref(p), _ptr(scratch),
                                            scratch.numel() * scratch.element_size(),
                                            _stream(stream)))
    return core


def prep_batched(pool: KvPool, qg: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 q_norm: torch.Tensor, k_norm: torch.Tensor, inv_freq: torch.Tensor, eps: float,
                 q_out: torch.Tensor, proj_stride: int, stream=None) -> torch.Tensor:
    """Prep of one new token per sequence at position lens[b]; appends K/V and advances lens."""
    p = capi.AttnPrepBatchedParams(_ptr(qg), _ptr(k), _ptr(v), _ptr(q_norm), _ptr(k_norm),
                                   _ptr(inv_freq), _ptr(pool.k), _ptr(pool.v), _ptr(pool.kv_row),
                                   _ptr(pool.lens), _ptr(q_out), pool.batch, proj_stride, eps)
    capi.check("miso_attn_prep_batched",
               capi.load().miso_attn_prep_batched(C.byref(p), _stream(stream)))
    return q_out
