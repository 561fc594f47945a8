"""Seeded inputs of the golden fixtures, shared by make_golden.py and the tests.

numpy's legacy RandomState stream is stable across numpy versions, so the fixtures store only
outputs; the inputs are regenerated bit for bit from these functions.
"""
from __future__ import annotations

import numpy as np

EPS = 1e-6
ROPE_BASE = 1.0e7


def inv_freq(base: float = ROPE_BASE, dim: int = 64) -> np.ndarray:
    i = np.arange(dim // 2, dtype=np.float32)
    return (np.float32(1.0) / np.power(np.float32(base), (2 * i) / np.float32(dim))).astype(
        np.float32)


def prep_inputs(seed: int = 11):
    r = np.random.RandomState(seed)
    qg = r.standard_normal((16, 512)).astype(np.float32) * np.float32(1.5)
    k = r.standard_normal((2, 256)).astype(np.float32)
    v = r.standard_normal((2, 256)).astype(np.float32)
    w_q = (r.standard_normal(256) * 0.1).astype(np.float32)  # HF weight; stored as 1 + w
    w_k = (r.standard_normal(256) * 0.1).astype(np.float32)
    return dict(qg=qg, k=k, v=v, q_norm=(1.0 + w_q).astype(np.float32),
                k_norm=(1.0 + w_k).astype(np.float32), w_q=w_q, w_k=w_k, pos=1234,
                inv_freq=inv_freq())


def decode_inputs(length: int = 200, seed: int = 12):
    """One sequence: q [16][256] (N(0, 2^2) like tests/test_attn_splitk.hip:110-111), qg gate
    N(0, 1), K/V fp16 N(0, 1) in a [2][max_ctx][256] cache with max_ctx = length + 7."""
    r = np.random.RandomState(seed)
    max_ctx = length + 7
    q = (2.0 * r.standard_normal((16, 256))).astype(np.float32)
    qg = r.standard_normal((16, 512)).astype(np.float32)
    k = r.standard_normal((2, max_ctx, 256)).astype(np.float16)
    v = r.standard_normal((2, max_ctx, 256)).astype(np.float16)
    return dict(q=q, qg=qg, k=k, v=v, len=length, max_ctx=max_ctx)


def prefill_inputs(pos0: int = 20, n: int = 17, seed: int = 13):
    r = np.random.RandomState(seed)
    max_ctx = pos0 + n + 5
    q = (2.0 * r.standard_normal((n, 16, 256))).astype(np.float32)
    qg = r.standard_normal((n, 16, 512)).astype(np.float32)
    k = r.standard_normal((2, max_ctx, 256)).astype(np.float16)
    v = r.standard_normal((2, max_ctx, 256)).astype(np.float16)
    return dict(q=q, qg=qg, k=k, v=v, pos0=pos0, n=n, max_ctx=max_ctx)


def deltanet_inputs(n: int = 70, seed: int = 14):
    """A short sequence in the reference's layouts (kernels/deltanet_step.hpp:22-36):
    qkv [n][8192], z [n][4096], a / b [n][32], conv_w [8192][4], conv history [8192][3],
    ssm_a / dt_bias [32], norm_w [128], state [32][128][128] (k-major)."""
    r = np.random.RandomState(seed)
    f = lambda *s, sc=1.0: (r.standard_normal(s) * sc).astype(np.float32)  # noqa: E731
    qkv = f(n, 8192, sc=0.5)
    z = f(n, 4096)
    a = f(n, 32)
    b = f(n, 32)
    conv_w = f(8192, 4, sc=0.5)
    conv_in = f(8192, 3, sc=0.5)
    ssm_a = (-np.exp(r.standard_normal(32) * 0.5)).astype(np.float32)
    dt_bias = f(32, sc=0.3)
    norm_w = (1.0 + r.standard_normal(128) * 0.1).astype(np.float32)
    state = f(32, 128, 128, sc=0.1)
    return dict(n=n, qkv=qkv, z=z, a=a, b=b, conv_w=conv_w, conv_in=conv_in, ssm_a=ssm_a,
                dt_bias=dt_bias, norm_w=norm_w, state=state)


# DeltaNet V heads whose outputs / final state the fixture stores (subset keeps it small).
DN_HEADS = (5, 16)
# V head whose final state the fixture stores.
DN_STATE_HEAD = 16
