"""CPU oracle of the attention hot path — TEST INFRASTRUCTURE ONLY.

A restatement of penta2himajin/miso's scalar references and kernel formulas in C (double
precision), loaded with ctypes. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline /
reference arm use it, and only as the checker or the timed CPU baseline; the product library
never calls it.

Every function takes numpy arrays (C-contiguous; float32 / uint16 / int64 / int32 as documented in
miso_oracle.h) and returns float64 numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libmiso_oracle.so")

_lib = None


REF = os.environ.get("MISO_REFERENCE_DIR",
                     os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
REF_QUANT = os.path.join(HERE, "_ref", "libref_quant.so")


def build() -> str:
    """Builds the C oracle; where the reference's sources are present, also its weight-format code
    (oracle/_ref/libref_quant.so) that pins oracle/quant.py."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    if os.path.exists(os.path.join(REF, "src", "repack.cpp")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={REF}"], check=True)
    return LIB


def ref_quant():
    """The reference's dequant / repack code (ctypes), or None when it was not built."""
    if not os.path.exists(REF_QUANT):
        return None
    lib = C.CDLL(REF_QUANT)
    lib.ref_dequant.argtypes = [C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_size_t]
    lib.ref_repack_q4k.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p]
    lib.ref_repack_q6k.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p, C.c_size_t]
    lib.ref_q6k_r1_row_bytes.argtypes = [C.c_size_t]
    lib.ref_q6k_r1_row_bytes.restype = C.c_size_t
    return lib


def _load() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        _lib = C.CDLL(LIB)
        _lib.oracle_half_to_double.restype = C.c_double
        _lib.oracle_half_to_double.argtypes = [C.c_uint16]
        _lib.oracle_attn_n_splits.restype = C.c_uint
        _lib.oracle_attn_n_splits.argtypes = [C.c_uint, C.c_uint]
        _lib.oracle_cpu_count.restype = C.c_int
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def cpu_count() -> int:
    return int(_load().oracle_cpu_count())


def half_to_double(bits: int) -> float:
    return float(_load().oracle_half_to_double(bits))


def attn_n_splits(length: int, max_splits: int) -> int:
    return int(_load().oracle_attn_n_splits(length, max_splits))


def attn_prep(qg, k, v, q_norm, k_norm, inv_freq, pos: int, eps: float):
    """Decode prep of one token: returns (q [16][256], k [2][256], v [2][256]) in float64."""
    q_out = np.zeros((16, 256)); k_out = np.zeros((2, 256)); v_out = np.zeros((2, 256))
    args = [_f32(x) for x in (qg, k, v, q_norm, k_norm, inv_freq)]
    _load().oracle_attn_prep(*[_p(x) for x in args], C.c_uint(pos), C.c_float(eps),
                             _p(q_out), _p(k_out), _p(v_out))
    return q_out, k_out, v_out


def attn_decode(q, qg, qg_stride: int, k_pool, v_pool, kv_row, lens, threads: int = 0):
    """Batched decode reference: out [batch][16][256]."""
    q = _f32(q); qg = _f32(qg)
    k_pool = np.ascontiguousarray(k_pool, dtype=np.uint16)
    v_pool = np.ascontiguousarray(v_pool, dtype=np.uint16)
    kv_row = np.ascontiguousarray(kv_row, dtype=np.int64)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    batch = lens.shape[0]
    out = np.zeros((batch, 16, 256))
    _load().oracle_attn_decode(C.c_uint(batch), _p(q), _p(qg), C.c_uint(qg_stride), _p(k_pool),
                               _p(v_pool), _p(kv_row), _p(lens), _p(out), C.c_int(threads))
    return out


def attn_prefill(n: int, pos0: int, q, qg, qg_stride: int, k_cache, v_cache, max_ctx: int,
                 rows=None, threads: int = 0):
    """Causal prefill reference: out [n or len(rows)][16][256]."""
    q = _f32(q); qg = _f32(qg)
    k_cache = np.ascontiguousarray(k_cache, dtype=np.uint16)
    v_cache = np.ascontiguousarray(v_cache, dtype=np.uint16)
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.uint32)
    nr = n if r is None else r.shape[0]
    out = np.zeros((nr, 16, 256))
    _load().oracle_attn_prefill(C.c_uint(n), C.c_uint(pos0), _p(q), _p(qg), C.c_uint(qg_stride),
                                _p(k_cache), _p(v_cache), C.c_uint(max_ctx), _p(r),
                                C.c_uint(0 if r is None else nr), _p(out), C.c_int(threads))
    return out


def attn_combine(part_m, part_l, part_o, qg, n_splits: int):
    out = np.zeros((16, 256))
    args = [_f32(x) for x in (part_m, part_l, part_o, qg)]
    _load().oracle_attn_combine(*[_p(x) for x in args], C.c_uint(n_splits), _p(out))
    return out


def deltanet_step(qkv, z, a, b, conv_w, conv, ssm_a, dt_bias, norm_w, state, eps: float,
                  threads: int = 0):
    """One decode step for a batch (leading axis) of sequences. conv ([B][8192][3]) and state
    ([B][32][128][128]) are float64 arrays updated in place; returns out [B][4096]."""
    qkv = _f32(qkv); z = _f32(z); a = _f32(a); b = _f32(b)
    assert conv.dtype == np.float64 and state.dtype == np.float64
    batch = qkv.reshape(-1, 8192).shape[0]
    out = np.zeros((batch, 4096))
    w = [_f32(x) for x in (conv_w, ssm_a, dt_bias, norm_w)]
    _load().oracle_deltanet_step(C.c_uint(batch), _p(qkv), _p(z), _p(a), _p(b), _p(w[0]),
                                 _p(conv), _p(w[1]), _p(w[2]), _p(w[3]), _p(state), _p(out),
                                 C.c_float(eps), C.c_int(threads))
    return out


def deltanet_seq(n: int, qkv, qkv_stride: int, zab, zab_stride: int, conv_w, conv, ssm_a,
                 dt_bias, norm_w, state, eps: float, z_off: int = 0, a_off: int = 4096,
                 b_off: int = 4128, threads: int = 0):
    """n-token recurrence. z / a / b live in one buffer `zab` (float32, flat or [n][zab_stride]):
    token t reads z at t * zab_stride + z_off, a at + a_off, b at + b_off (the reference's shared
    projection layout, src/engine/deltanet.hip:97-112). conv / state float64, updated in place;
    returns out [n][4096]."""
    qkv = _f32(qkv); zab = _f32(zab)
    out = np.zeros((n, 4096))
    w = [_f32(x) for x in (conv_w, ssm_a, dt_bias, norm_w)]
    base = zab.ctypes.data
    z, a, b = (C.c_void_p(base + 4 * off) for off in (z_off, a_off, b_off))
    _load().oracle_deltanet_seq(C.c_uint(n), _p(qkv), C.c_uint(qkv_stride), z, a, b,
                                C.c_uint(zab_stride), _p(w[0]), _p(conv), _p(w[1]), _p(w[2]),
                                _p(w[3]), _p(state), _p(out), C.c_float(eps), C.c_int(threads))
    return out


def deltanet_seq_heads(n: int, qkv, qkv_stride: int, zab, zab_stride: int, conv_w, conv, ssm_a,
                       dt_bias, norm_w, state, eps: float, heads, z_off: int = 0,
                       a_off: int = 4096, b_off: int = 4128, threads: int = 0):
    """deltanet_seq for the listed V heads only: state ([32][128][128] float64) updated in place
    for those heads; returns out [n][len(heads)][128] (the heads' outputs in list order). The conv
    history `conv` (float64 [8192][3]) is read, not updated."""
    qkv = _f32(qkv); zab = _f32(zab)
    hs = np.ascontiguousarray(heads, dtype=np.uint32)
    conv = np.ascontiguousarray(conv, dtype=np.float64)
    assert state.dtype == np.float64 and state.flags["C_CONTIGUOUS"]
    out = np.zeros((n, hs.shape[0], 128))
    w = [_f32(x) for x in (conv_w, ssm_a, dt_bias, norm_w)]
    base = zab.ctypes.data
    z, a, b = (C.c_void_p(base + 4 * off) for off in (z_off, a_off, b_off))
    _load().oracle_deltanet_seq_heads(C.c_uint(n), _p(qkv), C.c_uint(qkv_stride), z, a, b,
                                      C.c_uint(zab_stride), _p(w[0]), _p(conv), _p(w[1]),
                                      _p(w[2]), _p(w[3]), _p(state), _p(out), C.c_float(eps),
                                      _p(hs), C.c_uint(hs.shape[0]), C.c_int(threads))
    return out


def deltanet_prepare(n: int, qkv, a, b, conv_w, conv, ssm_a, dt_bias):
    """Conv + SiLU + norms of the chunked form: returns q, k, v, beta, log_a (float64)."""
    qkv = _f32(qkv); a = _f32(a); b = _f32(b)
    q = np.zeros((n, 16, 128)); k = np.zeros((n, 16, 128)); v = np.zeros((n, 32, 128))
    beta = np.zeros((n, 32)); log_a = np.zeros((n, 32))
    w = [_f32(x) for x in (conv_w, ssm_a, dt_bias)]
    _load().oracle_deltanet_prepare(C.c_uint(n), _p(qkv), _p(a), _p(b), _p(w[0]), _p(conv),
                                    _p(w[1]), _p(w[2]), _p(q), _p(k), _p(v), _p(beta), _p(log_a))
    return q, k, v, beta, log_a


def deltanet_chunk(n: int, q, k, v, beta, log_a, z, norm_w, state, eps: float, threads: int = 0):
    """Chunked delta rule from prepared inputs (float64); state updated in place; returns out."""
    arrs = [np.ascontiguousarray(x, dtype=np.float64) for x in (q, k, v, beta, log_a)]
    z = _f32(z); norm_w = _f32(norm_w)
    out = np.zeros((n, 4096))
    _load().oracle_deltanet_chunk(C.c_uint(n), *[_p(x) for x in arrs], _p(z), _p(norm_w),
                                  _p(state), _p(out), C.c_float(eps), C.c_int(threads))
    return out
