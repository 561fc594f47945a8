"""CPU oracle of the quantised weight formats and the projection / MoE arithmetic around the
attention path — TEST INFRASTRUCTURE ONLY (tests/ use it as the checker of the drop-in GEMV,
GEMM, embedding, norm, argmax and MoE kernels; the product never calls it).

Restated in numpy from the GGUF block formats as the reference reads them:
  * Q4_K (src/dequant.cpp, 144-byte blocks of 256: d, dmin, 12 packed 6-bit scale / min bytes,
    128 nibble bytes) and Q6_K (210-byte blocks: ql[128], qh[64], int8 scales[16], d) —
    dequantised with the reference's (and gguf-py's) FP32 rounding: Q4_K d*sc*q and dmin*m are
    exact and one subtraction rounds; Q6_K rounds (d*sc) * (q - 32) once.
  * the engine layouts of src/repack.cpp:9-78: Q4_K r1 (bytes 4..15 as four 24-bit scale / min
    fields) and Q6_K r1 (each row stored as ql / qh / scales / d sections, padded to 16 bytes).
  * the activation formats of kernels/q4k_gemv.hpp:18-21 (FP16 rounding; per-32 absmax INT8) and
    the MoE routing of kernels/moe_decode.hpp:3-11 (top 8 of 256 logits, ties to the lower index,
    softmax renormalised over the 8; the shared expert gated by sigmoid(logit 256)).
Pinned by tests/test_oracle_quant.py against the reference's fixture dequantisations
(tests/fixtures/tiny.q4_k.f32, tiny.q6_k.f32) and its compiled repack / dequant code.
"""
from __future__ import annotations

import numpy as np

Q4K_BYTES = 144
Q6K_BYTES = 210


def q4k_scale_min(blocks: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """6-bit (scale, min) of the 8 sub-blocks of GGUF Q4_K blocks [nb][144] -> two [nb][8]."""
    q = blocks[:, 4:16].astype(np.uint32)
    sc = np.empty((blocks.shape[0], 8), np.uint32)
    mn = np.empty_like(sc)
    for j in range(4):
        sc[:, j] = q[:, j] & 63
        mn[:, j] = q[:, j + 4] & 63
    for j in range(4, 8):
        sc[:, j] = (q[:, j + 4] & 0xF) | ((q[:, j - 4] >> 6) << 4)
        mn[:, j] = (q[:, j + 4] >> 4) | ((q[:, j] >> 6) << 4)
    return sc, mn


def q4k_nibbles(blocks: np.ndarray) -> np.ndarray:
    """The 256 4-bit codes of each block in element order: [nb][256]."""
    qs = blocks[:, 16:144].reshape(-1, 4, 32)  # nibble group g = bytes 32g..32g+31
    out = np.empty((blocks.shape[0], 4, 2, 32), np.uint8)
    out[:, :, 0, :] = qs & 15   # sub-block 2g: elements 64g + l
    out[:, :, 1, :] = qs >> 4   # sub-block 2g + 1: elements 64g + 32 + l
    return out.reshape(-1, 256)


def q4k_dequant(raw: np.ndarray) -> np.ndarray:
    """GGUF Q4_K bytes (any shape whose last axis is a multiple of 144) -> float32 values."""
    raw = np.ascontiguousarray(raw, np.uint8)
    blocks = raw.reshape(-1, Q4K_BYTES)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = blocks[:, 2:4].copy().view(np.float16).astype(np.float32)
    sc, mn = q4k_scale_min(blocks)
    q = q4k_nibbles(blocks).reshape(-1, 8, 32).astype(np.float32)
    a = (d * sc.astype(np.float32))[:, :, None] * q          # exact in FP32
    b = (dmin * mn.astype(np.float32))[:, :, None]            # exact in FP32
    y = (a - b).astype(np.float32)                              # the one rounding
    return y.reshape(raw.shape[:-1] + (raw.shape[-1] // Q4K_BYTES * 256,))


def q6k_codes(blocks: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """(6-bit codes [nb][256] in element order, int8 scale of each element's 16-group [nb][256])."""
    ql = blocks[:, 0:128].astype(np.uint32)
    qh = blocks[:, 128:192].astype(np.uint32)
    scales = blocks[:, 192:208].copy().view(np.int8).astype(np.int32)
    q = np.empty((blocks.shape[0], 2, 4, 32), np.uint32)
    s = np.empty((blocks.shape[0], 2, 4, 32), np.int32)
    for n in range(2):
        l = np.arange(32)
        lq, hq = ql[:, 64 * n:64 * n + 64], qh[:, 32 * n:32 * n + 32]
        q[:, n, 0] = (lq[:, :32] & 15) | ((hq >> 0) & 3) << 4
        q[:, n, 1] = (lq[:, 32:] & 15) | ((hq >> 2) & 3) << 4
        q[:, n, 2] = (lq[:, :32] >> 4) | ((hq >> 4) & 3) << 4
        q[:, n, 3] = (lq[:, 32:] >> 4) | ((hq >> 6) & 3) << 4
        for u in range(4):
            s[:, n, u] = scales[:, 8 * n + l // 16 + 2 * u]
    return q.reshape(-1, 256), s.reshape(-1, 256)


def q6k_dequant(raw: np.ndarray) -> np.ndarray:
    """GGUF Q6_K bytes (last axis a multiple of 210) -> float32 values."""
    raw = np.ascontiguousarray(raw, np.uint8)
    blocks = raw.reshape(-1, Q6K_BYTES)
    d = blocks[:, 208:210].copy().view(np.float16).astype(np.float32)
    q, s = q6k_codes(blocks)
    ds = (d * s.astype(np.float32)).astype(np.float32)          # exact
    y = (ds * (q.astype(np.float32) - np.float32(32))).astype(np.float32)
    return y.reshape(raw.shape[:-1] + (raw.shape[-1] // Q6K_BYTES * 256,))


def q4k_repack_r1(raw: np.ndarray) -> np.ndarray:
    """GGUF Q4_K bytes -> the engine's Q4_K r1 bytes (same size)."""
    raw = np.ascontiguousarray(raw, np.uint8)
    out = raw.copy().reshape(-1, Q4K_BYTES)
    sc, mn = q4k_scale_min(raw.reshape(-1, Q4K_BYTES))
    for g in range(4):
        v = sc[:, 2 * g] | mn[:, 2 * g] << 6 | sc[:, 2 * g + 1] << 12 | mn[:, 2 * g + 1] << 18
        for b in range(3):
            out[:, 4 + 3 * g + b] = (v >> (8 * b)) & 0xFF
    return out.reshape(raw.shape)


def q6k_r1_row_bytes(k: int) -> int:
    return (k // 256 * Q6K_BYTES + 15) // 16 * 16


def q6k_repack_r1(raw: np.ndarray, k: int) -> np.ndarray:
    """GGUF Q6_K rows of k elements ([rows][k / 256 * 210]) -> Q6_K r1 rows [rows][row_bytes]."""
    nb = k // 256
    blocks = np.ascontiguousarray(raw, np.uint8).reshape(-1, nb, Q6K_BYTES)
    rows = blocks.shape[0]
    out = np.zeros((rows, q6k_r1_row_bytes(k)), np.uint8)
    out[:, 0:nb * 128] = blocks[:, :, 0:128].reshape(rows, -1)
    out[:, nb * 128:nb * 192] = blocks[:, :, 128:192].reshape(rows, -1)
    out[:, nb * 192:nb * 208] = blocks[:, :, 192:208].reshape(rows, -1)
    out[:, nb * 208:nb * 210] = blocks[:, :, 208:210].reshape(rows, -1)
    return out


def q4k_r1_to_gguf(raw: np.ndarray) -> np.ndarray:
    """Q4_K r1 bytes -> GGUF Q4_K bytes: the 24-bit fields back into the 12-byte 6-bit packing
    (j < 4: scale / min in the low 6 bits of bytes j / j + 4; j >= 4: low nibbles in byte j + 4,
    top 2 bits in the high bits of bytes j - 4 / j)."""
    raw = np.ascontiguousarray(raw, np.uint8)
    b = raw.copy().reshape(-1, Q4K_BYTES)
    f = b[:, 4:16].astype(np.uint32).reshape(-1, 4, 3)
    v = f[:, :, 0] | f[:, :, 1] << 8 | f[:, :, 2] << 16
    sc = np.empty((b.shape[0], 8), np.uint32)
    mn = np.empty_like(sc)
    sc[:, 0::2], mn[:, 0::2] = v & 63, (v >> 6) & 63
    sc[:, 1::2], mn[:, 1::2] = (v >> 12) & 63, (v >> 18) & 63
    q = np.zeros((b.shape[0], 12), np.uint32)
    for j in range(4):
        q[:, j] |= sc[:, j]
        q[:, j + 4] |= mn[:, j]
    for j in range(4, 8):
        q[:, j + 4] = (sc[:, j] & 0xF) | (mn[:, j] & 0xF) << 4
        q[:, j - 4] |= (sc[:, j] >> 4) << 6
        q[:, j] |= (mn[:, j] >> 4) << 6
    b[:, 4:16] = q.astype(np.uint8)
    return b.reshape(raw.shape)


def q6k_r1_to_gguf(rows: np.ndarray, k: int) -> np.ndarray:
    """Q6_K r1 rows [rows][row_bytes] -> GGUF Q6_K rows [rows][k / 256 * 210]."""
    nb = k // 256
    rows = np.ascontiguousarray(rows, np.uint8).reshape(-1, q6k_r1_row_bytes(k))
    out = np.empty((rows.shape[0], nb, Q6K_BYTES), np.uint8)
    out[:, :, 0:128] = rows[:, 0:nb * 128].reshape(-1, nb, 128)
    out[:, :, 128:192] = rows[:, nb * 128:nb * 192].reshape(-1, nb, 64)
    out[:, :, 192:208] = rows[:, nb * 192:nb * 208].reshape(-1, nb, 16)
    out[:, :, 208:210] = rows[:, nb * 208:nb * 210].reshape(-1, nb, 2)
    return out.reshape(rows.shape[0], -1)


def random_q4k(rng: np.random.RandomState, rows: int, k: int, d_scale: float = 2e-3) -> np.ndarray:
    """Random GGUF Q4_K rows [rows][k / 256 * 144]: random codes and 6-bit scales / mins, d and
    dmin drawn around d_scale (positive FP16)."""
    nb = rows * k // 256
    b = rng.randint(0, 256, size=(nb, Q4K_BYTES)).astype(np.uint8)
    b[:, 0:2] = (d_scale * rng.uniform(0.5, 1.5, nb)).astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 2:4] = (d_scale * rng.uniform(0.5, 1.5, nb)).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(rows, -1)


def random_q6k(rng: np.random.RandomState, rows: int, k: int, d_scale: float = 1e-3) -> np.ndarray:
    """Random GGUF Q6_K rows [rows][k / 256 * 210] (random codes and int8 scales)."""
    nb = rows * k // 256
    b = rng.randint(0, 256, size=(nb, Q6K_BYTES)).astype(np.uint8)
    b[:, 208:210] = (d_scale * rng.uniform(0.5, 1.5, nb)).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(rows, -1)


def act_fp16(x: np.ndarray) -> np.ndarray:
    """The FP16 activation format: x rounded to binary16 (nearest even), as float64."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float64)


def act_int8(x: np.ndarray) -> np.ndarray:
    """The INT8 activation format: per 32 consecutive values amax = max |x|, q = rint((x * 127) /
    amax), x' = q * (amax / 127) (0 where amax = 0), each operation in FP32 as the kernels round
    it; returned as float64."""
    x = np.asarray(x, np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1, keepdims=True)
    safe = np.where(amax > 0, amax, np.float32(1))
    q = np.rint((x * np.float32(127)) / safe).astype(np.float32)
    xq = np.where(amax > 0, q * (safe / np.float32(127)), np.float32(0)).astype(np.float32)
    return xq.reshape(-1).astype(np.float64)


def gemv(w: np.ndarray, x_act: np.ndarray) -> np.ndarray:
    """y = W x in float64 for dequantised W [n][k] and already-converted activations [k]."""
    return w.astype(np.float64) @ x_act


def add_rmsnorm(res: np.ndarray, delta, weight: np.ndarray, eps: float):
    """Residual add + RMSNorm (kernels/rmsnorm.hpp:3-5): returns (new residual, out), float64."""
    h = res.astype(np.float64) + (0.0 if delta is None else delta.astype(np.float64))
    r = 1.0 / np.sqrt((h * h).mean(axis=-1, keepdims=True) + eps)
    return h, h * r * weight.astype(np.float64)


def bf16_to_f64(w: np.ndarray) -> np.ndarray:
    return (w.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def moe_topk(logits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Top 8 of logits[:256] (value descending, lower index first among equal values) and their
    softmax weights renormalised over the 8."""
    l = np.asarray(logits[:256], np.float64)
    ids = np.array(sorted(range(256), key=lambda i: (-l[i], i))[:8])
    e = np.exp(l[ids] - l[ids[0]])
    return ids, e / e.sum()


def silu(x):
    return x / (1.0 + np.exp(-x))


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))
