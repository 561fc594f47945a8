"""A synthetic model file for the reference engine's model-level tests — test data only.

Writes a GGUF with the architecture, tensor names, types and shapes of the reference's model
(qwen35moe: hidden 2048, 256 experts + a shared expert, Gated DeltaNet layers with a full
attention layer every 4th, as listed in the reference's tests/fixtures/ornith-q4km-tensors.tsv)
but with random weights, 4 layers and a small vocabulary, plus the per-layer tensors of layers 5
(a DeltaNet layer with Q4_K projections) and 11 (an attention layer with Q4_K q / k / v) that the
reference's tests/test_fused_gemv.hip loads on their own. A second file holds a prompt
(golden.token_ids, golden.continuation_ids) for tests/test_prefill.hip. The model-level tests
that compare against the real model's golden outputs cannot use it; the ones that compare the
engine against itself (prefill vs decode, fused vs separate GEMVs, staged vs plain uploads) can.

Weight scales keep every projection's output near unit variance for unit-variance inputs, so the
forward pass stays in range through the layers.
"""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import quant as Q  # noqa: E402

ARCH = "qwen35moe"
HIDDEN, EXPERTS, FF = 2048, 256, 512
Q4K, Q6K, F32 = 12, 14, 0


def _blocks(rng, n, size):
    return np.frombuffer(rng.bytes(n * size), np.uint8).reshape(n, size).copy()


def _q4k(rng, rows, k):
    """Q4_K rows with weights of standard deviation ~ 1 / sqrt(k) and mean ~ 0: with sc, m
    uniform on 0..63 and q on 0..15, w = d sc q - dmin m has standard deviation ~ 257 d when
    dmin = 7.5 d."""
    nb = rows * k // 256
    b = _blocks(rng, nb, Q.Q4K_BYTES)
    d = 1.0 / (257.0 * np.sqrt(k)) * rng.uniform(0.9, 1.1, nb)
    b[:, 0:2] = d.astype(np.float16).view(np.uint8).reshape(nb, 2)
    b[:, 2:4] = (7.5 * d).astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(rows, -1)


def _q6k(rng, rows, k):
    """Q6_K rows with weights of standard deviation ~ 1 / sqrt(k): int8 scales and 6-bit codes
    uniform give w = d sc (q - 32) a standard deviation of ~ 1370 d."""
    nb = rows * k // 256
    b = _blocks(rng, nb, Q.Q6K_BYTES)
    d = 1.0 / (1370.0 * np.sqrt(k)) * rng.uniform(0.9, 1.1, nb)
    b[:, 208:210] = d.astype(np.float16).view(np.uint8).reshape(nb, 2)
    return b.reshape(rows, -1)


def _bf16_exact(a):
    return (np.asarray(a, np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)


def tensors(rng, vocab: int, layers: int = 4, experts: int = EXPERTS, extra: bool = True,
            with_moe: bool = True):
    """(name, numpy shape, GGML type, data) for every tensor; quantised data as raw bytes.
    with_moe=False leaves out the MoE blocks (enough for loading single mixer layers)."""
    out = []

    def q(name, rows, k, t, lead=()):
        n = int(np.prod(lead)) * rows if lead else rows
        raw = _q4k(rng, n, k) if t == Q4K else _q6k(rng, n, k)
        out.append((name, tuple(lead) + (rows, k), t, raw.reshape(tuple(lead) + (rows, -1))))

    def f(name, a):
        out.append((name, a.shape, F32, np.ascontiguousarray(a, np.float32)))

    q("token_embd.weight", vocab, HIDDEN, Q4K)
    f("output_norm.weight", 1.0 + 0.1 * rng.standard_normal(HIDDEN))
    q("output.weight", vocab, HIDDEN, Q6K)

    def deltanet(i, qkv_t):
        p = f"blk.{i}."
        f(p + "attn_norm.weight", 1.0 + 0.1 * rng.standard_normal(HIDDEN))
        q(p + "attn_qkv.weight", 8192, HIDDEN, qkv_t)
        q(p + "attn_gate.weight", 4096, HIDDEN, Q4K)
        q(p + "ssm_alpha.weight", 32, HIDDEN, Q4K)
        q(p + "ssm_beta.weight", 32, HIDDEN, Q4K)
        q(p + "ssm_out.weight", HIDDEN, 4096, Q4K)
        f(p + "ssm_conv1d.weight", 0.5 * rng.standard_normal((8192, 4)))
        f(p + "ssm_a", -rng.uniform(0.5, 2.0, 32))
        f(p + "ssm_dt.bias", rng.uniform(-1.0, 1.0, 32))
        f(p + "ssm_norm.weight", 1.0 + 0.1 * rng.standard_normal(128))

    def attention(i, v_t):
        p = f"blk.{i}."
        f(p + "attn_norm.weight", 1.0 + 0.1 * rng.standard_normal(HIDDEN))
        q(p + "attn_q.weight", 8192, HIDDEN, Q4K)
        q(p + "attn_k.weight", 512, HIDDEN, Q4K)
        q(p + "attn_v.weight", 512, HIDDEN, v_t)
        q(p + "attn_output.weight", HIDDEN, 4096, Q4K)
        f(p + "attn_q_norm.weight", 1.0 + 0.1 * rng.standard_normal(256))
        f(p + "attn_k_norm.weight", 1.0 + 0.1 * rng.standard_normal(256))

    def moe(i):
        p = f"blk.{i}."
        f(p + "post_attention_norm.weight", 1.0 + 0.1 * rng.standard_normal(HIDDEN))
        f(p + "ffn_gate_inp.weight", _bf16_exact(0.05 * rng.standard_normal((experts, HIDDEN))))
        f(p + "ffn_gate_inp_shexp.weight", _bf16_exact(0.05 * rng.standard_normal(HIDDEN)))
        q(p + "ffn_gate_exps.weight", FF, HIDDEN, Q4K, lead=(experts,))
        q(p + "ffn_up_exps.weight", FF, HIDDEN, Q4K, lead=(experts,))
        q(p + "ffn_down_exps.weight", HIDDEN, FF, Q6K, lead=(experts,))
        q(p + "ffn_gate_shexp.weight", FF, HIDDEN, Q4K)
        q(p + "ffn_up_shexp.weight", FF, HIDDEN, Q4K)
        q(p + "ffn_down_shexp.weight", HIDDEN, FF, Q6K)

    for i in range(layers):
        if (i + 1) % 4 == 0:
            attention(i, Q6K)
        else:
            deltanet(i, Q6K)
        if with_moe:
            moe(i)
    if extra:
        deltanet(5, Q4K)
        attention(11, Q4K)
    return out


def write(model_path: str, golden_dir: str, vocab: int = 8192, seed: int = 0,
          experts: int = EXPERTS, n_prompt: int = 14, n_cont: int = 3,
          with_moe: bool = True) -> None:
    import gguf

    rng = np.random.RandomState(seed)
    w = gguf.GGUFWriter(model_path, ARCH)
    w.add_uint32(f"{ARCH}.block_count", 4)
    w.add_uint32(f"{ARCH}.nextn_predict_layers", 0)
    w.add_uint32(f"{ARCH}.full_attention_interval", 4)
    w.add_float32(f"{ARCH}.rope.freq_base", 10000000.0)
    w.add_uint32(f"{ARCH}.rope.dimension_count", 64)
    w.add_float32(f"{ARCH}.attention.layer_norm_rms_epsilon", 1e-6)
    for name, shape, t, data in tensors(rng, vocab, experts=experts, with_moe=with_moe):
        if t == F32:
            w.add_tensor(name, data)
        else:
            w.add_tensor(name, data, raw_dtype=gguf.GGMLQuantizationType(t))  # byte shape
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()

    os.makedirs(golden_dir, exist_ok=True)
    g = gguf.GGUFWriter(os.path.join(golden_dir, "ornith-layers.gguf"), ARCH)
    ids = rng.randint(0, vocab, n_prompt + n_cont)
    g.add_array("golden.token_ids", [int(v) for v in ids[:n_prompt]])
    g.add_array("golden.continuation_ids", [int(v) for v in ids[n_prompt:]])
    g.write_header_to_file()
    g.write_kv_data_to_file()
    g.write_tensors_to_file()
    g.close()


if __name__ == "__main__":
    # synthetic_model.py <model.gguf> <golden dir> [--mixers-only]
    write(sys.argv[1], sys.argv[2], with_moe="--mixers-only" not in sys.argv[3:])
