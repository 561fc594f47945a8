"""The CPU oracle pinned against the reference's known answers and against golden outputs of the
model's own reference code (transformers qwen3_5_moe + torch float64 attention), on CPU.

These tests make the oracle trustworthy before it is used to judge the CUDA kernels."""
import numpy as np
import pytest

import inputs as I
import oracle

GOLD = np.load(I.__file__.replace("inputs.py", "golden.npz"))


def rel_l2(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    den = np.sqrt(np.sum(ref * ref))
    return float(np.sqrt(np.sum((got - ref) ** 2)) / den) if den > 0 else float(np.abs(got).max())


def test_half_to_double_is_exact_for_every_finite_pattern():
    bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
    ref = bits.view(np.float16).astype(np.float64)
    finite = np.isfinite(ref)
    got = np.array([oracle.half_to_double(int(b)) for b in bits[finite][::37]])
    assert np.array_equal(got, ref[finite][::37])
    assert np.isinf(oracle.half_to_double(0x7C00)) and np.isnan(oracle.half_to_double(0x7E00))


# Known answers of tests/test_attn_splitk.hip:285-290.
KNOWN_SPLITS = [(3872, 60, 21), (33, 60, 2), (4096, 60, 22), (16384, 60, 57), (288, 60, 9)]


@pytest.mark.parametrize("length,max_splits,want", KNOWN_SPLITS)
def test_n_splits_known_answers(length, max_splits, want):
    assert oracle.attn_n_splits(length, max_splits) == want


def test_prep_matches_transformers_rmsnorm_and_rope():
    x = I.prep_inputs()
    q, k, v = oracle.attn_prep(x["qg"], x["k"], x["v"], x["q_norm"], x["k_norm"], x["inv_freq"],
                               x["pos"], I.EPS)
    assert rel_l2(q, GOLD["prep_q"]) < 2e-6
    assert rel_l2(k, GOLD["prep_k"]) < 2e-6
    assert np.array_equal(v, x["v"].astype(np.float64))


def test_decode_matches_float64_sdpa():
    x = I.decode_inputs()
    kv_row = np.array([[0, x["max_ctx"]]], np.int64)
    out = oracle.attn_decode(x["q"], x["qg"], 16 * 512, x["k"].view(np.uint16).reshape(-1, 256),
                             x["v"].view(np.uint16).reshape(-1, 256), kv_row,
                             np.array([x["len"]], np.int32))
    assert rel_l2(out[0], GOLD["decode_out"]) < 1e-6


def test_prefill_matches_float64_sdpa_with_causal_offset():
    x = I.prefill_inputs()
    out = oracle.attn_prefill(x["n"], x["pos0"], x["q"], x["qg"], 16 * 512,
                              x["k"].view(np.uint16), x["v"].view(np.uint16), x["max_ctx"])
    assert rel_l2(out, GOLD["prefill_out"]) < 1e-6
    rows = np.array([0, 7, x["n"] - 1], np.uint32)
    sub = oracle.attn_prefill(x["n"], x["pos0"], x["q"], x["qg"], 16 * 512,
                              x["k"].view(np.uint16), x["v"].view(np.uint16), x["max_ctx"],
                              rows=rows)
    assert np.array_equal(sub, out[rows])


def test_combine_of_split_partials_equals_unsplit_decode():
    """Split the keys by hand, form (m, l, o) partials in double, merge with the oracle combine."""
    x = I.decode_inputs(length=333, seed=3)
    L, ns = x["len"], 5
    kf = x["k"].astype(np.float64)
    vf = x["v"].astype(np.float64)
    per = -(-L // ns)
    pm = np.zeros((2, ns, 8), np.float32); pl = np.zeros_like(pm)
    po = np.zeros((2, ns, 8, 256), np.float32)
    for kvh in range(2):
        for c in range(ns):
            j0, j1 = c * per, min(L, (c + 1) * per)
            for hl in range(8):
                s = kf[kvh, j0:j1] @ x["q"][kvh * 8 + hl].astype(np.float64) / 16.0
                m = s.max(); e = np.exp(s - m)
                pm[kvh, c, hl], pl[kvh, c, hl] = m, e.sum()
                po[kvh, c, hl] = e @ vf[kvh, j0:j1]
    core = oracle.attn_combine(pm, pl, po, x["qg"], ns)
    full = oracle.attn_decode(x["q"], x["qg"], 8192, x["k"].view(np.uint16).reshape(-1, 256),
                              x["v"].view(np.uint16).reshape(-1, 256),
                              np.array([[0, x["max_ctx"]]], np.int64), np.array([L], np.int32))
    assert rel_l2(core, full[0]) < 1e-6  # partials were rounded to fp32


def _dn_seq(x):
    conv = x["conv_in"].astype(np.float64).copy()
    state = x["state"].astype(np.float64).copy()
    zab = np.zeros((x["n"], 4160), np.float32)
    zab[:, :4096], zab[:, 4096:4128], zab[:, 4128:] = x["z"], x["a"], x["b"]
    out = oracle.deltanet_seq(x["n"], x["qkv"], 8192, zab, 4160, x["conv_w"], conv, x["ssm_a"],
                              x["dt_bias"], x["norm_w"], state, I.EPS)
    return out, state, conv


def test_deltanet_recurrence_matches_transformers():
    x = I.deltanet_inputs()
    out, state, conv = _dn_seq(x)
    out = out.reshape(x["n"], 32, 128)
    assert rel_l2(out[:, list(I.DN_HEADS)], GOLD["dn_out_rec"]) < 1e-5
    assert rel_l2(state[I.DN_STATE_HEAD], GOLD["dn_state_rec"]) < 1e-5
    assert np.array_equal(conv, x["qkv"][-3:].T.astype(np.float64))


def test_deltanet_steps_equal_sequence():
    x = I.deltanet_inputs(n=6, seed=5)
    out_seq, st_seq, conv_seq = _dn_seq(x)
    conv = x["conv_in"].astype(np.float64)[None].copy()
    state = x["state"].astype(np.float64)[None].copy()
    outs = []
    for t in range(x["n"]):
        outs.append(oracle.deltanet_step(x["qkv"][t][None], x["z"][t][None], x["a"][t][None],
                                         x["b"][t][None], x["conv_w"], conv, x["ssm_a"],
                                         x["dt_bias"], x["norm_w"], state, I.EPS)[0])
    assert np.allclose(np.stack(outs), out_seq, rtol=0, atol=1e-12)
    assert np.allclose(state[0], st_seq, rtol=0, atol=1e-12)
    assert np.array_equal(conv[0], conv_seq)


def test_deltanet_chunked_form_matches_transformers_and_recurrence():
    x = I.deltanet_inputs()
    n = x["n"]
    conv = x["conv_in"].astype(np.float64).copy()
    q, k, v, beta, log_a = oracle.deltanet_prepare(n, x["qkv"], x["a"], x["b"], x["conv_w"],
                                                   conv, x["ssm_a"], x["dt_bias"])
    state = x["state"].astype(np.float64).copy()
    out = oracle.deltanet_chunk(n, q, k, v, beta, log_a, x["z"], x["norm_w"], state, I.EPS)
    out = out.reshape(n, 32, 128)
    assert rel_l2(out[:, list(I.DN_HEADS)], GOLD["dn_out_chunk"]) < 1e-5
    assert rel_l2(state[I.DN_STATE_HEAD], GOLD["dn_state_chunk"]) < 1e-5
    out_rec, st_rec, _ = _dn_seq(x)
    assert rel_l2(out, out_rec.reshape(n, 32, 128)) < 1e-12
    assert rel_l2(state, st_rec) < 1e-12


def test_deltanet_state_is_affine_in_the_incoming_state():
    """The property a parallel-in-segments scheme builds on: over a segment, the state update is
    S_out(S_in) = A S_in + S_out(0) per head (A a k x k matrix that depends on q, k, beta and the
    decays only), and A itself is the segment's state update of S_in = I with the value inputs
    (and their conv history) set to zero. Checked on the fp64 oracle of the token recurrence."""
    n = 70
    rng = np.random.RandomState(31)
    qkv = (0.5 * rng.standard_normal((n, 8192))).astype(np.float32)
    zab = (0.5 * rng.standard_normal((n, 4160))).astype(np.float32)
    conv_w = (0.5 * rng.standard_normal((8192, 4))).astype(np.float32)
    ssm_a = (-0.2 * (np.arange(32) % 5 + 1)).astype(np.float32)
    dt = (0.05 * np.arange(32)).astype(np.float32)
    norm_w = np.ones(128, np.float32)
    conv0 = 0.5 * rng.standard_normal((8192, 3))
    s_in = 0.1 * rng.standard_normal((32, 128, 128))

    def run(x, conv, state):
        c, s = conv.copy(), state.copy()
        oracle.deltanet_seq(n, x, 8192, zab, 4160, conv_w, c, ssm_a, dt, norm_w, s, 1e-6)
        return s

    s_full = run(qkv, conv0, s_in)
    s_zero = run(qkv, conv0, np.zeros_like(s_in))
    x_nov = qkv.copy()
    x_nov[:, 4096:] = 0.0
    conv_nov = conv0.copy()
    conv_nov[4096:] = 0.0
    a = run(x_nov, conv_nov, np.broadcast_to(np.eye(128), (32, 128, 128)).copy())
    pred = np.einsum("hkm,hmv->hkv", a, s_in) + s_zero
    assert np.abs(pred - s_full).max() <= 1e-12 * max(1.0, np.abs(s_full).max())


def test_head_subset_recurrence_equals_the_full_one():
    """oracle.deltanet_seq_heads (used to check long sequences on a few heads) gives exactly the
    full recurrence's state slices and output columns of the listed heads."""
    rng = np.random.RandomState(21)
    n = 37
    qkv = rng.standard_normal((n, 8192)).astype(np.float32)
    zab = rng.standard_normal((n, 4160)).astype(np.float32)
    cw = (0.5 * rng.standard_normal((8192, 4))).astype(np.float32)
    conv = rng.standard_normal((8192, 3))
    sa, dt = -np.ones(32, np.float32), np.zeros(32, np.float32)
    nw = np.ones(128, np.float32)
    s_full = 0.1 * rng.standard_normal((32, 128, 128))
    s_sub = s_full.copy()
    out = oracle.deltanet_seq(n, qkv, 8192, zab, 4160, cw, conv.copy(), sa, dt, nw, s_full, 1e-6)
    heads = [1, 16, 31]
    sub = oracle.deltanet_seq_heads(n, qkv, 8192, zab, 4160, cw, conv, sa, dt, nw, s_sub, 1e-6,
                                    heads)
    for i, h in enumerate(heads):
        assert np.array_equal(s_sub[h], s_full[h])
        assert np.array_equal(sub[:, i], out[:, h * 128:(h + 1) * 128])
