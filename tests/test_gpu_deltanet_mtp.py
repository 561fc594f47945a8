"""Speculative verification with commit / rollback of a variable number of accepted tokens (the
reference's planned multi-token-prediction path, docs/decisions/ADR_002-build-scope-numerics-ops.md
D8), through the C ABI on the B200:
  * miso_deltanet_seq_ckpt gives the outputs of miso_deltanet_seq bit for bit, leaves the layer's
    state and conv history untouched, and its checkpoint after token t equals, bit for bit, what
    miso_deltanet_seq leaves after the first t + 1 tokens;
  * miso_deltanet_commit(k) then makes the layer exactly the layer that saw only the k accepted
    tokens (k = 0: the one that saw none), so decoding continues as if the rejected drafts never
    existed — checked against the oracle too;
  * the KV side: rolling the cache length back and appending the next token gives the decode
    output of a cache that never held the rejected drafts, bit for bit."""
import ctypes as C

import numpy as np
import pytest
import torch

from miso_b200 import _capi as capi
from miso_b200 import attention as A
from miso_b200 import deltanet as DN
import oracle

from test_gpu_deltanet import DEV, T, chunk_test_inputs, ptr, rel, run_seq

pytestmark = pytest.mark.gpu


def run_ckpt(x, n):
    d = {k: T(x[k]) for k in ("qkv", "zab", "conv_w", "ssm_a", "dt", "norm_w")}
    st, ci = T(x["state"]), T(x["conv_in"])
    co = torch.full_like(ci, 7.0)
    out = torch.empty((n, 4096), device=DEV)
    sck = torch.empty((n, 32, 128, 128), device=DEV)
    cck = torch.empty((n, 8192, 3), device=DEV)
    zb = ptr(d["zab"])
    p = capi.DeltaNetSeqParams(ptr(d["qkv"]), zb, zb + 4096 * 4, zb + 4128 * 4, ptr(d["conv_w"]),
                               ptr(ci), ptr(co), ptr(d["ssm_a"]), ptr(d["dt"]), ptr(d["norm_w"]),
                               ptr(st), ptr(out), n, 1e-6, 4160, 8192)
    capi.check("ckpt", capi.load().miso_deltanet_seq_ckpt(C.byref(p), ptr(sck), ptr(cck), None))
    torch.cuda.synchronize()
    return dict(out=out, st=st, ci=ci, co=co, sck=sck, cck=cck)


def bits(a):
    return np.asarray(a).view(np.uint32)


@pytest.mark.parametrize("n", [1, 2, 4])
def test_checkpoints_equal_shorter_sequences_bitwise(n):
    x = chunk_test_inputs(n)
    r = run_ckpt(x, n)
    out_full, _, _ = run_seq(x)
    assert np.array_equal(bits(r["out"].cpu().numpy()), bits(out_full))
    assert np.array_equal(bits(r["st"].cpu().numpy()), bits(x["state"]))    # untouched
    assert torch.all(r["co"] == 7.0)                                          # untouched
    for t in range(n):
        xt = dict(x, n=t + 1, qkv=x["qkv"][:t + 1], zab=x["zab"][:t + 1])
        _, st_t, co_t = run_seq(xt)
        assert np.array_equal(bits(r["sck"][t].cpu().numpy()), bits(st_t))
        assert np.array_equal(bits(r["cck"][t].cpu().numpy()), bits(co_t))


@pytest.mark.parametrize("k", [0, 1, 2, 3])
def test_commit_then_continue_equals_never_seeing_the_rejected_drafts(k):
    n = 3  # draft tokens verified; k accepted, then one more real token
    x = chunk_test_inputs(n + 1)
    st = DN.DeltaNetState(device=DEV)
    st.s.copy_(T(x["state"]))
    st.conv[0].copy_(T(x["conv_in"]))
    ck = DN.DraftCheckpoints(4, device=DEV)
    w = {k_: T(x[k_]) for k_ in ("conv_w", "ssm_a", "dt", "norm_w")}
    proj = torch.zeros((n + 1, DN.PROJ), device=DEV)
    proj[:, :8192] = T(x["qkv"])
    proj[:, 8192:8192 + 4160] = T(x["zab"])
    out = torch.empty((n, 4096), device=DEV)
    DN.deltanet_verify_core(st, ck, proj, n, w["conv_w"], w["ssm_a"], w["dt"], w["norm_w"], out,
                            1e-6)
    DN.deltanet_commit(st, ck, k)
    # The real next token is the last row of x (position k in the accepted stream).
    nxt = torch.empty((1, 4096), device=DEV)
    DN.deltanet_prefill_core(st, proj[n:].contiguous(), 1, w["conv_w"], w["ssm_a"], w["dt"],
                             w["norm_w"], nxt, 1e-6)
    torch.cuda.synchronize()
    # The same layer fed only the k accepted tokens and then the next one.
    idx = list(range(k)) + [n]
    ref = dict(x, n=k + 1, qkv=x["qkv"][idx], zab=x["zab"][idx])
    out_ref, st_ref, co_ref = run_seq(ref)
    assert np.array_equal(bits(nxt.cpu().numpy()), bits(out_ref[k:k + 1]))
    assert np.array_equal(bits(st.s.cpu().numpy()), bits(st_ref))
    assert np.array_equal(bits(st.conv[st.parity].cpu().numpy()), bits(co_ref))
    # And against the fp64 oracle of the same token stream.
    conv64 = x["conv_in"].astype(np.float64).copy()
    s64 = x["state"].astype(np.float64).copy()
    o64 = oracle.deltanet_seq(k + 1, ref["qkv"], 8192, ref["zab"], 4160, x["conv_w"], conv64,
                              x["ssm_a"], x["dt"], x["norm_w"], s64, 1e-6)
    assert rel(nxt.cpu().numpy()[0], o64[k]) < 1e-5
    assert rel(st.s.cpu().numpy(), s64) < 1e-5


def test_kv_rollback_equals_a_cache_without_the_rejected_drafts():
    rng = np.random.RandomState(5)
    B, drafts, keep = 2, 3, 1
    lens0 = np.array([37, 300], np.int32)

    def fresh():
        pool = A.KvPool(batch=B, capacity=400, device=DEV)
        g = torch.Generator(device=DEV)
        g.manual_seed(3)
        pool.k.copy_(torch.randn(pool.k.shape, generator=g, device=DEV).half())
        pool.v.copy_(torch.randn(pool.v.shape, generator=g, device=DEV).half())
        pool.lens.copy_(T(lens0))
        return pool

    rows = [rng.standard_normal((B, 9216)).astype(np.float32) for _ in range(drafts + 1)]
    qn = T((1 + 0.1 * rng.standard_normal(256)).astype(np.float32))
    kn = T((1 + 0.1 * rng.standard_normal(256)).astype(np.float32))
    inv = T(A.rope_inv_freq())
    q = torch.empty((B, 16, 256), device=DEV)
    core = torch.empty((B, 16, 256), device=DEV)
    scratch = A.decode_scratch(B, device=DEV)

    def append_and_decode(pool, row):
        r = T(row)
        base = ptr(r)
        p = capi.AttnPrepBatchedParams(base, base + 8192 * 4, base + 8704 * 4, ptr(qn), ptr(kn),
                                       ptr(inv), ptr(pool.k), ptr(pool.v), ptr(pool.kv_row),
                                       ptr(pool.lens), ptr(q), B, 9216, 1e-6)
        capi.check("prep", capi.load().miso_attn_prep_batched(C.byref(p), None))
        A.decode_batched(pool, q, r, core, scratch, qg_stride=9216)
        torch.cuda.synchronize()
        return core.cpu().numpy().copy()

    # Verify `drafts` tokens, accept `keep`, roll the length back, then the next real token.
    pool = fresh()
    for i in range(drafts):
        append_and_decode(pool, rows[i])
    pool.lens.copy_(T(lens0 + keep))
    got = append_and_decode(pool, rows[drafts])
    # A cache that only ever saw the accepted tokens.
    ref_pool = fresh()
    for i in range(keep):
        append_and_decode(ref_pool, rows[i])
    want = append_and_decode(ref_pool, rows[drafts])
    assert np.array_equal(bits(got), bits(want))
