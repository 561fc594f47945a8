"""GPU parity at the sizes bench.py measures, against the fp64 CPU oracle.

Each case builds the bench's own inputs (same generator, seed and order) and runs the same entry
points, then checks the outputs against the oracle with BASELINE's bars: relative L2 <= 1e-3 and
max abs <= 1e-2 for fp32-accumulated outputs, DeltaNet state relative L2 <= 1e-3, argmax of each
(token, head) output row equal to the oracle's wherever the oracle's top-2 gap clears the error
bound.

* Config 3: the 8192-token causal gated prefill (prep + tcgen05 attention), 512 sampled query
  rows including the last, all 16 heads; the prep's fp16 queries and K cache rows of 64 sampled
  tokens against the oracle prep.
* A context-parallel chunk: 8192 queries at pos0 = 122880 against 131072 keys (the last zig-zag
  chunk of the 8-GPU config-5 layout), 64 sampled rows including its first and last.
* Config 4a: the 8192-token DeltaNet chunked prefill against the fp64 token recurrence: every
  output, the final state and the conv history.
* Config 5 at one GPU: the hybrid block (the context-parallel classes at world size 1) over
  131072 tokens; 48 sampled attention rows including the last, and for each of the 3 DeltaNet
  layers 8 of the 32 V heads (both halves of the K-head mapping) over the whole sequence: their
  outputs and final states.

The oracle's attention costs ~2 ms per (row, head, 1k keys) on one core and its recurrence
~35 us per (head, token), hence the sampling (heads are independent in the recurrence).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from miso_b200 import _capi as capi
from miso_b200 import attention as A
import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
PROJ = 9216
DN_PROJ = 12352
EPS = 1e-6


def rel(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.sqrt(((got - ref) ** 2).sum() / (ref ** 2).sum()))


def rel_per_head(got, ref):
    got = np.asarray(got, np.float64).reshape(-1, 256)
    ref = np.asarray(ref, np.float64).reshape(-1, 256)
    num = np.sqrt(((got - ref) ** 2).sum(1))
    den = np.sqrt((ref ** 2).sum(1))
    return float(np.max(num / np.maximum(den, 1e-300)))


def check_attention_rows(got, ref):
    assert np.isfinite(got).all()
    r, m = rel_per_head(got, ref), float(np.abs(got - ref).max())
    print(f"rows {got.shape[0]}: per-head rel-L2 {r:.3e}, max abs {m:.3e}")
    assert r <= 1e-3
    assert m <= 1e-2
    # Argmax of each row must agree wherever the oracle's top-2 gap exceeds twice the largest
    # error seen (then no error can swap the two). At long contexts the rows are averages over
    # many keys and the gaps small, so the bound follows the measured error, not a constant.
    g, o = got.reshape(-1, 256), ref.reshape(-1, 256)
    srt = np.sort(o, axis=1)
    clear = (srt[:, -1] - srt[:, -2]) > 2 * m + 1e-7
    assert clear.sum() >= min(64, clear.size // 4)
    assert np.array_equal(g[clear].argmax(1), o[clear].argmax(1))


def status_clear():
    s = C.c_int(-1)
    assert capi.load().miso_device_status(1, C.byref(s)) == 0
    return s.value == 0


def f16_ulps(got_bits, ref64):
    ref = ref64.astype(np.float16).view(np.uint16).astype(np.int32)
    return np.abs(got_bits.astype(np.int32) - ref)


def test_config3_prefill_8192_sampled_rows():
    """bench.py's prefill leg: inputs, prep and the tcgen05 attention of BASELINE config 3."""
    n = 8192
    g = torch.Generator(device=DEV)
    g.manual_seed(99)
    proj = torch.randn((n, PROJ), generator=g, device=DEV).bfloat16().float()
    ones = torch.ones(256, device=DEV)
    inv = torch.from_numpy(A.rope_inv_freq()).to(DEV)
    kc = torch.empty((2, n, 256), dtype=torch.float16, device=DEV)
    vc = torch.empty_like(kc)
    q16 = torch.empty((n, 16, 256), dtype=torch.float16, device=DEV)
    core = torch.full((n, 16, 256), float("nan"), device=DEV)
    lib = capi.load()
    base = proj.data_ptr()
    tok0 = capi.AttnPrepParams(base, base + 8192 * 4, base + 8704 * 4, ones.data_ptr(),
                               ones.data_ptr(), inv.data_ptr(), kc.data_ptr(), vc.data_ptr(), 0,
                               0, n, EPS)
    bp = capi.AttnPrepBatchParams(tok0, n, PROJ)
    capi.check("prep_f16", lib.miso_attn_prep_batch_f16(C.byref(bp), q16.data_ptr(), None))
    tp = capi.AttnPrefillTcParams(q16.data_ptr(), base, kc.data_ptr(), vc.data_ptr(),
                                  core.data_ptr(), 0, n, n, PROJ)
    capi.check("prefill_tc", lib.miso_attn_prefill_tc(C.byref(tp), None))
    torch.cuda.synchronize()
    assert status_clear()

    rng = np.random.RandomState(3)
    rows = np.unique(np.concatenate([rng.choice(n - 1, 511, replace=False), [n - 1]]))
    p = proj.cpu().numpy()
    q = q16.cpu().numpy()
    kb = kc.cpu().numpy().view(np.uint16)
    vb = vc.cpu().numpy().view(np.uint16)
    # the prep of 64 sampled tokens: fp16 queries and K rows within one fp16 ulp, V exact
    one = np.ones(256, np.float32)
    for t in rows[::8]:
        rq, rk, rv = oracle.attn_prep(p[t, :8192].reshape(16, 512),
                                      p[t, 8192:8704].reshape(2, 256), p[t, 8704:].reshape(2, 256),
                                      one, one, A.rope_inv_freq(), int(t), EPS)
        assert f16_ulps(q[t].view(np.uint16), rq).max() <= 1
        assert f16_ulps(kb[:, t], rk).max() <= 1
        assert np.array_equal(vb[:, t], rv.astype(np.float16).view(np.uint16))
    ref = oracle.attn_prefill(n, 0, q.astype(np.float32), p, PROJ, kb, vb, n, rows=rows)
    check_attention_rows(core.cpu().numpy()[rows], ref)


def test_prefill_at_a_context_parallel_chunk_position():
    """The last zig-zag chunk of the 8-GPU config-5 layout: queries [122880, 131072) against all
    131072 keys of the cache."""
    t, n = 131072, 8192
    pos0 = t - n
    g = torch.Generator(device=DEV)
    g.manual_seed(11)
    kc = torch.randn((2, t, 256), generator=g, device=DEV).half()
    vc = torch.randn((2, t, 256), generator=g, device=DEV).half()
    q16 = torch.randn((n, 16, 256), generator=g, device=DEV).half()
    qg = torch.randn((n, 16, 512), generator=g, device=DEV)
    core = torch.full((n, 16, 256), float("nan"), device=DEV)
    tp = capi.AttnPrefillTcParams(q16.data_ptr(), qg.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                  core.data_ptr(), pos0, n, t, 16 * 512)
    capi.check("prefill_tc", capi.load().miso_attn_prefill_tc(C.byref(tp), None))
    torch.cuda.synchronize()
    assert status_clear()
    rng = np.random.RandomState(4)
    rows = np.unique(np.concatenate([rng.choice(n, 62, replace=False), [0, n - 1]]))
    ref = oracle.attn_prefill(n, pos0, q16.cpu().numpy().astype(np.float32), qg.cpu().numpy(),
                              16 * 512, kc.cpu().numpy().view(np.uint16),
                              vc.cpu().numpy().view(np.uint16), t, rows=rows)
    check_attention_rows(core.cpu().numpy()[rows], ref)


def test_config4a_deltanet_prefill_8192_matches_fp64_recurrence():
    """bench.py's DeltaNet prefill leg (BASELINE config 4a), compared in full with the oracle."""
    n = 8192
    g = torch.Generator(device=DEV)
    g.manual_seed(1)
    proj = torch.randn((n, DN_PROJ), generator=g, device=DEV).bfloat16().float()
    conv_w = (0.5 * torch.randn((8192, 4), generator=g, device=DEV)).bfloat16().float()
    ssm_a = -torch.ones(32, device=DEV)
    dt = torch.zeros(32, device=DEV)
    norm_w = torch.ones(128, device=DEV)
    conv_in = torch.zeros((8192, 3), device=DEV)
    conv_out = torch.full((8192, 3), float("nan"), device=DEV)
    state = torch.zeros((32, 128, 128), device=DEV)
    out = torch.full((n, 4096), float("nan"), device=DEV)
    lib = capi.load()
    sb = lib.miso_deltanet_prefill_tc_scratch_bytes(n)
    scratch = torch.empty(sb, dtype=torch.uint8, device=DEV)
    base = proj.data_ptr()
    z = base + 8192 * 4
    p = capi.DeltaNetSeqParams(base, z, z + 4096 * 4, z + 4128 * 4, conv_w.data_ptr(),
                               conv_in.data_ptr(), conv_out.data_ptr(), ssm_a.data_ptr(),
                               dt.data_ptr(), norm_w.data_ptr(), state.data_ptr(), out.data_ptr(),
                               n, EPS, DN_PROJ, DN_PROJ)
    capi.check("dn_prefill_tc", lib.miso_deltanet_prefill_tc(C.byref(p), scratch.data_ptr(), sb,
                                                             None))
    torch.cuda.synchronize()
    assert status_clear()
    pr = proj.cpu().numpy()
    conv = np.zeros((8192, 3))
    s64 = np.zeros((32, 128, 128))
    ref = oracle.deltanet_seq(n, pr, DN_PROJ, pr, DN_PROJ, conv_w.cpu().numpy(), conv,
                              ssm_a.cpu().numpy(), dt.cpu().numpy(), norm_w.cpu().numpy(), s64,
                              EPS, z_off=8192, a_off=12288, b_off=12320)
    got = out.cpu().numpy()
    st = state.cpu().numpy()
    r_out, m_out, r_st = rel(got, ref), float(np.abs(got - ref).max()), rel(st, s64)
    print(f"config 4a: out rel-L2 {r_out:.3e} max abs {m_out:.3e}, state rel-L2 {r_st:.3e}")
    assert np.isfinite(got).all()
    assert r_out <= 1e-3 and m_out <= 1e-2 and r_st <= 1e-3
    assert np.array_equal(conv_out.cpu().numpy().astype(np.float64), conv)


def test_config5_block_at_one_gpu_sampled():
    """bench.py's config-5 block (prefill part) at one GPU: the same inputs, classes and streams;
    sampled attention rows and, per DeltaNet layer, 8 whole V heads against the oracle."""
    from miso_b200 import cp
    t, layers = 131072, 3
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    proj = torch.randn((t, cp.ATTN_PROJ), generator=g, device=DEV).bfloat16().float()
    projs = [torch.randn((t, cp.DN_PROJ), generator=g, device=DEV).bfloat16().float()
             for _ in range(layers)]
    ones = torch.ones(256, device=DEV)
    inv = torch.from_numpy(A.rope_inv_freq()).to(DEV)
    conv_w = (0.5 * torch.randn((8192, 4), generator=g, device=DEV)).bfloat16().float()
    ssm_a, dt = -torch.ones(32, device=DEV), torch.zeros(32, device=DEV)
    norm_w = torch.ones(128, device=DEV)
    stream = torch.cuda.current_stream(DEV)
    dn_stream = torch.cuda.Stream(device=DEV, priority=-100)
    attn = cp.GpuAttentionCp(t, 1, 0, proj, ones, ones, inv, EPS, stream)
    dn = cp.GpuDeltaNetWavefront(t, 1, 0, projs, conv_w, ssm_a, dt, norm_w, EPS, dn_stream)
    dn_stream.wait_stream(stream)
    dn.run()
    attn.run()
    stream.wait_stream(dn_stream)
    torch.cuda.synchronize()
    assert status_clear()

    # attention: 48 rows, both zig-zag chunks, the last row included
    rng = np.random.RandomState(6)
    rows = np.unique(np.concatenate([rng.choice(t - 1, 47, replace=False), [t - 1]]))
    kb = attn.k.cpu().numpy().view(np.uint16)
    vb = attn.v.cpu().numpy().view(np.uint16)
    got = attn.core[torch.from_numpy(rows).to(DEV)].cpu().numpy()
    q = attn.q16[torch.from_numpy(rows).to(DEV)].cpu().numpy().astype(np.float32)
    qg = proj[torch.from_numpy(rows).to(DEV)].cpu().numpy()
    ref = np.stack([oracle.attn_prefill(1, int(r), q[i:i + 1], qg[i:i + 1], PROJ, kb, vb, t)[0]
                    for i, r in enumerate(rows)])
    check_attention_rows(got, ref)
    del kb, vb

    heads = [0, 5, 11, 15, 16, 22, 27, 31]
    hsel = torch.tensor(heads, device=DEV)
    cw, sa, dtb, nw = (x.cpu().numpy() for x in (conv_w, ssm_a, dt, norm_w))
    for layer in range(layers):
        pr = projs[layer].cpu().numpy()
        s64 = np.zeros((32, 128, 128))
        ref = oracle.deltanet_seq_heads(t, pr, DN_PROJ, pr, DN_PROJ, cw, np.zeros((8192, 3)),
                                        sa, dtb, nw, s64, EPS, heads, z_off=8192, a_off=12288,
                                        b_off=12320)
        got = dn.out[layer].view(t, 32, 128)[:, hsel].cpu().numpy()
        st = dn.state[layer][hsel].cpu().numpy()
        r_out, m_out = rel(got, ref), float(np.abs(got - ref).max())
        r_st = rel(st, s64[heads])
        print(f"layer {layer}: out rel-L2 {r_out:.3e} max abs {m_out:.3e}, state rel {r_st:.3e}")
        assert np.isfinite(got).all()
        assert r_out <= 1e-3 and m_out <= 1e-2 and r_st <= 1e-3
        # conv history after the sequence: the last three raw input rows, exactly
        hist = dn.conv[layer].cpu().numpy()
        assert np.array_equal(hist, pr[t - 3:t, :8192].T)
        del pr
