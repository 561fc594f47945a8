"""GPU parity of the attention kernels (through the C ABI) against the CPU oracle.

Cases follow the reference's own tests (tests/test_attn_splitk.hip): same lengths, split counts,
(pos0, n) pairs, input distributions (q ~ 2 N(0,1), gate ~ N(0,1), K/V = fp16(N(0,1))) and the
same accuracy bar — relative L2 <= 1e-5 per head against double precision — plus the combine's
bit-exactness contract. The batched fast path is held to the same bar, with ragged batches,
empty sequences, tile tails and garbage (NaN) rows past each sequence's end.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

import miso_b200
from miso_b200 import _capi as capi
from miso_b200 import attention as A
import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
HERE = os.path.dirname(os.path.abspath(__file__))


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def ptr(t):
    return t.data_ptr()


def rel_per_head(got, ref):
    """Max over heads of the relative L2 error; got / ref [..., 16, 256]."""
    got = np.asarray(got, np.float64).reshape(-1, 256)
    ref = np.asarray(ref, np.float64).reshape(-1, 256)
    num = np.sqrt(((got - ref) ** 2).sum(1))
    den = np.sqrt((ref ** 2).sum(1))
    return float(np.max(num / np.maximum(den, 1e-300)))


def decode_case(length, seed, max_ctx=None):
    rng = np.random.RandomState(seed)
    max_ctx = max_ctx or length + 7
    q = (2.0 * rng.standard_normal((16, 256))).astype(np.float32)
    qg = rng.standard_normal((16, 512)).astype(np.float32)
    k = rng.standard_normal((2, max_ctx, 256)).astype(np.float16)
    v = rng.standard_normal((2, max_ctx, 256)).astype(np.float16)
    return q, qg, k, v, max_ctx


# ---- combine bit-exactness (tests/test_attn_splitk.hip:47-96,180-187) --------------------------

_support = None


def support():
    global _support
    if _support is None:
        _support = C.CDLL(os.path.join(HERE, "support", "libmiso_test_support.so"))
        _support.test_combine.argtypes = [C.c_int, C.c_int, C.POINTER(capi.AttnCombineParams),
                                          C.c_void_p]
    return _support


def run_combine(variant, partial, pm, pl, po, qg, n_splits, canary=-9123.5):
    core = torch.full((16 * 256,), canary, dtype=torch.float32, device=DEV)
    p = capi.AttnCombineParams(ptr(pm), ptr(pl), ptr(po), ptr(qg), ptr(core), n_splits)
    assert support().test_combine(variant, partial, C.byref(p), None) == 0
    torch.cuda.synchronize()
    return core.cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("splits", [1, 2, 3, 4, 5, 15, 16, 17, 31, 32, 33, 57, 60, 63, 64, 65,
                                    129])
def test_combine_variants_are_bit_identical(splits):
    for variant in (0, 1, 4):
        for extreme, partial in ((False, False), (True, False), (True, True)):
            rng = np.random.RandomState(9017 + splits)
            n = 2 * splits * 8
            pm = rng.uniform(-3, 3, n).astype(np.float32)
            pl = (1.0 + np.abs(rng.uniform(-3, 3, n))).astype(np.float32)
            po = rng.uniform(-3, 3, (n, 256)).astype(np.float32)
            if extreme:
                c = (np.arange(n) // 8) % splits
                pm += np.where(c % 2 == 0, 80.0, -80.0).astype(np.float32)
                empty = (c != 0) & (c % 3 == 0)
                pm[empty] = -np.inf
                pl[empty] = 0.0
                po[empty] = 0.0
                i = np.arange(16 * 512)
                qg = np.where(i % 3 == 0, -100.0, np.where(i % 3 == 1, 100.0, -0.0))
                qg = qg.astype(np.float32)
            else:
                qg = rng.uniform(-3, 3, 16 * 512).astype(np.float32)
            args = [T(x) for x in (pm, pl, po, qg)]
            ref = run_combine(-1, partial, *args, splits)
            got = run_combine(variant, partial, *args, splits)
            assert np.array_equal(got, ref), (variant, extreme, partial)


# ---- split-K decode, drop-in kernels (tests/test_attn_splitk.hip:101-176,189-200,281-290) -------


def run_split_combine(q, qg, k, v, length, max_ctx, max_splits):
    ns = A.n_splits(length, max_splits)
    dq, dqg, dk, dv = T(q), T(qg), T(k), T(v)
    pm = torch.empty(2 * ns * 8, device=DEV)
    pl = torch.empty(2 * ns * 8, device=DEV)
    po = torch.empty(2 * ns * 8 * 256, device=DEV)
    A.attn_split(capi.AttnSplitParams(ptr(dq), ptr(dk), ptr(dv), ptr(pm), ptr(pl), ptr(po),
                                      length, max_ctx, ns))
    core = torch.empty(16 * 256, device=DEV)
    A.attn_combine(capi.AttnCombineParams(ptr(pm), ptr(pl), ptr(po), ptr(dqg), ptr(core), ns))
    torch.cuda.synchronize()
    wide = run_combine(256, 0, pm, pl, po, dqg, ns)  # the reference test's <256> combine
    return core.cpu().numpy(), wide.view(np.float32), ns


@pytest.mark.parametrize("length,max_splits", [(1, 60), (31, 60), (32, 60), (33, 60), (257, 60),
                                               (1000, 60), (4096, 60), (32767, 60), (32768, 60),
                                               (32769, 60), (5000, 60), (3872, 60), (5000, 3)])
def test_split_decode_matches_fp64(length, max_splits):
    q, qg, k, v, max_ctx = decode_case(length, length)
    got, wide, ns = run_split_combine(q, qg, k, v, length, max_ctx, max_splits)
    assert np.array_equal(got.view(np.uint32), wide.view(np.uint32))  # production == <256>
    ref = oracle.attn_decode(q, qg, 8192, k.view(np.uint16).reshape(-1, 256),
                             v.view(np.uint16).reshape(-1, 256),
                             np.array([[0, max_ctx]], np.int64), np.array([length], np.int32))
    assert rel_per_head(got, ref) <= 1e-5


# ---- batched stream-K decode (fast path) -------------------------------------------------------


def make_pool(lens, capacity, seed, garbage=True):
    rng = np.random.RandomState(seed)
    batch = len(lens)
    pool = A.KvPool(batch, capacity, device=DEV)
    k = rng.standard_normal((pool.rows, 256)).astype(np.float16)
    v = rng.standard_normal((pool.rows, 256)).astype(np.float16)
    if garbage:  # rows past each sequence's end hold NaN bit patterns
        for b, n in enumerate(lens):
            for h in range(2):
                r0 = (2 * b + h) * capacity
                k[r0 + n:r0 + capacity] = np.float16(np.nan)
                v[r0 + n:r0 + capacity] = np.float16(np.nan)
    pool.k.copy_(T(k))
    pool.v.copy_(T(v))
    pool.lens.copy_(T(np.asarray(lens, np.int32)))
    q = (2.0 * rng.standard_normal((batch, 16, 256))).astype(np.float32)
    qg = rng.standard_normal((batch, 16, 512)).astype(np.float32)
    return pool, k, v, q, qg


def run_fast(pool, q, qg, scratch=None):
    core = torch.full((pool.batch, 16, 256), 7.0, device=DEV)
    scratch = scratch if scratch is not None else A.decode_scratch(pool.batch, device=DEV)
    A.decode_batched(pool, T(q), T(qg), core, scratch)
    torch.cuda.synchronize()
    return core.cpu().numpy(), scratch


def oracle_pool(pool, k, v, q, qg, lens):
    return oracle.attn_decode(q, qg, 8192, k.view(np.uint16), v.view(np.uint16),
                              pool.kv_row.cpu().numpy(), np.asarray(lens, np.int32))


def check_status():
    st = C.c_int(-1)
    assert capi.load().miso_device_status(1, C.byref(st)) == 0
    assert st.value == 0


@pytest.mark.parametrize("length", [1, 15, 16, 17, 63, 64, 65, 257, 1000, 4096, 32768, 32769])
def test_fast_decode_single_sequence(length):
    pool, k, v, q, qg = make_pool([length], length + 64, seed=length)
    got, _ = run_fast(pool, q, qg)
    ref = oracle_pool(pool, k, v, q, qg, [length])
    assert rel_per_head(got, ref) <= 1e-5
    check_status()


def test_fast_decode_ragged_batch_with_empty_sequences():
    rng = np.random.RandomState(99)
    lens = list(rng.randint(1, 3000, size=37))
    lens[3] = 0
    lens[20] = 0
    lens[36] = 64
    lens[10] = 1
    pool, k, v, q, qg = make_pool(lens, 3072, seed=5)
    got, scratch = run_fast(pool, q, qg)
    ref = oracle_pool(pool, k, v, q, qg, lens)
    live = [b for b, n in enumerate(lens) if n > 0]
    assert rel_per_head(got[live], ref[live]) <= 1e-5
    assert np.all(got[[3, 20]] == 0.0)
    # Same scratch again: counters were left zeroed, results are bitwise reproducible.
    again, _ = run_fast(pool, q, qg, scratch)
    assert np.array_equal(again.view(np.uint32), got.view(np.uint32))
    assert int(scratch[: 2 * len(lens)].abs().sum().item()) == 0
    check_status()


def test_fast_decode_ignores_leftover_counters_in_scratch():
    """A call whose kernel gave up on a bounded wait leaves arrival counters set. Each call zeroes
    its counters before its kernel, so a scratch buffer holding such leftovers (planted here from
    the host: every counter and partial set to garbage) still gives the oracle's result."""
    lens = [3000, 1, 777, 0, 2049, 64, 5000]
    pool, k, v, q, qg = make_pool(lens, 5120, seed=8)
    scratch = A.decode_scratch(pool.batch, device=DEV)
    scratch.fill_(0x3F00_0001)  # counters at ~1e9 arrivals, partials at 0.5-ish floats
    got, _ = run_fast(pool, q, qg, scratch)
    ref = oracle_pool(pool, k, v, q, qg, lens)
    live = [b for b, n in enumerate(lens) if n > 0]
    assert rel_per_head(got[live], ref[live]) <= 1e-5
    assert np.all(got[3] == 0.0)
    scratch[: 2 * len(lens)].fill_(-7)  # negative counts too
    again, _ = run_fast(pool, q, qg, scratch)
    assert np.array_equal(again.view(np.uint32), got.view(np.uint32))
    check_status()


def test_fast_decode_long_ragged_batch():
    rng = np.random.RandomState(0)
    lens = list(rng.randint(1024, 20000, size=8))
    pool, k, v, q, qg = make_pool(lens, 20000, seed=6, garbage=False)
    got, _ = run_fast(pool, q, qg)
    ref = oracle_pool(pool, k, v, q, qg, lens)
    assert rel_per_head(got, ref) <= 1e-5


def test_fast_decode_equals_drop_in_path_on_a_reference_cache():
    """A reference AttentionCache [2][max_ctx][256] is the pool with kv_row = {0, max_ctx}."""
    length = 4096
    q, qg, k, v, max_ctx = decode_case(length, 17)
    pool = A.KvPool(1, max_ctx, device=DEV)
    pool.k.copy_(T(k.reshape(-1, 256)))
    pool.v.copy_(T(v.reshape(-1, 256)))
    pool.lens.fill_(length)
    fast, _ = run_fast(pool, q[None], qg[None])
    drop, _, _ = run_split_combine(q, qg, k, v, length, max_ctx, 60)
    assert rel_per_head(fast[0], drop) <= 1e-5  # both within 1e-5 of fp64


# ---- prep (tests of the reference: via test_attention / prefill; formulas
#      kernels/attention_decode.hpp:41-71) -------------------------------------------------------


def prep_inputs(seed):
    rng = np.random.RandomState(seed)
    qg = (1.5 * rng.standard_normal((16, 512))).astype(np.float32)
    k = rng.standard_normal((2, 256)).astype(np.float32)
    v = rng.standard_normal((2, 256)).astype(np.float32)
    qn = (1.0 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    return qg, k, v, qn, kn, A.rope_inv_freq()


def f16_ulps(got_bits, ref64):
    ref = ref64.astype(np.float16).view(np.uint16).astype(np.int32)
    return np.abs(got_bits.astype(np.int32) - ref)


@pytest.mark.parametrize("pos", [0, 1, 777, 8191, 131071])
def test_prep_matches_oracle(pos):
    qg, k, v, qn, kn, inv = prep_inputs(pos)
    max_ctx = pos + 2
    kc = torch.zeros((2, max_ctx, 256), dtype=torch.float16, device=DEV)
    vc = torch.zeros_like(kc)
    qo = torch.empty((16, 256), device=DEV)
    d = [T(x) for x in (qg, k, v, qn, kn, inv)]
    A.attn_prep(capi.AttnPrepParams(*[ptr(x) for x in d], ptr(kc), ptr(vc), ptr(qo), pos,
                                    max_ctx, 1e-6))
    torch.cuda.synchronize()
    rq, rk, rv = oracle.attn_prep(qg, k, v, qn, kn, inv, pos, 1e-6)
    assert rel_per_head(qo.cpu().numpy(), rq) <= 2e-6
    kbits = kc[:, pos].cpu().numpy().view(np.uint16)
    vbits = vc[:, pos].cpu().numpy().view(np.uint16)
    assert f16_ulps(kbits, rk).max() <= 1
    assert np.array_equal(vbits, rv.astype(np.float16).view(np.uint16))


def test_batched_prep_equals_drop_in_prep_and_advances_lens():
    batch, cap = 5, 64
    pool = A.KvPool(batch, cap, device=DEV)
    pool.k.zero_(); pool.v.zero_()
    lens = np.array([0, 3, 17, 63, 40], np.int32)
    pool.lens.copy_(T(lens))
    proj = []
    for b in range(batch):
        qg, k, v, qn, kn, inv = prep_inputs(100 + b)
        proj.append(np.concatenate([qg.ravel(), k.ravel(), v.ravel()]))
    proj = np.stack(proj).astype(np.float32)  # [batch][9216]
    dproj = T(proj)
    dqn, dkn, dinv = T(qn), T(kn), T(inv)
    qo = torch.empty((batch, 16, 256), device=DEV)
    base = ptr(dproj)
    p = capi.AttnPrepBatchedParams(base, base + 8192 * 4, base + 8704 * 4, ptr(dqn), ptr(dkn),
                                   ptr(dinv), ptr(pool.k), ptr(pool.v), ptr(pool.kv_row),
                                   ptr(pool.lens), ptr(qo), batch, 9216, 1e-6)
    capi.check("miso_attn_prep_batched",
               capi.load().miso_attn_prep_batched(C.byref(p), None))
    torch.cuda.synchronize()
    assert np.array_equal(pool.lens.cpu().numpy(), lens + 1)
    for b in range(batch):
        kc = torch.zeros((2, cap, 256), dtype=torch.float16, device=DEV)
        vc = torch.zeros_like(kc)
        q1 = torch.empty((16, 256), device=DEV)
        pb = base + b * 9216 * 4
        A.attn_prep(capi.AttnPrepParams(pb, pb + 8192 * 4, pb + 8704 * 4, ptr(dqn), ptr(dkn),
                                        ptr(dinv), ptr(kc), ptr(vc), ptr(q1), int(lens[b]), cap,
                                        1e-6))
        torch.cuda.synchronize()
        assert torch.equal(q1, qo[b])
        for h in range(2):
            r = (2 * b + h) * cap + int(lens[b])
            assert torch.equal(pool.k[r], kc[h, lens[b]])
            assert torch.equal(pool.v[r], vc[h, lens[b]])


# ---- causal prefill, drop-in kernels (tests/test_attn_splitk.hip:204-279) ----------------------


@pytest.mark.parametrize("pos0,n", [(0, 1), (0, 3), (0, 4), (0, 5), (0, 33), (40, 17), (0, 128),
                                    (300, 77)])
def test_prefill_matches_fp64(pos0, n):
    length = pos0 + n
    max_ctx = length + 5
    rng = np.random.RandomState(1000 + 17 * pos0 + n)
    q = (2.0 * rng.standard_normal((n, 16, 256))).astype(np.float32)
    qg = rng.standard_normal((n, 16, 512)).astype(np.float32)
    k = rng.standard_normal((2, max_ctx, 256)).astype(np.float16)
    v = rng.standard_normal((2, max_ctx, 256)).astype(np.float16)
    core = torch.full((n, 16, 256), -1.0, device=DEV)
    dq, dqg, dk, dv = T(q), T(qg), T(k), T(v)
    A.attn_prefill(capi.AttnPrefillParams(ptr(dq), ptr(dqg), ptr(dk), ptr(dv), ptr(core), pos0,
                                          n, max_ctx, 16 * 512))
    torch.cuda.synchronize()
    ref = oracle.attn_prefill(n, pos0, q, qg, 8192, k.view(np.uint16), v.view(np.uint16),
                              max_ctx)
    assert rel_per_head(core.cpu().numpy(), ref) <= 1e-5


@pytest.mark.parametrize("cuts", [(13,), (1, 2, 3), (4, 8, 29), (16, 17)])
def test_prefill_does_not_depend_on_how_the_prompt_is_cut(cuts):
    """A token's core row is bitwise the same whether the prompt goes in one call or in several
    (each later call at pos0 = the tokens already cached), as the engine's chunked prefill and the
    reference's test_prefill expect: the row depends on the token's keys alone, not on the 4-token
    block it shares or the slabs the other tokens of the call reach."""
    n, pos0 = 37, 5
    max_ctx = pos0 + n
    rng = np.random.RandomState(77 + len(cuts))
    q = T((2.0 * rng.standard_normal((n, 16, 256))).astype(np.float32))
    qg = T(rng.standard_normal((n, 16, 512)).astype(np.float32))
    k = T(rng.standard_normal((2, max_ctx, 256)).astype(np.float16))
    v = T(rng.standard_normal((2, max_ctx, 256)).astype(np.float16))

    def run(a, b, core):
        A.attn_prefill(capi.AttnPrefillParams(ptr(q[a]), ptr(qg[a]), ptr(k), ptr(v), ptr(core[a]),
                                              pos0 + a, b - a, max_ctx, 16 * 512))

    whole = torch.full((n, 16, 256), -1.0, device=DEV)
    run(0, n, whole)
    parts = torch.full_like(whole, -2.0)
    edges = [0, *cuts, n]
    for a, b in zip(edges, edges[1:]):
        run(a, b, parts)
    torch.cuda.synchronize()
    assert torch.equal(whole.view(torch.int32), parts.view(torch.int32))


def test_engine_decode_sequence_matches_oracle():
    """attention_decode_core token by token (prep -> split -> combine), as the engine drives it."""
    rng = np.random.RandomState(4)
    cache = A.AttentionCache(64, device=DEV)
    sc = A.AttentionScratch(device=DEV)
    qn = T((1 + 0.1 * rng.standard_normal(256)).astype(np.float32))
    kn = T((1 + 0.1 * rng.standard_normal(256)).astype(np.float32))
    inv = T(A.rope_inv_freq())
    ks = np.zeros((2, 64, 256), np.float16); vs = np.zeros_like(ks)
    for t in range(40):
        qg = rng.standard_normal((16, 512)).astype(np.float32)
        k = rng.standard_normal((2, 256)).astype(np.float32)
        v = rng.standard_normal((2, 256)).astype(np.float32)
        core = A.attention_decode_core(cache, sc, T(qg), T(k), T(v), qn, kn, inv, 1e-6)
        torch.cuda.synchronize()
        rq, rk, rv = oracle.attn_prep(qg, k, v, qn.cpu().numpy(), kn.cpu().numpy(),
                                      inv.cpu().numpy(), t, 1e-6)
        ks[:, t] = cache.k[:, t].cpu().numpy()
        vs[:, t] = cache.v[:, t].cpu().numpy()
        ref = oracle.attn_decode(sc.q.cpu().numpy(), qg, 8192, ks.view(np.uint16).reshape(-1, 256),
                                 vs.view(np.uint16).reshape(-1, 256),
                                 np.array([[0, 64]], np.int64), np.array([t + 1], np.int32))
        assert rel_per_head(core.cpu().numpy(), ref) <= 1e-5
        assert rel_per_head(sc.q.cpu().numpy(), rq) <= 2e-6
    assert cache.len == 40


# ---- causal prefill on tcgen05 (fp16 queries; BASELINE bar: rel-L2 <= 1e-3, max-abs <= 1e-2) ---


def run_prefill_tc(q16, qg, k, v, pos0, n, max_ctx):
    core = torch.full((n, 16, 256), -3.0, device=DEV)
    dq, dqg, dk, dv = T(q16), T(qg), T(k), T(v)
    p = capi.AttnPrefillTcParams(ptr(dq), ptr(dqg), ptr(dk), ptr(dv), ptr(core), pos0, n, max_ctx,
                                 16 * 512)
    capi.check("miso_attn_prefill_tc", capi.load().miso_attn_prefill_tc(C.byref(p), None))
    torch.cuda.synchronize()
    return core.cpu().numpy()


@pytest.mark.parametrize("pos0,n", [(0, 1), (0, 15), (0, 16), (0, 17), (0, 100), (40, 17),
                                    (300, 77), (0, 512), (1000, 333), (0, 2048)])
def test_prefill_tc_matches_fp64(pos0, n):
    length = pos0 + n
    max_ctx = length + 5
    rng = np.random.RandomState(7000 + 13 * pos0 + n)
    q16 = rng.standard_normal((n, 16, 256)).astype(np.float16)
    qg = rng.standard_normal((n, 16, 512)).astype(np.float32)
    k = rng.standard_normal((2, max_ctx, 256)).astype(np.float16)
    v = rng.standard_normal((2, max_ctx, 256)).astype(np.float16)
    k[:, length:] = np.float16(np.nan)  # never read: outside the tensor maps
    v[:, length:] = np.float16(np.nan)
    got = run_prefill_tc(q16, qg, k, v, pos0, n, max_ctx)
    ref = oracle.attn_prefill(n, pos0, q16.astype(np.float32), qg, 8192, k.view(np.uint16),
                              v.view(np.uint16), max_ctx)
    assert rel_per_head(got, ref) <= 1e-3
    assert np.abs(got - ref).max() <= 1e-2
    # logits-proxy argmax over each output row is exact wherever the oracle's top-2 gap clears the
    # error bound
    srt = np.sort(ref.reshape(-1, 256), axis=1)
    clear = (srt[:, -1] - srt[:, -2]) > 2e-3
    assert clear.mean() > 0.5
    assert np.array_equal(got.reshape(-1, 256)[clear].argmax(1), ref.reshape(-1, 256)[clear].argmax(1))


def test_prep_batch_f16_matches_drop_in_prep():
    n, pos0, max_ctx = 37, 11, 64
    rng = np.random.RandomState(77)
    proj = (rng.standard_normal((n, 9216))).astype(np.float32)
    qn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    kn = (1 + 0.1 * rng.standard_normal(256)).astype(np.float32)
    dproj, dqn, dkn, dinv = T(proj), T(qn), T(kn), T(A.rope_inv_freq())
    caches = []
    for f16 in (False, True):
        kc = torch.zeros((2, max_ctx, 256), dtype=torch.float16, device=DEV)
        vc = torch.zeros_like(kc)
        q32 = torch.zeros((n, 16, 256), device=DEV)
        q16 = torch.zeros((n, 16, 256), dtype=torch.float16, device=DEV)
        base = ptr(dproj)
        tok0 = capi.AttnPrepParams(base, base + 8192 * 4, base + 8704 * 4, ptr(dqn), ptr(dkn),
                                   ptr(dinv), ptr(kc), ptr(vc), ptr(q32), pos0, max_ctx, 1e-6)
        bp = capi.AttnPrepBatchParams(tok0, n, 9216)
        if f16:
            capi.check("f16", capi.load().miso_attn_prep_batch_f16(C.byref(bp), ptr(q16), None))
        else:
            A.attn_prep_batch(bp)
        torch.cuda.synchronize()
        caches.append((kc.clone(), vc.clone(), q32.clone(), q16.clone()))
    (k0, v0, q32, _), (k1, v1, _, q16) = caches
    assert torch.equal(k0, k1) and torch.equal(v0, v1)
    assert torch.equal(q32.half(), q16)
