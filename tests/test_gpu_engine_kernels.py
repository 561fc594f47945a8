"""The drop-in kernels around the attention path, on the B200, against the numpy oracle of the
weight formats (oracle/quant.py, pinned to the reference's fixtures and code): Q4_K / Q6_K decode
GEMV (FP16 and INT8 activations; the engine's grids and rows-per-warp choices), the fused mixed
GEMV (bitwise equal to the separate kernels), the prefill GEMM and its activation prep (bitwise),
the Q4_K embedding (bitwise), add + RMSNorm, argmax (ties to the lowest index), and the MoE block
in its decode and prefill forms (routing identical to the oracle's on the kernel's logits; the
prefill router bitwise equal to the decode router; grouping equal to a stable sort by expert).
Launch configurations are the engine's (tests/support/engine_kernels.cu)."""
import ctypes as C
import os

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
DEV = torch.device("cuda")
P = C.c_void_p
U = C.c_uint

_lib = None


def lib():
    global _lib
    if _lib is None:
        L = C.CDLL(os.path.join(HERE, "support", "libmiso_test_support.so"))
        L.tk_q4k_gemv.argtypes = [P, P, P, U, U, C.c_int, C.c_int, U]
        L.tk_q6k_gemv.argtypes = [P, P, P, U, U, C.c_int, U]
        L.tk_mixed_gemv.argtypes = [P, P, P, P, P, U, U, C.c_int]
        L.tk_qgemm_act.argtypes = [P, P, P, U, U]
        L.tk_qgemm.argtypes = [C.c_int, P, P, P, P, U, U, U, U]
        L.tk_embed.argtypes = [P, P, P, U]
        L.tk_add_rmsnorm.argtypes = [P, P, P, P, C.c_float, U, U]
        L.tk_argmax.argtypes = [P, U, P, P, U, P]
        L.tk_moe_decode.argtypes = [C.c_int] + [P] * 13
        L.tk_moe_max_tasks.argtypes = [U]
        L.tk_moe_max_tasks.restype = U
        L.tk_moe_prefill.argtypes = [C.c_int, P, P, U] + [P] * 18
        _lib = L
    return _lib


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def ptr(t):
    """Device address of a tensor; the caller keeps the tensor alive until the kernel has run
    (a freed block can be handed to the next allocation, whose copy is ordered before the launch)."""
    return None if t is None else t.data_ptr()


def ok(rc):
    assert rc == 0, f"launch failed: {rc}"
    torch.cuda.synchronize()


def q4k_mag(g):
    """|d sc q| + |dmin m| per element of GGUF Q4_K rows (the scale of the kernels' FP32 error)."""
    blocks = g.reshape(-1, Q.Q4K_BYTES)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float64)
    dm = blocks[:, 2:4].copy().view(np.float16).astype(np.float64)
    sc, mn = Q.q4k_scale_min(blocks)
    q = Q.q4k_nibbles(blocks).reshape(-1, 8, 32).astype(np.float64)
    m = np.abs(d * sc)[:, :, None] * q + np.abs(dm * mn)[:, :, None]
    return m.reshape(g.shape[0], -1)


def within(got, ref, mag, rel):
    err = np.abs(np.asarray(got, np.float64) - ref)
    bound = rel * mag + 1e-30
    worst = np.max(err / bound)
    assert worst <= 1.0, f"error {worst:.3g} x the bound (max abs err {err.max():.3g})"


# ---- decode GEMV ---------------------------------------------------------------------------

@pytest.mark.parametrize("k,n,int8", [(2048, 100, 0), (2048, 2061, 0), (4096, 300, 0),
                                      (8192, 2, 0), (8192, 2, 1), (2048, 2061, 1), (4096, 64, 1)])
def test_q4k_gemv_matches_oracle(k, n, int8):
    rng = np.random.RandomState(k + n + int8)
    g = Q.random_q4k(rng, n, k)
    x = rng.standard_normal(k).astype(np.float32)
    w, y = dev(Q.q4k_repack_r1(g)), torch.full((n,), float("nan"), device=DEV)
    xd = dev(x)
    ok(lib().tk_q4k_gemv(ptr(w), ptr(xd), ptr(y), n, k, int8, 0, 0))
    xa = Q.act_int8(x) if int8 else Q.act_fp16(x)
    ref = Q.q4k_dequant(g).astype(np.float64) @ xa
    within(y.cpu().numpy(), ref, q4k_mag(g) @ np.abs(xa), 1e-5)


@pytest.mark.parametrize("k,n,rows,grid", [(2048, 300, 0, 0), (2048, 8192, 0, 0),
                                           (2048, 5000, 1, 1920), (4096, 4, 1, 1)])
def test_q6k_gemv_matches_oracle(k, n, rows, grid):
    rng = np.random.RandomState(k + n)
    g = Q.random_q6k(rng, n, k)
    x = rng.standard_normal(k).astype(np.float32)
    w, y, xd = dev(Q.q6k_repack_r1(g, k)), torch.full((n,), float("nan"), device=DEV), dev(x)
    ok(lib().tk_q6k_gemv(ptr(w), ptr(xd), ptr(y), n, k, rows, grid))
    xa = Q.act_fp16(x)
    wf = Q.q6k_dequant(g).astype(np.float64)
    within(y.cpu().numpy(), wf @ xa, np.abs(wf) @ np.abs(xa), 1e-5)


@pytest.mark.parametrize("n6,wide", [(8192, 1), (1000, 0)])
def test_mixed_gemv_equals_separate_kernels_bitwise(n6, wide):
    rng = np.random.RandomState(n6)
    g6, g4 = Q.random_q6k(rng, n6, 2048), Q.random_q4k(rng, 2048, 2048)
    x = dev(rng.standard_normal(2048).astype(np.float32))
    w6, w4 = dev(Q.q6k_repack_r1(g6, 2048)), dev(Q.q4k_repack_r1(g4))
    y6, y4 = torch.empty(n6, device=DEV), torch.empty(2048, device=DEV)
    s6, s4 = torch.empty_like(y6), torch.empty_like(y4)
    ok(lib().tk_mixed_gemv(ptr(w6), ptr(w4), ptr(x), ptr(y6), ptr(y4), n6, 2048, wide))
    ok(lib().tk_q6k_gemv(ptr(w6), ptr(x), ptr(s6), n6, 2048, 0, 0))
    ok(lib().tk_q4k_gemv(ptr(w4), ptr(x), ptr(s4), 2048, 2048, 0, 0, 0))
    assert torch.equal(y6.view(torch.int32), s6.view(torch.int32))
    assert torch.equal(y4.view(torch.int32), s4.view(torch.int32))


# ---- prefill GEMM --------------------------------------------------------------------------

def cpu_act(x):
    """FP16 rounding and per-32 sums in the kernels' FP32 order (((h0 + h1) + h2) + h3 per 4)."""
    h = x.astype(np.float16)
    f = h.astype(np.float32).reshape(-1, 8, 4)
    s = np.zeros(f.shape[0], np.float32)
    for c in range(8):
        s = s + (((f[:, c, 0] + f[:, c, 1]) + f[:, c, 2]) + f[:, c, 3])
    return h, s


def test_gemm_activation_prep_is_bitwise():
    rng = np.random.RandomState(1)
    x = (3 * rng.standard_normal((37, 2048))).astype(np.float32)
    xh = torch.empty((37, 2048), dtype=torch.float16, device=DEV)
    xs = torch.empty((37, 64), device=DEV)
    xd = dev(x)
    ok(lib().tk_qgemm_act(ptr(xd), ptr(xh), ptr(xs), 2048, 37))
    h, s = cpu_act(x)
    assert np.array_equal(xh.cpu().numpy().view(np.uint16), h.view(np.uint16).reshape(37, 2048))
    assert np.array_equal(xs.cpu().numpy().reshape(-1).view(np.uint32), s.view(np.uint32))


@pytest.mark.parametrize("q6,k,n,n_tok,ldy", [(0, 2048, 130, 70, 135), (1, 2048, 100, 65, 100),
                                              (0, 4096, 64, 1, 64), (1, 512, 2048, 9, 2048)])
def test_gemm_matches_oracle(q6, k, n, n_tok, ldy):
    rng = np.random.RandomState(n + n_tok)
    g = Q.random_q6k(rng, n, k) if q6 else Q.random_q4k(rng, n, k)
    w = dev(Q.q6k_repack_r1(g, k) if q6 else Q.q4k_repack_r1(g))
    x = rng.standard_normal((n_tok, k)).astype(np.float32)
    xh = torch.empty((n_tok, k), dtype=torch.float16, device=DEV)
    xs = torch.empty((n_tok, k // 32), device=DEV)
    xd = dev(x)
    ok(lib().tk_qgemm_act(ptr(xd), ptr(xh), ptr(xs), k, n_tok))
    y = torch.full((n_tok, ldy), 7.0, device=DEV)
    ok(lib().tk_qgemm(q6, ptr(w), ptr(xh), ptr(xs), ptr(y), k, n, n_tok, ldy))
    wf = (Q.q6k_dequant(g) if q6 else Q.q4k_dequant(g)).astype(np.float64)
    xa = Q.act_fp16(x).reshape(n_tok, k)
    got = y.cpu().numpy()
    mag = np.abs(xa) @ (q4k_mag(g) if not q6 else np.abs(wf)).T
    within(got[:, :n], xa @ wf.T, mag, k * 2.0 ** -24 + 1e-6)
    assert np.all(got[:, n:] == 7.0)


# ---- embedding, norm, argmax ---------------------------------------------------------------

def test_embedding_is_bitwise():
    rng = np.random.RandomState(2)
    g = Q.random_q4k(rng, 50, 2048)
    ids = np.array([0, 49, 7, 7, 23], np.int32)
    out = torch.full((5, 2048), float("nan"), device=DEV)
    table, idd = dev(Q.q4k_repack_r1(g)), dev(ids)  # alive until the kernel has run
    ok(lib().tk_embed(ptr(table), ptr(idd), ptr(out), 5))
    want = Q.q4k_dequant(g[ids])
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("with_delta,grid", [(1, 5), (1, 2), (0, 5)])
def test_add_rmsnorm(with_delta, grid):
    rng = np.random.RandomState(3)
    res = rng.standard_normal((5, 2048)).astype(np.float32)
    delta = rng.standard_normal((5, 2048)).astype(np.float32)
    wt = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    r, dl, w = dev(res), dev(delta), dev(wt)
    out = torch.empty((5, 2048), device=DEV)
    ok(lib().tk_add_rmsnorm(ptr(r), ptr(dl) if with_delta else None, ptr(w), ptr(out), 1e-6, 5,
                            grid))
    h, ref = Q.add_rmsnorm(res, delta if with_delta else None, wt, 1e-6)
    want_res = (res + delta) if with_delta else res
    assert np.array_equal(r.cpu().numpy().view(np.uint32), want_res.view(np.uint32))
    within(out.cpu().numpy(), ref, np.abs(ref), 1e-5)


@pytest.mark.parametrize("case", ["random", "ties", "all_equal", "small"])
def test_argmax_lowest_index_on_ties(case):
    rng = np.random.RandomState(4)
    n = 7 if case == "small" else 248320
    x = rng.standard_normal(n).astype(np.float32)
    if case == "ties":
        x[[100, 5000, 200000]] = x.max() + 1
    elif case == "all_equal":
        x[:] = 0.25
    elif case == "small":
        x[[2, 5]] = 9.0
    pv, pi = torch.empty(240, device=DEV), torch.empty(240, dtype=torch.int32, device=DEV)
    out = torch.full((1,), -1, dtype=torch.int32, device=DEV)
    xd = dev(x)
    ok(lib().tk_argmax(ptr(xd), n, ptr(pv), ptr(pi), 240, ptr(out)))
    assert int(out.item()) == int(np.argmax(x))


# ---- MoE -----------------------------------------------------------------------------------

Q4_ROW, Q6_ROW512 = 2048 // 256 * 144, Q.q6k_r1_row_bytes(512)


def rand_q4k_r1(rows, k, scale, gen):
    """Random Q4_K r1 rows generated on the device (any r1 scale fields are valid), d and dmin
    positive FP16 around `scale`."""
    nb = rows * k // 256
    b = torch.randint(0, 256, (nb, 144), dtype=torch.uint8, device=DEV, generator=gen)
    dd = torch.empty((nb, 2), dtype=torch.float16, device=DEV).uniform_(0.5 * scale, 1.5 * scale,
                                                                        generator=gen)
    b[:, 0:4] = dd.view(torch.uint8)
    return b.view(rows, -1)


def rand_q6k_r1(rows, k, scale, gen):
    """Random Q6_K r1 rows on the device: random codes / int8 scales, positive FP16 d, zero pad."""
    nb, rb = k // 256, Q.q6k_r1_row_bytes(k)
    b = torch.randint(0, 256, (rows, rb), dtype=torch.uint8, device=DEV, generator=gen)
    d = torch.empty((rows, nb), dtype=torch.float16, device=DEV).uniform_(0.5 * scale, 1.5 * scale,
                                                                          generator=gen)
    b[:, nb * 208:nb * 210] = d.view(torch.uint8)
    b[:, nb * 210:] = 0
    return b


class MoeWeights:
    def __init__(self, down_q6, seed):
        gen = torch.Generator(device=DEV)
        gen.manual_seed(seed)
        self.down_q6 = down_q6
        rng = np.random.RandomState(seed)
        rw = (0.05 * rng.standard_normal((257, 2048))).astype(np.float32)
        self.router_np = (rw.view(np.uint32) >> 16).astype(np.uint16)
        self.router = dev(self.router_np)
        self.gate = rand_q4k_r1(256 * 512, 2048, 2e-4, gen)
        self.up = rand_q4k_r1(256 * 512, 2048, 2e-4, gen)
        self.gate_sh = rand_q4k_r1(512, 2048, 2e-4, gen)
        self.up_sh = rand_q4k_r1(512, 2048, 2e-4, gen)
        if down_q6:
            self.down = rand_q6k_r1(256 * 2048, 512, 1e-4, gen)
            self.down_sh = rand_q6k_r1(2048, 512, 1e-4, gen)
        else:
            self.down = rand_q4k_r1(256 * 2048, 512, 1e-4, gen)
            self.down_sh = rand_q4k_r1(2048, 512, 1e-4, gen)
        self._cache = {}

    def rows(self, which, e):
        """Dequantised rows (float64) and per-element error magnitudes of expert e (256: shared)."""
        key = (which, e)
        if key not in self._cache:
            if which in ("gate", "up"):
                t = (self.gate if which == "gate" else self.up) if e < 256 else \
                    (self.gate_sh if which == "gate" else self.up_sh)
                r = t[e * 512:(e + 1) * 512] if e < 256 else t
                g = Q.q4k_r1_to_gguf(r.cpu().numpy())
                self._cache[key] = (Q.q4k_dequant(g).astype(np.float64), q4k_mag(g))
            else:
                t = self.down if e < 256 else self.down_sh
                r = (t[e * 2048:(e + 1) * 2048] if e < 256 else t).cpu().numpy()
                if self.down_q6:
                    wf = Q.q6k_dequant(Q.q6k_r1_to_gguf(r, 512)).astype(np.float64)
                    self._cache[key] = (wf, np.abs(wf))
                else:
                    g = Q.q4k_r1_to_gguf(r)
                    self._cache[key] = (Q.q4k_dequant(g).astype(np.float64), q4k_mag(g))
        return self._cache[key]

    def ptrs(self):
        return [ptr(t) for t in (self.gate, self.up, self.gate_sh, self.up_sh, self.down,
                                 self.down_sh)]


def check_routing(logits_t, ids_t, weights_t):
    want_ids, want_w = Q.moe_topk(logits_t)
    assert list(ids_t[:8]) == list(want_ids)
    within(weights_t[:8], want_w, np.abs(want_w), 1e-6)


def check_gate_up(W, x, e, h_got):
    """h = SiLU(gate . x) * (up . x) with FP16-rounded x; error bounded through both products."""
    xa = Q.act_fp16(x)
    (wg, mg), (wu, mu) = W.rows("gate", e), W.rows("up", e)
    g, u = wg @ xa, wu @ xa
    eg, eu = 1e-5 * (mg @ np.abs(xa)), 1e-5 * (mu @ np.abs(xa))
    within(h_got, Q.silu(g) * u, 1.1 * eg * np.abs(u) + np.abs(Q.silu(g)) * eu + 1e-3 * eg * eu,
           1.0)


def down_ref(W, e, h):
    wd, md = W.rows("down", e)
    ha = Q.act_fp16(h)
    return wd @ ha, md @ np.abs(ha)


@pytest.mark.parametrize("down_q6", [0, 1])
def test_moe_decode_matches_oracle(down_q6):
    W = MoeWeights(down_q6, 11 + down_q6)
    rng = np.random.RandomState(12)
    x = rng.standard_normal(2048).astype(np.float32)
    logits = torch.empty(257, device=DEV)
    h = torch.full((9, 512), float("nan"), device=DEV)
    ids = torch.empty(8, dtype=torch.int32, device=DEV)
    wts = torch.empty(8, device=DEV)
    out = torch.full((2048,), float("nan"), device=DEV)
    xd = dev(x)
    ok(lib().tk_moe_decode(down_q6, ptr(W.router), ptr(xd), ptr(logits), *W.ptrs(), ptr(h),
                           ptr(ids), ptr(wts), ptr(out)))
    lg = logits.cpu().numpy()
    rw = Q.bf16_to_f64(W.router_np)
    within(lg, rw @ x.astype(np.float64), np.abs(rw) @ np.abs(x.astype(np.float64)), 1e-5)
    ids_np, w_np, h_np = ids.cpu().numpy(), wts.cpu().numpy(), h.cpu().numpy()
    check_routing(lg, ids_np, w_np)
    experts = list(ids_np) + [256]
    for s, e in enumerate(experts):
        check_gate_up(W, x, e, h_np[s])
    ref, mag = np.zeros(2048), np.zeros(2048)
    coef = list(w_np.astype(np.float64)) + [Q.sigmoid(float(lg[256]))]
    for s, e in enumerate(experts):
        r, m = down_ref(W, e, h_np[s])
        ref += coef[s] * r
        mag += abs(coef[s]) * m
    within(out.cpu().numpy(), ref, mag, 2e-5)


@pytest.mark.parametrize("down_q6", [0, 1])
def test_moe_prefill_matches_oracle_and_decode_routing(down_q6):
    W = MoeWeights(down_q6, 21 + down_q6)
    rng = np.random.RandomState(22)
    n = 33
    base = rng.standard_normal(2048)
    x = np.empty((n, 2048), np.float32)
    x[:30] = base + 0.05 * rng.standard_normal((30, 2048))  # most tokens share their experts
    x[30:] = rng.standard_normal((3, 2048))
    L = lib()
    mt = L.tk_moe_max_tasks(n)
    z = lambda *s, dt=torch.float32: torch.zeros(s, dtype=dt, device=DEV)
    xh, xs, logits = z(n, 2048, dt=torch.float16), z(n, 64), z(n, 257)
    wts, ids, order = z(9 * n), z(9 * n, dt=torch.int32), z(9 * n, dt=torch.int32)
    n_tasks, tasks = z(1, dt=torch.int32), z(mt, 4, dt=torch.int32)
    ah, as_, part = z(9 * n, 512, dt=torch.float16), z(9 * n, 32), z(9 * n, 2048)
    out = torch.full((n, 2048), float("nan"), device=DEV)
    xd = dev(x)
    ok(L.tk_moe_prefill(down_q6, ptr(W.router), ptr(xd), n, *W.ptrs(), ptr(xh), ptr(xs),
                        ptr(logits), ptr(wts), ptr(ids), ptr(order), ptr(n_tasks), ptr(tasks),
                        ptr(ah), ptr(as_), ptr(part), ptr(out)))
    lg, ids_np, w_np = logits.cpu().numpy(), ids.cpu().numpy().reshape(n, 9), \
        wts.cpu().numpy().reshape(n, 9)

    # Routing: per token the decode routing, the shared expert as slot 8.
    for t in range(n):
        check_routing(lg[t], ids_np[t], w_np[t])
        assert ids_np[t, 8] == 256
        within(w_np[t, 8:9], np.array([Q.sigmoid(float(lg[t, 256]))]), np.ones(1), 1e-6)

    # The batched router is the decode router: bitwise equal logits, hence identical routing.
    dl = torch.empty(257, device=DEV)
    hd, idd, wd = z(9, 512), z(8, dt=torch.int32), z(8)
    outd = z(2048)
    for t in (0, 17, n - 1):
        ok(L.tk_moe_decode(down_q6, ptr(W.router), ptr(xd[t]), ptr(dl), *W.ptrs(), ptr(hd),
                           ptr(idd), ptr(wd), ptr(outd)))
        assert torch.equal(dl.view(torch.int32), logits[t].view(torch.int32))
        assert torch.equal(idd, ids[9 * t:9 * t + 8])
        d_out = outd.cpu().numpy().astype(np.float64)
        p_out = out[t].cpu().numpy().astype(np.float64)
        assert np.max(np.abs(d_out - p_out)) <= 1e-3 * np.max(np.abs(d_out)) + 1e-6

    # Grouping: a stable sort of the 9 n assignments by expert, cut into tasks of <= 16.
    flat = ids_np.reshape(-1)
    assert np.array_equal(order.cpu().numpy(), np.argsort(flat, kind="stable"))
    want_tasks = []
    start = 0
    for e in range(257):
        c = int((flat == e).sum())
        for q in range(0, c, 16):
            want_tasks.append([e, start + q, min(16, c - q), 0])
        start += c
    nt = int(n_tasks.item())
    assert nt == len(want_tasks) and nt <= mt
    assert np.array_equal(tasks.cpu().numpy()[:nt], np.array(want_tasks))
    assert max(t[2] for t in want_tasks) == 16  # some expert needed more than one task

    # Gate / up per assignment, then the weighted down projections and the slot sum.
    ah_np = ah.cpu().numpy().astype(np.float64)
    sums = ah_np.reshape(9 * n, 32, 16)
    within(as_.cpu().numpy(), sums.sum(axis=2), np.abs(sums).sum(axis=2), 1e-6)
    for a in range(9 * n):
        t, e = a // 9, int(flat[a])
        xa = Q.act_fp16(x[t])
        (wg, mg), (wu, mu) = W.rows("gate", e), W.rows("up", e)
        g, u = wg @ xa, wu @ xa
        hv = Q.silu(g) * u
        eg, eu = 1e-5 * (mg @ np.abs(xa)), 1e-5 * (mu @ np.abs(xa))
        bound = 1.1 * eg * np.abs(u) + np.abs(Q.silu(g)) * eu + 1e-3 * eg * eu + \
            np.abs(hv) * 2.0 ** -11  # ah is rounded to FP16
        within(ah_np[a], hv, bound, 1.0)
    ref, mag = np.zeros((n, 2048)), np.zeros((n, 2048))
    for a in range(9 * n):
        t, e = a // 9, int(flat[a])
        r, m = down_ref(W, e, ah_np[a])
        ref[t] += float(w_np.reshape(-1)[a]) * r
        mag[t] += abs(float(w_np.reshape(-1)[a])) * m
    within(out.cpu().numpy(), ref, mag, 2e-5)
