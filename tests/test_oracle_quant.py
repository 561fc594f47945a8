"""Pins the numpy restatement of the weight formats (oracle/quant.py) before it checks any
kernel: bit-exact against the reference's own fixture dequantisations (tests/fixtures/tiny.gguf
and tiny.q4_k.f32 / tiny.q6_k.f32, produced by gguf-py), against gguf-py's dequantize on random
blocks, and against the reference's repack / dequant code compiled from its sources
(oracle/_ref). Also the routing and activation helpers on hand-made cases."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle
from oracle import quant as Q

FIXTURES = os.path.join(oracle.REF, "tests", "fixtures")


def fixture_tensor(name):
    gguf = pytest.importorskip("gguf")
    path = os.path.join(FIXTURES, "tiny.gguf")
    if not os.path.exists(path):
        pytest.skip("needs the reference's fixture directory")
    for t in gguf.GGUFReader(path).tensors:
        if t.name == name:
            return np.asarray(t.data, np.uint8), [int(v) for v in t.shape]
    raise KeyError(name)


def golden(name):
    return np.fromfile(os.path.join(FIXTURES, f"tiny.{name}.f32"), dtype="<f4")


def test_q4k_dequant_equals_the_reference_fixture_bitwise():
    raw, shape = fixture_tensor("q4_k")
    got = Q.q4k_dequant(raw).reshape(-1)
    want = golden("q4_k")
    assert shape == [8192, 2] and got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q6k_dequant_equals_the_reference_fixture_bitwise():
    raw, shape = fixture_tensor("q6_k")
    got = Q.q6k_dequant(raw).reshape(-1)
    want = golden("q6_k")
    assert shape == [4096, 4] and got.shape == want.shape
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("kind", ["q4_k", "q6_k"])
def test_dequant_equals_gguf_py_on_random_blocks(kind):
    gguf = pytest.importorskip("gguf")
    rng = np.random.RandomState(5)
    if kind == "q4_k":
        raw, qt, f = Q.random_q4k(rng, 16, 2048), gguf.GGMLQuantizationType.Q4_K, Q.q4k_dequant
    else:
        raw, qt, f = Q.random_q6k(rng, 16, 2048), gguf.GGMLQuantizationType.Q6_K, Q.q6k_dequant
    want = np.asarray(gguf.quants.dequantize(raw, qt), np.float32)
    assert np.array_equal(f(raw).view(np.uint32), want.view(np.uint32))


def ref_lib():
    lib = oracle.ref_quant()
    if lib is None:
        pytest.skip("the reference's weight-format code was not built (oracle/_ref)")
    return lib


@pytest.mark.parametrize("kind,type_id", [("q4_k", 12), ("q6_k", 14)])
def test_dequant_equals_the_reference_code(kind, type_id):
    lib = ref_lib()
    rng = np.random.RandomState(6)
    raw = Q.random_q4k(rng, 8, 4096) if kind == "q4_k" else Q.random_q6k(rng, 8, 4096)
    want = np.empty(8 * 4096, np.float32)
    assert lib.ref_dequant(type_id, raw.ctypes.data, raw.nbytes, want.ctypes.data, want.size) == 0
    got = (Q.q4k_dequant if kind == "q4_k" else Q.q6k_dequant)(raw).reshape(-1)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q4k_r1_repack_equals_the_reference_code():
    lib = ref_lib()
    rng = np.random.RandomState(7)
    for raw in (Q.random_q4k(rng, 4, 2048), fixture_tensor("q4_k")[0]):
        raw = np.ascontiguousarray(raw)
        want = np.empty_like(raw)
        assert lib.ref_repack_q4k(raw.ctypes.data, raw.nbytes, want.ctypes.data) == 0
        assert np.array_equal(Q.q4k_repack_r1(raw), want)


@pytest.mark.parametrize("k", [512, 2048, 4096])
def test_q6k_r1_repack_equals_the_reference_code(k):
    lib = ref_lib()
    rng = np.random.RandomState(k)
    raw = Q.random_q6k(rng, 3, k)
    rb = Q.q6k_r1_row_bytes(k)
    assert lib.ref_q6k_r1_row_bytes(k) == rb
    want = np.empty((3, rb), np.uint8)
    assert lib.ref_repack_q6k(raw.ctypes.data, raw.nbytes, k, want.ctypes.data, want.nbytes) == 0
    assert np.array_equal(Q.q6k_repack_r1(raw, k), want)


def test_r1_layouts_invert_back_to_gguf():
    rng = np.random.RandomState(9)
    g4 = Q.random_q4k(rng, 5, 2048)
    assert np.array_equal(Q.q4k_r1_to_gguf(Q.q4k_repack_r1(g4)), g4)
    r1 = rng.randint(0, 256, size=(7, 144 * 8)).astype(np.uint8)  # any r1 bytes are valid
    assert np.array_equal(Q.q4k_repack_r1(Q.q4k_r1_to_gguf(r1)), r1)
    g6 = Q.random_q6k(rng, 5, 512)
    assert np.array_equal(Q.q6k_r1_to_gguf(Q.q6k_repack_r1(g6, 512), 512), g6)


def test_moe_topk_orders_ties_by_index_and_renormalises():
    l = np.full(257, -5.0)
    l[[3, 7, 9, 200]] = 2.0       # a four-way tie at the top
    l[[1, 50, 60, 70, 80]] = 1.0  # a five-way tie for the last four places
    ids, w = Q.moe_topk(l)
    assert list(ids) == [3, 7, 9, 200, 1, 50, 60, 70]
    assert abs(w.sum() - 1.0) < 1e-12
    assert np.allclose(w[:4], np.e / (4 * np.e + 4)) and np.allclose(w[4:], 1 / (4 * np.e + 4))


def test_int8_activation_format_bound():
    x = np.random.RandomState(8).standard_normal(4096)
    q = Q.act_int8(x)
    amax = np.abs(x.reshape(-1, 32)).max(axis=1).repeat(32)
    assert np.all(np.abs(q - x) <= 0.5 * amax / 127 * (1 + 1e-6))
