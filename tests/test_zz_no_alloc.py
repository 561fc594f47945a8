"""miso_attn_decode_noalloc: the batched decode for callers that cannot allocate device memory.

Some callers of this library may not allocate device memory themselves. Examples are a serving
framework that reserves nearly all of the GPU's memory for its own pool, a plugin inside such a
host that only receives the tensors it works on, and a latency-critical loop that cannot take
cudaMalloc's implicit synchronisation. The no-allocation entry point takes only inputs and
outputs and uses a fixed scratch array inside the library. This test calls it through the C ABI
and checks its output against miso_attn_decode, which uses caller-allocated scratch, within the
decode tests' tolerance (relative L2 <= 1e-5 per head). It does this on two calls in a row, so
the second call meets the first call's leftovers in the shared array. It also checks that a batch
beyond the fixed limit is refused with MISO_ERR_LIMIT.

Only calls that succeed are covered. Each call also zeroes the shared counters before its kernel,
which matters after a call whose kernel gave up on a bounded wait; no call here is made to give
up, so that zeroing is not exercised (a successful call leaves the counters at zero anyway). The
same zeroing in miso_attn_decode is tested with planted leftovers in test_gpu_attention.py.

The file name sorts last so that a run stopping at the first failure has already run every other
test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from miso_b200 import _capi as capi
from miso_b200 import attention as A

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def rel_per_head(got, ref):
    got = np.asarray(got, np.float64).reshape(-1, 256)
    ref = np.asarray(ref, np.float64).reshape(-1, 256)
    num = np.sqrt(((got - ref) ** 2).sum(1))
    den = np.sqrt((ref ** 2).sum(1))
    return float(np.max(num / np.maximum(den, 1e-300)))


def params(pool, q, qg, core):
    return capi.AttnDecodeParams(q.data_ptr(), qg.data_ptr(), pool.k.data_ptr(),
                                 pool.v.data_ptr(), pool.kv_row.data_ptr(), pool.lens.data_ptr(),
                                 core.data_ptr(), pool.rows, pool.batch, 16 * 512)


def test_noalloc_decode_matches_allocating_decode_on_two_calls():
    lib = capi.load()
    rng = np.random.RandomState(2024)
    lens = rng.randint(1, 6000, size=24).astype(np.int32)
    lens[5] = 0
    lens[11] = 64
    pool = A.KvPool(len(lens), 6016, device=DEV)
    pool.k.copy_(torch.from_numpy(rng.standard_normal((pool.rows, 256)).astype(np.float16)))
    pool.v.copy_(torch.from_numpy(rng.standard_normal((pool.rows, 256)).astype(np.float16)))
    pool.lens.copy_(torch.from_numpy(lens))
    scratch = A.decode_scratch(pool.batch, device=DEV)
    for call in range(2):
        q = torch.from_numpy((2 * rng.standard_normal((pool.batch, 16, 256)))
                             .astype(np.float32)).to(DEV)
        qg = torch.from_numpy(rng.standard_normal((pool.batch, 16, 512))
                              .astype(np.float32)).to(DEV)
        ref = torch.full((pool.batch, 16, 256), 5.0, device=DEV)
        got = torch.full((pool.batch, 16, 256), -5.0, device=DEV)
        p_ref = params(pool, q, qg, ref)
        capi.check("miso_attn_decode",
                   lib.miso_attn_decode(C.byref(p_ref), scratch.data_ptr(),
                                        scratch.numel() * 4, None))
        p = params(pool, q, qg, got)
        capi.check("miso_attn_decode_noalloc", lib.miso_attn_decode_noalloc(C.byref(p), None))
        torch.cuda.synchronize()
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        live = lens > 0
        assert rel_per_head(g[live], r[live]) <= 1e-5, f"call {call}"
        assert np.all(g[~live] == 0.0) and np.all(r[~live] == 0.0), f"call {call}"
    st = C.c_int(-1)
    assert lib.miso_device_status(1, C.byref(st)) == 0 and st.value == 0


def test_noalloc_decode_refuses_batches_beyond_its_limit():
    lib = capi.load()
    pool = A.KvPool(257, 64, device=DEV)
    pool.lens.fill_(1)
    q = torch.zeros((257, 16, 256), device=DEV)
    qg = torch.zeros((257, 16, 512), device=DEV)
    core = torch.zeros((257, 16, 256), device=DEV)
    p = params(pool, q, qg, core)
    assert lib.miso_attn_decode_noalloc(C.byref(p), None) == -5  # MISO_ERR_LIMIT
