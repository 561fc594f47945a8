"""The decode scratch contract of include/miso_cuda.h, checked without a GPU: the scratch may hold
anything when a call starts (a call whose kernel gave up on a bounded wait leaves arrival
counters set), because every miso_attn_decode call zeroes the counters it uses on its own stream
before its kernel; a scratch that cannot hold them is rejected before the device is touched.
The GPU side of the same contract (a call after counters were left set gives the oracle's
result) is tests/test_gpu_attention.py::test_fast_decode_ignores_leftover_counters_in_scratch."""
import ctypes as C
import os
import re

from miso_b200 import _capi as capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CAPI = os.path.join(ROOT, "miso_b200", "csrc", "capi.cu")
HEADER = os.path.join(ROOT, "include", "miso_cuda.h")


def function_body(src: str, name: str) -> str:
    start = src.index(f"int {name}(")
    depth, i = 0, src.index("{", start)
    for j in range(i, len(src)):
        depth += {"{": 1, "}": -1}.get(src[j], 0)
        if depth == 0:
            return src[i:j + 1]
    raise AssertionError(f"unterminated {name}")


def test_header_states_any_contents_and_the_per_call_reset():
    text = " ".join(open(HEADER).read().split())
    assert "256-byte aligned, any contents" in text
    assert "every call first zeroes the 2 * batch arrival counters" in text


def test_every_decode_call_zeroes_its_counters_before_the_kernel():
    """The allocating entry point and the no-allocation one both clear the counters on the
    caller's stream ahead of the decode kernel, with no early return in between."""
    src = open(CAPI).read() + open(os.path.join(ROOT, "miso_b200", "csrc",
                                                  "decode_noalloc.cu")).read()
    for name in ("miso_attn_decode", "miso_attn_decode_noalloc"):
        body = function_body(src, name)
        memset = re.search(r"cudaMemsetAsync\(\s*(\w+)\s*,\s*0\s*,", body)
        assert memset, f"{name}: no counter reset"
        launch = body.find("decode_kernel<<<")
        if launch < 0:  # the no-allocation entry point forwards to the shared launcher
            launch = body.rfind("return")
        assert memset.start() < launch, f"{name}: the reset must precede the launch"
        between = body[memset.end():launch]
        assert "return MISO_OK" not in between


def test_decode_rejects_scratch_it_cannot_use_before_touching_the_device():
    lib = capi.load()
    buf = (C.c_uint8 * 4096)()
    base = C.addressof(buf)
    aligned = (base + 255) & ~255
    q = (C.c_float * 16)()
    lens = (C.c_int32 * 1)(1)
    rows = (C.c_int64 * 2)(0, 1)
    pool = (C.c_uint16 * 1024)()
    pool_p = (C.addressof(pool) + 15) & ~15
    p = capi.AttnDecodeParams(C.addressof(q), C.addressof(q), pool_p, pool_p, C.addressof(rows),
                              C.addressof(lens), C.addressof(q), 2, 1, 8192)
    for scratch in (None, aligned + 8):  # missing, or not 256-byte aligned
        assert lib.miso_attn_decode(C.byref(p), scratch, 4096, None) == -1
