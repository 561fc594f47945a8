"""The C ABI without a GPU: the library loads, exports every declared symbol, its ctypes mirror
matches the C header layout, pure host functions give the reference's answers, and invalid
arguments are rejected before anything touches the device."""
import ctypes as C
import os
import re
import subprocess
import tempfile

import pytest

import miso_b200
from miso_b200 import _capi as capi
import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "miso_cuda.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(miso_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    lib = capi.load()
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
        assert name in capi.SIGNATURES, f"{name} has no ctypes signature"


def test_ctypes_structs_match_the_c_header():
    """Compiles a probe against include/miso_cuda.h and compares sizes and field offsets."""
    structs = {
        "miso_attn_prep_params": capi.AttnPrepParams,
        "miso_attn_prep_batch_params": capi.AttnPrepBatchParams,
        "miso_attn_split_params": capi.AttnSplitParams,
        "miso_attn_combine_params": capi.AttnCombineParams,
        "miso_attn_prefill_params": capi.AttnPrefillParams,
        "miso_deltanet_step_params": capi.DeltaNetStepParams,
        "miso_deltanet_seq_params": capi.DeltaNetSeqParams,
        "miso_deltanet_conv_params": capi.DeltaNetConvParams,
        "miso_deltanet_chunk_params": capi.DeltaNetChunkParams,
        "miso_attn_decode_params": capi.AttnDecodeParams,
        "miso_attn_prep_batched_params": capi.AttnPrepBatchedParams,
        "miso_attn_prefill_tc_params": capi.AttnPrefillTcParams,
        "miso_deltanet_step_batched_params": capi.DeltaNetStepBatchedParams,
    }
    lines = ['#include <stdio.h>', '#include <stddef.h>', f'#include "{HEADER}"', "int main(){"]
    for cname, py in structs.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "probe.c"), os.path.join(d, "probe")
        open(src, "w").write("\n".join(lines))
        subprocess.run(["gcc", "-std=c11", "-o", exe, src], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    seen = 0
    for line in out.splitlines():
        cname, field, value = line.split()
        py = structs[cname]
        want = C.sizeof(py) if field == "size" else getattr(py, field).offset
        assert int(value) == want, (cname, field)
        seen += 1
    assert seen == sum(len(p._fields_) + 1 for p in structs.values())


@pytest.mark.parametrize("length", [0, 1, 31, 32, 33, 257, 288, 1000, 3872, 4096, 5000, 16384,
                                    32767, 32768, 32769, 131072])
@pytest.mark.parametrize("max_splits", [3, 16, 60, 120])
def test_n_splits_matches_oracle(length, max_splits):
    got = miso_b200.attention.n_splits(length, max_splits)
    assert got == oracle.attn_n_splits(length, max_splits)


def test_n_splits_known_answers_through_the_abi():
    # tests/test_attn_splitk.hip:285-290
    for length, want in [(3872, 21), (33, 2), (4096, 22), (16384, 57), (288, 9)]:
        assert miso_b200.attention.n_splits(length, 60) == want


def test_prefill_items():
    for n in [1, 3, 4, 5, 33, 512]:
        assert miso_b200.attention.prefill_items(n) == 2 * ((n + 3) // 4)


def test_invalid_arguments_are_rejected_without_a_device():
    lib = capi.load()
    assert lib.miso_attn_decode(None, None, 0, None) == -1
    p = capi.AttnDecodeParams()
    assert lib.miso_attn_decode(C.byref(p), None, 0, None) == -1
    assert lib.miso_attn_split(None, None) == -1
    sp = capi.AttnSplitParams(1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 1 << 20, 10, 5, 1)
    assert lib.miso_attn_split(C.byref(sp), None) == -1  # len > max_ctx
    assert lib.miso_attn_combine(None, None) == -1
    assert lib.miso_attn_prefill(None, None) == -1
    assert lib.miso_deltanet_step(None, None) == -1
    assert lib.miso_deltanet_seq(None, None) == -1
    assert lib.miso_deltanet_chunk(None, None) == -1
    assert lib.miso_attn_prep_batched(None, None) == -1
    assert lib.miso_deltanet_step_batched(None, None) == -1
    assert lib.miso_attn_prefill_tc(None, None) == -1
    assert lib.miso_deltanet_prefill_tc(None, None, 0, None) == -1
    assert lib.miso_deltanet_prefill_tc_scratch_bytes(0) == 0
    sb = lib.miso_deltanet_prefill_tc_scratch_bytes(8192)
    assert sb >= 8192 * 16384 + 3 * 32 * 128 * 8192  # fp16 q/k/v and the three chunk tiles
    # conv_in == conv_out and a short scratch are refused before any device work.
    fake = 1 << 20
    dp = capi.DeltaNetSeqParams(fake, fake, fake, fake, fake, fake, fake, fake, fake, fake, fake,
                                fake, 64, 1e-6, 4160, 8192)
    assert lib.miso_deltanet_prefill_tc(C.byref(dp), fake, 1 << 30, None) == -1
    for stage in (lib.miso_deltanet_prefill_tc_front, lib.miso_deltanet_prefill_tc_recur):
        assert stage(None, fake, 1 << 30, None) == -1
        assert stage(C.byref(dp), fake, 1 << 30, None) == -1
    dp.conv_out = fake * 2
    assert lib.miso_deltanet_prefill_tc(C.byref(dp), fake, 1024, None) == -2
    for stage in (lib.miso_deltanet_prefill_tc_front, lib.miso_deltanet_prefill_tc_recur):
        assert stage(C.byref(dp), fake, 1024, None) == -2  # the same scratch contract
    # Speculative verification: checkpoints are required; commit refuses k_accepted > n and null
    # buffers, and with k_accepted = 0 it leaves everything as it was (no device work).
    assert lib.miso_deltanet_seq_ckpt(None, fake, fake, None) == -1
    assert lib.miso_deltanet_seq_ckpt(C.byref(dp), None, fake, None) == -1
    assert lib.miso_deltanet_seq_ckpt(C.byref(dp), fake, None, None) == -1
    assert lib.miso_deltanet_seq_ckpt(C.byref(dp), fake + 4, fake, None) == -1  # unaligned
    assert lib.miso_deltanet_commit(fake, fake, 3, 4, fake, fake, None) == -1
    assert lib.miso_deltanet_commit(None, fake, 3, 1, fake, fake, None) == -1
    assert lib.miso_deltanet_commit(fake, fake, 3, 1, fake, None, None) == -1
    assert lib.miso_deltanet_commit(fake, fake, 3, 0, fake, fake, None) == 0
    st = C.c_int(0)
    assert lib.miso_device_status(0, None) == -1
    assert st.value == 0


def test_version_string():
    assert b"sm_100a" in capi.load().miso_version()
