"""The reference's own test programs, built unchanged against the drop-in headers
(miso_b200/reference_engine.py), pass on the B200: the split-K decode / combine / causal prefill
cases of tests/test_attn_splitk.hip, the chunked delta rule of tests/test_deltanet_chunk.hip, the
axpy operator contract and the GEMM activation prep of tests/test_qgemm.hip — every case that needs
neither the model file nor the reference's fixture directory. The programs are built where the
reference checkout is (the build step) and travel with the repository; without them this skips."""
import pytest

from support import reference_programs as rp

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(rp.SELF_CONTAINED))
def test_reference_program_passes(name):
    if not (rp.BIN / name).exists():
        pytest.skip("reference programs not built (the build step needs the reference checkout)")
    args, want = rp.SELF_CONTAINED[name]
    rc, out, counts = rp.run(name, args)
    assert rc == 0, out[-4000:]
    assert counts["failed"] == 0 and counts["passed"] >= want, out[-2000:]


@pytest.mark.parametrize("name", rp.GGUF_GATED)
def test_gguf_gated_reference_program_runs(name):
    if not (rp.BIN / name).exists():
        pytest.skip("reference programs not built (the build step needs the reference checkout)")
    rc, out, counts = rp.run(name, [])
    assert rc == 0 and counts["failed"] == 0, out[-4000:]
