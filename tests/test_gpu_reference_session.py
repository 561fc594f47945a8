"""The reference's own model-level tests, built unchanged against the drop-in headers, pass on
the B200 on a synthetic model with the reference model's architecture and tensor layout
(tests/support/synthetic_model.py: 4 layers — 3 Gated DeltaNet + 1 gated attention, each with the
256-expert MoE — plus the per-layer tensors of layers 5 and 11, random weights):
  * tests/test_prefill.hip: chunked prefill (chunks of n, 7 and 1 tokens) leaves the same
    logits, KV cache, conv and recurrent state as token-by-token decode, every chunking is
    bitwise identical to the one-chunk prefill, one more decode step agrees, and ingest picks
    decode below the prefill threshold and prefill at it;
  * tests/test_fused_gemv.hip, test_gemv_dispatch.hip: fused / mixed-type projection GEMVs equal
    the separate kernels bit for bit;
  * tests/test_load_stage.hip: staged weight uploads are byte-identical to plain ones.
The whole decode and prefill of the engine (embedding, DeltaNet and attention mixers, MoE, LM
head, argmax) runs on this repository's kernels. The model file (~2.2 GB) is written next to the
built programs for the run and removed afterwards."""
import shutil
import sys

import pytest

from support import reference_programs as rp

pytestmark = pytest.mark.gpu

EXPECT = {"test_prefill": 2, "test_fused_gemv": 3, "test_gemv_dispatch": 2, "test_load_stage": 2}


@pytest.fixture(scope="module")
def model():
    if not all((rp.BIN / "synthetic" / n).exists() for n in EXPECT):
        pytest.skip("reference programs not built (the build step needs the reference checkout)")
    paths = rp.recipe().synthetic_paths()
    created = not paths["model"].exists()
    if created:
        from support import synthetic_model
        paths["dir"].mkdir(parents=True, exist_ok=True)
        synthetic_model.write(str(paths["model"]), str(paths["golden"]))
    yield paths
    if created:
        shutil.rmtree(paths["dir"], ignore_errors=True)


@pytest.mark.parametrize("name", sorted(EXPECT))
def test_reference_model_level_program_passes(model, name):
    rc, out, counts = rp.run(f"synthetic/{name}", [], timeout=900)
    sys.stdout.write(out[-3000:])
    assert rc == 0, out[-4000:]
    assert counts["failed"] == 0 and counts["skipped"] == 0, out[-2000:]
    assert counts["passed"] == EXPECT[name], out[-2000:]
