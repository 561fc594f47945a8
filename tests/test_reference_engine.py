"""The reference's engine (src/engine), its CLI and its kernel test programs compile and link
UNCHANGED as CUDA for sm_100a against this package's drop-in headers (miso_b200/reference_engine.py
builds them from the reference checkout; their GGUF-gated cases skip without the model file, as in
the reference's own CI). No GPU is needed: the programs are only listed and run to their skips."""
import pytest

from support import reference_programs as rp

pytestmark = pytest.mark.skipif(not rp.have_reference(),
                                reason="needs a checkout of the reference's sources")


@pytest.fixture(scope="module")
def built():
    return rp.recipe().build(rp.REFERENCE)


def test_engine_cli_and_tests_build(built):
    recipe = rp.recipe()
    assert set(built) == set(recipe.TESTS) | {"miso"} | set(recipe.BENCHES) | \
        {f"synthetic/{n}" for n in recipe.SYNTHETIC_TESTS}
    for name, path in built.items():
        assert path.exists() and path.stat().st_size > 0, name
    # The engine-level tests that link the whole engine library.
    for name in ("test_attention", "test_deltanet", "test_prefill"):
        assert name in built


@pytest.mark.parametrize("name", sorted(rp.recipe().TESTS) +
                         [f"synthetic/{n}" for n in rp.recipe().SYNTHETIC_TESTS])
def test_program_lists_its_cases(built, name):
    rc, out, _ = rp.run(name, ["--list-test-cases"], timeout=60)
    assert rc == 0, out[-2000:]
    assert "test cases passing the current filters" in out


@pytest.mark.parametrize("name", rp.GGUF_GATED)
def test_gguf_gated_programs_skip_cleanly_without_the_model(built, name):
    rc, out, counts = rp.run(name, [], timeout=120)
    assert rc == 0, out[-2000:]
    assert counts["failed"] == 0 and counts["skipped"] >= 1 and counts["passed"] == 0, out[-1000:]


def test_cli_prints_usage(built):
    import subprocess
    r = subprocess.run([str(built["miso"]), "--help"], capture_output=True, text=True, timeout=60)
    assert "usage: miso" in (r.stdout + r.stderr)


def test_synthetic_model_matches_the_reference_models_tensor_manifest(tmp_path):
    """The synthetic model the model-level GPU tests use has the real model's tensor names, GGML
    types and shapes (the reference's tests/fixtures/ornith-q4km-tensors.tsv), with the expert
    count and vocabulary scaled down here to keep the file small."""
    gguf = pytest.importorskip("gguf")
    manifest = rp.REFERENCE / "tests" / "fixtures" / "ornith-q4km-tensors.tsv"
    from support import synthetic_model as S
    S.write(str(tmp_path / "m.gguf"), str(tmp_path / "g"), vocab=512, experts=2)
    want = {}
    for line in manifest.read_text().splitlines():
        if line.startswith("#"):
            continue
        name, ty, dims = line.split("\t")[:3]
        want[name] = (int(ty), [int(v) for v in dims.split(",")])
    got = {t.name: (int(t.tensor_type), [int(v) for v in t.shape])
           for t in gguf.GGUFReader(str(tmp_path / "m.gguf")).tensors}
    assert len(got) == 93
    for name, (ty, dims) in got.items():
        wt, wd = want[name]
        if name.endswith("_exps.weight") or name.endswith("ffn_gate_inp.weight"):
            wd = wd[:-1] + [2]
        if name in ("token_embd.weight", "output.weight"):
            wd = wd[:-1] + [512]
        assert (ty, dims) == (wt, wd), name
    g = gguf.GGUFReader(str(tmp_path / "g" / "ornith-layers.gguf"))
    assert "golden.token_ids" in g.fields and "golden.continuation_ids" in g.fields


@pytest.mark.parametrize("kind,k", [("q4k", 2048), ("q4k", 4096), ("q6k", 512), ("q6k", 2048)])
def test_synthetic_weights_have_unit_variance_projections(kind, k):
    """The synthetic model's weights: standard deviation ~ 1 / sqrt(k) and mean ~ 0, so each
    projection maps unit-variance inputs to roughly unit-variance outputs."""
    import numpy as np
    from oracle import quant as Q
    from support import synthetic_model as S
    rng = np.random.RandomState(k)
    raw = S._q4k(rng, 64, k) if kind == "q4k" else S._q6k(rng, 64, k)
    w = (Q.q4k_dequant(raw) if kind == "q4k" else Q.q6k_dequant(raw)).astype(np.float64)
    assert 0.7 < w.std() * np.sqrt(k) < 1.4
    assert abs(w.mean()) < 0.1 * w.std()
