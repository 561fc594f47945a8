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
