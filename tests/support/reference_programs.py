"""Shared by the CPU and GPU tests of the reference's own engine and test programs built against
this package's drop-in headers (miso_b200/reference_engine.py): where the reference checkout and
the built programs are, and which doctest cases each program runs without the model file."""
import importlib.util
import os
import re
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
REFERENCE = Path(os.environ.get("MISO_REFERENCE_DIR", str(ROOT.parent / "reference")))
BIN = ROOT / "_build" / "reference_engine" / "bin"


def recipe():
    """The build recipe, imported by path (importing the package itself loads the CUDA library)."""
    spec = importlib.util.spec_from_file_location(
        "miso_reference_engine", ROOT / "miso_b200" / "reference_engine.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def have_reference() -> bool:
    return (REFERENCE / "src" / "engine" / "model.hip").exists()


# Programs whose every case is gated on the model file (doctest::skip when it is absent).
GGUF_GATED = ["test_attention", "test_deltanet", "test_prefill", "test_model", "test_fused_gemv",
              "test_gemv_dispatch", "test_norm_embed"]

# Programs with cases that need neither the model nor the reference's fixture directory:
# name -> (doctest arguments, number of cases that must pass).
SELF_CONTAINED = {
    # The first case asserts the reference's own card (gfx906, 60 CUs, 64-lane waves); the others
    # check hip_util.hpp's DeviceBuffer and error reporting.
    "test_device": (["--test-case-exclude=*MI50*"], 2),
    "test_axpy": ([], 2),
    "test_attn_splitk": ([], 5),
    "test_deltanet_chunk": ([], 1),
    "test_qgemm": (["--test-case=GEMM activation prep*"], 1),
}


def run(name: str, args: list[str], timeout: float = 600.0) -> tuple[int, str, dict]:
    """Runs a built program; returns (exit code, output, doctest's test-case summary counts)."""
    r = subprocess.run([str(BIN / name)] + args, capture_output=True, text=True, timeout=timeout)
    out = r.stdout + r.stderr
    m = re.search(r"test cases:\s*(\d+)\s*\|\s*(\d+) passed\s*\|\s*(\d+) failed\s*\|\s*(\d+) skipped",
                  out)
    counts = dict(zip(("total", "passed", "failed", "skipped"), map(int, m.groups()))) if m else {}
    return r.returncode, out, counts
