"""Builds penta2himajin/miso's own engine, CLI and kernel test programs — their sources unchanged,
where they lie in a checkout of the reference — as CUDA for sm_100a against this package's
drop-in headers: `csrc/compat` (the HIP runtime names the sources use, `hip_util.hpp`) and
`csrc/kernels` (every kernel header the engine includes). The reference's host library
(`src/gguf.cpp`, `dequant.cpp`, `repack.cpp`, `unicode.cpp`, `tokenizer.cpp`) is plain C++ and
is compiled with g++.

This is the proof that the engine drops in unchanged (the reference builds the same targets with
its CMakeLists.txt:64-80 and tests/CMakeLists.txt:1-58; this recipe does not run that build
system). Outputs go to `<out>/bin` (executables) and `<out>/obj`; a stamp of the inputs and flags
skips a rebuild when nothing changed.

    python -m miso_b200.reference_engine <reference checkout> [<out dir>]
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
DEFAULT_OUT = HERE.parent / "_build" / "reference_engine"

HOST_SOURCES = ["gguf", "dequant", "repack", "unicode", "tokenizer"]
ENGINE_SOURCES = ["weights", "deltanet", "attention", "moe", "model"]

# Test programs built (tests/CMakeLists.txt:18-58): name -> (sources, links the engine library).
TESTS = {
    "test_device": (["test_device.hip"], False),
    "test_axpy": (["test_axpy.hip"], False),
    "test_attn_splitk": (["test_attn_splitk.hip"], False),
    "test_deltanet_chunk": (["test_deltanet_chunk.hip"], False),
    "test_qgemm": (["test_qgemm.hip"], False),
    "test_q4k_gemv": (["test_q4k_gemv.hip"], False),
    "test_q6k_gemv": (["test_q6k_gemv.hip"], False),
    "test_norm_embed": (["test_norm_embed.hip"], False),
    "test_attention": (["test_attention.hip"], True),
    "test_deltanet": (["test_deltanet.hip"], True),
    "test_prefill": (["test_prefill.hip"], True),
    "test_model": (["test_model.hip"], True),
    "test_fused_gemv": (["test_fused_gemv.hip"], True),
    "test_gemv_dispatch": (["test_gemv_dispatch.hip"], True),
    "test_load_stage": (["test_load_stage.hip"], True),
}

# The reference's benchmarks (bench/CMakeLists.txt:12-35): name -> source under bench/. The
# per-layer decode benchmarks (bench_attention, bench_deltanet) take the model file as their first
# argument.
BENCHES = {  # name -> (source, links the engine library), as bench/CMakeLists.txt links them
    "bench_attention": ("attention/bench_attention.hip", True),
    "bench_deltanet": ("deltanet/bench_deltanet.hip", True),
    "bench_combine": ("attention/bench_combine.hip", False),
    "bench_q4k_gemv": ("gemv/bench_q4k_gemv.hip", False),
    "bench_q6k_gemv": ("gemv/bench_q6k_gemv.hip", False),
    "bench_qgemm": ("gemm/bench_qgemm.hip", False),
    "bench_norm": ("norm/bench_norm.hip", False),
    "bench_norm_chain": ("norm/bench_model_chain.hip", True),
    "bench_moe": ("moe/bench_moe.hip", True),
    "bench_decode": ("model/bench_decode.hip", True),
}

# Benchmarks not built, and why.
BENCHES_NOT_BUILT = {
    "bench_moe_coefficients": "compares against a frozen copy of the reference MoE kernel that "
                              "uses its private q4k_detail helpers",
    "bench_activation_prepare": "gfx906 DPP code (bench/deltanet/activation_prepare.hpp)",
}

# Test programs of the reference that are not built, and why.
NOT_BUILT = {
    "test_moe": "calls the reference kernels' private helpers (kernels::moe_topk, "
                "q4k_detail::SlotAct / load_slot) to compare against frozen copies of them",
    "test_moe_down_staging": "calls the private moe_detail::Down<> staging of the reference's "
                             "MoE down kernel",
    "test_deltanet_prepare": "includes bench/deltanet/activation_prepare.hpp, gfx906 DPP code",
}

# Model-level test programs that compare the engine with itself (prefill vs token-by-token decode,
# fused vs separate GEMVs, staged vs plain uploads). They are built a second time, into
# bin/synthetic/, reading a synthetic model with the reference model's architecture and tensor
# layout (tests/support/synthetic_model.py writes it to <out>/../synthetic_model/ where these
# paths point).
SYNTHETIC_TESTS = ["test_prefill", "test_fused_gemv", "test_gemv_dispatch", "test_load_stage"]

# The model file the GGUF-gated test cases look for (the reference's CMake default,
# CMakeLists.txt:83-85). Those cases skip themselves when it is absent.
DEFAULT_GGUF = os.environ.get(
    "MISO_ORNITH_GGUF",
    "/home/penta/llm-mi50/models/ornith-1.5-35b-a3b/Ornith-1.5-35B-Q4_K_M.gguf")

NVCC_FLAGS = ["-std=c++20", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-lineinfo"]


def _run(cmd: list[str]) -> tuple[int, str]:
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.returncode, (r.stdout + r.stderr)


def _stamp(ref: Path) -> str:
    h = hashlib.sha256()
    for p in sorted((CSRC / "compat").rglob("*")) + sorted((CSRC / "kernels").glob("*")):
        if p.is_file():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    for p in sorted((ref / "src").rglob("*")) + sorted((ref / "tests").glob("*.h*")) + \
            sorted((ref / "tests").glob("*.cpp")) + [ref / "bench" / s for s, _ in BENCHES.values()]:
        if p.is_file():
            h.update(str(p.relative_to(ref)).encode())
            h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS + [DEFAULT_GGUF] + SYNTHETIC_TESTS + list(BENCHES)).encode())
    return h.hexdigest()


def synthetic_paths(out: Path = DEFAULT_OUT) -> dict[str, Path]:
    """Where the synthetic model and its prompt file live for the bin/synthetic/ programs."""
    base = Path(out).resolve().parent / "synthetic_model"
    return {"dir": base, "model": base / "model.gguf", "golden": base / "golden"}


def build(ref: str | Path, out: str | Path = DEFAULT_OUT, jobs: int | None = None,
          verbose: bool = False) -> dict[str, Path]:
    """Compiles and links the engine library, the CLI (`miso`) and the test programs of TESTS.
    Returns {target name: executable path}. Raises RuntimeError with the compiler output of the
    first failure."""
    ref, out = Path(ref).resolve(), Path(out).resolve()
    obj, binp = out / "obj", out / "bin"
    obj.mkdir(parents=True, exist_ok=True)
    binp.mkdir(parents=True, exist_ok=True)
    targets = {name: binp / name for name in list(TESTS) + ["miso"]}
    targets.update({f"synthetic/{name}": binp / "synthetic" / name for name in SYNTHETIC_TESTS})
    targets.update({name: binp / name for name in BENCHES})
    (binp / "synthetic").mkdir(exist_ok=True)
    (obj / "synthetic").mkdir(exist_ok=True)
    synth = synthetic_paths(out)
    stamp = _stamp(ref)
    stamp_file = out / "stamp"
    if stamp_file.exists() and stamp_file.read_text() == stamp and \
            all(p.exists() for p in targets.values()):
        return targets

    inc = [f"-I{CSRC / 'compat'}", f"-I{CSRC / 'kernels'}", f"-I{ref / 'src'}",
           f"-I{ref / 'third_party'}"]
    defs = [f'-DMISO_FIXTURE_DIR="{ref / "tests" / "fixtures"}"',
            f'-DMISO_GOLDEN_DIR="{ref / "tests" / "golden"}"',
            f'-DMISO_ORNITH_GGUF="{DEFAULT_GGUF}"']
    nvcc = ["nvcc"] + NVCC_FLAGS + ["-x", "cu"] + inc + defs
    gxx = ["g++", "-std=c++20", "-O2", f"-I{ref / 'src'}"]

    compiles: list[tuple[str, list[str]]] = []
    for s in HOST_SOURCES:  # the reference compiles these with -ffp-contract=off
        compiles.append((s, gxx + ["-ffp-contract=off", "-c", str(ref / "src" / f"{s}.cpp"),
                                   "-o", str(obj / f"{s}.o")]))
    compiles.append(("test_main", gxx + [f"-I{ref / 'third_party'}", "-c",
                                         str(ref / "tests" / "test_main.cpp"),
                                         "-o", str(obj / "test_main.o")]))
    for s in ENGINE_SOURCES:
        compiles.append((s, nvcc + ["-c", str(ref / "src" / "engine" / f"{s}.hip"),
                                    "-o", str(obj / f"{s}.o")]))
    compiles.append(("miso_cli", nvcc + ["-c", str(ref / "src" / "cli" / "miso.hip"),
                                         "-o", str(obj / "miso_cli.o")]))
    for name, (srcs, _) in TESTS.items():
        for src in srcs:
            compiles.append((Path(src).stem, nvcc + ["-c", str(ref / "tests" / src),
                                                     "-o", str(obj / f"{Path(src).stem}.o")]))
    for name, (src, _) in BENCHES.items():
        compiles.append((name, nvcc + ["-c", str(ref / "bench" / src), "-o",
                                       str(obj / f"{name}.o")]))
    nvcc_synth = ["nvcc"] + NVCC_FLAGS + ["-x", "cu"] + inc + [
        f'-DMISO_FIXTURE_DIR="{ref / "tests" / "fixtures"}"',
        f'-DMISO_GOLDEN_DIR="{synth["golden"]}"', f'-DMISO_ORNITH_GGUF="{synth["model"]}"']
    for name in SYNTHETIC_TESTS:
        for src in TESTS[name][0]:
            compiles.append((f"synthetic/{Path(src).stem}",
                             nvcc_synth + ["-c", str(ref / "tests" / src), "-o",
                                           str(obj / "synthetic" / f"{Path(src).stem}.o")]))

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        results = list(ex.map(lambda c: (c[0], _run(c[1])), compiles))
    for name, (rc, log) in results:
        if verbose:
            print(f"compile {name}: rc={rc}")
        if rc != 0:
            raise RuntimeError(f"compiling {name} failed:\n{log[-4000:]}")

    host = [str(obj / f"{s}.o") for s in HOST_SOURCES]
    engine = [str(obj / f"{s}.o") for s in ENGINE_SOURCES]
    link = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a"]
    links = [("miso", link + ["-o", str(targets["miso"]), str(obj / "miso_cli.o")] + engine + host)]
    for name, (srcs, with_engine) in TESTS.items():
        objs = [str(obj / f"{Path(s).stem}.o") for s in srcs] + [str(obj / "test_main.o")]
        links.append((name, link + ["-o", str(targets[name])] + objs +
                      (engine if with_engine else []) + host))
    for name, (_, with_engine) in BENCHES.items():
        links.append((name, link + ["-o", str(targets[name]), str(obj / f"{name}.o")] +
                      (engine if with_engine else []) + host))
    for name in SYNTHETIC_TESTS:
        srcs, with_engine = TESTS[name]
        objs = [str(obj / "synthetic" / f"{Path(s).stem}.o") for s in srcs] + \
            [str(obj / "test_main.o")]
        links.append((f"synthetic/{name}", link + ["-o", str(targets[f"synthetic/{name}"])] +
                      objs + (engine if with_engine else []) + host))
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        results = list(ex.map(lambda c: (c[0], _run(c[1])), links))
    for name, (rc, log) in results:
        if verbose:
            print(f"link {name}: rc={rc}")
        if rc != 0:
            raise RuntimeError(f"linking {name} failed:\n{log[-4000:]}")
    stamp_file.write_text(stamp)
    return targets


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit(__doc__)
    built = build(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else DEFAULT_OUT, verbose=True)
    for name, path in built.items():
        print(f"{name}: {path}")
