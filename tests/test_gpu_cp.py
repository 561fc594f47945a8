"""Multi-GPU context-parallel prefill over NCCL (one process per GPU): attention zig-zag chunks
with the direct KV exchange, and the DeltaNet state hand-off wavefront, bit-identical to the
single-GPU kernels over the whole sequence. Needs at least two GPUs (skipped otherwise)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
WORKER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "support", "cp_gpu_worker.py")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("world", [2])
def test_context_parallel_prefill_matches_single_gpu(world):
    world = min(world, torch.cuda.device_count())
    port = free_port()
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([sys.executable, WORKER, "--rank", str(r), "--world", str(world),
                               "--port", str(port)], env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT) for r in range(world)]
    outs = []
    try:
        for p in procs:
            outs.append(p.communicate(timeout=300)[0].decode(errors="replace"))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    for r, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {r} failed:\n{o[-3000:]}"
