"""One rank (one GPU) of the multi-GPU context-parallel test: runs the CUDA / NCCL path of
miso_b200.cp and compares it, on the same GPU, with the single-GPU kernels over the whole
sequence. Zig-zag chunks and DeltaNet segments are multiples of 64 tokens, so the tiles and
chunks of both runs coincide and the results must be bit-identical.

  python cp_gpu_worker.py --rank R --world W --port P
"""
import argparse
import ctypes
import datetime
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from miso_b200 import _capi as capi  # noqa: E402
from miso_b200 import attention as A  # noqa: E402
from miso_b200 import cp  # noqa: E402


def attention_check(rank, world, dev, stream):
    t = 2048 * world
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    proj = torch.randn((t, cp.ATTN_PROJ), generator=g, device=dev).bfloat16().float()
    ones = torch.ones(256, device=dev)
    inv = torch.from_numpy(A.rope_inv_freq()).to(dev)
    run = cp.GpuAttentionCp(t, world, rank, proj, ones, ones, inv, 1e-6, stream)
    run.run()
    # Single-GPU reference over the whole sequence.
    lib = capi.load()
    k = torch.zeros((2, t, 256), dtype=torch.float16, device=dev)
    v = torch.zeros_like(k)
    q16 = torch.empty((t, 16, 256), dtype=torch.float16, device=dev)
    core = torch.empty((t, 16, 256), device=dev)
    base = proj.data_ptr()
    tok0 = capi.AttnPrepParams(base, base + 8192 * 4, base + 8704 * 4, ones.data_ptr(),
                               ones.data_ptr(), inv.data_ptr(), k.data_ptr(), v.data_ptr(), 0, 0,
                               t, 1e-6)
    with torch.cuda.stream(stream):
        capi.check("prep", lib.miso_attn_prep_batch_f16(
            ctypes.byref(capi.AttnPrepBatchParams(tok0, t, cp.ATTN_PROJ)), q16.data_ptr(),
            stream.cuda_stream))
        capi.check("prefill", lib.miso_attn_prefill_tc(ctypes.byref(capi.AttnPrefillTcParams(
            q16.data_ptr(), base, k.data_ptr(), v.data_ptr(), core.data_ptr(), 0, t, t,
            cp.ATTN_PROJ)), stream.cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(run.k, k) and torch.equal(run.v, v), "gathered KV cache differs"
    for start, n in cp.zigzag_chunks(t, world, rank):
        assert torch.equal(run.core[start:start + n], core[start:start + n]), \
            f"attention rows {start}..{start + n} differ"


def deltanet_check(rank, world, dev, stream):
    t, layers = 256 * world, 2
    g = torch.Generator(device=dev)
    g.manual_seed(12)
    projs = [torch.randn((t, cp.DN_PROJ), generator=g, device=dev).bfloat16().float()
             for _ in range(layers)]
    conv_w = 0.5 * torch.randn((8192, 4), generator=g, device=dev)
    ssm_a, dt = -torch.ones(32, device=dev), torch.zeros(32, device=dev)
    norm_w = torch.ones(128, device=dev)
    run = cp.GpuDeltaNetWavefront(t, world, rank, projs, conv_w, ssm_a, dt, norm_w, 1e-6, stream)
    run.run()
    torch.cuda.synchronize()
    lib = capi.load()
    start, n = cp.contiguous_segment(t, world, rank)
    sb = lib.miso_deltanet_prefill_tc_scratch_bytes(t)
    scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
    for layer in range(layers):
        st = torch.zeros((32, 128, 128), device=dev)
        ci, co = torch.zeros((8192, 3), device=dev), torch.zeros((8192, 3), device=dev)
        out = torch.empty((t, 4096), device=dev)
        base = projs[layer].data_ptr()
        z = base + 8192 * 4
        p = capi.DeltaNetSeqParams(base, z, z + 4096 * 4, z + 4128 * 4, conv_w.data_ptr(),
                                   ci.data_ptr(), co.data_ptr(), ssm_a.data_ptr(), dt.data_ptr(),
                                   norm_w.data_ptr(), st.data_ptr(), out.data_ptr(), t, 1e-6,
                                   cp.DN_PROJ, cp.DN_PROJ)
        with torch.cuda.stream(stream):
            capi.check("dn", lib.miso_deltanet_prefill_tc(ctypes.byref(p), scratch.data_ptr(), sb,
                                                         stream.cuda_stream))
        torch.cuda.synchronize()
        assert torch.equal(run.out[layer][start:start + n], out[start:start + n]), \
            f"layer {layer}: rows {start}..{start + n} differ"
        if rank == world - 1:
            assert torch.equal(run.state[layer], st), f"layer {layer}: final state differs"
            assert torch.equal(run.conv[layer], co), f"layer {layer}: conv history differs"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--world", type=int, required=True)
    ap.add_argument("--port", type=int, required=True)
    a = ap.parse_args()
    dev = torch.device(f"cuda:{a.rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{a.port}", rank=a.rank,
                            world_size=a.world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    stream = torch.cuda.Stream()
    try:
        attention_check(a.rank, a.world, dev, stream)
        deltanet_check(a.rank, a.world, dev, stream)
        st = ctypes.c_int(-1)
        capi.check("status", capi.load().miso_device_status(1, ctypes.byref(st)))
        assert st.value == 0, f"device status {st.value:#x}"
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
