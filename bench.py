#!/usr/bin/env python
"""Benchmark of the attention hot path on B200 (one JSON line on rank 0).

Headline workload ("batched GQA decode"): per GPU, 32 sequences with context
lengths uniform in [1024, 32768] (seed 0), 16 query / 2 KV heads, head_dim 256, fp16 KV cache
N(0, 1), fp32 queries and gate logits N(0, 1). One step = one decode token for every sequence:
batched prep (RMSNorm + RoPE + KV append, lens advance) then the stream-K split-K decode with
the gated combine fused in. Metric: decode tokens/s (whole job), with the decode kernel's HBM
GB/s against the measured HBM peak.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl miso|reference]

Multi-GPU: one process per GPU under torchrun; each rank decodes its own batch of 32
(independent sequences, no collective on the data path: weak scaling); the step time is the
max over ranks of device-event time.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BATCH = 32
LEN_LO, LEN_HI = 1024, 32768
Q_HEADS, KV_HEADS, DIM = 16, 2, 256
PROJ = 9216  # per-token projection row [q+gate 8192 | k 512 | v 512]
EPS = 1e-6
KV_BYTES_PER_POS = KV_HEADS * DIM * 2 * 2  # K and V, fp16: 2048 B per position
QGO_BYTES_PER_SEQ = 3 * Q_HEADS * DIM * 4  # q read, gate read, core written


def lens_config() -> np.ndarray:
    return np.random.RandomState(0).randint(LEN_LO, LEN_HI + 1, size=BATCH).astype(np.int32)


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        d = json.load(open(path))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "source": "measured (MEASURED_PEAKS.json)"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class Clocks:
    """Samples nvidia-smi clocks / throttle reasons while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p is not None:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self) -> dict:
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------------------------- reference arm


CPU_SAMPLE = ("the whole batch of {b} sequences per step (the GPU arm's lens), fp64 restatement "
              "of the reference's decode reference (tests/test_attn_splitk.hip:153-173)")


def cpu_decode_batch(lens: np.ndarray, seed: int, threads: int):
    """Host data for one decode step of the whole batch (K / V N(0, 1) fp16, q, gate N(0, 1)) and
    a callable that runs the oracle decode on it. Both CPU figures of the benchmark (the
    reference arm and the GPU arm's cpu_baseline) time this same callable."""
    import oracle
    rng = np.random.default_rng(seed)
    b = len(lens)
    cap = int(lens.max())
    rows = b * KV_HEADS * cap
    k = np.empty((rows, DIM), np.uint16)
    v = np.empty((rows, DIM), np.uint16)
    kv_row = (np.arange(b * KV_HEADS, dtype=np.int64) * cap).reshape(-1, KV_HEADS)
    for i in range(b * KV_HEADS):  # only the rows each sequence uses are filled
        n = int(lens[i // KV_HEADS])
        r0 = i * cap
        k[r0:r0 + n] = rng.standard_normal((n, DIM), dtype=np.float32).astype(np.float16).view(
            np.uint16)
        v[r0:r0 + n] = rng.standard_normal((n, DIM), dtype=np.float32).astype(np.float16).view(
            np.uint16)
    q = rng.standard_normal((b, Q_HEADS, DIM), dtype=np.float32)
    qg = rng.standard_normal((b, Q_HEADS, 2 * DIM), dtype=np.float32)
    lens = np.ascontiguousarray(lens, np.int32)
    return lambda: oracle.attn_decode(q, qg, Q_HEADS * 2 * DIM, k, v, kv_row, lens,
                                      threads=threads)


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle
    oracle.build()
    threads = oracle.cpu_count()
    fn = cpu_decode_batch(lens_config(), seed=100, threads=threads)
    steps = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        fn()
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            steps.append(dt)
    t = sum(steps) / len(steps)
    value = BATCH / t
    line = {
        "impl": "reference", "metric": "attn decode tok/s", "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * t, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": CPU_SAMPLE.format(b=BATCH)},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(n_gpus: int) -> dict:
    return {"workload": "batched GQA decode (BASELINE config 2)", "batch_per_gpu": BATCH,
            "global_batch": BATCH * n_gpus, "ctx_len": f"U[{LEN_LO}, {LEN_HI}] seed 0",
            "mean_ctx": float(lens_config().mean()), "q_heads": Q_HEADS, "kv_heads": KV_HEADS,
            "head_dim": DIM, "kv_dtype": "fp16", "q_dtype": "fp32",
            "parallelism": f"dp{n_gpus} (independent sequences per GPU)",
            "l2": "inputs larger than L2 (KV stream ~1.1 GB per step per GPU)"}


# ------------------------------------------------------------------------------------- miso arm


class DecodeBatch:
    """A batch of sequences in one KV pool (fp16 N(0, 1), lens given, `extra` free rows per
    sequence for appended tokens), their projection rows and the two launches of a decode step:
    batched prep (norms, RoPE, KV append, lens advance) and the stream-K split-K decode."""

    def __init__(self, dev, lens: np.ndarray, extra: int, seed: int, stream):
        import torch
        from miso_b200 import attention as A
        from miso_b200 import capi
        self.capi, self.lib, self.stream = capi, capi.load(), stream
        self.batch = b = len(lens)
        self.lens0 = lens.astype(np.int64)
        seg_caps = np.repeat(self.lens0 + extra, KV_HEADS)
        starts = np.concatenate([[0], np.cumsum(seg_caps)[:-1]]).astype(np.int64)
        self.rows = rows = int(seg_caps.sum())
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        pool = A.KvPool.__new__(A.KvPool)
        pool.batch, pool.capacity, pool.rows = b, None, rows
        pool.k = torch.randn((rows, DIM), generator=g, device=dev, dtype=torch.float16)
        pool.v = torch.randn((rows, DIM), generator=g, device=dev, dtype=torch.float16)
        pool.kv_row = torch.from_numpy(starts.reshape(b, KV_HEADS)).to(dev)
        pool.lens = torch.from_numpy(lens.astype(np.int32)).to(dev)
        self.pool = pool
        self.proj = torch.randn((b, PROJ), generator=g, device=dev, dtype=torch.float32)
        self.q_norm = (1.0 + 0.1 * torch.randn(DIM, generator=g, device=dev)).float()
        self.k_norm = (1.0 + 0.1 * torch.randn(DIM, generator=g, device=dev)).float()
        self.inv_freq = torch.from_numpy(A.rope_inv_freq()).to(dev)
        self.q = torch.empty((b, Q_HEADS, DIM), device=dev)
        self.core = torch.empty((b, Q_HEADS, DIM), device=dev)
        self.scratch = A.decode_scratch(b, device=dev)

    def prep(self, src_base: int):
        capi, pool = self.capi, self.pool
        p = capi.AttnPrepBatchedParams(src_base, src_base + 8192 * 4, src_base + 8704 * 4,
                                       self.q_norm.data_ptr(), self.k_norm.data_ptr(),
                                       self.inv_freq.data_ptr(), pool.k.data_ptr(),
                                       pool.v.data_ptr(), pool.kv_row.data_ptr(),
                                       pool.lens.data_ptr(), self.q.data_ptr(), self.batch, PROJ,
                                       EPS)
        capi.check("miso_attn_prep_batched",
                   self.lib.miso_attn_prep_batched(ctypes.byref(p), self.stream.cuda_stream))

    def decode(self, qg_base: int, out=None, kv_row=None):
        capi, pool = self.capi, self.pool
        out = self.core if out is None else out
        kv_row = pool.kv_row.data_ptr() if kv_row is None else kv_row
        dp = capi.AttnDecodeParams(self.q.data_ptr(), qg_base, pool.k.data_ptr(),
                                   pool.v.data_ptr(), kv_row, pool.lens.data_ptr(),
                                   out.data_ptr(), self.rows, self.batch, PROJ)
        capi.check("miso_attn_decode",
                   self.lib.miso_attn_decode(ctypes.byref(dp), self.scratch.data_ptr(),
                                             self.scratch.numel() * 4, self.stream.cuda_stream))

    def time_device(self, steps: int, warmup: int, barrier):
        """Device-resident decode steps (prep + decode) timed with CUDA events: returns (step ms,
        decode-kernel ms, algorithmic bytes per decode launch), averaged over the timed steps.
        The bytes: K and V of every cached position (after the step's append), q and gate
        reads and the output write."""
        import torch
        stream, base = self.stream, self.proj.data_ptr()
        for _ in range(warmup):
            self.prep(base)
            self.decode(base)
        torch.cuda.synchronize()
        lens_start = self.pool.lens.cpu().numpy().astype(np.int64)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(steps)]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for i in range(steps):
            self.prep(base)
            ev[i][0].record(stream)
            self.decode(base)
            ev[i][1].record(stream)
        end.record(stream)
        torch.cuda.synchronize()
        barrier()
        dec_ms = sum(a.elapsed_time(b) for a, b in ev) / steps
        nbytes = sum(float(((lens_start + i + 1) * KV_BYTES_PER_POS).sum() +
                           self.batch * QGO_BYTES_PER_SEQ) for i in range(steps)) / steps
        return start.elapsed_time(end) / steps, dec_ms, nbytes


def bench_decode_32k(args, dev, stream, max_over_ranks, barrier, world, rank) -> dict:
    """BASELINE's "@32k ctx" decode figure: config 2 with every sequence at 32768 cached
    positions (32 sequences per GPU, 2.147 GB of K / V per step)."""
    b = args.batch
    db = DecodeBatch(dev, np.full(b, 32768, np.int32), args.warmup + args.steps + 4,
                     4321 + rank, stream)
    step_ms, dec_ms, nbytes = db.time_device(args.steps, args.warmup, barrier)
    step_ms, dec_ms = max_over_ranks(step_ms), max_over_ranks(dec_ms)
    pk = peaks()
    achieved = nbytes / (dec_ms * 1e-3) / 1e9
    return {"metric": "attn decode tok/s @32k ctx", "value": world * b / (step_ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": step_ms, "batch_per_gpu": b, "ctx_len": 32768,
            "bytes_per_step": nbytes, "gbs": achieved,
            "config": "config 2 shapes with all lens = 32768; step = batched prep + split-K "
                      "decode (inputs larger than L2)",
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "traffic": nbytes * DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE,
                         "kernel": "decode_kernel", "kernel_ms": dec_ms,
                         "peak_source": pk["source"]},
            "gpu_launches": 2 * args.steps}


C1_CTX = 4096
C1_COPIES = 32  # 32 x 8.4 MB of K / V rotate, so a step never finds its cache in the 126 MB L2


def bench_decode_config1(args, dev, stream, max_over_ranks, barrier, world, rank) -> dict:
    """one sequence, 16 Q / 2 KV heads, head_dim 256, context 4096, fp16 K / V
    cache and fp32 queries N(0, 1), fp32 output [16][256] (the reference's CPU-runnable decode
    step). One step = the attention decode over the cache. 32 copies of the cache rotate from
    step to step so that the 8.4 MB are read from HBM, not L2. Timed two ways: the fast
    stream-K decode (one launch), and the drop-in split + combine pair that the reference
    engine launches (miso_attn_split / miso_attn_combine, caller geometry). Steps are captured
    in a CUDA graph so that the host's launch cost does not pace a single sequence."""
    import torch
    from miso_b200 import attention as A
    from miso_b200 import capi
    lib = capi.load()
    db = DecodeBatch(dev, np.full(C1_COPIES, C1_CTX, np.int32), 0, 777 + rank, stream)
    # batch 1 over the pool: copy c is pool rows kv_row[c]
    kv_rows = db.pool.kv_row.contiguous()
    lens1 = torch.full((1,), C1_CTX, dtype=torch.int32, device=dev)
    db.pool.lens = lens1
    db.batch = 1
    q = torch.randn((1, Q_HEADS, DIM), device=dev)
    db.q = q
    qg = db.proj[:1]
    out = torch.empty((1, Q_HEADS, DIM), device=dev)
    ns = A.n_splits(C1_CTX, A.MAX_SPLITS)
    sc = A.AttentionScratch(device=dev)
    # a reference AttentionCache per copy: the pool's two KV-head segments of copy c are
    # [2][C1_CTX][256] contiguous (capacity C1_CTX, no extra rows)
    seg = C1_CTX * DIM * 2

    def fast(i, st):
        db.stream = st
        db.decode(qg.data_ptr(), out, kv_rows.data_ptr() + (i % C1_COPIES) * 16)

    def drop_in(i, st):
        c = i % C1_COPIES
        kb = db.pool.k.data_ptr() + 2 * c * seg
        vb = db.pool.v.data_ptr() + 2 * c * seg
        sp = capi.AttnSplitParams(q.data_ptr(), kb, vb, sc.part_m.data_ptr(),
                                  sc.part_l.data_ptr(), sc.part_o.data_ptr(), C1_CTX, C1_CTX, ns)
        capi.check("miso_attn_split", lib.miso_attn_split(ctypes.byref(sp), st.cuda_stream))
        cp_ = capi.AttnCombineParams(sc.part_m.data_ptr(), sc.part_l.data_ptr(),
                                     sc.part_o.data_ptr(), qg.data_ptr(), out.data_ptr(), ns)
        capi.check("miso_attn_combine", lib.miso_attn_combine(ctypes.byref(cp_), st.cuda_stream))

    def timed(fn) -> float:
        n = max(args.steps, C1_COPIES)
        for i in range(max(args.warmup, C1_COPIES)):
            fn(i, stream)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(stream)
        with torch.cuda.graph(graph, stream=cap):
            for i in range(n):
                fn(i, cap)
        graph.replay()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        del graph
        return max_over_ranks(e0.elapsed_time(e1) / n)

    fast_ms = timed(fast)
    drop_ms = timed(drop_in)
    nbytes = C1_CTX * KV_BYTES_PER_POS + QGO_BYTES_PER_SEQ
    pk = peaks()
    a_fast = nbytes / (fast_ms * 1e-3) / 1e9
    return {"metric": "attn decode tok/s, 1 sequence @4096 ctx (config 1)",
            "value": world / (fast_ms * 1e-3), "unit": "tokens/s", "ms_per_step": fast_ms,
            "bytes_per_step": nbytes, "gbs": a_fast,
            "drop_in": {"ms_per_step": drop_ms, "value": world / (drop_ms * 1e-3),
                        "gbs": nbytes / (drop_ms * 1e-3) / 1e9, "n_splits": ns,
                        "launches": "attn_split_kernel<256> (n_splits x 2) + "
                                    "attn_combine_kernel<64, true, 4>"},
            "config": "BASELINE config 1: 1 sequence, ctx 4096, fp16 KV, fp32 q, gate; 32 "
                      "rotating cache copies (268 MB > L2); steps replayed from a CUDA graph",
            "roofline": {"bound": "hbm", "achieved": a_fast, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": a_fast / pk["hbm_gbs"], "traffic": None,
                         "kernel": "decode_kernel", "kernel_ms": fast_ms,
                         "peak_source": pk["source"],
                         "note": "8.4 MB per step: launch- and latency-bound, far from the HBM "
                                 "roofline by construction"},
            "gpu_launches": 2 * max(args.steps, C1_COPIES) * 3}


def run_miso(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)

    import miso_b200
    from miso_b200 import attention as A
    from miso_b200 import capi

    lens0 = lens_config()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Room for the appended tokens: the device-timed loop and the end-to-end loop each append
    # warmup + steps tokens to every sequence.
    db = DecodeBatch(dev, lens0, 2 * (args.warmup + args.steps) + 4, 1234 + rank, stream)
    step, decode, base = db.prep, db.decode, db.proj.data_ptr()
    pool = db.pool

    # ---- device-resident timing ---------------------------------------------------------------
    with Clocks(local) as clk:
        step_ms, dec_avg_ms, dec_bytes = db.time_device(args.steps, args.warmup, barrier)
    step_ms_max = max_over_ranks(step_ms)
    achieved = dec_bytes / (dec_avg_ms * 1e-3) / 1e9
    pk = peaks()

    # ---- end to end through the C ABI with host buffers ---------------------------------------
    # A serving loop: every step's inputs are uploaded from pinned host memory and its output is
    # downloaded to pinned host memory, inside the timed region. Inputs and outputs are double
    # buffered and the copies run on their own streams, so the upload of step i + 1 and the
    # download of step i overlap step i's kernels; events order every reuse of a buffer.
    host_in = [torch.randn((BATCH, PROJ), dtype=torch.float32).pin_memory() for _ in range(2)]
    host_out = [torch.empty((BATCH, Q_HEADS, DIM), dtype=torch.float32).pin_memory()
                for _ in range(2)]
    dev_in = [torch.empty((BATCH, PROJ), device=dev) for _ in range(2)]
    dev_out = [torch.empty((BATCH, Q_HEADS, DIM), device=dev) for _ in range(2)]
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def serve(n: int) -> None:
        uploaded = [torch.cuda.Event() for _ in range(2)]    # input b is on the device
        consumed = [torch.cuda.Event() for _ in range(2)]    # step using buffer b has finished
        downloaded = [torch.cuda.Event() for _ in range(2)]  # output b is in host memory
        t0 = torch.cuda.Event()
        t0.record(stream)
        h2d.wait_event(t0)
        with torch.cuda.stream(h2d):
            dev_in[0].copy_(host_in[0], non_blocking=True)
        uploaded[0].record(h2d)
        for i in range(n):
            b = i % 2
            if i + 1 < n:  # upload the next step's input while this step computes
                if i >= 1:
                    h2d.wait_event(consumed[1 - b])
                with torch.cuda.stream(h2d):
                    dev_in[1 - b].copy_(host_in[1 - b], non_blocking=True)
                uploaded[1 - b].record(h2d)
            stream.wait_event(uploaded[b])
            if i >= 2:
                stream.wait_event(downloaded[b])  # step i - 2's output has left buffer b
            step(dev_in[b].data_ptr())
            decode(dev_in[b].data_ptr(), dev_out[b])
            consumed[b].record(stream)
            d2h.wait_event(consumed[b])
            with torch.cuda.stream(d2h):
                host_out[b].copy_(dev_out[b], non_blocking=True)
            downloaded[b].record(d2h)
        for b in range(min(n, 2)):
            stream.wait_event(downloaded[b])

    serve(args.warmup)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    serve(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    last = (args.steps - 1) % 2  # the last step's output reached host memory intact
    assert torch.equal(host_out[last], dev_out[last].cpu()), "end-to-end download mismatch"
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)

    decode_32k = None if args.no_decode_legs else bench_decode_32k(args, dev, stream,
                                                                   max_over_ranks, barrier,
                                                                   world, rank)
    decode_c1 = None if args.no_decode_legs else bench_decode_config1(args, dev, stream,
                                                                      max_over_ranks, barrier,
                                                                      world, rank)
    prefill = None if args.no_prefill else bench_prefill(args, dev, stream, max_over_ranks,
                                                         barrier, world)
    dn_step = None if args.no_deltanet else bench_deltanet_step(args, dev, stream,
                                                                max_over_ranks, barrier, world)
    dn_prefill = None if args.no_deltanet else bench_deltanet_prefill(args, dev, stream,
                                                                      max_over_ranks, barrier,
                                                                      world)
    cp_block = None if args.no_cp else bench_cp_block(args, dev, stream, max_over_ranks,
                                                      barrier, world, rank)

    st = ctypes.c_int(-1)
    capi.check("miso_device_status", capi.load().miso_device_status(1, st))
    if st.value != 0:
        raise RuntimeError(f"device status {st.value} after the timed region")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        oracle.build()
        threads = oracle.cpu_count()
        fn = cpu_decode_batch(lens0, seed=100, threads=threads)
        fn()
        t0 = time.perf_counter()
        reps = 0
        while True:
            fn()
            reps += 1
            if time.perf_counter() - t0 > 10.0 or reps >= 20:
                break
        t = (time.perf_counter() - t0) / reps
        cpu = {"value": BATCH / t, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": CPU_SAMPLE.format(b=BATCH) + f", {reps} steps"}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    value = world * BATCH / (step_ms_max * 1e-3)
    line = {
        "metric": "attn decode tok/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms_max,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16kv-f32",
        "data": "synthetic", "config": workload_config(world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "traffic": dec_bytes * DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE,
                     "traffic_source": "ncu dram read + write of a batch-8 capture "
                                       "(profiles/decode_kernel_b8_ncu.md) scaled by the KV "
                                       "bytes of a full launch",
                     "kernel": "decode_kernel", "kernel_ms": dec_avg_ms,
                     "peak_source": pk["source"]},
        "e2e": {"value": world * BATCH / (e2e_ms * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": BATCH * PROJ * 4,
                "d2h_bytes_per_step": BATCH * Q_HEADS * DIM * 4},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
        "cpu_baseline": cpu,
        "decode_32k": decode_32k,
        "decode_config1": decode_c1,
        "prefill": prefill,
        "deltanet_step": dn_step,
        "deltanet_prefill": dn_prefill,
        "cp_block": cp_block,
    }
    print(json.dumps(line), flush=True)


PREFILL_N = 8192
# ncu DRAM bytes (read + write) per algorithmic byte of the decode kernel: batch-8 capture, 257.0 +
# 6.3 MB for 256.8 MB of K / V / q / gate (profiles/decode_kernel_b8_ncu.md).
DECODE_TRAFFIC_PER_ALGORITHMIC_BYTE = (257.0 + 6.3) / 256.8
# ncu DRAM bytes (read + write) of one full-size launch (profiles/prefill_kernel_8k_ncu.md,
# profiles/deltanet_prefill_tc_8k_ncu.md).
PREFILL_8K_TRAFFIC = (237.3 + 101.1) * 1e6
# DRAM bytes (read + write inside each launch) of the three kernels of a piece of 1024 tokens
# (front 49.9 + 15.8 MB, chain 69.3 + 3.1 MB, gate 33.6 + 0.0 MB; ncu, caches flushed before each
# launch), times the 8 such token ranges of a call at 8192 tokens (every byte is per token: the
# records are written and read once whatever the piece size).
DN_PREFILL_8K_TRAFFIC = 8 * (49.94 + 15.80 + 69.26 + 3.08 + 33.56) * 1e6
# DRAM bytes inside one launch of step_batched_kernel at batch 64 (ncu: read 143.9 MB, write
# 87.6 MB; the remaining state writes leave L2 after the launch ends).
DN_STEP_B64_TRAFFIC = (143.86 + 87.64) * 1e6


def prefill_flops(n: int, pos0: int = 0) -> float:
    """Causal QK^T + PV FLOPs of 16 heads x 256 dims: 4 * 16 * 256 * sum_t (pos0 + t + 1)."""
    return 4.0 * 16 * 256 * (n * pos0 + n * (n + 1) / 2)


def bench_prefill(args, dev, stream, max_over_ranks, barrier, world) -> dict:
    """one 8192-token causal gated prefill per GPU (bf16 inputs, fp16 tensor
    operands, fp32 softmax / accumulation). Step = prep (norm, RoPE, fp16 KV append) + tcgen05
    attention; TFLOP/s counts the causal attention FLOPs 8192 n (n + 1)."""
    import torch
    from miso_b200 import attention as A
    from miso_b200 import capi

    n = args.prefill_n
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    proj = torch.randn((n, PROJ), generator=g, device=dev).bfloat16().float()  # bf16 values
    ones = torch.ones(DIM, device=dev)
    inv_freq = torch.from_numpy(A.rope_inv_freq()).to(dev)
    kc = torch.empty((KV_HEADS, n, DIM), dtype=torch.float16, device=dev)
    vc = torch.empty_like(kc)
    q16 = torch.empty((n, Q_HEADS, DIM), dtype=torch.float16, device=dev)
    core = torch.empty((n, Q_HEADS, DIM), device=dev)
    base = proj.data_ptr()
    tok0 = capi.AttnPrepParams(base, base + 8192 * 4, base + 8704 * 4, ones.data_ptr(),
                               ones.data_ptr(), inv_freq.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                               0, 0, n, EPS)
    bp = capi.AttnPrepBatchParams(tok0, n, PROJ)
    tp = capi.AttnPrefillTcParams(q16.data_ptr(), base, kc.data_ptr(), vc.data_ptr(),
                                  core.data_ptr(), 0, n, n, PROJ)
    lib = capi.load()

    def step(ev=None):
        capi.check("prep_f16", lib.miso_attn_prep_batch_f16(ctypes.byref(bp), q16.data_ptr(),
                                                            stream.cuda_stream))
        if ev is not None:
            ev[0].record(stream)
        capi.check("prefill_tc", lib.miso_attn_prefill_tc(ctypes.byref(tp), stream.cuda_stream))
        if ev is not None:
            ev[1].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(args.steps):
        step(evs[i])
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    step_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    kern_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in evs) / args.steps)
    flops = prefill_flops(n)
    pk = peaks()
    achieved = flops / (kern_ms * 1e-3) / 1e12
    return {"metric": f"prefill TFLOP/s @{n}", "value": world * flops / (step_ms * 1e-3) / 1e12,
            "unit": "TFLOP/s", "ms_per_step": step_ms, "n_tokens": n,
            "config": "BASELINE config 3: 1 x 8192 tokens per GPU, causal, 16 Q / 2 KV heads, "
                      "d 256, RoPE 64 dims theta 1e7, sigmoid gate, bf16 inputs, fp16 tensor "
                      "operands, fp32 softmax / accumulate; step = prep + attention",
            "flops_per_step": flops,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                         "traffic": PREFILL_8K_TRAFFIC if n == 8192 else None,
                         "kernel": "prefill_kernel", "kernel_ms": kern_ms,
                         "peak_source": pk["source"] + " (dense bf16 burst; fp16 equal)"},
            "gpu_launches": 2 * args.steps}


DN_BATCH = 64
DN_STATE_BYTES = 32 * 128 * 128 * 4
DN_PROJ = 12352  # [qkv 8192 | z 4096 | a 32 | b 32]


def bench_deltanet_step(args, dev, stream, max_over_ranks, barrier, world) -> dict:
    """BASELINE config 4b: one Gated DeltaNet decode step for 64 sequences per GPU on fp32
    [32][128][128] states (zero-initialised), qkv / z / a / b N(0,1) bf16 values, conv_w
    N(0, 0.5), ssm_a = -1, dt_bias = 0. HBM-bound: algorithmic bytes per step = state read +
    write (268 MB) + conv history read + write + inputs + outputs."""
    import torch
    from miso_b200 import capi

    B = DN_BATCH
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    proj = torch.randn((B, DN_PROJ), generator=g, device=dev).bfloat16().float()
    conv_w = 0.5 * torch.randn((8192, 4), generator=g, device=dev)
    ssm_a = -torch.ones(32, device=dev)
    dt = torch.zeros(32, device=dev)
    norm_w = torch.ones(128, device=dev)
    conv = [torch.zeros((B, 8192, 3), device=dev) for _ in range(2)]
    state = torch.zeros((B, 32, 128, 128), device=dev)
    out = torch.empty((B, 4096), device=dev)
    lib = capi.load()
    base = proj.data_ptr()
    params = [capi.DeltaNetStepBatchedParams(base, base + 8192 * 4, base + 12288 * 4,
                                             base + 12320 * 4, conv_w.data_ptr(),
                                             ssm_a.data_ptr(), dt.data_ptr(), norm_w.data_ptr(),
                                             conv[i].data_ptr(), conv[1 - i].data_ptr(),
                                             state.data_ptr(), out.data_ptr(), B, DN_PROJ, EPS)
              for i in range(2)]

    def step(i):
        capi.check("dn_step", lib.miso_deltanet_step_batched(ctypes.byref(params[i % 2]),
                                                             stream.cuda_stream))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    nbytes = (2 * B * DN_STATE_BYTES + 2 * B * 8192 * 3 * 4 + B * DN_PROJ * 4 + B * 4096 * 4 +
              8192 * 4 * 4)
    achieved = nbytes / (ms * 1e-3) / 1e9
    pk = peaks()
    return {"metric": "DeltaNet decode tok/s (batch 64)", "value": world * B / (ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": ms,
            "config": "BASELINE config 4b: 64 sequences per GPU, 16 K / 32 V heads, d 128, fp32 "
                      "states (zero-init), bf16-valued inputs; one launch per step",
            "bytes_per_step": nbytes,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "traffic": DN_STEP_B64_TRAFFIC if B == 64 else None,
                         "kernel": "step_batched_kernel", "kernel_ms": ms,
                         "peak_source": pk["source"]},
            "gpu_launches": args.steps}


DN_PREFILL_T = 8192
# pieces per miso_deltanet_prefill_tc call: 16 chunks, then 32 each (the last one the remainder)
DN_PIECES = 1 + -(-(DN_PREFILL_T // 64 - 16) // 32)
# Algorithmic FLOPs of the chunked rule per (V head, chunk of 64): 2 (3 C d^2 + 3 C^2 d)
# = 9.44 MFLOP (QK^T / KK^T, the UT-transform products, S updates), 32 heads x T / 64 chunks.
DN_PREFILL_FLOPS_PER_HEAD_CHUNK = 2.0 * (3 * 64 * 128 * 128 + 3 * 64 * 64 * 128)


def bench_deltanet_prefill(args, dev, stream, max_over_ranks, barrier, world) -> dict:
    """BASELINE config 4a: Gated DeltaNet chunked prefill of T = 8192 tokens per GPU (one
    sequence per rank), bf16-valued N(0,1) projections, conv_w N(0, 0.5), ssm_a = -1,
    dt_bias = 0, zero initial state and conv history; one step = miso_deltanet_prefill_tc (conv +
    norms, per-chunk UT transform, state recurrence with the gated RMS-norm output)."""
    import torch
    from miso_b200 import capi

    T = DN_PREFILL_T
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    proj = torch.randn((T, DN_PROJ), generator=g, device=dev).bfloat16().float()
    conv_w = (0.5 * torch.randn((8192, 4), generator=g, device=dev)).bfloat16().float()
    ssm_a = -torch.ones(32, device=dev)
    dt = torch.zeros(32, device=dev)
    norm_w = torch.ones(128, device=dev)
    conv = [torch.zeros((8192, 3), device=dev) for _ in range(2)]
    state = torch.zeros((32, 128, 128), device=dev)
    out = torch.empty((T, 4096), device=dev)
    lib = capi.load()
    sb = lib.miso_deltanet_prefill_tc_scratch_bytes(T)
    scratch = torch.empty(sb, dtype=torch.uint8, device=dev)
    base = proj.data_ptr()
    z = base + 8192 * 4
    params = [capi.DeltaNetSeqParams(base, z, z + 4096 * 4, z + 4128 * 4, conv_w.data_ptr(),
                                     conv[i].data_ptr(), conv[1 - i].data_ptr(), ssm_a.data_ptr(),
                                     dt.data_ptr(), norm_w.data_ptr(), state.data_ptr(),
                                     out.data_ptr(), T, EPS, DN_PROJ, DN_PROJ)
              for i in range(2)]

    def step(i):
        capi.check("dn_prefill", lib.miso_deltanet_prefill_tc(
            ctypes.byref(params[i % 2]), scratch.data_ptr(), sb, stream.cuda_stream))

    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(args.steps):
        step(i)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    flops = 32 * (T // 64) * DN_PREFILL_FLOPS_PER_HEAD_CHUNK
    nbytes = T * (8192 + 4096 + 64) * 4 + T * 4096 * 4 + 2 * 32 * 128 * 128 * 4
    pk = peaks()
    tflops = flops / (ms * 1e-3) / 1e12
    return {"metric": "DeltaNet chunked prefill tok/s @8192", "value": world * T / (ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": ms, "n_tokens": T,
            "config": "BASELINE config 4a: 1 x 8192 tokens per GPU, 16 K / 32 V heads, d 128, "
                      "chunk 64, bf16-valued inputs, zero initial state; fp16 hi/lo tensor "
                      "operands, fp32 accumulation and state; one call per step = 5 pieces "
                      "(1024, 3 x 2048, 1024 tokens) x 3 launches (per-chunk records, state recurrence, gated "
                      "norm) on three streams",
            "flops_per_step": flops, "tflops": tflops, "bytes_per_step": nbytes,
            "gbs": nbytes / (ms * 1e-3) / 1e9,
            "roofline": {"bound": "tensor", "achieved": tflops, "peak": pk["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": tflops / pk["bf16_tflops"],
                         "traffic": DN_PREFILL_8K_TRAFFIC,
                         "kernel": "front_kernel + chain_kernel + gate_kernel", "kernel_ms": ms,
                         "peak_source": pk["source"],
                         "traffic_source": "ncu DRAM bytes of one piece's three launches x 8 "
                                           "pieces (profiles/deltanet_prefill_tc_8k_ncu.md)",
                         "note": "latency-bound: the state recurrence is sequential over the "
                                 "128 chunks of each of the 32 heads; the records of each chunk "
                                 "go through HBM between the front and the chain"},
            "gpu_launches": 3 * DN_PIECES * args.steps}


CP_T = 131072
CP_DN_LAYERS = 3
CP_DEC_BATCH = 8
CP_DEC_STEPS = 256


def cp_block_decode(args, dev, stream, max_over_ranks, barrier, world, rank, attn, dn, dn_group,
                    g) -> dict:
    """BASELINE config 5 (decode part): 256 decode steps of the block at a total batch of 8
    sequences that continue from the context-parallel prefix. The 8 sequences are split over the
    ranks; each rank already holds the whole prefix KV cache (from the prefill's KV exchange) and
    receives the DeltaNet states at the end of the prefix from the last rank (a broadcast). Step
    = batched attention prep + split-K decode, then the batched DeltaNet step of each layer."""
    import torch
    import torch.distributed as dist
    from miso_b200 import _capi as capi
    from miso_b200 import attention as A

    t, steps = attn.t, args.cp_decode_steps
    nb = CP_DEC_BATCH // world + (1 if rank < CP_DEC_BATCH % world else 0)
    if world > 1:
        for layer in range(CP_DN_LAYERS):
            dist.broadcast(dn.state[layer], world - 1, group=dn_group)
            dist.broadcast(dn.conv[layer], world - 1, group=dn_group)
    torch.cuda.synchronize()
    if nb == 0:  # take part in the same collectives as the ranks that decode
        barrier()
        barrier()
        max_over_ranks(0.0)
        barrier()
        return None
    lib = capi.load()
    cap = t + steps + args.warmup + 8
    rows = nb * KV_HEADS * cap
    pk_, pv_ = (torch.empty((rows, DIM), dtype=torch.float16, device=dev) for _ in range(2))
    kv_row = torch.arange(nb * KV_HEADS, dtype=torch.int64, device=dev).reshape(nb, KV_HEADS) * cap
    for b in range(nb):
        for h in range(KV_HEADS):
            r0 = (b * KV_HEADS + h) * cap
            pk_[r0:r0 + t] = attn.k[h]
            pv_[r0:r0 + t] = attn.v[h]
    lens = torch.full((nb,), t, dtype=torch.int32, device=dev)
    aproj = torch.randn((steps, nb, PROJ), generator=g, device=dev).bfloat16().float()
    dproj = torch.randn((steps, CP_DN_LAYERS, nb, DN_PROJ), generator=g,
                        device=dev).bfloat16().float()
    ones = torch.ones(DIM, device=dev)
    inv = torch.from_numpy(A.rope_inv_freq()).to(dev)
    q = torch.empty((nb, Q_HEADS, DIM), device=dev)
    core = torch.empty_like(q)
    scratch = A.decode_scratch(nb, device=dev)
    conv_w, ssm_a, dt, norm_w = dn.w
    states = [dn.state[layer].unsqueeze(0).repeat(nb, 1, 1, 1).contiguous()
              for layer in range(CP_DN_LAYERS)]
    convs = [[dn.conv[layer].unsqueeze(0).repeat(nb, 1, 1).contiguous(),
              torch.empty((nb, 8192, 3), device=dev)] for layer in range(CP_DN_LAYERS)]
    dout = torch.empty((nb, 4096), device=dev)

    def step(i, st):
        src = aproj[i % steps].data_ptr()
        pp = capi.AttnPrepBatchedParams(src, src + 8192 * 4, src + 8704 * 4, ones.data_ptr(),
                                        ones.data_ptr(), inv.data_ptr(), pk_.data_ptr(),
                                        pv_.data_ptr(), kv_row.data_ptr(), lens.data_ptr(),
                                        q.data_ptr(), nb, PROJ, EPS)
        capi.check("prep_batched", lib.miso_attn_prep_batched(ctypes.byref(pp),
                                                              st.cuda_stream))
        dp = capi.AttnDecodeParams(q.data_ptr(), src, pk_.data_ptr(), pv_.data_ptr(),
                                   kv_row.data_ptr(), lens.data_ptr(), core.data_ptr(), rows, nb,
                                   PROJ)
        capi.check("decode", lib.miso_attn_decode(ctypes.byref(dp), scratch.data_ptr(),
                                                  scratch.numel() * 4, st.cuda_stream))
        for layer in range(CP_DN_LAYERS):
            base = dproj[i % steps, layer].data_ptr()
            cin, cout = convs[layer][i % 2], convs[layer][1 - i % 2]
            sp = capi.DeltaNetStepBatchedParams(base, base + 8192 * 4, base + 12288 * 4,
                                                base + 12320 * 4, conv_w.data_ptr(),
                                                ssm_a.data_ptr(), dt.data_ptr(), norm_w.data_ptr(),
                                                cin.data_ptr(), cout.data_ptr(),
                                                states[layer].data_ptr(), dout.data_ptr(), nb,
                                                DN_PROJ, EPS)
            capi.check("dn_step", lib.miso_deltanet_step_batched(ctypes.byref(sp),
                                                                 st.cuda_stream))

    for i in range(args.warmup):
        step(i, stream)
    torch.cuda.synchronize()
    # The 256 steps (5 launches each, one token per sequence) are captured once into a CUDA graph
    # and replayed, so the host's per-launch cost does not pace one-sequence-per-rank decoding.
    graph = torch.cuda.CUDAGraph()
    cap_stream = torch.cuda.Stream(device=dev)
    cap_stream.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap_stream):
        for i in range(steps):
            step(i, cap_stream)
    lens.fill_(t)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    barrier()
    del graph
    return {"metric": "hybrid block decode tok/s after the prefix", "value":
            CP_DEC_BATCH * steps / (ms * 1e-3), "unit": "tokens/s", "steps": steps,
            "ms": ms, "batch": CP_DEC_BATCH, "sequences_per_rank": nb, "context": t,
            "scaling": "strong", "gpu_launches": steps * (2 + CP_DN_LAYERS)}


def bench_cp_block(args, dev, stream, max_over_ranks, barrier, world, rank) -> dict:
    """BASELINE config 5 (prefill part): one hybrid block (3 Gated DeltaNet + 1 gated GQA layer,
    independent seeded bf16-valued N(0,1) mixer inputs, no projections) over one sequence of
    T = 131072 tokens, context-parallel over the ranks: attention with zig-zag chunks and the KV
    direct KV exchange, DeltaNet with the state hand-off wavefront (miso_b200.cp). At one GPU the same
    code runs the whole sequence locally. Step = the block's prefill; tokens/s = T / step."""
    import torch
    from miso_b200 import attention as A
    from miso_b200 import cp

    t = args.cp_t
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    proj = torch.randn((t, cp.ATTN_PROJ), generator=g, device=dev).bfloat16().float()
    projs = [torch.randn((t, cp.DN_PROJ), generator=g, device=dev).bfloat16().float()
             for _ in range(CP_DN_LAYERS)]
    ones = torch.ones(DIM, device=dev)
    inv = torch.from_numpy(A.rope_inv_freq()).to(dev)
    conv_w = (0.5 * torch.randn((8192, 4), generator=g, device=dev)).bfloat16().float()
    ssm_a, dt = -torch.ones(32, device=dev), torch.zeros(32, device=dev)
    norm_w = torch.ones(128, device=dev)
    # The DeltaNet wavefront runs on its own stream and NCCL communicator, concurrently with the
    # attention layer (the layers are independent here), so that attention work fills the
    # wavefront's idle segments.
    # Higher priority: when attention CTAs retire, the block scheduler starts the wavefront's
    # CTAs first, so the sequential DeltaNet chain is not queued behind the whole attention grid.
    dn_stream = torch.cuda.Stream(device=dev, priority=-100)  # clamped to the highest
    dn_group = None
    if world > 1:
        import torch.distributed as dist
        # The state hand-off's NCCL kernels run on the communicator's own stream: at normal
        # priority the block scheduler holds them behind the attention grid's pending CTAs, so a
        # rank's DeltaNet could start only once the whole attention layer had been dispatched.
        opts = dist.ProcessGroupNCCL.Options(is_high_priority_stream=True)
        dn_group = dist.new_group(list(range(world)), backend="nccl", pg_options=opts)
        # The attention's KV exchange likewise: each exchange part needs every rank's send /
        # receive kernels, so one rank whose GPU is full of pending attention CTAs would stall it
        # for all ranks.
        ring_group = dist.new_group(list(range(world)), backend="nccl", pg_options=opts)
    else:
        ring_group = None
    attn = cp.GpuAttentionCp(t, world, rank, proj, ones, ones, inv, EPS, stream,
                             group=ring_group)
    dn = cp.GpuDeltaNetWavefront(t, world, rank, projs, conv_w, ssm_a, dt, norm_w, EPS,
                                 dn_stream, group=dn_group)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]

    def step(record=False):
        if record:
            ev[0].record(stream)
        dn_stream.wait_stream(stream)
        # The attention's prep and KV exchange are enqueued before the DeltaNet fronts (whose
        # high-priority grids would otherwise be dispatched first and hold the exchange back);
        # its big attention grids, enqueued here too, yield to the DeltaNet kernels by priority.
        attn.run()
        dn.run()
        if record:
            ev[1].record(stream)
            ev[2].record(dn_stream)
        stream.wait_stream(dn_stream)
        if record:
            ev[3].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    attn_ms = dn_ms = tot_ms = 0.0
    for _ in range(args.cp_steps):
        barrier()
        torch.cuda.synchronize()
        step(record=True)
        torch.cuda.synchronize()
        barrier()
        attn_ms += max_over_ranks(ev[0].elapsed_time(ev[1]))
        dn_ms += max_over_ranks(ev[0].elapsed_time(ev[2]))
        tot_ms += max_over_ranks(ev[0].elapsed_time(ev[3]))
    k = args.cp_steps
    attn_ms, dn_ms, tot_ms = attn_ms / k, dn_ms / k, tot_ms / k
    decode = cp_block_decode(args, dev, stream, max_over_ranks, barrier, world, rank, attn, dn,
                             dn_group, g)
    a_flops = 8192.0 * t * (t + 1)
    d_flops = CP_DN_LAYERS * 32 * (t // 64) * DN_PREFILL_FLOPS_PER_HEAD_CHUNK
    pk = peaks()
    a_tf = a_flops / (attn_ms * 1e-3) / 1e12
    return {"metric": f"hybrid block prefill tok/s @{t}", "value": t / (tot_ms * 1e-3),
            "unit": "tokens/s", "ms_per_step": tot_ms, "steps": k, "n_tokens": t,
            "scaling": "strong",
            "config": "BASELINE config 5 prefill: 1 x 131072 tokens over the ranks; 1 gated GQA "
                      "layer (config 3 shapes) context-parallel with zig-zag chunks and an NCCL "
                      "direct KV exchange; 3 Gated DeltaNet layers (config 4 shapes) as a state "
                      "hand-off wavefront over contiguous segments",
            "attention": {"ms": attn_ms, "tflops_per_gpu": a_tf / world, "flops": a_flops,
                          "frac_of_peak_per_gpu": a_tf / world / pk["bf16_tflops"],
                          "note": "time from the step start to the end of the attention layer, "
                                  "which shares the GPUs with the concurrent DeltaNet layers"},
            "deltanet": {"ms": dn_ms, "flops": d_flops, "layers": CP_DN_LAYERS,
                         "note": "time from the step start to the end of the wavefront (own "
                                 "stream and NCCL communicator, concurrent with attention)"},
            "decode": decode,
            "gpu_launches": k * (4 + 3 * CP_DN_LAYERS)}


def main():
    global BATCH
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["miso", "reference"], default="miso")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the prefill leg (BASELINE config 3) of the JSON line")
    ap.add_argument("--no-deltanet", action="store_true",
                    help="skip the DeltaNet legs (BASELINE config 4) of the JSON line")
    ap.add_argument("--prefill-n", type=int, default=PREFILL_N,
                    help="prefill tokens (default 8192, the BASELINE config; smaller only for "
                         "profiling captures)")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="sequences per GPU (default 32, the BASELINE config; smaller only for "
                         "profiling captures)")
    ap.add_argument("--cp-t", type=int, default=CP_T,
                    help="tokens of the context-parallel hybrid block (BASELINE config 5)")
    ap.add_argument("--cp-steps", type=int, default=3,
                    help="timed steps of the config 5 block (each is a 131072-token prefill)")
    ap.add_argument("--cp-decode-steps", type=int, default=CP_DEC_STEPS,
                    help="decode steps of the config 5 block after the prefix")
    ap.add_argument("--no-cp", action="store_true", help="skip the config 5 block")
    ap.add_argument("--no-decode-legs", action="store_true",
                    help="skip the fixed-32k and config-1 decode legs")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    BATCH = args.batch
    if args.impl == "reference":
        run_reference(args)
    else:
        run_miso(args)


if __name__ == "__main__":
    main()
