"""Context-parallel prefill (miso_b200.cp): the partition arithmetic, and the multi-rank
orchestration run as gloo ranks on the CPU with the oracle in place of the kernels (attention:
zig-zag chunks + direct KV exchange; DeltaNet: state hand-off wavefront), bit-exact against a
single-process run."""
import os
import socket
import subprocess
import sys

import pytest

from miso_b200 import cp

WORKER = os.path.join(os.path.dirname(os.path.abspath(__file__)), "support", "cp_worker.py")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_zigzag_partition_covers_and_balances(world):
    t = 2 * world * 1024
    seen = []
    for r in range(world):
        for start, n in cp.zigzag_chunks(t, world, r):
            seen.extend(range(start, start + n))
            assert cp.chunk_owner(t, world, start // n) == r
    assert sorted(seen) == list(range(t))
    work = [cp.causal_work(cp.zigzag_chunks(t, world, r)) for r in range(world)]
    assert max(work) / min(work) < 1.001
    with pytest.raises(ValueError):
        cp.zigzag_chunks(t + 1, world, 0)


@pytest.mark.parametrize("world", [1, 3, 8])
def test_contiguous_segments_cover(world):
    t = 1000
    segs = [cp.contiguous_segment(t, world, r) for r in range(world)]
    assert segs[0][0] == 0 and sum(n for _, n in segs) == t
    assert all(a[0] + a[1] == b[0] for a, b in zip(segs, segs[1:]))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(case: str, world: int) -> None:
    port = free_port()
    env = dict(os.environ, OMP_NUM_THREADS="1")
    procs = [subprocess.Popen([sys.executable, WORKER, "--case", case, "--rank", str(r),
                               "--world", str(world), "--port", str(port)], env=env,
                              stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
             for r in range(world)]
    outs = []
    try:
        for p in procs:
            outs.append(p.communicate(timeout=240)[0].decode(errors="replace"))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    for r, (p, o) in enumerate(zip(procs, outs)):
        assert p.returncode == 0, f"rank {r} of {case} (world {world}) failed:\n{o[-3000:]}"


@pytest.mark.parametrize("world", [2, 3])
def test_attention_context_parallel_gloo(world):
    run_ranks("attention", world)


@pytest.mark.parametrize("world", [2, 3])
def test_deltanet_wavefront_gloo(world):
    run_ranks("deltanet", world)


@pytest.mark.parametrize("world", [2, 3])
def test_deltanet_affine_schedule_gloo(world):
    """Per-segment affine maps, all-gathered and composed, give the sequential recurrence."""
    run_ranks("deltanet_affine", world)


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_attention_exchange_schedule(world):
    """Per rank: prep of both own chunks, then the two exchange parts (low chunks, high chunks),
    then the low chunk r attended after part 0 (rank 0: without waiting), when the keys of
    chunks 0..r are present, and the high chunk after part 1. Part p sends this rank's chunk p to
    every other rank and receives theirs, so afterwards every rank holds every chunk."""
    t = 64 * world
    s = t // (2 * world)
    for rank in range(world):
        calls = []
        rec = lambda name: (lambda *a: calls.append((name,) + a))  # noqa: E731
        cp.AttentionCp(t, world, rank, rec("prep"), rec("exchange"), rec("attend")).run()
        low, high = cp.zigzag_chunks(t, world, rank)
        expect = [("prep",) + low, ("prep",) + high]
        if world > 1:
            expect += [("exchange", 0), ("exchange", 1)]
        expect += [("attend",) + low + (0 if rank > 0 else -1,),
                   ("attend",) + high + (1 if world > 1 else -1,)]
        assert calls == expect
        held = {low[0], high[0]}
        for part in (0, 1):
            pairs = cp.exchange_chunks(t, world, rank, part)
            assert sorted(p for p, _, _ in pairs) == [p for p in range(world) if p != rank]
            for peer, mine, theirs in pairs:
                assert mine == (low, high)[part][0]
                assert theirs == cp.zigzag_chunks(t, world, peer)[part][0]
                # symmetric: the peer sends this rank exactly what this rank receives
                assert (rank, theirs, mine) in cp.exchange_chunks(t, world, peer, part)
                held.add(theirs)
            if part == 0:  # the low chunk's keys: chunks 0..rank
                assert {c * s for c in range(rank + 1)} <= held
        assert held == {c * s for c in range(2 * world)}


@pytest.mark.parametrize("world", [1, 2, 4])
def test_deltanet_wavefront_call_order(world):
    """Per rank: the conv halos first (no compute behind them), then the state-independent front
    of every layer, then per layer receive state -> recurrence -> send state; rank 0 starts from
    reset() instead of a received halo / state, the last rank sends nothing."""
    layers, t = 3, 64 * world
    for rank in range(world):
        calls = []
        rec = lambda name: (lambda *a: calls.append((name,) + a))  # noqa: E731
        wf = cp.DeltaNetWavefront(t, world, rank, layers, rec("front"), rec("recur"),
                                  rec("reset"), rec("halo_recv"), rec("halo_send"), rec("recv"),
                                  rec("send"))
        wf.run()
        start, n = cp.contiguous_segment(t, world, rank)
        first, last = rank == 0, rank == world - 1
        expect = []
        for layer in range(layers):
            expect.append(("reset", layer) if first else ("halo_recv", layer))
            if not last:
                expect.append(("halo_send", layer))
        expect += [("front", layer, start, n) for layer in range(layers)]
        for layer in range(layers):
            if not first:
                expect.append(("recv", layer))
            expect.append(("recur", layer, start, n))
            if not last:
                expect.append(("send", layer))
        assert calls == expect


def test_deltanet_wavefront_rejects_segments_shorter_than_the_conv_halo():
    noop = lambda *a: None  # noqa: E731
    wf = cp.DeltaNetWavefront(4, 2, 0, 1, noop, noop, noop, noop, noop, noop, noop)
    with pytest.raises(ValueError):
        wf.run()


def test_deltanet_affine_composes_the_earlier_segments_in_order():
    """Rank r composes the maps of ranks 0 .. r - 1, in order, onto the initial state, after
    every layer's own maps were computed (no rank waits on a recurrence of another)."""
    world, layers, t = 4, 2, 64
    for rank in range(world):
        log = []
        af = cp.DeltaNetAffine(
            t, world, rank, layers,
            maps=lambda layer, s, n: (log.append(("maps", layer)) or (f"A{layer}", f"B{layer}")),
            gather=lambda layer, a, b: (log.append(("gather", layer)) or
                                        ([f"A{layer}r{r}" for r in range(world)],
                                         [f"B{layer}r{r}" for r in range(world)])),
            initial=lambda layer: "S0",
            compose=lambda a, s, b: f"({a}*{s}+{b})",
            final=lambda layer, s, n, st: log.append(("final", layer, st)),
            reset=lambda layer: log.append(("reset", layer)),
            halo_recv=lambda layer: log.append(("halo_recv", layer)),
            halo_send=lambda layer: log.append(("halo_send", layer)))
        af.run()
        kinds = [e[0] for e in log]
        assert kinds.index("gather") > max(i for i, k in enumerate(kinds) if k == "maps")
        finals = [e for e in log if e[0] == "final"]
        assert len(finals) == layers
        for layer, (_, lay, st) in enumerate(finals):
            want = "S0"
            for r in range(rank):
                want = f"(A{layer}r{r}*{want}+B{layer}r{r})"
            assert lay == layer and st == want
