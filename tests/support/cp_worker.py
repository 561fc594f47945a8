"""One rank of the gloo (CPU) tests of miso_b200.cp: the context-parallel orchestration with the
CPU oracle standing in for the kernels. Exits non-zero if this rank's checks fail.

  python cp_worker.py --case attention|deltanet --rank R --world W --port P
"""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import oracle  # noqa: E402
from miso_b200 import cp  # noqa: E402


def attention_case(rank: int, world: int) -> None:
    t = 16 * world
    rng = np.random.RandomState(5)
    k_full = (0.5 * rng.standard_normal((2, t, 256))).astype(np.float16)
    v_full = rng.standard_normal((2, t, 256)).astype(np.float16)
    q = (0.3 * rng.standard_normal((t, 16, 256))).astype(np.float32)
    qg = rng.standard_normal((t, 8192)).astype(np.float32)
    k_loc = torch.zeros((2, t, 256), dtype=torch.float16)
    v_loc = torch.zeros_like(k_loc)
    out = np.zeros((t, 16, 256))

    def prep(start, n):
        k_loc[:, start:start + n] = torch.from_numpy(k_full[:, start:start + n])
        v_loc[:, start:start + n] = torch.from_numpy(v_full[:, start:start + n])

    def exchange(part):
        s = t // (2 * world)
        # Pairwise in a fixed order (lower rank sends first) so that blocking gloo calls pair up.
        for peer, mine, theirs in cp.exchange_chunks(t, world, rank, part):
            for cache in (k_loc, v_loc):
                for h in range(2):
                    buf = torch.empty((s, 256), dtype=torch.float16)
                    if rank < peer:
                        dist.send(cache[h, mine:mine + s].contiguous(), peer)
                        dist.recv(buf, peer)
                    else:
                        dist.recv(buf, peer)
                        dist.send(cache[h, mine:mine + s].contiguous(), peer)
                    cache[h, theirs:theirs + s] = buf

    def attend(start, n, after):
        kb = k_loc.numpy().view(np.uint16)
        vb = v_loc.numpy().view(np.uint16)
        out[start:start + n] = oracle.attn_prefill(n, start, q[start:start + n],
                                                   qg[start:start + n], 8192, kb, vb, t)

    cp.AttentionCp(t, world, rank, prep, exchange, attend).run()
    # Every rank now holds the whole cache.
    assert np.array_equal(k_loc.numpy(), k_full) and np.array_equal(v_loc.numpy(), v_full)
    total = torch.from_numpy(out)
    dist.all_reduce(total)  # each row is written by exactly one rank
    ref = oracle.attn_prefill(t, 0, q, qg, 8192, k_full.view(np.uint16), v_full.view(np.uint16), t)
    assert np.array_equal(total.numpy(), ref), "context-parallel attention differs"


def deltanet_case(rank: int, world: int) -> None:
    t, layers = 5 * world + 2, 2
    ins = []
    for layer in range(layers):
        rng = np.random.RandomState(100 + layer)
        nd = lambda *s: (0.5 * rng.standard_normal(s)).astype(np.float32)  # noqa: E731
        ins.append(dict(qkv=nd(t, 8192), zab=nd(t, 4160), conv_w=nd(8192, 4),
                        ssm_a=(-0.05 * (np.arange(32) + 1)).astype(np.float32),
                        dt=(0.1 * np.arange(32)).astype(np.float32),
                        norm_w=(1.0 + 0.01 * (np.arange(128) - 64)).astype(np.float32)))
    state = [np.zeros((32, 128, 128)) for _ in range(layers)]
    conv = [np.zeros((8192, 3)) for _ in range(layers)]
    out = [np.zeros((t, 4096)) for _ in range(layers)]

    def front(layer, start, n):
        pass  # the oracle runs the conv and the recurrence together in recur()

    def recur(layer, start, n):
        x = ins[layer]
        out[layer][start:start + n] = oracle.deltanet_seq(
            n, x["qkv"][start:start + n], 8192, x["zab"][start:start + n], 4160, x["conv_w"],
            conv[layer], x["ssm_a"], x["dt"], x["norm_w"], state[layer], 1e-6)

    def reset(layer):
        state[layer][:] = 0
        conv[layer][:] = 0

    def halo_recv(layer):
        buf = torch.empty(conv[layer].shape, dtype=torch.float64)
        dist.recv(buf, rank - 1)
        conv[layer][:] = buf.numpy()

    def halo_send(layer):
        start, n = cp.contiguous_segment(t, world, rank)
        rows = ins[layer]["qkv"][start + n - 3:start + n].astype(np.float64)  # [3][8192]
        dist.send(torch.from_numpy(np.ascontiguousarray(rows.T)), rank + 1)

    def recv(layer):
        buf = torch.empty(state[layer].shape, dtype=torch.float64)
        dist.recv(buf, rank - 1)
        state[layer][:] = buf.numpy()

    def send(layer):
        dist.send(torch.from_numpy(state[layer].copy()), rank + 1)

    cp.DeltaNetWavefront(t, world, rank, layers, front, recur, reset, halo_recv, halo_send, recv,
                         send).run()
    for layer in range(layers):
        total = torch.from_numpy(out[layer])
        dist.all_reduce(total)
        x = ins[layer]
        s64, c64 = np.zeros((32, 128, 128)), np.zeros((8192, 3))
        ref = oracle.deltanet_seq(t, x["qkv"], 8192, x["zab"], 4160, x["conv_w"], c64,
                                  x["ssm_a"], x["dt"], x["norm_w"], s64, 1e-6)
        assert np.array_equal(total.numpy(), ref), f"layer {layer}: outputs differ"
        if rank == world - 1:
            assert np.array_equal(state[layer], s64), f"layer {layer}: final state differs"
            assert np.array_equal(conv[layer], c64), f"layer {layer}: conv history differs"


def deltanet_affine_case(rank: int, world: int) -> None:
    """The affine schedule with the fp64 oracle as the segment runs: outputs and final state
    within 1e-10 of one process running the whole sequence (the composition reassociates)."""
    t, layers = 5 * world + 2, 2
    ins = []
    for layer in range(layers):
        rng = np.random.RandomState(200 + layer)
        nd = lambda *s: (0.5 * rng.standard_normal(s)).astype(np.float32)  # noqa: E731
        ins.append(dict(qkv=nd(t, 8192), zab=nd(t, 4160), conv_w=nd(8192, 4),
                        ssm_a=(-0.05 * (np.arange(32) + 1)).astype(np.float32),
                        dt=(0.1 * np.arange(32)).astype(np.float32),
                        norm_w=(1.0 + 0.01 * (np.arange(128) - 64)).astype(np.float32)))
    halo = [np.zeros((8192, 3)) for _ in range(layers)]
    out = [np.zeros((t, 4096)) for _ in range(layers)]
    final_state = [None] * layers

    def run_segment(layer, start, n, qkv, conv, state):
        x = ins[layer]
        return oracle.deltanet_seq(n, np.ascontiguousarray(qkv), 8192,
                                   x["zab"][start:start + n], 4160, x["conv_w"], conv,
                                   x["ssm_a"], x["dt"], x["norm_w"], state, 1e-6)

    def maps(layer, start, n):
        qkv = ins[layer]["qkv"][start:start + n]
        qkv0 = qkv.copy()
        qkv0[:, 4096:] = 0.0               # value channels
        conv0 = halo[layer].copy()
        conv0[4096:] = 0.0
        a = np.broadcast_to(np.eye(128), (32, 128, 128)).copy()
        run_segment(layer, start, n, qkv0, conv0, a)
        b = np.zeros((32, 128, 128))
        run_segment(layer, start, n, qkv, halo[layer].copy(), b)
        return a, b

    def gather(layer, a, b):
        a_all = [torch.empty(a.shape, dtype=torch.float64) for _ in range(world)]
        b_all = [torch.empty(b.shape, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(a_all, torch.from_numpy(a))
        dist.all_gather(b_all, torch.from_numpy(b))
        return [x.numpy() for x in a_all], [x.numpy() for x in b_all]

    def final(layer, start, n, s):
        state = s.copy()
        out[layer][start:start + n] = run_segment(layer, start, n,
                                                  ins[layer]["qkv"][start:start + n],
                                                  halo[layer].copy(), state)
        final_state[layer] = state

    def reset(layer):
        halo[layer][:] = 0

    def halo_recv(layer):
        buf = torch.empty(halo[layer].shape, dtype=torch.float64)
        dist.recv(buf, rank - 1)
        halo[layer][:] = buf.numpy()

    def halo_send(layer):
        start, n = cp.contiguous_segment(t, world, rank)
        rows = ins[layer]["qkv"][start + n - 3:start + n].astype(np.float64)
        dist.send(torch.from_numpy(np.ascontiguousarray(rows.T)), rank + 1)

    cp.DeltaNetAffine(t, world, rank, layers, maps, gather, lambda layer: np.zeros((32, 128, 128)),
                      lambda a, s, b: np.einsum("hkm,hmv->hkv", a, s) + b, final, reset,
                      halo_recv, halo_send).run()
    for layer in range(layers):
        total = torch.from_numpy(out[layer])
        dist.all_reduce(total)
        x = ins[layer]
        s64, c64 = np.zeros((32, 128, 128)), np.zeros((8192, 3))
        ref = oracle.deltanet_seq(t, x["qkv"], 8192, x["zab"], 4160, x["conv_w"], c64,
                                  x["ssm_a"], x["dt"], x["norm_w"], s64, 1e-6)
        err = np.abs(total.numpy() - ref).max() / np.abs(ref).max()
        assert err < 1e-10, f"layer {layer}: outputs differ by {err:.3g}"
        if rank == world - 1:
            serr = np.abs(final_state[layer] - s64).max() / np.abs(s64).max()
            assert serr < 1e-10, f"layer {layer}: final state differs by {serr:.3g}"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True)
    ap.add_argument("--rank", type=int, required=True)
    ap.add_argument("--world", type=int, required=True)
    ap.add_argument("--port", type=int, required=True)
    a = ap.parse_args()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{a.port}", rank=a.rank,
                            world_size=a.world)
    try:
        {"attention": attention_case, "deltanet": deltanet_case,
         "deltanet_affine": deltanet_affine_case}[a.case](a.rank, a.world)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
