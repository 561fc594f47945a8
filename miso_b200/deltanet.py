"""Host side of the Gated DeltaNet hot path over torch device tensors.

Mirrors the kernel part of the reference engine's DeltaNet mixer (src/engine/deltanet.hip
:56-118): DeltaNetState with the double-buffered conv history and the fp32 [32][128][128] state
(src/engine/deltanet.hpp:24-33), decode = one step kernel then a parity flip, prefill = the fused
n-token recurrence then a parity flip. The chunked form (conv -> norm -> chunk) is exposed as in
the reference's test harness (tests/test_deltanet_chunk.hip:76-88).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _capi as capi
from .attention import _ptr, _stream

K_HEADS, V_HEADS, DIM, CHUNK = 16, 32, 128, 64
CHANNELS = 2 * K_HEADS * DIM + V_HEADS * DIM  # 8192
PROJ = 12352  # DeltaNetScratch::kProj: [qkv 8192 | z 4096 | a 32 | b 32]


class DeltaNetState:
    def __init__(self, device="cuda"):
        self.conv = [torch.zeros((CHANNELS, 3), dtype=torch.float32, device=device)
                     for _ in range(2)]
        self.s = torch.zeros((V_HEADS, DIM, DIM), dtype=torch.float32, device=device)
        self.parity = 0

    def reset(self):
        for c in self.conv:
            c.zero_()
        self.s.zero_()
        self.parity = 0


def step(p: capi.DeltaNetStepParams, stream=None) -> None:
    capi.check("miso_deltanet_step", capi.load().miso_deltanet_step(C.byref(p), _stream(stream)))


def seq(p: capi.DeltaNetSeqParams, stream=None) -> None:
    capi.check("miso_deltanet_seq", capi.load().miso_deltanet_seq(C.byref(p), _stream(stream)))


def conv(p: capi.DeltaNetConvParams, stream=None) -> None:
    capi.check("miso_deltanet_conv", capi.load().miso_deltanet_conv(C.byref(p), _stream(stream)))


def norm(p: capi.DeltaNetConvParams, stream=None) -> None:
    capi.check("miso_deltanet_norm", capi.load().miso_deltanet_norm(C.byref(p), _stream(stream)))


def chunk(p: capi.DeltaNetChunkParams, stream=None) -> None:
    capi.check("miso_deltanet_chunk",
               capi.load().miso_deltanet_chunk(C.byref(p), _stream(stream)))


def deltanet_decode_core(st: DeltaNetState, proj: torch.Tensor, conv_w, ssm_a, dt_bias, norm_w,
                         out: torch.Tensor, eps: float, stream=None) -> torch.Tensor:
    """One token from its [12352] projection row (src/engine/deltanet.hip:66-81)."""
    base = proj.data_ptr()
    p = capi.DeltaNetStepParams(base, base + 8192 * 4, base + 12288 * 4, base + 12320 * 4,
                                _ptr(conv_w), _ptr(st.conv[st.parity]),
                                _ptr(st.conv[1 - st.parity]), _ptr(ssm_a), _ptr(dt_bias),
                                _ptr(norm_w), _ptr(st.s), _ptr(out), eps)
    step(p, stream)
    st.parity = 1 - st.parity
    return out


def deltanet_prefill_core(st: DeltaNetState, proj: torch.Tensor, n: int, conv_w, ssm_a, dt_bias,
                          norm_w, out: torch.Tensor, eps: float, stream=None) -> torch.Tensor:
    """n tokens from a [n][12352] projection buffer (src/engine/deltanet.hip:97-115)."""
    base = proj.data_ptr()
    z = base + 8192 * 4
    p = capi.DeltaNetSeqParams(base, z, z + 4096 * 4, z + 4128 * 4, _ptr(conv_w),
                               _ptr(st.conv[st.parity]), _ptr(st.conv[1 - st.parity]),
                               _ptr(ssm_a), _ptr(dt_bias), _ptr(norm_w), _ptr(st.s), _ptr(out),
                               n, eps, PROJ, PROJ)
    seq(p, stream)
    st.parity = 1 - st.parity
    return out


class DraftCheckpoints:
    """Per-token state / conv-history checkpoints of a speculative verification pass of up to
    max_tokens draft tokens (multi-token prediction: the reference's planned commit / rollback of
    2-4 accepted tokens, docs/decisions/ADR_002-build-scope-numerics-ops.md D8)."""

    def __init__(self, max_tokens: int, device="cuda"):
        self.max_tokens = max_tokens
        self.state = torch.empty((max_tokens, V_HEADS, DIM, DIM), dtype=torch.float32,
                                 device=device)
        self.conv = torch.empty((max_tokens, CHANNELS, 3), dtype=torch.float32, device=device)
        self.n = 0


def deltanet_verify_core(st: DeltaNetState, ck: DraftCheckpoints, proj: torch.Tensor, n: int,
                         conv_w, ssm_a, dt_bias, norm_w, out: torch.Tensor, eps: float,
                         stream=None) -> torch.Tensor:
    """n draft tokens from a [n][12352] projection buffer: outputs as deltanet_prefill_core, the
    layer state left as it was and checkpoints taken after every token."""
    if not 0 < n <= ck.max_tokens:
        raise ValueError(f"verify: {n} tokens, checkpoints hold {ck.max_tokens}")
    base = proj.data_ptr()
    z = base + 8192 * 4
    p = capi.DeltaNetSeqParams(base, z, z + 4096 * 4, z + 4128 * 4, _ptr(conv_w),
                               _ptr(st.conv[st.parity]), None, _ptr(ssm_a), _ptr(dt_bias),
                               _ptr(norm_w), _ptr(st.s), _ptr(out), n, eps, PROJ, PROJ)
    capi.check("miso_deltanet_seq_ckpt",
               capi.load().miso_deltanet_seq_ckpt(C.byref(p), _ptr(ck.state), _ptr(ck.conv),
                                                  _stream(stream)))
    ck.n = n
    return out


def deltanet_commit(st: DeltaNetState, ck: DraftCheckpoints, k_accepted: int,
                    stream=None) -> None:
    """Keeps the first k_accepted verified tokens (0 keeps the state from before the pass)."""
    capi.check("miso_deltanet_commit",
               capi.load().miso_deltanet_commit(_ptr(ck.state), _ptr(ck.conv), ck.n, k_accepted,
                                                _ptr(st.s), _ptr(st.conv[1 - st.parity]),
                                                _stream(stream)))
    if k_accepted > 0:
        st.parity = 1 - st.parity
