"""Generates tests/golden/golden.npz: outputs of the model's own reference implementations on the
seeded inputs of inputs.py. Run in a container that has `transformers` (the model code the
reference's golden tooling drives: tools/golden/make_golden.py:51-105, pinned there as
transformers==5.17.0; generated here with the installed version, recorded in the fixture).

  * prep:     Qwen3_5MoeRMSNorm (q_norm / k_norm) + apply_rotary_pos_emb (partial NEOX RoPE on 64
              dims) from transformers.models.qwen3_5_moe, cos / sin formed the HF way
              (fp32 inv_freq x position).
  * decode /  torch scaled_dot_product_attention in float64 with GQA (8 query heads per KV head),
    prefill   scale 1/16, causal offset mask for prefill, times sigmoid(gate) — the eager attention
              + gate of Qwen3_5MoeAttention.forward, evaluated in double.
  * deltanet: torch_causal_conv1d_update -> l2norm -> torch_recurrent_gated_delta_rule and
              torch_chunk_gated_delta_rule (chunk 64) -> Qwen3_5MoeRMSNormGated, with the tiled
              V-head order of the GGUF (V head h reads K head h % 16) made explicit by expanding
              q / k per V head.

The fixture stores outputs only (inputs are regenerated from the seeds) and, for DeltaNet, only
the V heads in inputs.DN_HEADS (outputs) and inputs.DN_STATE_HEAD (final state), all
as float32.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch
import torch.nn.functional as F
import transformers
from transformers.models.qwen3_5_moe import modeling_qwen3_5_moe as m

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import inputs as I  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


def golden_prep():
    x = I.prep_inputs()
    qn = m.Qwen3_5MoeRMSNorm(256, eps=I.EPS)
    kn = m.Qwen3_5MoeRMSNorm(256, eps=I.EPS)
    with torch.no_grad():
        qn.weight.copy_(torch.from_numpy(x["w_q"]))
        kn.weight.copy_(torch.from_numpy(x["w_k"]))
        q = torch.from_numpy(x["qg"][:, :256]).reshape(1, 16, 1, 256)
        k = torch.from_numpy(x["k"]).reshape(1, 2, 1, 256)
        q, k = qn(q), kn(k)
        inv = torch.from_numpy(x["inv_freq"])
        freqs = inv[None, :] * torch.tensor([[float(x["pos"])]], dtype=torch.float32)
        emb = torch.cat([freqs, freqs], dim=-1)  # [1, 64]
        cos, sin = emb.cos()[None], emb.sin()[None]  # [1, 1, 64]
        q, k = m.apply_rotary_pos_emb(q, k, cos, sin, unsqueeze_dim=1)
    return dict(prep_q=q.reshape(16, 256).numpy(), prep_k=k.reshape(2, 256).numpy())


def attend(q, k, v, gate, mask=None):
    """q [T, 16, 256], k / v [S, 2, 256] (float64), gate [T, 16, 256] -> [T, 16, 256]."""
    qq = torch.from_numpy(q).permute(1, 0, 2)[None]  # [1, 16, T, 256]
    kk = torch.from_numpy(k).permute(1, 0, 2)[None].repeat_interleave(8, dim=1)
    vv = torch.from_numpy(v).permute(1, 0, 2)[None].repeat_interleave(8, dim=1)
    o = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=1.0 / 16.0)
    o = o[0].permute(1, 0, 2).numpy()
    return o * (1.0 / (1.0 + np.exp(-gate)))


def golden_decode():
    x = I.decode_inputs()
    L = x["len"]
    k = x["k"][:, :L].astype(np.float64).transpose(1, 0, 2)
    v = x["v"][:, :L].astype(np.float64).transpose(1, 0, 2)
    out = attend(x["q"].astype(np.float64)[None], k, v, x["qg"][None, :, 256:].astype(np.float64))
    return dict(decode_out=out[0])


def golden_prefill():
    x = I.prefill_inputs()
    S = x["pos0"] + x["n"]
    k = x["k"][:, :S].astype(np.float64).transpose(1, 0, 2)
    v = x["v"][:, :S].astype(np.float64).transpose(1, 0, 2)
    t = np.arange(x["n"])[:, None] + x["pos0"]
    mask = torch.from_numpy(np.arange(S)[None, :] <= t)  # token t sees keys <= pos0 + t
    out = attend(x["q"].astype(np.float64), k, v, x["qg"][:, :, 256:].astype(np.float64), mask)
    return dict(prefill_out=out)


def golden_deltanet():
    x = I.deltanet_inputs()
    n = x["n"]
    with torch.no_grad():
        hs = torch.from_numpy(x["qkv"]).T[None]  # [1, 8192, n]
        conv_state = torch.from_numpy(x["conv_in"]).clone()[None]  # [1, 8192, 3]
        y = m.torch_causal_conv1d_update(hs, conv_state, torch.from_numpy(x["conv_w"]),
                                         activation="silu")[0].T  # [n, 8192]
        q = y[:, :2048].reshape(n, 16, 128)
        k = y[:, 2048:4096].reshape(n, 16, 128)
        v = y[:, 4096:].reshape(n, 32, 128)
        heads = torch.arange(32) % 16  # tiled V-head order: V head h <- K head h % 16
        qe, ke = q[:, heads][None], k[:, heads][None]  # [1, n, 32, 128]
        a = torch.from_numpy(x["a"]).double()
        g = (torch.from_numpy(x["ssm_a"]).double()[None]
             * F.softplus(a + torch.from_numpy(x["dt_bias"]).double()[None])).float()[None]
        beta = torch.sigmoid(torch.from_numpy(x["b"]))[None]
        s0 = torch.from_numpy(x["state"])[None]
        o_rec, s_rec = m.torch_recurrent_gated_delta_rule(
            qe, ke, v[None], g, beta, initial_state=s0, output_final_state=True,
            use_qk_l2norm_in_kernel=True)
        o_chk, s_chk = m.torch_chunk_gated_delta_rule(
            qe, ke, v[None], g, beta, chunk_size=64, initial_state=s0, output_final_state=True,
            use_qk_l2norm_in_kernel=True)
        norm = m.Qwen3_5MoeRMSNormGated(128, eps=I.EPS)
        norm.weight.copy_(torch.from_numpy(x["norm_w"]))
        z = torch.from_numpy(x["z"]).reshape(n, 32, 128)
        out_rec = norm(o_rec[0], z)
        out_chk = norm(o_chk[0], z)
    hs_ = list(I.DN_HEADS)
    sh = I.DN_STATE_HEAD
    return dict(dn_out_rec=out_rec[:, hs_].numpy(), dn_state_rec=s_rec[0, sh].numpy(),
                dn_out_chunk=out_chk[:, hs_].numpy(), dn_state_chunk=s_chk[0, sh].numpy())


def main():
    torch.manual_seed(0)
    d = {}
    for fn in (golden_prep, golden_decode, golden_prefill, golden_deltanet):
        d.update(fn())
    d = {k: np.asarray(v, dtype=np.float32) for k, v in d.items()}
    d["transformers_version"] = np.array(transformers.__version__)
    d["torch_version"] = np.array(torch.__version__)
    np.savez_compressed(OUT, **d)
    print(OUT, {k: v.shape for k, v in d.items()})


if __name__ == "__main__":
    main()
