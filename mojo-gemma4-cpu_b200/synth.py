"""Seeded synthetic Gemma-4 MoE layers and tokens.

The reference publishes no checkpoint-free benchmark inputs, so tests and the
benchmark use synthetic tensors with the shapes of Gemma-4-26B-A4B's MoE block:
activations x ~ N(0,1), router/expert weights ~ N(0, 0.02) in bf16, norm gains
and per-expert scales 1.0 (HF init), optionally a "stress" variant with gains
~ N(1, 0.25) including negative entries (exercises the split-gain bake).

Butterquant layers are produced with the library's on-device restatement of
the reference quantizer (gm_bq_quantize_rows + gm_vnni_pack + router centering
+ the load-time bakes), i.e. the same procedure quant/quantizer.mojo and
Gemma4.model_init run, so no CPU code is involved.

torch provides the RNG and device memory only.
"""
import numpy as np
import torch

import gmoe

H, E, I, GU = gmoe.HIDDEN, gmoe.NUM_EXPERTS, gmoe.INTERMEDIATE, gmoe.GATE_UP


def _gen(seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_tokens(T, seed=0x6E6D6F45, device="cpu"):
    g = _gen(seed + 1, device)
    return torch.randn(T, H, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)


def make_layer(seed=0x6E6D6F45, device="cpu", weight_std=0.02, router_std=0.02,
               stress_gains=False, num_experts=E):
    """Raw (un-baked, un-quantised) bf16 tensors of one MoE layer."""
    g = _gen(seed, device)

    def normal(*shape, std=1.0, mean=0.0):
        t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
        return (t * std + mean).to(torch.bfloat16)

    L = {
        "router_proj": normal(E, H, std=router_std),
        "gate_up": normal(num_experts, GU, H, std=weight_std),
        "down": normal(num_experts, H, I, std=weight_std),
    }
    if stress_gains:
        L["router_scale"] = normal(H, std=0.25, mean=1.0)
        L["per_expert_scale"] = normal(E, std=0.25, mean=1.0)
        L["pre_ffn_norm_2"] = normal(H, std=0.25, mean=1.0)
    else:
        L["router_scale"] = torch.ones(H, dtype=torch.bfloat16, device=device)
        L["per_expert_scale"] = torch.ones(E, dtype=torch.bfloat16, device=device)
        L["pre_ffn_norm_2"] = torch.ones(H, dtype=torch.bfloat16, device=device)
    return L


def bake_router_scale(rs, stream=None):
    out = torch.empty_like(rs)
    gmoe.call("gm_bake_router_scale", rs, out, rs.numel(), gmoe._stream(stream))
    return out


def bf16_layer(raw):
    """Device tensors for gm_moe_register_layer_bf16 (router scale baked as
    modeling/gemma4_topology.mojo:362-388 does at model_init)."""
    d = {k: v.cuda().contiguous() for k, v in raw.items()}
    return {
        "gate_up": d["gate_up"], "down": d["down"], "router_proj": d["router_proj"],
        "router_scale": bake_router_scale(d["router_scale"]),
        "per_expert_scale": d["per_expert_scale"], "pre_ffn_norm_2": d["pre_ffn_norm_2"],
    }


def bq_layer(raw, keep_rowmajor=False):
    """Device tensors for gm_moe_register_layer_bq, produced by the reference's
    quantizer recipe (MoeGateUp = PerRowQuant(128, SplitGamma(pre_ffn_norm_2)),
    MoeDown = PerRowQuant(64, NoGamma), Router = SoftmaxRouterCenter;
    modeling/gemma_4_moe_bq.mojo:91-121) and load-time bakes."""
    d = {k: v.cuda().contiguous() for k, v in raw.items()}
    ne = d["gate_up"].shape[0]
    gu_q = torch.empty(ne * GU, H, dtype=torch.int8, device="cuda")
    gu_s = torch.empty(ne * GU, dtype=torch.float32, device="cuda")
    gmoe.call("gm_bq_quantize_rows", d["gate_up"], ne * GU, H, d["pre_ffn_norm_2"], 128, gu_q, gu_s,
              None)
    dn_q = torch.empty(ne * H, I, dtype=torch.int8, device="cuda")
    dn_s = torch.empty(ne * H, dtype=torch.float32, device="cuda")
    gmoe.call("gm_bq_quantize_rows", d["down"], ne * H, I, None, 64, dn_q, dn_s, None)
    gu_p = torch.empty_like(gu_q)
    gmoe.call("gm_vnni_pack", gu_q, ne * GU, H, gu_p, None)
    dn_p = torch.empty_like(dn_q)
    gmoe.call("gm_vnni_pack", dn_q, ne * H, I, dn_p, None)
    rc = torch.empty_like(d["router_proj"])
    gmoe.call("gm_router_center", d["router_proj"], E, H, rc, None)
    g2 = torch.empty_like(d["pre_ffn_norm_2"])
    gmoe.call("gm_bake_split_gain", d["pre_ffn_norm_2"], g2, H, None)
    out = {
        "gate_up": gu_p, "gate_up_scale": gu_s, "down": dn_p, "down_scale": dn_s,
        "router_centered": rc, "router_scale": bake_router_scale(d["router_scale"]),
        "per_expert_scale": d["per_expert_scale"], "pre_ffn_norm_2": g2,
    }
    if keep_rowmajor:
        out["gate_up_rowmajor"] = gu_q
        out["down_rowmajor"] = dn_q
    else:
        del gu_q, dn_q
    return out


def to_numpy_u16(t):
    """bf16 torch tensor -> uint16 numpy bit patterns (host)."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_numpy(t):
    if t.dtype == torch.bfloat16:
        return to_numpy_u16(t)
    return t.detach().contiguous().cpu().numpy()
