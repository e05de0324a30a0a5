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
TOPK_K = gmoe.TOP_K


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


# ---------------------------------------------------------------- Zipf routing
ZIPF_S = 1.1
ZIPF_C = 16.0   # token shift along u (|x| is about sqrt(2816) = 53)


def zipf_targets(T, s=ZIPF_S):
    """Per-expert route counts for T tokens: 8T * i^-s / sum_j j^-s for the
    expert of rank i (expert i-1), capped at T (an expert is picked at most
    once per token); the overflow is re-spread over the uncapped experts in
    proportion to their shares."""
    w = np.arange(1, E + 1, dtype=np.float64) ** -s
    tgt = 8.0 * T * w / w.sum()
    capped = np.zeros(E, bool)
    for _ in range(E):
        over = tgt > T
        if not over.any():
            break
        capped |= over
        excess = float((tgt[over] - T).sum())
        tgt[over] = T
        free = ~capped
        tgt[free] += excess * w[free] / w[free].sum()
    return tgt


def zipf_direction(seed=0x6E6D6F45):
    """The fixed unit vector u of the skew (host f32)."""
    g = _gen(seed + 7, "cpu")
    u = torch.randn(H, generator=g, dtype=torch.float64)
    return (u / u.norm()).to(torch.float32)


def zipf_tokens(T, seed=0x6E6D6F45, device="cpu", c=ZIPF_C, u=None):
    """x + c*u (bf16) for x ~ N(0,1)."""
    u = zipf_direction() if u is None else u
    g = _gen(seed + 1, device)
    x = torch.randn(T, H, generator=g, device=device, dtype=torch.float32)
    return (x + c * u.to(device)).to(torch.bfloat16)


def apply_zipf(raw, T_cal=4096, iters=80, c=ZIPF_C, cal_seed=0x5A1F):
    """Adds beta_e * u to router row e so that the top-8 route counts of
    tokens x + c*u track zipf_targets (the skew direction of the synthetic
    Zipf(1.1) configs).  beta is calibrated on the host side from routed
    counts of T_cal calibration tokens: each round moves every expert's logit
    bias by a damped step of log(target) - log(count) until the counts track
    the targets.  Routing ranks are invariant to a common logit shift, so the
    butterquant router's centring (which removes the mean of beta) keeps the
    skew.  Returns the new raw dict (router_proj replaced)."""
    # computed on the host CPU so that every process derives identical weights
    dev = raw["router_proj"].device
    u = zipf_direction()
    x = zipf_tokens(T_cal, seed=cal_seed, device="cpu", c=c, u=u).float()
    inv = torch.rsqrt((x * x).mean(dim=1, keepdim=True) + 1e-6)
    rs = raw["router_scale"].float().cpu() * (H ** -0.5)
    sv = x * rs * inv                                  # router input, as the kernels form it
    W = raw["router_proj"].float().cpu()
    base = sv @ W.t()                                  # [T, E]
    us = sv @ u                                        # [T]: per-token weight of the bias
    tgt = torch.tensor(zipf_targets(T_cal), dtype=torch.float32)
    sigma = float(base.std())
    b = torch.zeros(E)
    for it in range(iters):
        lg = base + us[:, None] * (b / us.mean())[None, :]
        top = lg.topk(TOPK_K, dim=1).indices
        cnt = torch.bincount(top.reshape(-1), minlength=E).float()
        step = sigma * (0.5 if it < iters // 2 else 0.2)
        b = b + step * (torch.log(tgt + 1.0) - torch.log(cnt + 1.0))
    beta = b / us.mean()
    out = dict(raw)
    out["router_proj"] = (W + beta[:, None] * u[None, :]).to(torch.bfloat16).to(dev)
    return out


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


DENSE_I = 2112


def make_dense(seed=0x0D3E, device="cpu", weight_std=0.02, stress_gains=True):
    """Raw bf16 tensors of one layer's dense MLP (gate/up [2112][2816], down
    [2816][2112], pre_feedforward_layernorm gain)."""
    g = _gen(seed, device)

    def normal(*shape, std=1.0, mean=0.0):
        t = torch.randn(*shape, generator=g, device=device, dtype=torch.float32)
        return (t * std + mean).to(torch.bfloat16)

    return {"gate": normal(DENSE_I, H, std=weight_std), "up": normal(DENSE_I, H, std=weight_std),
            "down": normal(H, DENSE_I, std=weight_std),
            "pre_ffn_norm": normal(H, std=0.25 if stress_gains else 0.0, mean=1.0)}


def dense_layer(raw, keep_rowmajor=False):
    """Device tensors for gm_moe_register_dense_bq: the reference's DenseGateUp
    (PerRowQuant(128, SplitGamma(pre_feedforward_layernorm))) and DenseDown
    (PerRowQuant(64, NoGamma)) recipes, VNNI-packed, split gain baked."""
    d = {k: v.cuda().contiguous() for k, v in raw.items()}
    out = {}
    for name, rows, cols, gamma, block in (("gate", DENSE_I, H, d["pre_ffn_norm"], 128),
                                           ("up", DENSE_I, H, d["pre_ffn_norm"], 128),
                                           ("down", H, DENSE_I, None, 64)):
        q = torch.empty(rows, cols, dtype=torch.int8, device="cuda")
        sc = torch.empty(rows, dtype=torch.float32, device="cuda")
        gmoe.call("gm_bq_quantize_rows", d[name], rows, cols, gamma, block, q, sc, None)
        p = torch.empty_like(q)
        gmoe.call("gm_vnni_pack", q, rows, cols, p, None)
        out[name], out[name + "_scale"] = p, sc
        if keep_rowmajor:
            out[name + "_rowmajor"] = q
    g = torch.empty_like(d["pre_ffn_norm"])
    gmoe.call("gm_bake_split_gain", d["pre_ffn_norm"], g, H, None)
    out["pre_ffn_norm"] = g
    return out


def to_numpy_u16(t):
    """bf16 torch tensor -> uint16 numpy bit patterns (host)."""
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def to_numpy(t):
    if t.dtype == torch.bfloat16:
        return to_numpy_u16(t)
    return t.detach().contiguous().cpu().numpy()
