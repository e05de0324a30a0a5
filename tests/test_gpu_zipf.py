"""Prefill-size parity under the skewed routing of the benchmark configs
(configs 3 and 4: Zipf(1.1) expert load, synth.apply_zipf), against the CPU
oracle, through the C ABI.

The layer is the parity tests' stress layer (router std 1.0, gains with
negative entries) with the Zipf bias added to its router rows; the tokens are
x + c*u (synth.zipf_tokens).  The head expert then takes about one route per
token -- 32 m-tiles of 128 routes at 4096 tokens, 128 at 16384 -- which
exercises the tcgen05 kernels' multi-tile experts, the multi-CTA schedule and
the workspace at the sizes the benchmark runs.

Bars: expert indices bit-exact wherever the oracle's
top-8/9th logit margin exceeds 1e-3; outputs within 3e-2 (butterquant) /
2e-2 (bf16) of max|ref| on the tokens whose routing matches.  The oracle runs
in chunks of 1024 tokens (chunked = unchunked bit for bit, tests/test_oracle.py)."""
import numpy as np
import pytest
import torch

import gmoe
import synth
from oracle import oracle as O
from helpers import stress_layer, oracle_bf16_layer, rel_err, topk_margin, routes_by_expert

pytestmark = pytest.mark.gpu

H, E, TOPK = O.H, O.E, O.TOPK
TOL_BQ, TOL_BF16, MARGIN = 3e-2, 2e-2, 1e-3


def u16(t):
    return synth.to_numpy(t) if t.is_cuda else t.contiguous().view(torch.int16).numpy().view(np.uint16)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


@pytest.fixture(scope="module")
def zipf_layer():
    """(raw numpy, oracle bq layer, device bq layer, device bf16 layer) of the
    stress layer with the Zipf(1.1) router bias."""
    raw, ref = stress_layer()
    t = {k: torch.from_numpy(v.view(np.int16)).view(torch.bfloat16) for k, v in raw.items()}
    z = synth.apply_zipf(t)
    raw_z = dict(raw)
    raw_z["router_proj"] = u16(z["router_proj"])
    ref_z = dict(ref)
    ref_z["router_centered"] = O.router_center(raw_z["router_proj"])
    gq = synth.bq_layer(z)
    gb = synth.bf16_layer(z)
    return raw_z, ref_z, gq, gb


def oracle_chunked(fwd, x, layer, chunk=1024):
    outs, idxs, lgs = [], [], []
    for c in range(0, x.shape[0], chunk):
        o, i, _, lg = fwd(x[c:c + chunk], layer)
        outs.append(o)
        idxs.append(i)
        lgs.append(lg)
    return np.concatenate(outs), np.concatenate(idxs), np.concatenate(lgs)


def device_routes(g, router_key, x):
    T = x.shape[0]
    lg = torch.empty(gmoe.lib().gm_router_workspace_bytes(T) // 4, dtype=torch.float32, device="cuda")
    idx = torch.empty(T, TOPK, dtype=torch.int32, device="cuda")
    w = torch.empty(T, TOPK, dtype=torch.float32, device="cuda")
    gmoe.call("gm_router_select", x, g[router_key], g["router_scale"], g["per_expert_scale"], T, lg, idx,
              w, None)
    torch.cuda.synchronize()
    return synth.to_numpy(idx)


def check(out, gidx, rout, ridx, rlg, tol):
    margin = topk_margin(rlg)
    same = (routes_by_expert(gidx) == routes_by_expert(ridx)).all(axis=1)
    assert same[margin > MARGIN].all()
    assert (margin > MARGIN).mean() > 0.9
    err = rel_err(out, rout, rows=same)
    assert err < tol, err
    return err


def head_routes(idx):
    return np.bincount(idx.reshape(-1), minlength=E)


@pytest.mark.parametrize("T", [4096, 16384])
def test_forward_bq_zipf(T, zipf_layer):
    raw, ref, g, _ = zipf_layer
    x = synth.zipf_tokens(T, seed=0x2F + T)
    x_np = u16(x)
    xd = x.cuda()
    blk = gmoe.MoeBlock(T, 1)
    blk.register_bq(0, g["gate_up"], g["gate_up_scale"], g["down"], g["down_scale"], g["router_centered"],
                    g["router_scale"], g["per_expert_scale"], g["pre_ffn_norm_2"])
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    blk.profile(True)
    blk.forward(0, xd, out, T)
    stats, _ = blk.profile_read()
    torch.cuda.synchronize()
    assert blk.device_status() == 0
    assert "bq_phase2_down.tc" in stats  # the prefill kernels ran
    gidx = device_routes(g, "router_centered", xd)
    # the skew is there: the head expert takes about one route per token
    cnt = head_routes(gidx)
    assert cnt.max() > 0.7 * T and cnt[np.argsort(-cnt)[:4]].sum() > 2.5 * T
    rout, ridx, rlg = oracle_chunked(O.bq_forward, x_np, ref)
    check(synth.to_numpy(out), gidx, rout, ridx, rlg, TOL_BQ)
    if T == 4096:
        # the HBM-streaming decode kernels give the same bits on the same routing
        blk.set_option(gmoe.OPT_TC_MIN_TOKENS, 1 << 30)
        out2 = torch.empty_like(out)
        blk.forward(0, xd, out2, T)
        torch.cuda.synchronize()
        assert blk.device_status() == 0
        assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    blk.close()


def test_forward_bf16_zipf_4096(zipf_layer):
    raw, _, _, gb = zipf_layer
    T = 4096
    x = synth.zipf_tokens(T, seed=0x3F)
    x_np = u16(x)
    xd = x.cuda()
    blk = gmoe.MoeBlock(T, 1)
    blk.register_bf16(0, gb["gate_up"], gb["down"], gb["router_proj"], gb["router_scale"],
                      gb["per_expert_scale"], gb["pre_ffn_norm_2"])
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    blk.profile(True)
    blk.forward(0, xd, out, T)
    stats, _ = blk.profile_read()
    torch.cuda.synchronize()
    assert blk.device_status() == 0
    assert "phase2_down.tc" in stats
    gidx = device_routes(gb, "router_proj", xd)
    assert head_routes(gidx).max() > 0.7 * T
    rout, ridx, rlg = oracle_chunked(O.bf16_forward, x_np, oracle_bf16_layer(raw))
    check(synth.to_numpy(out), gidx, rout, ridx, rlg, TOL_BF16)
    blk.close()


def test_ep_group_zipf_prefill_one_gpu(zipf_layer):
    """Config 4's shape on one GPU: 4 members of an in-process expert-parallel
    group, 4096 Zipf tokens each (16384 in all), balanced expert placement;
    equal to the oracle's forward within the bq tolerance."""
    raw, ref, g, _ = zipf_layer
    G, T = 4, 4096
    x = synth.zipf_tokens(G * T, seed=0x4F)
    x_np = u16(x)
    xd = x.cuda()
    epr = E // G
    blks = []
    for r in range(G):
        b = gmoe.MoeBlock(T, 1, rank=r, degree=G)
        lo, hi = r * epr, (r + 1) * epr
        b.register_bq(0, g["gate_up"][lo * 1408:hi * 1408], g["gate_up_scale"][lo * 1408:hi * 1408],
                      g["down"][lo * H:hi * H], g["down_scale"][lo * H:hi * H], g["router_centered"],
                      g["router_scale"], g["per_expert_scale"], g["pre_ffn_norm_2"])
        blks.append(b)
    gmoe.ep_init_group(blks)
    gmoe.ep_set_placement_group(blks, gmoe.balanced_placement(synth.zipf_targets(T), G))
    outs = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(G)]
    gmoe.ep_forward_group(blks, 0, [xd[r * T:(r + 1) * T] for r in range(G)], outs, [T] * G)
    torch.cuda.synchronize()
    for b in blks:
        assert b.device_status() == 0
    got = synth.to_numpy(torch.cat(outs))
    gidx = device_routes(g, "router_centered", xd)
    rout, ridx, rlg = oracle_chunked(O.bq_forward, x_np, ref)
    check(got, gidx, rout, ridx, rlg, TOL_BQ)
    for b in blks:
        b.close()
