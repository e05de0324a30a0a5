"""Expert parallelism on ONE GPU: an in-process group of G handles
(gm_moe_ep_init_group), each holding 128/G experts and its own tokens, runs
the whole exchange of the multi-process forward -- plan, pack by peer stores,
the flag waits, the receiver's schedule and experts, the combine's stores into
the sources' contribution blocks, the rank-order final sum -- through
gm_moe_ep_forward_group.  The result must equal, bit for bit, the rank-order
sum of the degree-G partials that plain degree-G handles compute over all
tokens (the reference's sharded experts plus dispatch_allreduce_inplace,
kernels/reductions.mojo:186-204), and match the oracle's degree-G forward
within the north-star tolerance.

Failure detection, in the forms allowed on a shared GPU: a member whose peer
never runs its forward waits on flags that nothing sets and the wait bound
(GM_OPT_EP_TIMEOUT_MS) turns that into GM_ETIMEOUT from gm_moe_device_status;
a communicator whose second rank never joins returns GM_ETIMEOUT from
gm_moe_ep_init (host-side deadline, no kernel involved)."""
import time

import numpy as np
import pytest
import torch

import gmoe
import synth
from oracle import oracle as O
from helpers import stress_layer, tokens_np, oracle_bf16_layer, rel_err, topk_margin

pytestmark = pytest.mark.gpu

H, E, GU, TOPK = O.H, O.E, O.GU, O.TOPK
TOL_BQ, TOL_BF16, MARGIN = 3e-2, 2e-2, 1e-3


def raw_to_torch(raw):
    return {k: torch.from_numpy(v.view(np.int16)).view(torch.bfloat16) for k, v in raw.items()}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).cuda()


@pytest.fixture(scope="module")
def layers():
    raw, ref = stress_layer()
    t = raw_to_torch(raw)
    return raw, ref, synth.bq_layer(t), synth.bf16_layer(t)


def register(blk, fmt, g, rank, degree):
    epr = E // degree
    lo, hi = rank * epr, (rank + 1) * epr
    if fmt == "bq":
        blk.register_bq(0, g["gate_up"][lo * GU:hi * GU], g["gate_up_scale"][lo * GU:hi * GU],
                        g["down"][lo * H:hi * H], g["down_scale"][lo * H:hi * H],
                        g["router_centered"], g["router_scale"], g["per_expert_scale"],
                        g["pre_ffn_norm_2"])
    else:
        blk.register_bf16(0, g["gate_up"][lo:hi], g["down"][lo:hi], g["router_proj"],
                          g["router_scale"], g["per_expert_scale"], g["pre_ffn_norm_2"])


def make_group(fmt, g, G, T):
    blks = [gmoe.MoeBlock(T, 1, rank=r, degree=G) for r in range(G)]
    for r, b in enumerate(blks):
        register(b, fmt, g, r, G)
    gmoe.ep_init_group(blks)
    return blks


def partial_sum(fmt, g, G, x_all):
    """Rank-order f32 sum of the degree-G bf16 partials over all tokens."""
    n = x_all.shape[0]
    acc = torch.zeros(n, H, dtype=torch.float32, device="cuda")
    for r in range(G):
        b = gmoe.MoeBlock(n, 1, rank=r, degree=G)
        register(b, fmt, g, r, G)
        p = torch.empty(n, H, dtype=torch.bfloat16, device="cuda")
        b.forward(0, x_all, p, n)
        acc += p.float()
        torch.cuda.synchronize()
        b.close()
    return acc.to(torch.bfloat16)


# T per member: decode size, and >= 512 so that the G*T received rows run the
# tcgen05 prefill kernels (>= 1024 rows).  The members and the reference
# handles over all G*T tokens must pick the same router kernel (the FMA one
# below 512 tokens, the tcgen05 one from 512), whose logits differ in their
# last bits: both T and G*T lie on the same side of 512.
@pytest.mark.parametrize("fmt,G,T", [("bq", 2, 64), ("bq", 4, 64), ("bq", 2, 640), ("bq", 4, 640),
                                     ("bf16", 2, 48), ("bf16", 2, 512)])
def test_ep_group_one_gpu_bit_exact(fmt, G, T, layers):
    raw, ref, gq, gb = layers
    g = gq if fmt == "bq" else gb
    x_np = tokens_np(G * T, seed=5000 + 7 * G + T)
    x_all = dev(x_np)
    blks = make_group(fmt, g, G, T)
    xs = [x_all[r * T:(r + 1) * T] for r in range(G)]
    outs = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(G)]
    for b in blks:
        b.profile(True)
    first = None
    for it in range(3):  # both parities of the exchange regions, then reuse
        gmoe.ep_forward_group(blks, 0, xs, outs, [T] * G)
        torch.cuda.synchronize()
        got = torch.cat(outs)
        if first is None:
            first = got.clone()
        else:
            assert torch.equal(got.view(torch.int16), first.view(torch.int16))
    for b in blks:
        assert b.device_status() == 0
    stats, launches = blks[0].profile_read()
    for label in ("ep_plan", "ep_pack.p2p", "ep_dispatch.wait", "ep_schedule", "combine.p2p",
                  "ep_combine.wait", "ep_final"):
        assert label in stats, sorted(stats)
    assert stats["ep_final"]["calls"] == 3 and launches > 0
    if fmt == "bq" and G * T >= 1024:
        assert "bq_phase2_down.tc" in stats
    # bit for bit the reference's sharded experts plus all-reduce
    want = partial_sum(fmt, g, G, x_all)
    assert torch.equal(first.view(torch.int16), want.view(torch.int16))
    # and the oracle's degree-G forward where routing is unambiguous
    if fmt == "bq":
        rout, _, _, rlg = O.bq_forward(x_np, ref, degree=G)
        tol = TOL_BQ
    else:
        rout, _, _, rlg = O.bf16_forward(x_np, oracle_bf16_layer(raw), degree=G)
        tol = TOL_BF16
    checked = topk_margin(rlg) > MARGIN
    assert checked.mean() > 0.9
    assert rel_err(synth.to_numpy(first), rout, rows=checked) < tol
    for b in blks:
        b.close()


def test_ep_group_uneven_tokens_and_empty_member(layers):
    """Members pass different token counts, one of them none."""
    raw, ref, g, _ = layers
    G, cap = 4, 96
    Ts = [96, 0, 17, 64]
    x_np = tokens_np(sum(Ts), seed=5100)
    x_all = dev(x_np)
    blks = make_group("bq", g, G, cap)
    off = np.r_[0, np.cumsum(Ts)]
    xs = [x_all[off[r]:off[r + 1]] if Ts[r] else x_all[:1] for r in range(G)]
    outs = [torch.empty(max(t, 1), H, dtype=torch.bfloat16, device="cuda") for t in Ts]
    gmoe.ep_forward_group(blks, 0, xs, outs, Ts)
    torch.cuda.synchronize()
    for b in blks:
        assert b.device_status() == 0
    got = torch.cat([outs[r][:Ts[r]] for r in range(G) if Ts[r]])
    want = partial_sum("bq", g, G, x_all)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    for b in blks:
        b.close()


def test_ep_group_placement_one_gpu(layers):
    """gm_moe_ep_set_placement_group: experts moved between the members by
    load; equals the oracle's per-rank partials over the placed experts summed
    in rank order (the multi-process placement test's criterion)."""
    from test_ep_protocol import placement_tables, rank_weights, rank_partial
    raw, ref, g, _ = layers
    G, T = 4, 160
    load = np.arange(E, 0, -1).astype(float) ** 1.1
    rank_of = np.array(gmoe.balanced_placement(load, G), np.int32)
    blks = make_group("bq", g, G, T)
    gmoe.ep_set_placement_group(blks, rank_of)
    x_np = tokens_np(G * T, seed=5200)
    x_all = dev(x_np)
    xs = [x_all[r * T:(r + 1) * T] for r in range(G)]
    outs = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(G)]
    for _ in range(2):
        gmoe.ep_forward_group(blks, 0, xs, outs, [T] * G)
    torch.cuda.synchronize()
    for b in blks:
        assert b.device_status() == 0
    got = synth.to_numpy(torch.cat(outs))
    idx, w, lg = O.router(x_np, ref["router_centered"], ref["router_scale"], ref["pes"])
    xi8, xsa = O.bq_norm_quant(x_np, ref["gamma2"])
    epr = E // G
    local_of = placement_tables(rank_of, G)
    acc = np.zeros((x_np.shape[0], H), np.float32)
    for r in range(G):
        Wr = rank_weights(ref, [e for e in range(E) if rank_of[e] == r])
        ridx = np.where(rank_of[idx] == r, r * epr + local_of[idx], -1).astype(np.int32)
        acc = acc + O.bf16_to_f32(rank_partial(xi8, xsa, ridx, w, Wr, r, epr))
    want = O.f32_to_bf16(acc)
    checked = topk_margin(lg) > MARGIN
    assert checked.mean() > 0.9
    assert rel_err(got, want, rows=checked) < TOL_BQ
    for b in blks:
        b.close()


def test_ep_wait_bound_expires_when_a_peer_never_runs(layers):
    """Member 0 runs its forward alone: the flags of member 1 are never
    published, the bounded waits give up after GM_OPT_EP_TIMEOUT_MS and the
    status reports GM_ETIMEOUT; the GPU context stays usable."""
    raw, ref, g, _ = layers
    T = 16
    blks = make_group("bq", g, 2, T)
    blks[0].set_option(gmoe.OPT_EP_TIMEOUT_MS, 50)
    x = dev(tokens_np(T, seed=5300))
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    t0 = time.time()
    blks[0].forward(0, x, out, T)
    with pytest.raises(gmoe.GmoeError, match="GM_ETIMEOUT"):
        blks[0].device_status()
    assert time.time() - t0 < 20
    # the context is intact: a plain handle still computes
    plain = gmoe.MoeBlock(T, 1)
    register(plain, "bq", g, 0, 1)
    plain.forward(0, x, out, T)
    torch.cuda.synchronize()
    assert plain.device_status() == 0
    plain.close()
    # destroying one member dissolves the group
    blks[1].close()
    with pytest.raises(gmoe.GmoeError, match="GM_ESTATE"):
        blks[0].forward(0, x, out, T)
    blks[0].close()


def test_ep_group_argument_checks(layers):
    raw, ref, g, _ = layers
    T = 8
    blks = make_group("bq", g, 2, T)
    x = dev(tokens_np(2 * T, seed=5400))
    outs = [torch.empty(T, H, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    xs = [x[:T], x[T:]]
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):  # one GPU, two streams
        gmoe.ep_forward_group(blks, 0, xs, outs, [T, T], [s1, s2])
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):  # members out of order
        gmoe.ep_forward_group(blks[::-1], 0, xs, outs, [T, T])
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):  # too many tokens
        gmoe.ep_forward_group(blks, 0, xs, outs, [T + 1, T])
    with pytest.raises(gmoe.GmoeError, match="GM_ESTATE"):  # no communicator in a group
        blks[0].set_option(gmoe.OPT_EP_TRANSPORT, 0)
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):
        blks[0].set_option(gmoe.OPT_EP_TIMEOUT_MS, 0)
    with pytest.raises(gmoe.GmoeError, match="GM_ESTATE"):  # already in a group
        gmoe.ep_init_group(blks)
    other = gmoe.MoeBlock(T, 1, rank=1, degree=2)
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):  # rank 0 slot holds rank 1
        gmoe.ep_init_group([other, other])
    # one stream for both (the same stream object) runs
    gmoe.ep_forward_group(blks, 0, xs, outs, [T, T], [s1, s1])
    torch.cuda.synchronize()
    assert blks[0].device_status() == 0 and blks[1].device_status() == 0
    for b in blks + [other]:
        b.close()


def test_ep_init_deadline_when_a_rank_never_joins():
    """Rank 1 of a 2-rank communicator never calls gm_moe_ep_init: rank 0's
    non-blocking initialisation is polled against GM_OPT_EP_INIT_TIMEOUT_MS,
    aborted, and returns GM_ETIMEOUT (host side only; no kernel runs)."""
    blk = gmoe.MoeBlock(8, 1, rank=0, degree=2)
    blk.set_option(gmoe.OPT_EP_INIT_TIMEOUT_MS, 1500)
    uid = gmoe.ep_unique_id()
    t0 = time.time()
    with pytest.raises(gmoe.GmoeError, match="GM_ETIMEOUT"):
        blk.ep_init(uid, 2)
    assert time.time() - t0 < 60
    blk.close()
