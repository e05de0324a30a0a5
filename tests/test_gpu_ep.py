"""Expert-parallel forward on 2 GPUs (one process per GPU, NCCL inside the
library).  Each rank passes only its own tokens; the result must equal, bit
for bit, the rank-order sum of the degree-2 partial outputs that the
non-parallel handles compute over all tokens (the reference's sharded experts
plus all-reduce), and match the oracle's degree-2 forward within tolerance."""
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import gmoe
import synth
from oracle import oracle as O
from helpers import raw_layer_np, tokens_np, oracle_bq_layer, oracle_bf16_layer, rel_err, topk_margin

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

H, E, GU, TOPK = O.H, O.E, O.GU, O.TOPK
WORLD = 2
TOL_BQ, TOL_BF16, MARGIN = 3e-2, 2e-2, 1e-3


def raw_to_torch(raw):
    return {k: torch.from_numpy(v.view(np.int16)).view(torch.bfloat16) for k, v in raw.items()}


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


def worker(rank, fmt, T, uid, tmp, placement=None):
    torch.cuda.set_device(rank)
    raw = raw_layer_np(seed=4321, router_std=1.0, stress=True)
    g = synth.bq_layer(raw_to_torch(raw)) if fmt == "bq" else synth.bf16_layer(raw_to_torch(raw))
    x_all = torch.from_numpy(tokens_np(WORLD * T, seed=500 + T).view(np.int16)).view(torch.bfloat16).cuda()
    # expert-parallel handle: this rank's tokens only
    ep = gmoe.MoeBlock(T, 1, device=rank, rank=rank, degree=WORLD)
    register(ep, fmt, g, rank, WORLD)
    ep.ep_init(uid, WORLD)
    if placement is not None:
        ep.ep_set_placement(placement)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    x_loc = x_all[rank * T:(rank + 1) * T]
    ep.profile(True)
    for _ in range(3):  # later calls reuse every buffer (both parities)
        ep.forward(0, x_loc, out, T)
    stats, _ = ep.profile_read()
    ep.profile(False)
    assert "ep_pack.p2p" in stats, sorted(stats)  # peer-memory transport by default
    # the NCCL transport computes the same result bit for bit
    out_nccl = torch.empty_like(out)
    ep.set_option(gmoe.OPT_EP_TRANSPORT, 0)
    ep.forward(0, x_loc, out_nccl, T)
    ep.set_option(gmoe.OPT_EP_TRANSPORT, 1)
    torch.cuda.synchronize()
    assert torch.equal(out, out_nccl)
    # the fused post-MoE tail on the expert-parallel path (rank-order sum,
    # then the three norms and the residual on the same row)
    rng = np.random.default_rng(7)
    bf = lambda a: torch.from_numpy(O.f32_to_bf16(np.asarray(a, np.float32)).view(np.int16)).view(torch.bfloat16).cuda()
    gains = [bf(1.0 + 0.2 * rng.standard_normal(H)) for _ in range(3)]
    dense_all = bf(rng.standard_normal((WORLD * T, H)) * 2.0)
    ep.register_post(0, gains[0], gains[1], gains[2], 0.75)
    x_main = x_all[rank * T:(rank + 1) * T].clone()
    ep.forward_ffn(0, x_main, dense_all[rank * T:(rank + 1) * T].contiguous(), T)
    torch.cuda.synchronize()
    assert ep.device_status() == 0
    np.save(os.path.join(tmp, "ffn%d.npy" % rank), synth.to_numpy(x_main))
    if fmt == "bq":
        # the whole FFN under expert parallelism: the dense MLP (replicated) on
        # the dense stream, joined before the EP final sum's post tail, equals
        # the MoE tail given that dense MLP's output
        D = synth.dense_layer(synth.make_dense(seed=77, device="cuda"))
        ep.register_dense(0, D["gate"], D["gate_scale"], D["up"], D["up_scale"], D["down"],
                          D["down_scale"], D["pre_ffn_norm"])
        x0 = x_all[rank * T:(rank + 1) * T]
        dense_loc = torch.empty(T, gmoe.HIDDEN, dtype=torch.bfloat16, device="cuda")
        ep.dense_forward(0, x0, dense_loc, T)
        a = x0.clone()
        ep.forward_ffn(0, a, dense_loc, T)
        b = x0.clone()
        ep.ffn_forward(0, b, T)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
    np.save(os.path.join(tmp, "dense.npy"), synth.to_numpy(dense_all))
    np.save(os.path.join(tmp, "gains.npy"), np.stack([synth.to_numpy(g_) for g_ in gains]))
    # plain degree-2 handle: this rank's partial over all tokens
    part = gmoe.MoeBlock(WORLD * T, 1, device=rank, rank=rank, degree=WORLD)
    register(part, fmt, g, rank, WORLD)
    p = torch.empty(WORLD * T, H, dtype=torch.bfloat16, device="cuda")
    part.forward(0, x_all, p, WORLD * T)
    torch.cuda.synchronize()
    np.save(os.path.join(tmp, "ep%d.npy" % rank), synth.to_numpy(out))
    np.save(os.path.join(tmp, "part%d.npy" % rank), synth.to_numpy(p))
    ep.close()
    part.close()


@pytest.mark.parametrize("fmt,T", [("bq", 200), ("bq", 640), ("bf16", 64)])
def test_ep_forward_two_gpus(fmt, T, tmp_path):
    uid = gmoe.ep_unique_id()
    mp.spawn(worker, args=(fmt, T, uid, str(tmp_path)), nprocs=WORLD, join=True)
    got = np.concatenate([np.load(tmp_path / ("ep%d.npy" % r)) for r in range(WORLD)])
    parts = [np.load(tmp_path / ("part%d.npy" % r)) for r in range(WORLD)]
    acc = np.zeros(parts[0].shape, np.float32)
    for p in parts:  # rank order, from +0.0, as the all-reduce of the reference
        acc = acc + O.bf16_to_f32(p)
    assert np.array_equal(got, O.f32_to_bf16(acc))
    # fused post-MoE tail: the oracle's tail applied to the EP output
    ffn = np.concatenate([np.load(tmp_path / ("ffn%d.npy" % r)) for r in range(WORLD)])
    g3 = np.load(tmp_path / "gains.npy")
    want = O.post_moe(got, np.load(tmp_path / "dense.npy"), tokens_np(WORLD * T, seed=500 + T),
                      g3[0], g3[1], g3[2], 0.75)
    assert rel_err(ffn, want) < 1e-2 and (ffn == want).mean() > 0.97
    # against the oracle's degree-2 forward, on tokens whose top-8 margin
    # guarantees the device picks the same experts
    raw = raw_layer_np(seed=4321, router_std=1.0, stress=True)
    x = tokens_np(WORLD * T, seed=500 + T)
    if fmt == "bq":
        rout, _, _, rlg = O.bq_forward(x, oracle_bq_layer(raw), degree=WORLD)
        tol = TOL_BQ
    else:
        rout, _, _, rlg = O.bf16_forward(x, oracle_bf16_layer(raw), degree=WORLD)
        tol = TOL_BF16
    checked = topk_margin(rlg) > MARGIN
    assert checked.mean() > 0.9
    assert rel_err(got, rout, rows=checked) < tol


def test_ep_forward_two_gpus_with_placement(tmp_path):
    """gm_moe_ep_set_placement: experts moved between the ranks (load-based);
    the output equals each rank's bf16 partial over its placed experts summed
    in rank order (the oracle's stages, on the tokens whose top-8 margin
    guarantees the device routes like the oracle) within the bq tolerance."""
    from test_ep_protocol import placement_tables, rank_weights, rank_partial
    T = 200
    load = np.arange(E, 0, -1).astype(float) ** 1.1
    rank_of = np.array(gmoe.balanced_placement(load, WORLD), np.int32)
    uid = gmoe.ep_unique_id()
    mp.spawn(worker, args=("bq", T, uid, str(tmp_path), [int(r) for r in rank_of]), nprocs=WORLD,
             join=True)
    got = np.concatenate([np.load(tmp_path / ("ep%d.npy" % r)) for r in range(WORLD)])
    raw = raw_layer_np(seed=4321, router_std=1.0, stress=True)
    ref = oracle_bq_layer(raw)
    x = tokens_np(WORLD * T, seed=500 + T)
    idx, w, lg = O.router(x, ref["router_centered"], ref["router_scale"], ref["pes"])
    xi8, xsa = O.bq_norm_quant(x, ref["gamma2"])
    epr = E // WORLD
    local_of = placement_tables(rank_of, WORLD)
    acc = np.zeros((x.shape[0], H), np.float32)
    for r in range(WORLD):
        Wr = rank_weights(ref, [e for e in range(E) if rank_of[e] == r])
        ridx = np.where(rank_of[idx] == r, r * epr + local_of[idx], -1).astype(np.int32)
        acc = acc + O.bf16_to_f32(rank_partial(xi8, xsa, ridx, w, Wr, r, epr))
    want = O.f32_to_bf16(acc)
    checked = topk_margin(lg) > MARGIN
    assert checked.mean() > 0.9
    assert rel_err(got, want, rows=checked) < TOL_BQ
