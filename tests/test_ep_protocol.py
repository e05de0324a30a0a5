"""Expert-parallel exchange protocol on CPU: two gloo processes run the same
steps as the library's EP forward (ep.cu: plan -> pack -> dispatch all-to-all
-> this rank's experts over the received rows -> combine all-to-all -> sum in
rank order), with the oracle's stages as the expert arithmetic, and must
reproduce the oracle's degree-2 forward (the reference's sharded experts plus
all-reduce) bit for bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from helpers import raw_layer_np, tokens_np, oracle_bq_layer

H, E, I, GU, TOPK = O.H, O.E, O.I, O.GU, O.TOPK
WORLD, T_RANK = 2, 24


def plan(idx, G, epr):
    """pos[t][d]: row of token t in destination d's block (token order) or -1."""
    T = idx.shape[0]
    mask = np.zeros((T, G), bool)
    for d in range(G):
        mask[:, d] = ((idx // epr) == d).any(axis=1)
    pos = np.where(mask, np.cumsum(mask, axis=0) - 1, -1).astype(np.int32)
    return pos, mask.sum(axis=0)


def a2a(t, world):
    out = torch.empty_like(t)
    dist.all_to_all_single(out, t)
    return out


def rank_partial(rx, rsa, ridx, rw, ref, rank, epr):
    """This rank's experts over the received rows: bf16(sum over its experts)."""
    n = rx.shape[0]
    off, routes = O.build_schedules(ridx, rw, rank * epr, epr)
    g0, d0 = rank * epr * GU, rank * epr * H
    bucket = O.bq_phase1(rx, rsa, off, routes, ref["gu_q"][g0:], ref["gu_scale"][g0:],
                         ref["gu_cs"][g0:], epr)
    bi8, bsa = O.bq_block_quant(bucket)
    dn_cs = ref["dn_cs"].reshape(-1)
    return O.bq_phase2(bi8, bsa, off, routes, ref["dn_q"][d0:], ref["dn_scale"][d0:], dn_cs[d0:],
                       E * H, epr, n)


def worker(rank, world, port, tmp):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    O.lib().orc_set_num_threads(4)
    with np.load(os.path.join(tmp, "layer.npz")) as z:
        ref = {k: z[k] for k in z.files}
    x = tokens_np(WORLD * T_RANK, seed=77)[rank * T_RANK:(rank + 1) * T_RANK]
    epr, cap = E // world, T_RANK
    # 1. local prep and routing
    xi8, xsa = O.bq_norm_quant(x, ref["gamma2"])
    idx, w, _ = O.router(x, ref["router_centered"], ref["router_scale"], ref["pes"])
    # 2. plan and pack blocks of `cap` rows per destination
    pos, count = plan(idx, world, epr)
    sx = np.zeros((world, cap, H), np.int8)
    ssa = np.zeros((world, cap), np.float32)
    sidx = np.full((world, cap, TOPK), -1, np.int32)
    sw = np.zeros((world, cap, TOPK), np.float32)
    for t in range(T_RANK):
        for d in range(world):
            p = pos[t, d]
            if p >= 0:
                sx[d, p], ssa[d, p], sidx[d, p], sw[d, p] = xi8[t], xsa[t], idx[t], w[t]
    # 3. dispatch
    rx = a2a(torch.from_numpy(sx), world).numpy().reshape(world * cap, H)
    rsa = a2a(torch.from_numpy(ssa), world).numpy().reshape(world * cap)
    ridx = a2a(torch.from_numpy(sidx), world).numpy().reshape(world * cap, TOPK)
    rw = a2a(torch.from_numpy(sw), world).numpy().reshape(world * cap, TOPK)
    # 4. experts, 5. combine exchange
    part = rank_partial(rx, rsa, ridx, rw, ref, rank, epr)
    # bf16 rows travel as int32 pairs (gloo has no 16-bit integer type)
    contrib = a2a(torch.from_numpy(np.ascontiguousarray(part).view(np.int32).reshape(world, cap, H // 2)),
                  world).numpy().view(np.uint16).reshape(world, cap, H)
    # 6. rank-order sum
    out = np.empty((T_RANK, H), np.uint16)
    for t in range(T_RANK):
        acc = np.zeros(H, np.float32)
        for d in range(world):
            if pos[t, d] >= 0:
                acc = acc + O.bf16_to_f32(contrib[d, pos[t, d]])
        out[t] = O.f32_to_bf16(acc)
    np.save(os.path.join(tmp, "out%d.npy" % rank), out)
    np.save(os.path.join(tmp, "count%d.npy" % rank), count)
    dist.barrier()
    dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_protocol_matches_degree2_oracle(tmp_path):
    raw = raw_layer_np(seed=4321, router_std=1.0, stress=True)
    ref = oracle_bq_layer(raw)
    np.savez(tmp_path / "layer.npz", **ref)
    mp.spawn(worker, args=(WORLD, free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    x = tokens_np(WORLD * T_RANK, seed=77)
    rout, _, _, _ = O.bq_forward(x, ref, degree=WORLD)
    got = np.concatenate([np.load(tmp_path / ("out%d.npy" % r)) for r in range(WORLD)])
    assert np.array_equal(got, rout)
    # every token reaches at least one rank, and some reach both
    counts = np.stack([np.load(tmp_path / ("count%d.npy" % r)) for r in range(WORLD)])
    assert counts.sum(axis=1).min() >= T_RANK and counts.max() <= T_RANK
