"""CPU self-checks of the oracle (the reference restatement used as checker).

The reference has no golden vectors for its MoE path, so these pin the
oracle against mathematics and against independent numpy restatements:
FWHT orthonormality, the quantizer's spec identities
(quantization_docs/butterquant.md 1.1-1.4, 2.4-2.5), the VNNI layout
formula, the router against softmax->argsort->renorm on the same logits, the
router-merge invariant of benchmarks/benchmark_router_merge.mojo:120-135,
the stable schedule order of kernels/moe_router.mojo:72-101, float64
restatements of the whole bf16 block and of the butterquant expert
arithmetic, degree-G partial sums, token independence and chunking."""
import numpy as np
import pytest

from oracle import oracle as O
from helpers import stress_layer, tokens_np, oracle_bf16_layer, rel_err, topk_margin, routes_by_expert

H, E, I, GU, TOPK = O.H, O.E, O.I, O.GU, O.TOPK


def sylvester(n):
    m = np.array([[1.0]])
    while m.shape[0] < n:
        m = np.block([[m, m], [m, -m]])
    return m


@pytest.mark.parametrize("block", [64, 128])
def test_fwht_matches_hadamard_and_is_involution(block):
    rng = np.random.default_rng(0)
    v = rng.standard_normal((5, 3 * block)).astype(np.float32)
    w = O.fwht_rows(v, block)
    Hm = sylvester(block) / np.sqrt(block)
    ref = np.concatenate([v[:, b * block:(b + 1) * block] @ Hm.T for b in range(3)], axis=1)
    assert np.abs(w - ref).max() < 1e-5
    assert np.abs(O.fwht_rows(w, block) - v).max() < 1e-5


def test_fast_exp_error_profile():
    L = O.lib()
    xs = np.linspace(-30, 0, 2001)
    sm = np.array([L.orc_fast_exp_softmax_biased(float(x)) for x in xs])
    rel = (sm - np.exp(xs)) / np.exp(xs)
    # simd_math/exponential.mojo:161-170: undershooting, max rel error ~6.88e-3
    assert rel.max() <= 1e-6 and rel.min() > -7.5e-3
    xf = np.linspace(-20, 0, 2001)
    ef = np.array([L.orc_exp_f32_fast(float(x)) for x in xf])
    assert np.abs(ef / np.exp(xf) - 1).max() < 4e-3   # simd_math/ops.mojo:76 "~0.3%"


def test_gelu_tanh_close_to_exact():
    L = O.lib()
    xs = np.linspace(-8, 8, 801)
    got = np.array([L.orc_gelu_tanh(float(x)) for x in xs])
    exact = 0.5 * xs * (1 + np.tanh(np.sqrt(2 / np.pi) * (xs + 0.044715 * xs ** 3)))
    assert np.abs(got - exact).max() < 1e-2


def test_bf16_rne():
    vals = np.array([1.0, 1.00390625, 1.0078125, 3.14159, -2.5e-3, 65504.0], np.float32)
    b = O.f32_to_bf16(vals)
    for v, bb in zip(vals, b):
        assert O.lib().orc_f2bf(float(v)) == bb
    # ties to even: 1 + 2^-8 lies halfway between 1 and 1+2^-7 -> 1
    assert O.bf16_to_f32(O.f32_to_bf16(np.array([1.00390625], np.float32)))[0] == 1.0


@pytest.mark.parametrize("block,gamma", [(128, True), (64, False)])
def test_quantizer_spec_identities(block, gamma):
    rng = np.random.default_rng(1)
    cols = H if block == 128 else I
    w = O.f32_to_bf16(rng.standard_normal((64, cols)).astype(np.float32) * 0.02)
    g = O.f32_to_bf16(rng.standard_normal(cols).astype(np.float32) * 0.25 + 1.0) if gamma else None
    q, s = O.quantize_rows(w, block, g)
    wf = O.bf16_to_f32(w).reshape(64, cols)
    if gamma:
        wf = wf * np.sqrt(np.abs(O.bf16_to_f32(g)))
    rot = O.fwht_rows(wf, block)
    amax = np.abs(rot).max(axis=1)
    # scale stored pre-divided by 127 (butterquant.md 2.4)
    assert np.allclose(s, amax / 127, rtol=1e-6)
    assert q.min() >= -128 and q.max() <= 127
    # reconstruction error <= S/254 (butterquant.md 1.2), plus f32 slack
    err = np.abs(q * s[:, None] - rot)
    assert (err <= (amax / 254)[:, None] * 1.0001 + 1e-9).all()
    # the absmax element maps to +-127
    assert (np.abs(q).max(axis=1) == 127).all()


def test_vnni_layout_formula_and_roundtrip():
    rng = np.random.default_rng(2)
    q = rng.integers(-128, 128, size=(96, 192), dtype=np.int8)
    p = O.vnni_pack(q)
    # offset = t*32*K + ks*2048 + half*1024 + (k%64//4)*64 + n*4 + k%4
    ref = q.reshape(3, 2, 16, 3, 16, 4).transpose(0, 3, 1, 4, 2, 5).reshape(96, 192)
    assert np.array_equal(p.reshape(-1), ref.reshape(-1))
    assert np.array_equal(O.vnni_unpack(p, 96, 192), q)


def test_colsum_layouts():
    rng = np.random.default_rng(3)
    q = rng.integers(-128, 128, size=(64, 704), dtype=np.int8)
    rm = O.colsum(q, 64, True)
    bm = O.colsum(q, 64, False)
    ref = q.reshape(64, 11, 64).astype(np.int64).sum(axis=2)
    assert np.array_equal(rm, ref.astype(np.float32))
    assert np.array_equal(bm, ref.T.astype(np.float32))


@pytest.fixture(scope="module")
def router_inputs():
    rng = np.random.default_rng(4)
    T = 37
    x = tokens_np(T, seed=5)
    wr = O.f32_to_bf16(rng.standard_normal((E, H)).astype(np.float32) * 0.5)
    rs = O.bake_router_scale(O.f32_to_bf16(np.ones(H, np.float32)))
    pes = O.f32_to_bf16(np.ones(E, np.float32))
    return x, wr, rs, pes


def test_router_matches_softmax_argsort_renorm(router_inputs):
    x, wr, rs, pes = router_inputs
    idx, w, lg = O.router(x, wr, rs, pes)
    # self-check (iv): same f32 logits -> softmax over 128 -> stable argsort -> renorm
    p = np.exp(lg.astype(np.float64) - lg.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    order = np.argsort(-p, axis=1, kind="stable")[:, :TOPK]
    assert np.array_equal(idx, order)
    ref_w = np.take_along_axis(p, order, axis=1)
    ref_w /= ref_w.sum(axis=1, keepdims=True)
    assert np.abs(w - ref_w).max() < 1e-2
    # benchmarks/benchmark_router_merge.mojo:120-135 verify_softmax
    assert ((idx >= 0) & (idx < E)).all()
    assert np.abs(w.sum(axis=1) - 1).max() <= 1e-3


def test_router_logits_match_float64(router_inputs):
    x, wr, rs, pes = router_inputs
    _, _, lg = O.router(x, wr, rs, pes)
    xf = O.bf16_to_f32(x).astype(np.float64)
    inv = 1 / np.sqrt((xf ** 2).mean(axis=1) + 1e-6)
    s = xf * O.bf16_to_f32(rs)[None, :] * inv[:, None]
    ref = s @ O.bf16_to_f32(wr).astype(np.float64).T
    assert np.abs(lg - ref).max() < 1e-4 * np.abs(ref).max()


def test_router_tie_breaks_to_lower_expert():
    # identical router rows -> identical logits -> lowest ids win, in id order
    x = tokens_np(3, seed=6)
    row = O.f32_to_bf16(np.random.default_rng(7).standard_normal(H).astype(np.float32))
    wr = np.tile(row, (E, 1))
    rs = O.f32_to_bf16(np.ones(H, np.float32))
    pes = O.f32_to_bf16(np.ones(E, np.float32))
    idx, w, _ = O.router(x, wr, rs, pes)
    assert (idx == np.arange(8)[None, :]).all()
    assert np.allclose(w, 1 / 8, atol=1e-6)


def test_zero_tokens_and_empty_batches():
    """Edge rows of the front end: an all-zero token (RMSNorm with only the
    epsilon, butterquant_kernels/linear.mojo:58-82: scale 0, int8 0; every logit
    0, so the top 8 are experts 0..7 with weights pes/8), an all-zero bucket row
    (block scales 0, int8 0), and empty batches."""
    rng = np.random.default_rng(9)
    zero = np.zeros((2, H), np.uint16)
    wr = O.f32_to_bf16(rng.standard_normal((E, H)).astype(np.float32))
    rs = O.bake_router_scale(O.f32_to_bf16(np.ones(H, np.float32)))
    pes = O.f32_to_bf16((1.0 + 0.25 * rng.standard_normal(E)).astype(np.float32))
    idx, w, lg = O.router(zero, wr, rs, pes)
    assert (lg == 0).all() and (idx == np.arange(8)[None, :]).all()
    assert np.allclose(w, O.bf16_to_f32(pes)[:8][None, :] / 8, rtol=1e-5)
    g2 = O.bake_split_gain(O.f32_to_bf16(np.ones(H, np.float32)))
    q, sa = O.bq_norm_quant(zero, g2)
    assert not q.any() and not sa.any()
    bq, bsa = O.bq_block_quant(np.zeros((3, I), np.uint16))
    assert not bq.any() and not bsa.any()
    idx0, w0, lg0 = O.router(np.zeros((0, H), np.uint16), wr, rs, pes)
    assert idx0.shape == (0, TOPK) and lg0.shape == (0, E)
    q0, sa0 = O.bq_norm_quant(np.zeros((0, H), np.uint16), g2)
    assert q0.shape == (0, H) and sa0.shape == (0,)


def np_schedule(idx, w, base, epr):
    off = np.zeros(epr + 1, np.int32)
    recs = [[] for _ in range(epr)]
    T = idx.shape[0]
    for t in range(T):
        for k in range(TOPK):
            e = idx[t, k] - base
            if 0 <= e < epr:
                recs[e].append((t, w[t, k]))
    out = []
    for e in range(epr):
        off[e + 1] = off[e] + len(recs[e])
        out += recs[e]
    return off, out


@pytest.mark.parametrize("base,epr", [(0, 128), (32, 32), (96, 32)])
def test_schedule_stable_order(base, epr):
    rng = np.random.default_rng(8)
    T = 300
    idx = np.stack([rng.permutation(E)[:TOPK] for _ in range(T)]).astype(np.int32)
    w = rng.random((T, TOPK)).astype(np.float32)
    off, routes = O.build_schedules(idx, w, base, epr)
    roff, rrec = np_schedule(idx, w, base, epr)
    assert np.array_equal(off, roff)
    assert [int(t) for t in routes["token"]] == [t for t, _ in rrec]
    assert np.array_equal(routes["weight"], np.array([x for _, x in rrec], np.float32))


def _edge_routes(kind, T):
    rng = np.random.default_rng(len(kind) + T)
    if kind == "hot":        # every token picks experts 0..7
        idx = np.tile(np.arange(TOPK, dtype=np.int32), (T, 1))
    elif kind == "remote":   # nothing lands in the rank's block (experts 64..127)
        idx = np.stack([rng.permutation(64)[:TOPK] for _ in range(T)]).astype(np.int32)
    else:                    # reversed ids: the schedule order is by token, not by rank in the top 8
        idx = np.stack([np.sort(rng.permutation(E)[:TOPK])[::-1] for _ in range(T)]).astype(np.int32)
    return idx, rng.random((T, TOPK)).astype(np.float32)


@pytest.mark.parametrize("kind,T,base,epr", [("hot", 0, 0, 128), ("hot", 1, 0, 128), ("hot", 1024, 0, 1),
                                             ("remote", 50, 64, 64), ("reversed", 97, 0, 128),
                                             ("reversed", 97, 120, 8)])
def test_schedule_edge_cases(kind, T, base, epr):
    """The stable schedule (kernels/moe_router.mojo:72-101) on the edge cases
    its GPU restatement must handle: an empty batch, one token, one expert
    taking every route, a rank receiving no route, reversed top-8 order."""
    idx, w = _edge_routes(kind, T)
    off, routes = O.build_schedules(idx, w, base, epr)
    roff, rrec = np_schedule(idx, w, base, epr)
    assert np.array_equal(off, roff)
    assert [int(t) for t in routes["token"]] == [t for t, _ in rrec]
    assert np.array_equal(routes["weight"], np.array([x for _, x in rrec], np.float32))
    if kind == "remote":
        assert off[-1] == 0
    if kind == "hot" and epr == 1:
        assert off.tolist() == [0, T]


@pytest.fixture(scope="module")
def bq_small():
    return stress_layer()


def test_bq_forward_degree_partials_close(bq_small):
    raw, L = bq_small
    x = tokens_np(24, seed=12)
    out1, idx1, _, _ = O.bq_forward(x, L, degree=1)
    out2, idx2, _, _ = O.bq_forward(x, L, degree=2)
    assert np.array_equal(idx1, idx2)
    # reference degree-G semantics round each rank's partial to bf16 first
    assert rel_err(out2, out1) < 1e-2


def test_bq_forward_tokens_independent(bq_small):
    _, L = bq_small
    x = tokens_np(20, seed=13)
    full, _, _, _ = O.bq_forward(x, L)
    part, _, _, _ = O.bq_forward(x[:7], L)
    assert np.array_equal(full[:7], part)


def test_bq_forward_chunked_equals_unchunked(bq_small):
    """Self-check (ii): the reference runs prefill in chunks of at most 1024
    tokens (its scratch plan, modeling/gemma_4_moe_bq.mojo:275-360); the
    block's output does not depend on the chunking, bit for bit."""
    _, L = bq_small
    x = tokens_np(1100, seed=15)
    full, idx, w, _ = O.bq_forward(x, L)
    a = O.bq_forward(x[:1024], L)
    b = O.bq_forward(x[1024:], L)
    assert np.array_equal(full, np.concatenate([a[0], b[0]]))
    assert np.array_equal(idx, np.concatenate([a[1], b[1]]))
    assert np.array_equal(w, np.concatenate([a[2], b[2]]))


def _f64(a):
    return O.bf16_to_f32(a).astype(np.float64)


def _bf16_round(a):
    return _f64(O.f32_to_bf16(np.asarray(a, np.float32)))


def _gelu_tanh64(g):
    return 0.5 * g * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (g + 0.044715 * g ** 3)))


def _fwht64_blocks(v, block):
    """Orthonormal FWHT in blocks along the last axis (float64)."""
    v = v.reshape(-1, block).copy()
    h = 1
    while h < block:
        a = v.reshape(v.shape[0], block // (2 * h), 2, h)
        x, y = a[:, :, 0, :].copy(), a[:, :, 1, :].copy()
        a[:, :, 0, :], a[:, :, 1, :] = x + y, x - y
        h *= 2
    return (v / np.sqrt(block)).reshape(-1)


def test_bf16_forward_matches_float64(bq_small):
    """The oracle's bf16 block against an independent float64 restatement of
    its specification (kernels/rmsnorm.mojo:21-47, kernels/moe_router.mojo:
    164-293, kernels/moe_experts.mojo:16-319: RMSNorm with the gain rounded to
    bf16, softmax top-8 renormalised times the per-expert scale, GeGLU bucket
    rounded to bf16, down product, weighted sum): routing weights within the
    reference's fast-exp error (1e-2), output within 1e-2 of max|ref| (half
    the bf16 tolerance; 4e-3 measured).  The experts are the oracle's own
    selection."""
    raw, _ = bq_small
    T = 6
    x = tokens_np(T, seed=16)
    out, idx, w, lg = O.bf16_forward(x, oracle_bf16_layer(raw))
    p = np.exp(lg.astype(np.float64) - lg.max(axis=1, keepdims=True))
    ref_w = np.take_along_axis(p, idx, axis=1)
    ref_w = ref_w / ref_w.sum(axis=1, keepdims=True) * _f64(raw["per_expert_scale"])[idx]
    assert (np.abs(w - ref_w) <= 1e-2 * np.abs(ref_w)).all()
    xf = _f64(x)
    inv = np.sqrt(H) / np.sqrt((xf * xf).sum(axis=1, keepdims=True) + H * 1e-6)
    xn = _bf16_round(xf * inv * _f64(raw["pre_ffn_norm_2"]))
    ref = np.zeros((T, H))
    for t in range(T):
        for k in range(TOPK):
            e = idx[t, k]
            gu = _f64(raw["gate_up"][e]) @ xn[t]
            h = _bf16_round(_gelu_tanh64(gu[:I]) * gu[I:])
            ref[t] += ref_w[t, k] * (_f64(raw["down"][e]) @ h)
    got = _f64(out)
    assert np.abs(got - ref).max() <= 1e-2 * np.abs(ref).max()


def test_bq_forward_matches_float64_dequantized(bq_small):
    """The oracle's butterquant expert arithmetic against float64 on the same
    int8 operands: dequantised dots (x_i8 * sa/127) . (W_i8 * scale) in the
    rotated domain, exact GeGLU, the bucket rounded to bf16 and rotated by
    FWHT64 (unquantised here), the dequantised down product, the oracle's
    routing weights: within 1.5e-2 of max|ref| (half the butterquant
    tolerance; 6e-3 measured)."""
    _, L = bq_small
    T = 6
    x = tokens_np(T, seed=17)
    out, idx, w, _ = O.bq_forward(x, L)
    xq, xsa = O.bq_norm_quant(x, L["gamma2"])
    ref = np.zeros((T, H))
    for t in range(T):
        a = xq[t].astype(np.float64) * (float(xsa[t]) / 127.0)
        for k in range(TOPK):
            e = idx[t, k]
            rows = slice(e * GU, (e + 1) * GU)
            gu = (L["gu_q"][rows].astype(np.float64) * L["gu_scale"][rows, None].astype(np.float64)) @ a
            h = _fwht64_blocks(_bf16_round(_gelu_tanh64(gu[:I]) * gu[I:]), 64)
            drows = slice(e * H, (e + 1) * H)
            wd = L["dn_q"][drows].astype(np.float64) * L["dn_scale"][drows, None].astype(np.float64)
            ref[t] += float(w[t, k]) * (wd @ h)
    got = _f64(out)
    assert np.abs(got - ref).max() <= 1.5e-2 * np.abs(ref).max()


def test_bq_close_to_bf16_path(bq_small):
    """Butterquant output approximates the unquantised model (the int8 error
    is the only difference; FWHT rotations cancel): self-check (i)."""
    raw, Lq = bq_small
    Lb = oracle_bf16_layer(raw)
    x = tokens_np(64, seed=14)
    ob, ib, _, lgb = O.bf16_forward(x, Lb)
    oq, iq, _, lgq = O.bq_forward(x, Lq)
    # the centred router keeps the selected set (the gauge x.mean(W) shifts
    # every logit of a token alike); only tokens whose 8th/9th margin is below
    # the bf16 rounding of the centred weights may select differently
    keep = (routes_by_expert(ib) == routes_by_expert(iq)).all(axis=1)
    assert keep[topk_margin(lgb) > 1e-3].all()
    assert keep.mean() > 0.9
    assert rel_err(oq, ob, rows=keep) < 0.1


def test_post_moe_tail():
    """orc_post_moe (modeling/gemma_4_moe_bq.mojo:785-805): identities, and a
    float64 restatement of the three norms within bf16 rounding."""
    rng = np.random.default_rng(5)
    T = 6
    bf = lambda a: O.f32_to_bf16(np.asarray(a, np.float32))
    moe, dense, x = (bf(rng.standard_normal((T, H)) * s) for s in (0.3, 2.0, 1.0))
    w1, w2, w = (bf(1.0 + 0.2 * rng.standard_normal(H)) for _ in range(3))
    zero = np.zeros(H, np.uint16)
    # all gains zero: x_main * layer_scalar
    out = O.post_moe(moe, dense, x, zero, zero, zero, 0.5)
    assert np.array_equal(out, bf(O.bf16_to_f32(x) * np.float32(0.5)))

    def inv(v):
        v = v.astype(np.float64)
        return np.sqrt(H) / np.sqrt((v * v).sum(axis=1, keepdims=True) + H * 1e-6)

    f = lambda a: O.bf16_to_f32(a).astype(np.float64)
    d1 = f(dense) * inv(f(dense)) * f(w1)
    d2 = d1 + f(moe) * inv(f(moe)) * f(w2)
    ref = (f(x) + d2 * inv(d2) * f(w)) * 0.75
    got = f(O.post_moe(moe, dense, x, w1, w2, w, 0.75))
    assert np.abs(got - ref).max() <= 0.02 * np.abs(ref).max()


def test_norm_residual_add_oracle():
    """orc_norm_residual_add (kernels/rmsnorm.mojo:48-64): with a zero
    residual it is rms_norm bit for bit; composed with rms_norm it rebuilds the
    post-MoE tail's two norm-residual steps bit for bit (layer scalar 1)."""
    rng = np.random.default_rng(6)
    T = 5
    bf = lambda a: O.f32_to_bf16(np.asarray(a, np.float32))
    moe, dense, x = (bf(rng.standard_normal((T, H)) * s) for s in (0.3, 2.0, 1.0))
    w1, w2, w = (bf(1.0 + 0.2 * rng.standard_normal(H)) for _ in range(3))
    zeros = np.zeros((T, H), np.uint16)
    assert np.array_equal(O.norm_residual_add(moe, zeros, w2), O.rms_norm(moe, w2))
    d2 = O.norm_residual_add(moe, O.rms_norm(dense, w1), w2)
    assert np.array_equal(O.norm_residual_add(d2, x, w), O.post_moe(moe, dense, x, w1, w2, w, 1.0))


def test_dense_mlp_oracle():
    """orc_dense_mlp (modeling/gemma_4_moe_bq.mojo:749-783): equals its own
    stages composed, the signed-dot form of bq_linear (the u8 x s8 - 128*colsum
    identity, exact here), and a float64 restatement of the unquantised MLP
    within the int8 quantisation tolerance."""
    from helpers import raw_dense_np, oracle_dense_layer
    raw = raw_dense_np(seed=31)
    d = oracle_dense_layer(raw)
    x = tokens_np(5, seed=8)
    out, hb, hq, hs = O.dense_mlp(x, d)
    xi8, xsa = O.bq_norm_quant(x, d["gamma"])
    g = O.bq_linear(xi8, xsa, d["wg"], d["wgs"], d["wgcs"])
    u = O.bq_linear(xi8, xsa, d["wu"], d["wus"], d["wucs"])
    assert np.array_equal(O.gelu_gate_up(g, u), hb)
    q, s = O.bq_block_quant(hb)
    assert np.array_equal(q, hq) and np.array_equal(s, hs)
    assert np.array_equal(O.bq_block_linear(hq, hs, d["wd"], d["wds"], d["wdcs"]), out)
    # signed dots: f32(dot) * (sa/127) * sw, rounded to bf16
    dot = xi8.astype(np.int64) @ d["wg"].astype(np.int64).T
    ad = (xsa * np.float32(1.0 / 127.0)).astype(np.float32)
    ref_g = O.f32_to_bf16((dot.astype(np.float32) * ad[:, None]) * d["wgs"][None, :])
    assert np.array_equal(ref_g, g)
    # float64 MLP on the raw weights
    f = lambda a: O.bf16_to_f32(a).astype(np.float64)
    xf = f(x)
    xn = xf * (np.sqrt(H) / np.sqrt((xf * xf).sum(1, keepdims=True) + H * 1e-6)) * f(raw["pre_ffn_norm"])
    gg, uu = xn @ f(raw["gate"]).T, xn @ f(raw["up"]).T
    gel = 0.5 * gg * (1 + np.tanh(np.sqrt(2 / np.pi) * (gg + 0.044715 * gg ** 3)))
    ref = (gel * uu) @ f(raw["down"]).T
    got = f(out)
    assert np.abs(got - ref).max() <= 0.03 * np.abs(ref).max()
