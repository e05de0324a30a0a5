"""The oracle's restatement of the reference's butterquant attention
(butterquant/head_prep.mojo, butterquant_kernels/attention.mojo,
kernels/attention_ops.mojo, kernels/logsum_merge.mojo) against float64
restatements of the same mathematics: head prep (RMSNorm with the head gain,
RoPE, FWHT over the head, int8) and decode attention (softmax over the
dequantised int8 scores, V in the rotated domain, partials merged)."""
import numpy as np
import pytest

from oracle import oracle as O

SLIDING = dict(head_dim=256, num_q=16, num_kv=8, rope_half=128, pair_stride=128)
FULL = dict(head_dim=512, num_q=16, num_kv=2, rope_half=64, pair_stride=256)


def bf(a):
    return O.f32_to_bf16(np.asarray(a, np.float32))


def f(a):
    return O.bf16_to_f32(a).astype(np.float64)


def rope_tables(max_pos, rope_half, base):
    """Standard RoPE tables [pos][rope_half] (the caller's tables; both sides
    read the same values)."""
    inv = base ** (-np.arange(rope_half, dtype=np.float64) / rope_half)
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def fwht64(v):
    """Orthonormal FWHT along the last axis (float64)."""
    v = v.copy()
    n = v.shape[-1]
    h = 1
    while h < n:
        a = v.reshape(v.shape[:-1] + (n // (2 * h), 2, h))
        x, y = a[..., 0, :].copy(), a[..., 1, :].copy()
        a[..., 0, :], a[..., 1, :] = x + y, x - y
        h *= 2
    return v / np.sqrt(n)


def prep_f64(src, gamma, c, s, cfg, rope=True):
    x = f(src)
    hd = cfg["head_dim"]
    x = x * np.sqrt(hd) / np.sqrt((x * x).sum(-1, keepdims=True) + hd * 1e-6)
    if gamma is not None:
        x = x * f(gamma)
    if rope:
        rh, ps = cfg["rope_half"], cfg["pair_stride"]
        lo, hi = x[..., :rh].copy(), x[..., ps:ps + rh].copy()
        x[..., :rh] = lo * c - hi * s
        x[..., ps:ps + rh] = hi * c + lo * s
    return fwht64(x)


@pytest.mark.parametrize("cfg", [SLIDING, FULL], ids=["sliding", "full"])
def test_attn_prep_matches_float64(cfg):
    rng = np.random.default_rng(3)
    hd, nq, nkv = cfg["head_dim"], cfg["num_q"], cfg["num_kv"]
    T = 3
    q = bf(rng.standard_normal((T, nq * hd)) * 2.0)
    k = bf(rng.standard_normal((T, nkv * hd)))
    v = bf(rng.standard_normal((T, nkv * hd)) * 0.5)
    qn, kn = bf(1.0 + 0.3 * rng.standard_normal(hd)), bf(1.0 + 0.3 * rng.standard_normal(hd))
    cos, sin = rope_tables(64, cfg["rope_half"], 10000.0)
    pos = np.array([0, 17, 63], np.int32)
    slot = np.array([5, -1, 2], np.int32)
    q_i8, qb, fq, kc, ks, vc, vs = O.bq_attn_prep(q, k, v, qn, kn, pos, slot, hd, nq, nkv,
                                                   cfg["rope_half"], cfg["pair_stride"], cos, sin, 8)
    # qi_bias = 128 * sum(q_i8), f_q = absmax
    qh = q_i8.reshape(T, nq, hd).astype(np.int64)
    assert np.array_equal(qb, (qh.sum(-1) * 128).astype(np.float32))
    for t in range(T):
        c, s = cos[pos[t]].astype(np.float64), sin[pos[t]].astype(np.float64)
        ref = prep_f64(q[t].reshape(nq, hd), qn, c, s, cfg)
        assert np.allclose(fq[t], np.abs(ref).max(-1), rtol=1e-4)
        deq = qh[t] * (fq[t][:, None] / 127.0)
        assert np.abs(deq - ref).max() <= 0.51 * fq[t].max() / 127.0 + 1e-4
        if slot[t] >= 0:
            rk = prep_f64(k[t].reshape(nkv, hd), kn, c, s, cfg)
            rv = prep_f64(v[t].reshape(nkv, hd), None, c, s, cfg, rope=False)
            kd = kc[slot[t]].reshape(nkv, hd) * (ks[slot[t]][:, None] / 127.0)
            vd = vc[slot[t]].reshape(nkv, hd) * (vs[slot[t]][:, None] / 127.0)
            assert np.abs(kd - rk).max() <= 0.51 * ks[slot[t]].max() / 127.0 + 1e-4
            assert np.abs(vd - rv).max() <= 0.51 * vs[slot[t]].max() / 127.0 + 1e-4
    # tokens with slot -1 write no cache row
    assert not kc[[0, 1, 3, 4, 6, 7]].any()


def random_cache(rng, n_slots, cfg):
    hd, nkv = cfg["head_dim"], cfg["num_kv"]
    kc = rng.integers(-127, 128, size=(n_slots, nkv * hd), dtype=np.int8)
    vc = rng.integers(-127, 128, size=(n_slots, nkv * hd), dtype=np.int8)
    ks = (rng.random((n_slots, nkv)) * 2 + 0.5).astype(np.float32)
    vs = (rng.random((n_slots, nkv)) * 2 + 0.5).astype(np.float32)
    return kc, ks, vc, vs


def decode_f64(q_i8, fq, kc, ks, vc, vs, slots, kv_len, cfg):
    hd, nq, nkv = cfg["head_dim"], cfg["num_q"], cfg["num_kv"]
    T = q_i8.shape[0]
    out = np.zeros((T, nq, hd))
    for t in range(T):
        rows = slots[t, :kv_len[t]]
        for h in range(nq):
            g = h // (nq // nkv)
            q = q_i8[t, h * hd:(h + 1) * hd].astype(np.float64) * fq[t, h] / 127.0
            k = kc[rows][:, g * hd:(g + 1) * hd].astype(np.float64) * ks[rows, g][:, None] / 127.0
            v = vc[rows][:, g * hd:(g + 1) * hd].astype(np.float64) * vs[rows, g][:, None] / 127.0
            sc = k @ q
            p = np.exp(sc - sc.max())
            out[t, h] = (p / p.sum()) @ v
    return out.reshape(T, nq * hd)


@pytest.mark.parametrize("cfg", [SLIDING, FULL], ids=["sliding", "full"])
def test_flash_decode_matches_float64(cfg):
    rng = np.random.default_rng(4)
    hd, nq, nkv = cfg["head_dim"], cfg["num_q"], cfg["num_kv"]
    n_slots, T, max_kv = 300, 3, 200
    kc, ks, vc, vs = random_cache(rng, n_slots, cfg)
    # small scores keep the softmax soft (many rows contribute)
    ks *= 0.05
    q_i8 = rng.integers(-127, 128, size=(T, nq * hd), dtype=np.int8)
    fq = (rng.random((T, nq)) + 0.5).astype(np.float32)
    qb = (q_i8.reshape(T, nq, hd).astype(np.int64).sum(-1) * 128).astype(np.float32)
    kv_len = np.array([1, 37, 200], np.int32)
    slots = np.stack([rng.permutation(n_slots)[:max_kv] for _ in range(T)]).astype(np.int32)
    ref = decode_f64(q_i8, fq, kc, ks, vc, vs, slots, kv_len, cfg)
    outs = []
    for ns in (1, 3, 20):
        got = O.bf16_to_f32(O.bq_flash_decode(q_i8, qb, fq, kc, ks, vc, vs, slots, kv_len, hd, nq,
                                              nkv, ns)).astype(np.float64)
        assert np.abs(got - ref).max() <= 1e-2 * np.abs(ref).max()
        outs.append(got)
    # the split count changes only rounding
    assert np.abs(outs[0] - outs[2]).max() <= 1e-2 * np.abs(ref).max()


def run_scenario_oracle(n_splits=4, full=False):
    """A reference test's ten steps through the oracle (prep into the paged
    cache, then the flash decode of every token of the step); per step
    (tokens, q_i8, f_q, output, cache after the step)."""
    import attention_scenario as S
    if full:
        hd, nq, nkv, rh, ps = S.FULL_HEAD_DIM, S.FULL_NUM_Q, S.FULL_NUM_KV, 64, 256
        n_slots, slot_of, slots_of = S.FULL_NUM_PAGES * S.PAGE_LEN, S.full_slot, S.full_slots
    else:
        hd, nq, nkv, rh, ps = S.HEAD_DIM, S.NUM_Q, S.NUM_KV, 128, 128
        n_slots, slot_of, slots_of = S.NUM_PAGES * S.PAGE_LEN, S.ring_slot, S.window_slots
    kvs = nkv * hd
    kc = np.zeros((n_slots, kvs), np.int8)
    vc = np.zeros_like(kc)
    ks = np.zeros((n_slots, nkv), np.float32)
    vs = np.zeros_like(ks)
    cos, sin = S.identity_rope(rh)
    g = S.unit_gain(hd)
    steps = []
    for step in range(len(S.STEPS)):
        toks, _ = S.step_tokens(step)
        q, k, v = S.step_inputs(step, hd, nq, nkv)
        pos = np.array([p for _, p in toks], np.int32)
        slot = np.array([slot_of(p, seq) for seq, p in toks], np.int32)
        q_i8, qb, fq, kc1, ks1, vc1, vs1 = O.bq_attn_prep(
            q, k, v, g, g, pos, slot, hd, nq, nkv, rh, ps, cos, sin, n_slots)
        kc[slot], ks[slot], vc[slot], vs[slot] = kc1[slot], ks1[slot], vc1[slot], vs1[slot]
        lists = [slots_of(seq, p) for seq, p in toks]
        kv_len = np.array([len(x) for x in lists], np.int32)
        slots = np.zeros((len(toks), max(kv_len)), np.int32)
        for t, x in enumerate(lists):
            slots[t, :len(x)] = x
        out = O.bq_flash_decode(q_i8, qb, fq, kc, ks, vc, vs, slots, kv_len, hd, nq, nkv, n_splits)
        steps.append((toks, q_i8, fq, out, (kc.copy(), ks.copy(), vc.copy(), vs.copy())))
    return steps


@pytest.mark.parametrize("full", [False, True], ids=["sliding", "full"])
def test_reference_attention_scenario(full):
    """The scenarios and acceptance bound of the reference's own tests
    (tests/test_sliding_attention_degree_parity.mojo,
    tests/test_full_attention_degree_parity.mojo at degree 1): every token of
    every step within 0.05 of its f32 exact-exp reference_head."""
    import attention_scenario as S
    hd, nq = (S.FULL_HEAD_DIM, S.FULL_NUM_Q) if full else (S.HEAD_DIM, S.NUM_Q)
    worst = 0.0
    for toks, q_i8, fq, out, (kc, ks, vc, vs) in run_scenario_oracle(full=full):
        got = O.bf16_to_f32(out)
        for t, (seq, p) in enumerate(toks):
            for h in range(nq):
                ref = S.reference_head(kc, ks, vc, vs, seq, p, q_i8[t, h * hd:(h + 1) * hd], fq[t, h], h,
                                       full=full)
                worst = max(worst, float(np.abs(got[t, h * hd:(h + 1) * hd] - ref).max()))
    assert worst <= S.TOL, worst
