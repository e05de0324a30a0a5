"""Butterquant decode attention on the GPU (gm_bq_attn_prep,
gm_bq_attention_decode) against the oracle's restatement of the reference's
attention (butterquant_kernels/attention.mojo, kernels/attention_ops.mojo,
kernels/logsum_merge.mojo).

The prep (RMSNorm, RoPE, FWHT, int8 into the paged cache) is bit-identical.
The decode output is a sum of exponentially weighted V rows whose order of
accumulation differs from the reference's 16-position tiles (as the
reference's own output differs between worker counts), so it is checked
within 1e-2 of max|ref| against the oracle and against a float64 softmax."""
import numpy as np
import pytest
import torch

import gmoe
from oracle import oracle as O
from test_attention_oracle import SLIDING, FULL, bf, rope_tables, random_cache, decode_f64
import golden_cases as G
from helpers import golden

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

PAGE = 64
SHIFT = 6


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    return torch.from_numpy(a).cuda()


def host(t):
    t = t.detach().cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def runs_array(runs):
    return np.array(runs, np.int32).reshape(-1, 4)


def slot_of(base_rows, run, p, page_mask):
    return base_rows[run[2] + ((p >> SHIFT) & page_mask)] + (p & (PAGE - 1))


@pytest.mark.parametrize("cfg,page_mask", [(SLIDING, 1), (FULL, -1)], ids=["sliding", "full"])
def test_attn_prep_bit_exact(cfg, page_mask):
    rng = np.random.default_rng(11)
    hd, nq, nkv = cfg["head_dim"], cfg["num_q"], cfg["num_kv"]
    # two runs (sequences): 3 prefill-chunk tokens at positions 62..64 (crossing
    # a page) and one decode token at position 200 (ring wraps for sliding)
    runs = [(0, 62, 0, 2), (3, 200, 2, 4)]
    base_rows = np.array([128, 0, 320, 192, 64, 256], np.int32)
    T = 4
    q = bf(rng.standard_normal((T, nq * hd)) * 1.5)
    k = bf(rng.standard_normal((T, nkv * hd)))
    v = k.copy() if cfg is FULL else bf(rng.standard_normal((T, nkv * hd)) * 0.7)
    qn, kn = bf(1.0 + 0.3 * rng.standard_normal(hd)), bf(1.0 + 0.3 * rng.standard_normal(hd))
    cos, sin = rope_tables(256, cfg["rope_half"], 10000.0)
    pos = np.array([62, 63, 64, 200], np.int32)
    run_of = [0, 0, 0, 1]
    slot = np.array([slot_of(base_rows, runs[run_of[t]], pos[t], page_mask) for t in range(T)], np.int32)
    n_slots = 384
    want = O.bq_attn_prep(q, k, v, qn, kn, pos, slot, hd, nq, nkv, cfg["rope_half"],
                          cfg["pair_stride"], cos, sin, n_slots)
    q_i8 = torch.zeros(T, nq * hd, dtype=torch.int8, device="cuda")
    qb = torch.zeros(T, nq, dtype=torch.float32, device="cuda")
    fq = torch.zeros_like(qb)
    kc = torch.zeros(n_slots, nkv * hd, dtype=torch.int8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.zeros(n_slots, nkv, dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    dq, dk = dev(q), dev(k)
    dv = dk if cfg is FULL else dev(v)
    gmoe.call("gm_bq_attn_prep", dq, dk, dv, dev(qn), dev(kn), q_i8, qb, fq, kc, ks, vc, vs,
              dev(cos), dev(sin), dev(runs_array(runs)), len(runs), dev(base_rows), T, hd, nq, nkv,
              cfg["rope_half"], cfg["pair_stride"], 1, 0, SHIFT, PAGE - 1, page_mask, None)
    torch.cuda.synchronize()
    for got, exp in zip((q_i8, qb, fq, kc, ks, vc, vs), want):
        assert np.array_equal(host(got), exp)
    # degree 2, rank 1: only odd positions reach this rank's cache (row pos // 2)
    kc.zero_()
    slot2 = np.array([slot_of(base_rows, runs[run_of[t]], pos[t] // 2, page_mask)
                      if pos[t] % 2 == 1 else -1 for t in range(T)], np.int32)
    want2 = O.bq_attn_prep(q, k, v, qn, kn, pos, slot2, hd, nq, nkv, cfg["rope_half"],
                           cfg["pair_stride"], cos, sin, n_slots)
    gmoe.call("gm_bq_attn_prep", dq, dk, dv, dev(qn), dev(kn), q_i8, qb, fq, kc, ks, vc, vs,
              dev(cos), dev(sin), dev(runs_array(runs)), len(runs), dev(base_rows), T, hd, nq, nkv,
              cfg["rope_half"], cfg["pair_stride"], 2, 1, SHIFT, PAGE - 1, page_mask, None)
    torch.cuda.synchronize()
    assert np.array_equal(host(kc), want2[3])


def decode_case(cfg, window, page_mask, positions, rng):
    hd, nq, nkv = cfg["head_dim"], cfg["num_q"], cfg["num_kv"]
    T = len(positions)
    pages_per_run = 2 if page_mask == 1 else (max(positions) >> SHIFT) + 1
    n_slots = T * pages_per_run * PAGE
    perm = rng.permutation(T * pages_per_run)
    base_rows = (perm * PAGE).astype(np.int32)
    runs = [(t, positions[t], t * pages_per_run, pages_per_run) for t in range(T)]
    kc, ks, vc, vs = random_cache(rng, n_slots, cfg)
    ks *= 0.03
    q_i8 = rng.integers(-127, 128, size=(T, nq * hd), dtype=np.int8)
    fq = (rng.random((T, nq)) + 0.5).astype(np.float32)
    qb = (q_i8.reshape(T, nq, hd).astype(np.int64).sum(-1) * 128).astype(np.float32)
    max_kv = max(min(p + 1, window) if window else p + 1 for p in positions)
    slots = np.zeros((T, max_kv), np.int32)
    kv_len = np.zeros(T, np.int32)
    for t, p in enumerate(positions):
        valid = min(p + 1, window) if window else p + 1
        start = p - valid + 1 if window else 0
        kv_len[t] = valid
        for i in range(valid):
            slots[t, i] = slot_of(base_rows, runs[t], start + i, page_mask)
    return dict(q_i8=q_i8, fq=fq, qb=qb, kc=kc, ks=ks, vc=vc, vs=vs, slots=slots, kv_len=kv_len,
                runs=runs, base_rows=base_rows, max_kv=max_kv)


@pytest.mark.parametrize("cfg,window,page_mask,positions", [
    (SLIDING, 64, 1, [0, 5, 63, 64, 100, 127, 128, 300]),
    (FULL, 0, -1, [0, 1, 31, 64, 200, 511]),
    (SLIDING, 64, 1, [90]),
], ids=["sliding", "full", "sliding-b1"])
def test_attention_decode_matches_oracle(cfg, window, page_mask, positions):
    rng = np.random.default_rng(len(positions) + cfg["head_dim"])
    hd, nq, nkv = cfg["head_dim"], cfg["num_q"], cfg["num_kv"]
    c = decode_case(cfg, window, page_mask, positions, rng)
    T = len(positions)
    want = O.bf16_to_f32(O.bq_flash_decode(c["q_i8"], c["qb"], c["fq"], c["kc"], c["ks"], c["vc"], c["vs"],
                                           c["slots"], c["kv_len"], hd, nq, nkv, 1)).astype(np.float64)
    ref = decode_f64(c["q_i8"], c["fq"], c["kc"], c["ks"], c["vc"], c["vs"], c["slots"], c["kv_len"], cfg)
    ws_bytes = gmoe.lib().gm_bq_attention_workspace_bytes(T, hd, nq, nkv, c["max_kv"])
    ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device="cuda")
    out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device="cuda")
    gmoe.call("gm_bq_attention_decode", dev(c["q_i8"]), dev(c["fq"]), dev(c["kc"]), dev(c["ks"]),
              dev(c["vc"]), dev(c["vs"]), dev(runs_array(c["runs"])), dev(c["base_rows"]), T, hd, nq, nkv,
              window, 1, 0, SHIFT, PAGE - 1, page_mask, c["max_kv"], out, ws, ws_bytes, None)
    torch.cuda.synchronize()
    got = O.bf16_to_f32(host(out)).astype(np.float64)
    scale = np.abs(ref).max()
    assert np.abs(got - want).max() <= 1e-2 * scale
    assert np.abs(got - ref).max() <= 1e-2 * scale
    # a too-small workspace is refused
    with pytest.raises(gmoe.GmoeError, match="workspace"):
        gmoe.call("gm_bq_attention_decode", dev(c["q_i8"]), dev(c["fq"]), dev(c["kc"]), dev(c["ks"]),
                  dev(c["vc"]), dev(c["vs"]), dev(runs_array(c["runs"])), dev(c["base_rows"]), T, hd, nq,
                  nkv, window, 1, 0, SHIFT, PAGE - 1, page_mask, c["max_kv"], out, ws, ws_bytes - 4, None)


@pytest.mark.parametrize("full", [False, True], ids=["sliding", "full"])
def test_reference_attention_scenario_on_gpu(full):
    """The reference's own attention test scenarios
    (tests/test_sliding_attention_degree_parity.mojo,
    tests/test_full_attention_degree_parity.mojo at degree 1: three sequences
    on paged caches, ten steps of prefill chunks and decode tokens) through the
    C ABI: the prep of every step (multi-token runs) writes the same cache and
    q_i8 as the oracle, bit for bit, and every token's attention output is
    within the reference tests' bound (0.05) of their f32 reference_head."""
    import attention_scenario as S
    from test_attention_oracle import run_scenario_oracle
    oracle_steps = run_scenario_oracle(full=full)
    if full:
        hd, nq, nkv, rh, ps = S.FULL_HEAD_DIM, S.FULL_NUM_Q, S.FULL_NUM_KV, 64, 256
        n_slots, window, page_mask, max_kv = S.FULL_NUM_PAGES * S.PAGE_LEN, 0, -1, 256
        lists = [S.full_base_rows(q) for q in range(3)]
    else:
        hd, nq, nkv, rh, ps = S.HEAD_DIM, S.NUM_Q, S.NUM_KV, 128, 128
        n_slots, window, page_mask, max_kv = S.NUM_PAGES * S.PAGE_LEN, S.WINDOW, S.RING_PAGES - 1, S.WINDOW
        lists = [S.base_rows(q) for q in range(3)]
    rows_off = np.cumsum([0] + [len(x) for x in lists])[:3]
    kvs = nkv * hd
    kc = torch.zeros(n_slots, kvs, dtype=torch.int8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.zeros(n_slots, nkv, dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    cos, sin = S.identity_rope(rh)
    g = dev(S.unit_gain(hd))
    base_rows = dev(np.concatenate(lists))
    worst = 0.0
    for step, (toks, q_o, fq_o, out_o, cache_o) in enumerate(oracle_steps):
        T = len(toks)
        _, runs = S.step_tokens(step)
        q, k, v = S.step_inputs(step, hd, nq, nkv)
        prep_runs = runs_array([(b, p, rows_off[seq], len(lists[seq])) for b, p, seq in runs])
        q_i8 = torch.empty(T, nq * hd, dtype=torch.int8, device="cuda")
        qb = torch.empty(T, nq, dtype=torch.float32, device="cuda")
        fq = torch.empty_like(qb)
        gmoe.call("gm_bq_attn_prep", dev(q), dev(k), dev(v), g, g, q_i8, qb, fq, kc, ks, vc, vs,
                  dev(cos), dev(sin), dev(prep_runs), len(runs), base_rows, T, hd, nq, nkv, rh, ps,
                  1, 0, 6, S.PAGE_LEN - 1, page_mask, None)
        # every token (prefill chunks too) as the newest position of its own run
        tok_runs = runs_array([(t, p, rows_off[seq], len(lists[seq])) for t, (seq, p) in enumerate(toks)])
        wsb = gmoe.lib().gm_bq_attention_workspace_bytes(T, hd, nq, nkv, max_kv)
        ws = torch.empty(wsb // 4 + 1, dtype=torch.float32, device="cuda")
        out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device="cuda")
        gmoe.call("gm_bq_attention_decode", q_i8, fq, kc, ks, vc, vs, dev(tok_runs), base_rows, T,
                  hd, nq, nkv, window, 1, 0, 6, S.PAGE_LEN - 1, page_mask, max_kv, out, ws, wsb, None)
        # the prefill kernel over the prep's own runs gives the same outputs
        pout = torch.empty_like(out)
        gmoe.call("gm_bq_attention_prefill", q_i8, fq, kc, ks, vc, vs, dev(prep_runs), len(runs), base_rows, T,
                  hd, nq, nkv, window, 6, S.PAGE_LEN - 1, page_mask, pout, None)
        torch.cuda.synchronize()
        assert np.array_equal(host(q_i8), q_o) and np.array_equal(host(fq), fq_o)
        pgot = O.bf16_to_f32(host(pout))
        assert np.abs(pgot - O.bf16_to_f32(out_o)).max() <= 2e-2
        kc_o, ks_o, vc_o, vs_o = cache_o
        assert np.array_equal(host(kc), kc_o) and np.array_equal(host(vc), vc_o)
        assert np.array_equal(host(ks), ks_o) and np.array_equal(host(vs), vs_o)
        got = O.bf16_to_f32(host(out))
        assert np.abs(got - O.bf16_to_f32(out_o)).max() <= 2e-2
        if step in G.ATTN_STEPS:
            # the committed golden vectors of the same step
            name = "full" if full else "sliding"
            ga = golden("attention")
            assert np.array_equal(host(fq), ga[f"{name}_fq_s{step}"])
            assert np.abs(got - O.bf16_to_f32(ga[f"{name}_out_s{step}"])).max() <= 2e-2
        for t, (seq, p) in enumerate(toks):
            for h in range(nq):
                ref = S.reference_head(kc_o, ks_o, vc_o, vs_o, seq, p, q_o[t, h * hd:(h + 1) * hd],
                                       fq_o[t, h], h, full=full)
                worst = max(worst, float(np.abs(got[t, h * hd:(h + 1) * hd] - ref).max()),
                            float(np.abs(pgot[t, h * hd:(h + 1) * hd] - ref).max()))
    assert worst <= S.TOL, worst


@pytest.mark.parametrize("degree", [2, 4])
def test_sharded_full_cache_partials_and_merge(degree):
    """A full-layer cache sharded by position over `degree` ranks (position p
    on rank p % degree at row p // degree, kernels/attention_ops.mojo:167-173):
    each rank's gm_bq_attention_partial over its positions, merged in rank
    order by gm_bq_attention_merge (kernels/logsum_merge.mojo:29-117), equals
    the unsharded decode within the attention tolerance and the float64
    softmax within 1e-2 of max|ref|; a rank that holds no position of a token
    (position 0 on rank 1) contributes nothing."""
    cfg = FULL
    hd, nq, nkv = cfg["head_dim"], cfg["num_q"], cfg["num_kv"]
    rng = np.random.default_rng(77 + degree)
    positions = [0, 1, 5, 64, 200, 511]
    c = decode_case(cfg, 0, -1, positions, rng)
    T = len(positions)
    runs = dev(runs_array(c["runs"]))
    ws_bytes = gmoe.lib().gm_bq_attention_workspace_bytes(T, hd, nq, nkv, c["max_kv"])
    ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device="cuda")
    whole = torch.empty(T, nq * hd, dtype=torch.bfloat16, device="cuda")
    gmoe.call("gm_bq_attention_decode", dev(c["q_i8"]), dev(c["fq"]), dev(c["kc"]), dev(c["ks"]),
              dev(c["vc"]), dev(c["vs"]), runs, dev(c["base_rows"]), T, hd, nq, nkv, 0, 1, 0, SHIFT,
              PAGE - 1, -1, c["max_kv"], whole, ws, ws_bytes, None)
    pbytes = gmoe.lib().gm_bq_attention_partial_bytes(T, hd, nq)
    parts = []
    for r in range(degree):
        kc, ks = np.zeros_like(c["kc"]), np.zeros_like(c["ks"])
        vc, vs = np.zeros_like(c["vc"]), np.zeros_like(c["vs"])
        for t, pmax in enumerate(positions):
            for p in range(r, pmax + 1, degree):
                src = slot_of(c["base_rows"], c["runs"][t], p, -1)
                dst = slot_of(c["base_rows"], c["runs"][t], p // degree, -1)
                kc[dst], ks[dst], vc[dst], vs[dst] = c["kc"][src], c["ks"][src], c["vc"][src], c["vs"][src]
        part = torch.empty(pbytes // 4, dtype=torch.float32, device="cuda")
        gmoe.call("gm_bq_attention_partial", dev(c["q_i8"]), dev(c["fq"]), dev(kc), dev(ks), dev(vc), dev(vs),
                  runs, dev(c["base_rows"]), T, hd, nq, nkv, 0, degree, r, SHIFT, PAGE - 1, -1, c["max_kv"],
                  part, ws, ws_bytes, None)
        parts.append(part)
    out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device="cuda")
    ptrs = (gmoe.C.c_void_p * degree)(*[p.data_ptr() for p in parts])
    gmoe.check(gmoe.lib().gm_bq_attention_merge(ptrs, degree, T, nq, hd, out.data_ptr(), None))
    torch.cuda.synchronize()
    got = O.bf16_to_f32(host(out)).astype(np.float64)
    ref = decode_f64(c["q_i8"], c["fq"], c["kc"], c["ks"], c["vc"], c["vs"], c["slots"], c["kv_len"], cfg)
    scale = np.abs(ref).max()
    assert np.abs(got - O.bf16_to_f32(host(whole))).max() <= 1e-2 * scale
    assert np.abs(got - ref).max() <= 1e-2 * scale
    # position 0's token lives on rank 0 alone: its rank-1 partial is empty
    p1 = host(parts[1]).reshape(T, nq, hd + 2)
    assert (p1[0, :, 1] == 0).all()
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):  # sliding windows are never sharded
        gmoe.call("gm_bq_attention_partial", dev(c["q_i8"]), dev(c["fq"]), dev(c["kc"]), dev(c["ks"]),
                  dev(c["vc"]), dev(c["vs"]), runs, dev(c["base_rows"]), T, hd, nq, nkv, 64, degree, 0, SHIFT,
                  PAGE - 1, -1, c["max_kv"], parts[0], ws, ws_bytes, None)


@pytest.mark.parametrize("cfg,window", [(SLIDING, 128), (SLIDING, 1024), (FULL, 0)],
                         ids=["sliding-128", "sliding-1024", "full"])
def test_attention_prefill_chunks(cfg, window):
    """gm_bq_attention_prefill (attention.mojo:150-332) over two runs of one
    step -- a 300-token chunk continuing a sequence at position 500 and a new
    37-token sequence -- on randomly placed pages: every token equals the
    decode kernel's output for the same token (each token as the newest
    position of its own run) and a float64 softmax, within 1e-2 of max|ref|."""
    rng = np.random.default_rng(150 + window)
    hd, nq, nkv = cfg["head_dim"], cfg["num_q"], cfg["num_kv"]
    seqs = [(500, 300), (0, 37)]  # (first position, tokens)
    pages = [(p0 + n + PAGE - 1) // PAGE for p0, n in seqs]
    perm = rng.permutation(sum(pages))
    base_rows = (perm * PAGE).astype(np.int32)
    rows_off = [0, pages[0]]
    runs, tok_runs, positions = [], [], []
    for i, (p0, n) in enumerate(seqs):
        runs.append((len(positions), p0, rows_off[i], pages[i]))
        for j in range(n):
            tok_runs.append((len(positions), p0 + j, rows_off[i], pages[i]))
            positions.append((i, p0 + j))
    T = len(positions)
    kc, ks, vc, vs = random_cache(rng, sum(pages) * PAGE, cfg)
    ks *= 0.03
    q_i8 = rng.integers(-127, 128, size=(T, nq * hd), dtype=np.int8)
    fq = (rng.random((T, nq)) + 0.5).astype(np.float32)
    max_kv = max(min(p + 1, window) if window else p + 1 for _, p in positions)
    dq, dfq, dkc, dks, dvc, dvs, drows = (dev(x) for x in (q_i8, fq, kc, ks, vc, vs, base_rows))
    out = torch.empty(T, nq * hd, dtype=torch.bfloat16, device="cuda")
    gmoe.call("gm_bq_attention_prefill", dq, dfq, dkc, dks, dvc, dvs, dev(runs_array(runs)), len(runs), drows, T,
              hd, nq, nkv, window, SHIFT, PAGE - 1, -1, out, None)
    ws_bytes = gmoe.lib().gm_bq_attention_workspace_bytes(T, hd, nq, nkv, max_kv)
    ws = torch.empty(ws_bytes // 4, dtype=torch.float32, device="cuda")
    dec = torch.empty_like(out)
    gmoe.call("gm_bq_attention_decode", dq, dfq, dkc, dks, dvc, dvs, dev(runs_array(tok_runs)), drows, T, hd, nq,
              nkv, window, 1, 0, SHIFT, PAGE - 1, -1, max_kv, dec, ws, ws_bytes, None)
    torch.cuda.synchronize()
    got = O.bf16_to_f32(host(out)).astype(np.float64)
    want = O.bf16_to_f32(host(dec)).astype(np.float64)
    scale = np.abs(want).max()
    assert np.abs(got - want).max() <= 1e-2 * scale
    # float64 on a sample of tokens: both ends of each run and its window edge
    sample = sorted({0, 1, 15, 16, 17, 63, 64, 299, 300, 301, 320, T - 1})
    slots = np.zeros((len(sample), max_kv), np.int32)
    kv_len = np.zeros(len(sample), np.int32)
    for k, t in enumerate(sample):
        i, p = positions[t]
        valid = min(p + 1, window) if window else p + 1
        start = p - valid + 1
        kv_len[k] = valid
        for j in range(valid):
            q = start + j
            slots[k, j] = base_rows[rows_off[i] + (q >> SHIFT)] + (q & (PAGE - 1))
    ref = decode_f64(q_i8[sample], fq[sample], kc, ks, vc, vs, slots, kv_len, cfg)
    assert np.abs(got[sample] - ref).max() <= 1e-2 * scale


def test_attention_prefill_argument_checks():
    z = torch.zeros(16, dtype=torch.int8, device="cuda")
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):  # 4 query heads per KV head at 256
        gmoe.call("gm_bq_attention_prefill", z, z, z, z, z, z, z, 1, z, 1, 256, 16, 4, 0, 6, 63, -1, z, None)
    with pytest.raises(gmoe.GmoeError, match="GM_EINVAL"):  # tokens without runs
        gmoe.call("gm_bq_attention_prefill", z, z, z, z, z, z, z, 0, z, 1, 512, 16, 2, 0, 6, 63, -1, z, None)
